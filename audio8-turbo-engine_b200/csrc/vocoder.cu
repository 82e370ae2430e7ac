// The streaming codec decoder step and its per-slot state arena, as sequences of the library's kernels
// (serve/fast_engine.py:312-494 StreamingVocoder).
//
//   codes -> code tables (k_codec_embed) -> window transformer (stack_forward, ring = window)
//         -> n_ups x [GEMM (transposed conv k=s=2), dwconv+LayerNorm (k_ups_dwln), GEMM+GELU, GEMM+LayerScale+res]
//         -> conv program: per op, context+snake (k_snake_cat) then the implicit-GEMM conv (k_conv); the last op
//            writes tanh audio.
#include "common.cuh"

namespace a8 {

int stack_forward(const A8StackDesc& d, const A8StackRun& r, cudaStream_t s);
int voc_decode(const A8Vocoder& v, const void* u, int b, cudaStream_t s);

static int voc_gemm(const void* x, int ldx, const void* w, int N, int K, int M, void* y, int ldy, const A8Epilogue& e,
                    cudaStream_t s) {
  GemmPlan p;
  int rc = gemm_plan(&p, x, ldx, w, N, K, M, y, ldy, &e, 0);
  if (rc) return rc;
  return gemm_launch(&p, s, true);
}

// after_read (may be null): recorded once the codes have been read
int voc_step(const A8Vocoder& v, const int64_t* codes, int b, cudaStream_t s, cudaEvent_t after_read) {
  if (b <= 0 || b > v.B || v.n_ups > A8_MAX_UPS || v.n_ops > A8_MAX_CONV_OPS || v.n_ops <= 0) return A8_ERR_ARG;
  const int C = v.C;
  int rc = codec_embed(codes, v.ncb, v.t_sem, v.v_sem, v.t_res, v.v_res, C, v.x, v.pos, v.pos_c, v.lens, v.max_pos,
                       v.window, b, s);
  if (rc) return rc;
  if (after_read != nullptr && cudaEventRecord(after_read, s) != cudaSuccess) return A8_ERR_CUDA;
  A8StackRun r = {};
  r.x = v.x;
  r.ldx = C;
  r.rows = b;
  r.pos = v.pos_c;
  r.lens = v.lens;
  r.lens_max = v.window;
  r.max_len = v.window;
  r.scratch = v.scratch;
  rc = stack_forward(v.post, r, s);
  if (rc) return rc;

  // upsample stages: rows (b, t) of [b * T, C]; ubuf 0 = transposed conv out (the residual), 1 = LayerNorm out,
  // 2 = GELU out, 3 = the stage's output (the next stage's input)
  const void* xs = v.scratch.h;
  int T = 1;
  for (int i = 0; i < v.n_ups; ++i) {
    const A8Upsample& u = v.ups[i];
    A8Epilogue e = {};
    e.kind = A8_EPI_BF16;
    e.bias = u.tb;
    if ((rc = voc_gemm(xs, C, u.tw, 2 * C, C, b * T, v.ubuf[0], 2 * C, e, s))) return rc;
    T *= 2;
    if ((rc = ups_dwln(v.ubuf[0], T, C, u.st, u.st_bs, u.K, u.dww, u.dwb, u.lnw, u.lnb, u.eps, v.ubuf[1], b, s)))
      return rc;
    A8Epilogue g = {};
    g.kind = A8_EPI_GELU;
    g.bias = u.b1;
    if ((rc = voc_gemm(v.ubuf[1], C, u.w1, u.mlp, C, b * T, v.ubuf[2], u.mlp, g, s))) return rc;
    A8Epilogue l = {};
    l.kind = A8_EPI_LSRES;
    l.bias = u.b2;
    l.gamma = u.gamma;
    l.res = v.ubuf[0];
    l.ldres = C;
    if ((rc = voc_gemm(v.ubuf[2], u.mlp, u.w2, C, u.mlp, b * T, v.ubuf[3], C, l, s))) return rc;
    xs = v.ubuf[3];
  }

  return voc_decode(v, xs, b, s);
}

// The conv decoder on u (bf16 [b, T0, C], T0 = the first op's T): the first op's input rows from u; each op's epilogue
// writes the next op's input rows (activated) and, where a later residual needs it, its raw output; the last op writes
// the audio; then every context advances one frame.
int voc_decode(const A8Vocoder& v, const void* u, int b, cudaStream_t s) {
  if (b <= 0 || b > v.B || v.n_ops > A8_MAX_CONV_OPS || v.n_ops <= 0) return A8_ERR_ARG;
  const A8ConvOp& op0 = v.ops[0];
  int rc = conv_input(u, 1, (long long)op0.T * op0.Cin, op0.T, op0.Cin, op0.xin, op0.ctx, op0.alpha, op0.inv, b, s);
  if (rc) return rc;
  for (int i = 0; i < v.n_ops; ++i) {
    const A8ConvOp& op = v.ops[i];
    if (op.raw < -1 || op.raw > 1 || op.res < -1 || op.res > 1 || op.xin == nullptr) return A8_ERR_ARG;
    ConvPlan p;
    if ((rc = conv_plan(&p, op.xin, b, op.T, op.Cin, op.ctx, op.w, op.N, op.taps, op.dil))) return rc;
    ConvArgs& a = p.args;
    a.bias = reinterpret_cast<const float*>(op.bias);
    if (op.res >= 0) {
      a.res = reinterpret_cast<const __half*>(v.act[op.res]);
      a.res_bs = (long long)op.T * op.N;
      a.res_ts = op.N;
    }
    if (op.raw >= 0) {
      a.raw = reinterpret_cast<__half*>(v.act[op.raw]);
      a.raw_bs = (long long)op.T * op.N;
      a.raw_ts = op.N;
    }
    if (i + 1 < v.n_ops) {
      const A8ConvOp& nx = v.ops[i + 1];
      if (op.N % nx.Cin || nx.T != op.T * (op.N / nx.Cin)) return A8_ERR_ARG;
      a.nxt = reinterpret_cast<__half*>(nx.xin);
      a.nxt_bs = (long long)(nx.ctx + nx.T) * nx.Cin;
      a.nxt_off = (long long)nx.ctx * nx.Cin;
      a.cout = nx.Cin;
      a.alpha = nx.alpha;
      a.inv = nx.inv;
    } else {
      if (op.T != v.up) return A8_ERR_ARG;
      a.audio = v.audio;
      a.audio_bs = v.up;
    }
    if (v.conv_ctas > 0 && (int)p.grid.x > v.conv_ctas) p.grid.x = v.conv_ctas;
    if ((rc = conv_launch(&p, s))) return rc;
  }
  // every context advances one frame
  if (v.n_ctx > 0 && (rc = ctx_shift_launch(v.ctx_table, v.n_ctx, b, s))) return rc;
  return A8_OK;
}

// ------------------------------------------------------------------------------------------------ state arena
// grid (parts, nseg, nslots): part p of segment g for slot slots[z] -- the segment's words (chunk-major) split evenly;
// 16-byte words where every address and size of the segment allows, else 4-byte words
template <typename W>
__device__ __forceinline__ void state_copy(const A8StateSeg& g, uint8_t* row, uint8_t* blob, int op) {
  const long long per_chunk = g.chunk_bytes / (long long)sizeof(W);
  const long long total = per_chunk * g.nchunks;
  const long long part = (total + gridDim.x - 1) / gridDim.x;
  const long long lo = blockIdx.x * part, hi = min(total, lo + part);
  W* bl = reinterpret_cast<W*>(blob != nullptr ? blob + g.blob_off : nullptr);
  for (long long i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const long long k = i / per_chunk, o = i % per_chunk;
    W* p = reinterpret_cast<W*>(row + k * g.chunk_stride) + o;
    if (op == A8_STATE_CLEAR)
      *p = W{};
    else if (op == A8_STATE_LOAD)
      *p = bl[i];
    else
      bl[i] = *p;
  }
}

__global__ void k_state_rows(const A8StateSeg* __restrict__ segs, const int* __restrict__ slots, int op,
                             uint8_t* __restrict__ blob) {
  pdl_launch();
  pdl_wait();
  const A8StateSeg g = segs[blockIdx.y];
  const int slot = slots[blockIdx.z];
  uint8_t* row = reinterpret_cast<uint8_t*>(g.base) + (size_t)slot * g.slot_stride;
  const long long any = reinterpret_cast<long long>(row) | g.chunk_bytes | g.chunk_stride | g.blob_off;
  if ((any & 15) == 0)
    state_copy<uint4>(g, row, blob, op);
  else
    state_copy<uint32_t>(g, row, blob, op);
}

}  // namespace a8

using namespace a8;

extern "C" int a8_voc_step(const A8Vocoder* v, const int64_t* codes, int b, a8_stream_t stream) {
  if (v == nullptr || codes == nullptr) return A8_ERR_ARG;
  return voc_step(*v, codes, b, reinterpret_cast<cudaStream_t>(stream), nullptr);
}

extern "C" int a8_voc_decode(const A8Vocoder* v, const void* u, int b, a8_stream_t stream) {
  if (v == nullptr || u == nullptr) return A8_ERR_ARG;
  return voc_decode(*v, u, b, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int a8_state_rows(const A8StateSeg* segs, int nseg, const int* slots, int nslots, int op, void* blob,
                             a8_stream_t stream) {
  if (segs == nullptr || slots == nullptr || nseg <= 0 || nslots <= 0 || op < 0 || op > 2) return A8_ERR_ARG;
  if (op != A8_STATE_CLEAR && blob == nullptr) return A8_ERR_ARG;
  if (op == A8_STATE_SNAPSHOT) nslots = 1;
  if ((reinterpret_cast<uintptr_t>(blob) & 15)) return A8_ERR_ALIGN;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(16, nseg, nslots);
  cfg.blockDim = dim3(256);
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  ++g_launches;
  uint8_t* bp = reinterpret_cast<uint8_t*>(blob);
  return cudaLaunchKernelEx(&cfg, k_state_rows, segs, slots, op, bp) == cudaSuccess ? A8_OK : A8_ERR_CUDA;
}
