// Memory-bound kernels of the streaming codec decoder (serve/fast_engine.py:312-494, StreamingVocoder.step):
//   k_codec_embed   codes -> code-table sum (fp32) -> bf16 transformer input; the window transformer's positions
//   k_conv_input    a conv's input rows (after its carried context) from a tensor, activated or copied
//   k_ups_dwln      upsample stage: causal 7-tap depthwise conv with carried tail + LayerNorm (bf16 op by op)
// All are PDL secondaries; a batch row's carried state is updated inside one block.
#include "common.cuh"

namespace a8 {

// codes [rows, ncb] (the LLM's codes; clamped like the codec): x[r] = bf16(t_sem[c0] + sum_k t_res[k, c_k]) with the
// sum over the residual tables first, in k order. Positions of the window transformer: pos_c = min(pos, max_pos - 1),
// lens = min(pos + 1, window); pos advances by one frame (serve/fast_engine.py:472-477, :493).
__global__ void k_codec_embed(const int64_t* __restrict__ codes, int ncb, const float* __restrict__ t_sem, int v_sem,
                              const float* __restrict__ t_res, int v_res, int C, __nv_bfloat16* __restrict__ x,
                              int* pos, int* pos_c, int* lens, int max_pos, int window, int rows) {
  pdl_launch();
  pdl_wait();
  const int r = blockIdx.x;
  if (r >= rows) return;
  const int64_t* cr = codes + (size_t)r * ncb;
  long long c0 = cr[0];
  c0 = c0 < 0 ? 0 : (c0 >= v_sem ? v_sem - 1 : c0);
  for (int c = threadIdx.x * 4; c < C; c += blockDim.x * 4) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 1; k < ncb; ++k) {
      long long ck = cr[k];
      ck = ck < 0 ? 0 : (ck >= v_res ? v_res - 1 : ck);
      const float4 t = *reinterpret_cast<const float4*>(t_res + ((size_t)(k - 1) * v_res + ck) * C + c);
      s.x += t.x; s.y += t.y; s.z += t.z; s.w += t.w;
    }
    const float4 e = *reinterpret_cast<const float4*>(t_sem + (size_t)c0 * C + c);
    *reinterpret_cast<uint2*>(x + (size_t)r * C + c) =
        make_uint2(pack_bf16(e.x + s.x, e.y + s.y), pack_bf16(e.z + s.z, e.w + s.w));
  }
  if (threadIdx.x == 0) {
    const int p = pos[r];
    pos_c[r] = p < max_pos - 1 ? p : max_pos - 1;
    lens[r] = p + 1 < window ? p + 1 : window;
    pos[r] = p + 1;
  }
}

// 8 consecutive 16-bit values -> fp32
__device__ __forceinline__ void load8(const __half* p, float* v) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack_f16(w[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* v) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack_bf16(w[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// A conv's input rows from a tensor: xin[b, ctx + t, c] = fp16(act(x[b, t, c])), act(v) = v + inv * sin(alpha v)^2
// in fp32 (serve/fast_kernels.py:695-729 snake_cat; the context rows [0, ctx) already hold the carried context);
// alpha == null: plain fp16 copy. grid (rows, parts): part p of batch row b, 8 channels a thread.
template <typename TIn>
__global__ void k_conv_input(const TIn* __restrict__ x, long long x_bs, int T, int C, __half* __restrict__ xin,
                             int ctx, const float* __restrict__ alpha, const float* __restrict__ inv, int rows) {
  pdl_launch();
  pdl_wait();
  const int b = blockIdx.x;
  if (b >= rows) return;
  __half* xb = xin + ((size_t)b * (ctx + T) + ctx) * C;
  const TIn* src = x + (size_t)b * x_bs;
  const int total = T * C;
  for (int idx = (blockIdx.y * blockDim.x + threadIdx.x) * 8; idx < total; idx += gridDim.y * blockDim.x * 8) {
    const int c = idx % C;                             // C is a multiple of 8: the 8 channels share a row
    float v[8];
    load8(src + idx, v);
    if (alpha != nullptr) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float s = sinf(v[i] * alpha[c + i]);
        v[i] = v[i] + inv[c + i] * s * s;
      }
    }
    *reinterpret_cast<uint4*>(xb + idx) =
        make_uint4(pack_f16(v[0], v[1]), pack_f16(v[2], v[3]), pack_f16(v[4], v[5]), pack_f16(v[6], v[7]));
  }
}

// Upsample stage tail (serve/fast_engine.py:484-489): y[t] = dwb + sum_j xin[t + j] * w[j] with a bf16 rounding after
// every product and every add (as the reference's eager bf16 ops), xin = [st (k-1 rows) ; u (T rows)], then
// st = xin[T:], then LayerNorm over C (fp32 statistics, bf16 out). One block per batch row, C / 4 threads.
__global__ void k_ups_dwln(const __nv_bfloat16* __restrict__ u, int T, int C, __nv_bfloat16* st, long long st_bs, int K,
                           const __nv_bfloat16* __restrict__ dww, const __nv_bfloat16* __restrict__ dwb,
                           const __nv_bfloat16* __restrict__ lnw, const __nv_bfloat16* __restrict__ lnb, float eps,
                           __nv_bfloat16* __restrict__ z, int rows) {
  __shared__ float red[2][32];
  pdl_launch();
  pdl_wait();
  const int b = blockIdx.x;
  if (b >= rows) return;
  const int ctx = K - 1;
  const __nv_bfloat16* ub = u + (size_t)b * T * C;
  __nv_bfloat16* sb = st + (size_t)b * st_bs;
  const int c0 = threadIdx.x * 4;                     // blockDim.x * 4 == C
  float w[8][4], bias[4];
  for (int j = 0; j < K; ++j)
    for (int i = 0; i < 4; ++i) w[j][i] = __bfloat162float(dww[(size_t)j * C + c0 + i]);
  for (int i = 0; i < 4; ++i) bias[i] = __bfloat162float(dwb[c0 + i]);
  auto xin = [&](int row, int i) -> float {
    return row < ctx ? __bfloat162float(sb[(size_t)row * C + c0 + i]) : __bfloat162float(ub[(size_t)(row - ctx) * C + c0 + i]);
  };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int t = 0; t < T; ++t) {
    float y[4];
    for (int i = 0; i < 4; ++i) {
      float acc = bf16r(bias[i] + bf16r(xin(t, i) * w[0][i]));
      for (int j = 1; j < K; ++j) acc = bf16r(acc + bf16r(xin(t + j, i) * w[j][i]));
      y[i] = acc;
    }
    float s = y[0] + y[1] + y[2] + y[3];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffff, s, o);
    if (lane == 0) red[0][warp] = s;
    __syncthreads();
    float mean = 0.f;
    for (int k = 0; k < nw; ++k) mean += red[0][k];
    mean /= C;
    float q = 0.f;
    for (int i = 0; i < 4; ++i) q += (y[i] - mean) * (y[i] - mean);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffff, q, o);
    if (lane == 0) red[1][warp] = q;
    __syncthreads();
    float var = 0.f;
    for (int k = 0; k < nw; ++k) var += red[1][k];
    var /= C;
    const float rs = rsqrtf(var + eps);
    __nv_bfloat16* zr = z + ((size_t)b * T + t) * C + c0;
    for (int i = 0; i < 4; ++i)
      zr[i] = __float2bfloat16_rn((y[i] - mean) * rs * __bfloat162float(lnw[c0 + i]) + __bfloat162float(lnb[c0 + i]));
    __syncthreads();                                   // red[] is reused by the next row
  }
  // carried tail: st = xin[T : T + ctx] (rows of the old tail when T < ctx): read everything, then write
  float nt[8][4];
  for (int i = 0; i < ctx; ++i)
    for (int k = 0; k < 4; ++k) nt[i][k] = xin(T + i, k);
  __syncthreads();
  for (int i = 0; i < ctx; ++i)
    for (int k = 0; k < 4; ++k) sb[(size_t)i * C + c0 + k] = __float2bfloat16_rn(nt[i][k]);
}

static cudaError_t launch_rows(const void* fn, int rows, int threads, void** args, cudaStream_t s, int parts = 1) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rows, parts);
  cfg.blockDim = dim3(threads);
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  ++g_launches;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

int codec_embed(const int64_t* codes, int ncb, const float* t_sem, int v_sem, const float* t_res, int v_res, int C,
                void* x, int* pos, int* pos_c, int* lens, int max_pos, int window, int rows, cudaStream_t s) {
  __nv_bfloat16* xp = reinterpret_cast<__nv_bfloat16*>(x);
  void* args[] = {&codes, &ncb, &t_sem, &v_sem, &t_res, &v_res, &C, &xp, &pos, &pos_c, &lens, &max_pos, &window, &rows};
  return launch_rows((const void*)k_codec_embed, rows, 256, args, s) == cudaSuccess ? A8_OK : A8_ERR_CUDA;
}

int conv_input(const void* x, int x_bf16, long long x_bs, int T, int C, void* xin, int ctx, const float* alpha,
               const float* inv, int rows, cudaStream_t s) {
  if (C % 8 || x_bs % 8) return A8_ERR_ARG;
  __half* xp = reinterpret_cast<__half*>(xin);
  const int parts = std::max(1, std::min(64, (T * C / 8 + 255) / 256));
  if (x_bf16) {
    const __nv_bfloat16* xs = reinterpret_cast<const __nv_bfloat16*>(x);
    void* args[] = {&xs, &x_bs, &T, &C, &xp, &ctx, &alpha, &inv, &rows};
    return launch_rows((const void*)k_conv_input<__nv_bfloat16>, rows, 256, args, s, parts) == cudaSuccess
               ? A8_OK
               : A8_ERR_CUDA;
  }
  const __half* xs = reinterpret_cast<const __half*>(x);
  void* args[] = {&xs, &x_bs, &T, &C, &xp, &ctx, &alpha, &inv, &rows};
  return launch_rows((const void*)k_conv_input<__half>, rows, 256, args, s, parts) == cudaSuccess ? A8_OK
                                                                                                   : A8_ERR_CUDA;
}

int ups_dwln(const void* u, int T, int C, void* st, long long st_bs, int K, const void* dww, const void* dwb,
             const void* lnw, const void* lnb, float eps, void* z, int rows, cudaStream_t s) {
  if (C % 128 || C > 4096 || K > 8) return A8_ERR_ARG;
  const __nv_bfloat16* up = reinterpret_cast<const __nv_bfloat16*>(u);
  __nv_bfloat16* sp = reinterpret_cast<__nv_bfloat16*>(st);
  const __nv_bfloat16 *wp = reinterpret_cast<const __nv_bfloat16*>(dww), *bp = reinterpret_cast<const __nv_bfloat16*>(dwb);
  const __nv_bfloat16 *lw = reinterpret_cast<const __nv_bfloat16*>(lnw), *lb = reinterpret_cast<const __nv_bfloat16*>(lnb);
  __nv_bfloat16* zp = reinterpret_cast<__nv_bfloat16*>(z);
  void* args[] = {&up, &T, &C, &sp, &st_bs, &K, &wp, &bp, &lw, &lb, &eps, &zp, &rows};
  return launch_rows((const void*)k_ups_dwln, rows, C / 4, args, s) == cudaSuccess ? A8_OK : A8_ERR_CUDA;
}

}  // namespace a8

using namespace a8;

extern "C" int a8_conv_input(const void* x, int x_bf16, long long x_bs, int T, int C, void* xin, int ctx,
                             const float* alpha, const float* inv, int rows, a8_stream_t stream) {
  if (x == nullptr || xin == nullptr || rows <= 0 || T <= 0 || ctx < 0 || (alpha != nullptr && inv == nullptr))
    return A8_ERR_ARG;
  return conv_input(x, x_bf16, x_bs, T, C, xin, ctx, alpha, inv, rows, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int a8_ups_dwln(const void* u, int T, int C, void* st, long long st_bs, int K, const void* dww, const void* dwb,
                           const void* lnw, const void* lnb, float eps, void* z, int rows, a8_stream_t stream) {
  if (u == nullptr || st == nullptr || z == nullptr || rows <= 0) return A8_ERR_ARG;
  return ups_dwln(u, T, C, st, st_bs, K, dww, dwb, lnw, lnb, eps, z, rows, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int a8_codec_embed(const int64_t* codes, int ncb, const float* t_sem, int v_sem, const float* t_res,
                              int v_res, int C, void* x, int* pos, int* pos_c, int* lens, int max_pos, int window,
                              int rows, a8_stream_t stream) {
  if (codes == nullptr || t_sem == nullptr || t_res == nullptr || x == nullptr || pos == nullptr || rows <= 0 ||
      (C % 4))
    return A8_ERR_ARG;
  return codec_embed(codes, ncb, t_sem, v_sem, t_res, v_res, C, x, pos, pos_c, lens, max_pos, window, rows,
                     reinterpret_cast<cudaStream_t>(stream));
}
