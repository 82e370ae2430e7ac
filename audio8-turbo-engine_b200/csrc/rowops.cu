// Row-wise memory-bound kernels of the tick: residual add + RMSNorm, the slow AR input embedding, the fast AR
// input rows. One warp per row, 16-byte vector loads; every kernel is a PDL secondary (griddepcontrol.wait before
// its first dependent read).
#include "common.cuh"

namespace a8 {

constexpr int MAXV = 4;   // 16-byte vectors per lane: rows of up to 32 * 4 * 8 = 1024 bf16

__device__ __forceinline__ void ld8(const __nv_bfloat16* p, float* f) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  float2 a = unpack_bf16(u.x), b = unpack_bf16(u.y), c = unpack_bf16(u.z), d = unpack_bf16(u.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y; f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}
__device__ __forceinline__ void st8(__nv_bfloat16* p, const float* f) {
  *reinterpret_cast<uint4*>(p) =
      make_uint4(pack_bf16(f[0], f[1]), pack_bf16(f[2], f[3]), pack_bf16(f[4], f[5]), pack_bf16(f[6], f[7]));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  return v;
}

// HF RMSNorm with the reference's rounding points (serve/fast_kernels.py:30-46):
//   h = bf16(x + res) (stored back to res), var = mean(h^2) in fp32, y = bf16(w * bf16(h * rsqrt(var + eps)))
__global__ void k_rmsnorm(const __nv_bfloat16* __restrict__ x, int ldx, __nv_bfloat16* res, int ldr,
                          const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ y, int ldy, int rows, int N,
                          float eps) {
  pdl_launch();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  // the weight (never written by a previous kernel) is read before waiting for that kernel
  float wv[MAXV][8];
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c = (lane + 32 * i) * 8;
    if (c < N) ld8(w + c, wv[i]);
  }
  pdl_wait();
  if (row >= rows) return;
  const int nv = N >> 3;
  float v[MAXV][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c = (lane + 32 * i) * 8;
    if (c < N) {
      ld8(x + (size_t)row * ldx + c, v[i]);
      if (res != nullptr) {
        float r[8];
        ld8(res + (size_t)row * ldr + c, r);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[i][k] = bf16r(v[i][k] + r[k]);
        st8(res + (size_t)row * ldr + c, v[i]);
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) ss += v[i][k] * v[i][k];
    }
  }
  (void)nv;
  ss = warp_sum(ss);
  const float rs = rsqrtf(ss / (float)N + eps);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c = (lane + 32 * i) * 8;
    if (c < N) {
      float o[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) o[k] = wv[i][k] * bf16r(v[i][k] * rs);
      st8(y + (size_t)row * ldy + c, o);
    }
  }
}

// Slow AR input of an audio frame (serve/fast_engine.py:715-717): emb[sem] + sum_k cbemb[codes_k + 4096 k];
// the codebook sum is one bf16 rounding of an fp32 sum, then a bf16 add.
__global__ void k_embed_frame(const int64_t* __restrict__ sem, const int64_t* __restrict__ codes, int ncb, int cbk,
                              const __nv_bfloat16* __restrict__ emb, const __nv_bfloat16* __restrict__ cbemb,
                              __nv_bfloat16* __restrict__ x, int ldx, int rows, int H, int vocab) {
  pdl_launch();
  pdl_wait();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  long long s = sem[row];
  s = s < 0 ? 0 : (s >= vocab ? vocab - 1 : s);
  for (int c = lane * 8; c < H; c += 256) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int k = 0; k < ncb; ++k) {
      long long cd = codes[(size_t)row * ncb + k];
      cd = cd < 0 ? 0 : (cd >= cbk ? cbk - 1 : cd);
      float e[8];
      ld8(cbemb + ((size_t)k * cbk + cd) * H + c, e);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += e[i];
    }
    float e0[8];
    ld8(emb + (size_t)s * H + c, e0);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = e0[i] + bf16r(acc[i]);
    st8(x + (size_t)row * ldx + c, acc);
  }
}

// Packed prompt rows (serve/fast_engine.py:941-945, _prompt_embeds): ids[r] = (sem, audio, code_0 .. code_{ncb-1})
// (int32): x[r] = emb[sem] on text positions, bf16(emb[sem] + bf16(sum_k cbemb[code_k + cbk k])) on audio positions
// (the codebook sum in fp32, k in order, rounded once).
__global__ void k_embed_prompt(const int* __restrict__ ids, int ncb, int cbk, const __nv_bfloat16* __restrict__ emb,
                               const __nv_bfloat16* __restrict__ cbemb, __nv_bfloat16* __restrict__ x, int ldx,
                               int rows, int H, int vocab) {
  pdl_launch();
  pdl_wait();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int* id = ids + (size_t)row * (2 + ncb);
  int s = id[0];
  s = s < 0 ? 0 : (s >= vocab ? vocab - 1 : s);
  const bool audio = id[1] != 0;
  for (int c = lane * 8; c < H; c += 256) {
    float e0[8];
    ld8(emb + (size_t)s * H + c, e0);
    if (audio) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int k = 0; k < ncb; ++k) {
        int cd = id[2 + k];
        cd = cd < 0 ? 0 : (cd >= cbk ? cbk - 1 : cd);
        float e[8];
        ld8(cbemb + ((size_t)k * cbk + cd) * H + c, e);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] += e[i];
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) e0[i] += bf16r(acc[i]);
    }
    st8(x + (size_t)row * ldx + c, e0);
  }
}

// Tick start (serve/fast_engine.py:742-749, :705): tok_in = tok; code0 = clamp(tok - sb, 0, cbk-1) into codes[:, 0];
// the fast AR's 2-token rows x[2r] = hid[r], x[2r+1] = fast_emb[code0]; block 0 also draws this tick's number
// from the counter (tick_id[0] = ctr[0]++).
__global__ void k_tick_start(const int64_t* __restrict__ tok, int64_t* __restrict__ tok_in, int64_t* __restrict__ codes,
                             int ncb, long long sb, int cbk, const __nv_bfloat16* __restrict__ hid,
                             const __nv_bfloat16* __restrict__ fast_emb, __nv_bfloat16* __restrict__ x2, int rows, int H,
                             long long* ctr, long long* tick_id) {
  pdl_launch();
  pdl_wait();
  if (blockIdx.x == 0 && threadIdx.x == 0 && ctr != nullptr) {
    tick_id[0] = ctr[0];
    ctr[0] = ctr[0] + 1;
  }
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const long long t = tok[row];
  long long c0 = t - sb;
  c0 = c0 < 0 ? 0 : (c0 >= cbk ? cbk - 1 : c0);
  if (lane == 0) {
    tok_in[row] = t;
    codes[(size_t)row * ncb] = c0;
  }
  for (int c = lane * 8; c < H; c += 256) {
    *reinterpret_cast<uint4*>(x2 + (size_t)(2 * row) * H + c) = *reinterpret_cast<const uint4*>(hid + (size_t)row * H + c);
    *reinterpret_cast<uint4*>(x2 + (size_t)(2 * row + 1) * H + c) =
        *reinterpret_cast<const uint4*>(fast_emb + (size_t)c0 * H + c);
  }
}

// Gather rows: y[r] = src[idx[r] * idx_stride] (bf16 rows of H), e.g. the last packed prefill row of each request.
__global__ void k_gather_rows(const __nv_bfloat16* __restrict__ src, int lds, const int* __restrict__ idx,
                              __nv_bfloat16* __restrict__ y, int ldy, int rows, int H) {
  pdl_launch();
  pdl_wait();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int s = idx[row];
  for (int c = lane * 8; c < H; c += 256)
    *reinterpret_cast<uint4*>(y + (size_t)row * ldy + c) = *reinterpret_cast<const uint4*>(src + (size_t)s * lds + c);
}

static cudaError_t launch_pdl(const void* fn, dim3 grid, dim3 block, void** args, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  ++g_launches;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace a8

using namespace a8;

extern "C" int a8_rmsnorm(const void* x, int ldx, void* res, int ldr, const void* w, void* y, int ldy, int rows, int N,
                          float eps, a8_stream_t stream) {
  if (x == nullptr || w == nullptr || y == nullptr || rows <= 0 || N <= 0 || N > 1024 || (N % 8)) return A8_ERR_ARG;
  if ((ldx % 8) || (ldy % 8) || (res != nullptr && (ldr % 8))) return A8_ERR_ALIGN;
  const __nv_bfloat16* xp = reinterpret_cast<const __nv_bfloat16*>(x);
  __nv_bfloat16* rp = reinterpret_cast<__nv_bfloat16*>(res);
  const __nv_bfloat16* wp = reinterpret_cast<const __nv_bfloat16*>(w);
  __nv_bfloat16* yp = reinterpret_cast<__nv_bfloat16*>(y);
  void* args[] = {&xp, &ldx, &rp, &ldr, &wp, &yp, &ldy, &rows, &N, &eps};
  return launch_pdl((const void*)k_rmsnorm, dim3((rows + 3) / 4), dim3(128), args,
                    reinterpret_cast<cudaStream_t>(stream)) == cudaSuccess ? A8_OK : A8_ERR_CUDA;
}

extern "C" int a8_embed_frame(const int64_t* sem, const int64_t* codes, int ncb, int cbk, const void* emb,
                              const void* cbemb, void* x, int ldx, int rows, int H, int vocab, a8_stream_t stream) {
  if (sem == nullptr || codes == nullptr || emb == nullptr || cbemb == nullptr || x == nullptr || rows <= 0 ||
      (H % 8))
    return A8_ERR_ARG;
  const __nv_bfloat16* ep = reinterpret_cast<const __nv_bfloat16*>(emb);
  const __nv_bfloat16* cp = reinterpret_cast<const __nv_bfloat16*>(cbemb);
  __nv_bfloat16* xp = reinterpret_cast<__nv_bfloat16*>(x);
  void* args[] = {&sem, &codes, &ncb, &cbk, &ep, &cp, &xp, &ldx, &rows, &H, &vocab};
  return launch_pdl((const void*)k_embed_frame, dim3((rows + 3) / 4), dim3(128), args,
                    reinterpret_cast<cudaStream_t>(stream)) == cudaSuccess ? A8_OK : A8_ERR_CUDA;
}

extern "C" int a8_embed_prompt(const int* ids, int ncb, int cbk, const void* emb, const void* cbemb, void* x, int ldx,
                               int rows, int H, int vocab, a8_stream_t stream) {
  if (ids == nullptr || emb == nullptr || cbemb == nullptr || x == nullptr || rows <= 0 || (H % 8) || ncb < 0 ||
      cbk <= 0 || vocab <= 0)
    return A8_ERR_ARG;
  if ((ldx % 8) || (reinterpret_cast<uintptr_t>(x) & 15)) return A8_ERR_ALIGN;
  const __nv_bfloat16* ep = reinterpret_cast<const __nv_bfloat16*>(emb);
  const __nv_bfloat16* cp = reinterpret_cast<const __nv_bfloat16*>(cbemb);
  __nv_bfloat16* xp = reinterpret_cast<__nv_bfloat16*>(x);
  void* args[] = {&ids, &ncb, &cbk, &ep, &cp, &xp, &ldx, &rows, &H, &vocab};
  return launch_pdl((const void*)k_embed_prompt, dim3((rows + 3) / 4), dim3(128), args,
                    reinterpret_cast<cudaStream_t>(stream)) == cudaSuccess ? A8_OK : A8_ERR_CUDA;
}

extern "C" int a8_tick_start(const int64_t* tok, int64_t* tok_in, int64_t* codes, int ncb, long long sb, int cbk,
                             const void* hid, const void* fast_emb, void* x2, int rows, int H, long long* ctr,
                             long long* tick_id, a8_stream_t stream) {
  if (tok == nullptr || tok_in == nullptr || codes == nullptr || hid == nullptr || fast_emb == nullptr ||
      x2 == nullptr || rows <= 0 || (H % 8))
    return A8_ERR_ARG;
  const __nv_bfloat16* hp = reinterpret_cast<const __nv_bfloat16*>(hid);
  const __nv_bfloat16* fp = reinterpret_cast<const __nv_bfloat16*>(fast_emb);
  __nv_bfloat16* xp = reinterpret_cast<__nv_bfloat16*>(x2);
  void* args[] = {&tok, &tok_in, &codes, &ncb, &sb, &cbk, &hp, &fp, &xp, &rows, &H, &ctr, &tick_id};
  return launch_pdl((const void*)k_tick_start, dim3((rows + 3) / 4), dim3(128), args,
                    reinterpret_cast<cudaStream_t>(stream)) == cudaSuccess ? A8_OK : A8_ERR_CUDA;
}

extern "C" int a8_gather_rows(const void* src, int lds, const int* idx, void* y, int ldy, int rows, int H,
                              a8_stream_t stream) {
  if (src == nullptr || idx == nullptr || y == nullptr || rows <= 0 || (H % 8)) return A8_ERR_ARG;
  const __nv_bfloat16* sp = reinterpret_cast<const __nv_bfloat16*>(src);
  __nv_bfloat16* yp = reinterpret_cast<__nv_bfloat16*>(y);
  void* args[] = {&sp, &lds, &idx, &yp, &ldy, &rows, &H};
  return launch_pdl((const void*)k_gather_rows, dim3((rows + 3) / 4), dim3(128), args,
                    reinterpret_cast<cudaStream_t>(stream)) == cudaSuccess ? A8_OK : A8_ERR_CUDA;
}
