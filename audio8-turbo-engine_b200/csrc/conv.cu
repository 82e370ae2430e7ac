// Channels-last causal convolution / polyphase transposed convolution of the codec's conv decoder as a tcgen05
// implicit GEMM (serve/fast_kernels.py:551-623 conv_cl; serve/fast_engine.py:178-232 _CLConv).
//
//   out[b, t, n] = epi( sum_j sum_c xin[b, t + j*dil, c] * W[n, j*Cin + c] ),   t in [0, T)
//
// xin is the context-padded input [rows, ctx + T, Cin] (fp16, the left context first). A transposed conv (stride s,
// kernel 2s, right crop s) is a 2-tap conv whose N = s * Cout holds every phase (n = p * Cout + c), so row (b, t) of
// the result is already output rows t*s .. t*s+s-1 of [rows, T*s, Cout].
//
// One CTA = 128 token rows (TB batch rows x TT timesteps) x ntile output channels. The A tile of K block (tap j,
// channel block c) is ONE 3-D TMA box {KC, TT, TB} at (c*KC, t0 + j*dil, b0) of xin viewed as [rows][ctx+T][Cin] --
// the tap shift is just a coordinate. B = weight tile {KC, ntile}. fp16 x fp16 -> fp32 accumulator in TMEM
// (tcgen05.mma kind::f16), a TMA ring of stages, one producer lane, one MMA lane, four epilogue warps (thread = token
// row, tcgen05.ld 32 channels at a time): + bias, + residual, fp16 store; or tanh into fp32 audio (conv_out).
#include "common.cuh"

namespace a8 {

constexpr int KERNEL_ID_CONV = 4;

struct ConvArgs {
  int rows, T, Cin, N, taps, dil, ctx;
  int KC;                 // channels per K block: 64 (128-byte swizzle) or 32 (64-byte swizzle)
  int TT, TB;             // token tile: TB batch rows x TT timesteps (TT * TB == 128)
  int ntile, n_tiles;
  int kb_total, stages;
  uint32_t tmem_cols;
  const __half* bias;     // [N] or null
  const __half* res;      // residual, same indexing as out (fp16) or null
  long long res_bs, res_ts;
  void* out;
  long long out_bs, out_ts;   // element strides of a batch row and of a timestep row
  int mode;               // 0: fp16 out; 1: tanh of column 0 into fp32 out[b * out_bs + t]
};

template <int KC>
__global__ void __launch_bounds__(128, 1)
    k_conv(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW, const ConvArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int stages = a.stages;
  const uint32_t a_bytes = 128 * KC * 2, b_bytes = a.ntile * KC * 2;
  const uint32_t stage_bytes = a_bytes + b_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + stages * stage_bytes);
  uint64_t* empty = full + stages;
  uint64_t* accum = empty + stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tiles_t = a.T / a.TT;
  const int mt = blockIdx.x;                      // token tile: (batch group, time block)
  const int b0 = (mt / tiles_t) * a.TB, t0 = (mt % tiles_t) * a.TT;
  const int n0 = blockIdx.y * a.ntile;
  const int cblocks = a.Cin / KC;

  if (tid == 0) {
    tma_prefetch(&tmX);
    tma_prefetch(&tmW);
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, a.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch();

  auto tileA = [&](int s) { return smem + s * stage_bytes; };
  auto tileB = [&](int s) { return smem + s * stage_bytes + a_bytes; };
  const int nkb = a.kb_total;
  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_last(), pol_x = policy_evict_first();
      const int pre = min(stages, nkb);
      for (int i = 0; i < pre; ++i) {           // weights do not depend on the previous kernel
        mbar_arrive_expect_tx(&full[i], stage_bytes);
        const int j = i / cblocks, c = i % cblocks;
        tma_load_2d(tileB(i), &tmW, &full[i], j * a.Cin + c * KC, n0, pol_w);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i) {
        const int j = i / cblocks, c = i % cblocks;
        tma_load_3d(tileA(i), &tmX, &full[i], c * KC, t0 + j * a.dil, b0, pol_x);
      }
      int issued = pre;
      for (int i = pre; i < nkb; ++i) {
        const int s = i % stages;
        if (!mbar_wait(&empty[s], ((i / stages) - 1) & 1, ERR_TIMEOUT_EMPTY, KERNEL_ID_CONV)) break;
        const int j = i / cblocks, c = i % cblocks;
        mbar_arrive_expect_tx(&full[s], stage_bytes);
        tma_load_2d(tileB(s), &tmW, &full[s], j * a.Cin + c * KC, n0, pol_w);
        tma_load_3d(tileA(s), &tmX, &full[s], c * KC, t0 + j * a.dil, b0, pol_x);
        issued = i + 1;
      }
      for (int i = max(0, issued - stages); i < issued; ++i)
        mbar_wait(&full[i % stages], (i / stages) & 1, ERR_TIMEOUT_FULL, KERNEL_ID_CONV);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc(128, a.ntile, 0);   // fp16 x fp16 -> fp32
      for (int i = 0; i < nkb; ++i) {
        const int s = i % stages;
        if (!mbar_wait(&full[s], (i / stages) & 1, ERR_TIMEOUT_FULL, KERNEL_ID_CONV)) break;
        tc_fence_after();
        uint64_t da, db;
        if constexpr (KC == 64) {
          da = umma_desc_sw128(tileA(s));
          db = umma_desc_sw128(tileB(s));
        } else {
          da = umma_desc_sw64(tileA(s));
          db = umma_desc_sw64(tileB(s));
        }
#pragma unroll
        for (int k = 0; k < KC / 16; ++k) umma_f16(tmem, da + 2 * k, db + 2 * k, idesc, (i | k) != 0);
        umma_commit(&empty[s]);
      }
      umma_commit(accum);
    }
  }
  __syncwarp();
  pdl_wait();
  const bool ok = mbar_wait(accum, 0, ERR_TIMEOUT_ACCUM, KERNEL_ID_CONV);
  __syncthreads();
  tc_fence_after();

  // epilogue: thread = token row
  const int r = warp * 32 + lane;
  const int b = b0 + r / a.TT, t = t0 + r % a.TT;
  const bool live = b < a.rows;
  const uint32_t trow = tmem + (uint32_t(warp * 32) << 16);
  if (a.mode == 1) {
    float v[32];
    tmem_ld32(trow, v);
    if (live && ok) {
      const float bias = a.bias != nullptr ? __half2float(a.bias[0]) : 0.f;
      reinterpret_cast<float*>(a.out)[(size_t)b * a.out_bs + t] = tanhf(f16r(v[0] + bias));
    }
  } else {
    const int nch = (min(a.ntile, a.N - n0) + 31) / 32;
    for (int ch = 0; ch < (a.ntile + 31) / 32; ++ch) {
      float v[32];
      tmem_ld32(trow + ch * 32, v);
      if (!live || ch >= nch) continue;
      const int nb = n0 + ch * 32;
      const int nn = min(32, a.N - nb);
      float o[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        float x = ok ? v[i] : 0.f;
        if (a.bias != nullptr && i < nn) x += __half2float(a.bias[nb + i]);
        o[i] = x;
      }
      if (a.res != nullptr) {
        const __half* rp = a.res + (size_t)b * a.res_bs + (size_t)t * a.res_ts + nb;
        if (nn == 32) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 u = reinterpret_cast<const uint4*>(rp)[q];
            const float2 x0 = unpack_f16(u.x), x1 = unpack_f16(u.y), x2 = unpack_f16(u.z), x3 = unpack_f16(u.w);
            o[8 * q] += x0.x; o[8 * q + 1] += x0.y; o[8 * q + 2] += x1.x; o[8 * q + 3] += x1.y;
            o[8 * q + 4] += x2.x; o[8 * q + 5] += x2.y; o[8 * q + 6] += x3.x; o[8 * q + 7] += x3.y;
          }
        } else {
          for (int i = 0; i < nn; ++i) o[i] += __half2float(rp[i]);
        }
      }
      __half* op = reinterpret_cast<__half*>(a.out) + (size_t)b * a.out_bs + (size_t)t * a.out_ts + nb;
      if (nn == 32) {
        uint4* d4 = reinterpret_cast<uint4*>(op);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          d4[q] = make_uint4(pack_f16(o[8 * q], o[8 * q + 1]), pack_f16(o[8 * q + 2], o[8 * q + 3]),
                             pack_f16(o[8 * q + 4], o[8 * q + 5]), pack_f16(o[8 * q + 6], o[8 * q + 7]));
      } else {
        for (int i = 0; i < nn; ++i) op[i] = __float2half_rn(o[i]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, a.tmem_cols);
}

// ------------------------------------------------------------------------------------------------ host
struct ConvPlan {
  CUtensorMap tmX, tmW;
  ConvArgs args;
  dim3 grid;
  int smem;
};

// xin: fp16 [rows, ctx + T, Cin]; w: fp16 [N, taps * Cin] (K-major)
int conv_plan(ConvPlan* p, const void* xin, int rows, int T, int Cin, int ctx, const void* w, int N, int taps, int dil,
              const void* bias, const void* res, long long res_bs, long long res_ts, void* out, long long out_bs,
              long long out_ts, int mode) {
  if (xin == nullptr || w == nullptr || out == nullptr || rows <= 0 || T <= 0 || Cin <= 0 || N <= 0 || taps <= 0)
    return A8_ERR_ARG;
  if (Cin % 32) return A8_ERR_ARG;
  if ((taps - 1) * dil > ctx) return A8_ERR_ARG;
  ConvArgs& a = p->args;
  a.rows = rows;
  a.T = T;
  a.Cin = Cin;
  a.N = N;
  a.taps = taps;
  a.dil = dil;
  a.ctx = ctx;
  a.KC = (Cin % 64 == 0) ? 64 : 32;
  a.TT = T >= 128 ? 128 : T;
  if (128 % a.TT || T % a.TT) return A8_ERR_ARG;
  a.TB = 128 / a.TT;
  const int nt = (N + 255) / 256;
  a.ntile = std::max(16, ((N + nt - 1) / nt + 15) / 16 * 16);
  a.n_tiles = (N + a.ntile - 1) / a.ntile;
  a.kb_total = taps * (Cin / a.KC);
  a.tmem_cols = a.ntile <= 32 ? 32 : a.ntile <= 64 ? 64 : a.ntile <= 128 ? 128 : 256;
  const int stage_bytes = 128 * a.KC * 2 + a.ntile * a.KC * 2;
  a.stages = std::max(2, std::min(6, (200 * 1024) / stage_bytes));
  a.stages = std::min(a.stages, std::max(2, a.kb_total));
  a.bias = reinterpret_cast<const __half*>(bias);
  a.res = reinterpret_cast<const __half*>(res);
  a.res_bs = res_bs;
  a.res_ts = res_ts;
  a.out = out;
  a.out_bs = out_bs;
  a.out_ts = out_ts;
  a.mode = mode;
  const CUtensorMapSwizzle sw = a.KC == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  int rc = encode_map_3d(&p->tmX, xin, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, Cin, ctx + T, rows, (uint64_t)Cin * 2,
                         (uint64_t)(ctx + T) * Cin * 2, a.KC, a.TT, a.TB, sw);
  if (rc) return rc;
  rc = encode_map_2d(&p->tmW, w, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)taps * Cin, N, (uint64_t)taps * Cin * 2,
                     a.KC, a.ntile, sw);
  if (rc) return rc;
  p->grid = dim3((T / a.TT) * ((rows + a.TB - 1) / a.TB), a.n_tiles);
  p->smem = a.stages * stage_bytes + 1024 + 256;
  return A8_OK;
}

int conv_launch(const ConvPlan* p, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = p->grid;
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = p->smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  ++g_launches;
  cudaError_t e;
  if (p->args.KC == 64) {
    static bool attr = false;
    if (!attr) {
      cudaFuncSetAttribute(k_conv<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
      attr = true;
    }
    e = cudaLaunchKernelEx(&cfg, k_conv<64>, p->tmX, p->tmW, p->args);
  } else {
    static bool attr = false;
    if (!attr) {
      cudaFuncSetAttribute(k_conv<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
      attr = true;
    }
    e = cudaLaunchKernelEx(&cfg, k_conv<32>, p->tmX, p->tmW, p->args);
  }
  return e == cudaSuccess ? A8_OK : A8_ERR_CUDA;
}

}  // namespace a8

using namespace a8;

extern "C" int a8_conv(const void* xin, int rows, int T, int Cin, int ctx, const void* w, int N, int taps, int dil,
                       const void* bias, const void* res, long long res_bs, long long res_ts, void* out,
                       long long out_bs, long long out_ts, int mode, a8_stream_t stream) {
  ConvPlan p;
  int rc = conv_plan(&p, xin, rows, T, Cin, ctx, w, N, taps, dil, bias, res, res_bs, res_ts, out, out_bs, out_ts,
                     mode);
  if (rc) return rc;
  return conv_launch(&p, reinterpret_cast<cudaStream_t>(stream));
}
