// tcgen05 GEMM with fused epilogues for the decode tick:  Y = epilogue( X[M,K] . W[N,K]^T ).
//
// Layout ("swap AB"): the weight supplies the 128-row UMMA M dimension and the token rows the UMMA N dimension
// (16..256), so a decode batch of a few dozen rows still fills whole 128-lane tensor-core tiles and every weight
// byte is read from HBM once per launch. One CTA = 128 weight rows x ntok token rows x a K range:
//   warp 0 / one lane : TMA producer (128B-swizzled K-major tiles of W and X, a ring of `stages` smem slots)
//   warp 1 / one lane : MMA issuer (tcgen05.mma kind::f16, fp32 accumulator in TMEM, commit frees a slot)
//   all 16 warps      : epilogue (tcgen05.ld 32 lanes x 32 columns per warp; four 32-column chunks at once, each
//                       staged transposed through smem and finished by a 128-thread group)
// K splits of a tile (blockIdx.z) run as one thread-block cluster: each CTA sends its fp32 partial of every token
// column to the column's owner rank with asynchronous distributed-shared-memory stores (counted by the owner's
// mbarrier); the owner adds them in split order (deterministic) and runs the epilogue. Launched with programmatic
// dependent launch: the weight tiles of the first stages are requested before griddepcontrol.wait, i.e. while the
// previous kernel is still finishing.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "gemm.cuh"

namespace a8 {

long long g_launches = 0;               // kernels this library has launched (host-side count, for benchmarks)

constexpr int BK = 64;                  // K elements per stage (128 bytes of bf16: one swizzle atom)
constexpr int TILE_A_BYTES = 128 * BK * 2;
constexpr int STAGE_PITCH = 132;        // fp32 epilogue staging row pitch (bank-conflict-free float4 reads)
constexpr int KERNEL_ID_GEMM = 1;
constexpr int GEMM_PARTS = 4;           // warps per TMEM lane quarter in the epilogue
constexpr int GEMM_THREADS = 128 * GEMM_PARTS;
constexpr int NORM_WARP0 = 2;           // warps 2-15 normalise X tiles during the mainloop (operand RMSNorm)
constexpr int NORM_WARPS = GEMM_THREADS / 32 - NORM_WARP0;
constexpr int NORM_MAX_K = 1024;
// operand-normalisation shared memory: normed barriers (<= 8), rstd[256], norm weight[NORM_MAX_K] (bf16)
constexpr int NORM_SMEM = 8 * 8 + 16 + 256 * 4 + NORM_MAX_K * 2;   // (+16: alignment of rstd)

struct EpiCtx {
  const GemmArgs* a;
  int n0, m_base;
};

// ------------------------------------------------------------------------------------------------ operand norm
// bf16 pair (x0, x1) -> bf16 pair (bf16(x0 * r), bf16(x1 * r)), the products in fp32
__device__ __forceinline__ uint32_t scale_bf16x2(uint32_t u, float r) {
  const float2 f = unpack_bf16(u);
  return pack_bf16(f.x * r, f.y * r);
}
// bf16 pairs multiplied lane-wise, each product rounded to nearest once
__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// ------------------------------------------------------------------------------------------------ epilogues
// 8 bf16 (16-byte aligned) -> fp32
__device__ __forceinline__ void load8_bf16(const __nv_bfloat16* p, float* o) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack_bf16(w[i]);
    o[2 * i] = f.x;
    o[2 * i + 1] = f.y;
  }
}

// Every epilogue sees one chunk of 32 token columns: stage[j][r] = fp32 result of weight row n0 + r, token m_base + j.
// Thread t handles token j = t / 4 and the 32 weight rows [32 (t % 4), +32) of the tile.
template <int KIND>
__device__ __forceinline__ void epilogue_chunk(const GemmArgs& a, const float* stage, int n0, int mb, int mend,
                                               int tid) {
  const int j = tid >> 2, seg = tid & 3;
  const int m = mb + j;
  if (m >= mend) return;
  const float* src = stage + j * STAGE_PITCH + seg * 32;
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; i += 4) {
    float4 f = *reinterpret_cast<const float4*>(src + i);
    v[i] = f.x; v[i + 1] = f.y; v[i + 2] = f.z; v[i + 3] = f.w;
  }
  const A8Epilogue& e = a.epi;
  const int nb = n0 + seg * 32;
  if constexpr (KIND == A8_EPI_BF16 || KIND == A8_EPI_GELU || KIND == A8_EPI_LSRES) {
    const __nv_bfloat16* bias = reinterpret_cast<const __nv_bfloat16*>(e.bias);
    __nv_bfloat16* y = reinterpret_cast<__nv_bfloat16*>(a.y) + (size_t)m * a.ldy;
    float o[32];
    const bool vec = nb + 32 <= a.N;                 // whole segment: 16-byte loads of bias / residual / gamma
    if (vec && (KIND == A8_EPI_LSRES || bias != nullptr)) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float bx[8];
        if (bias != nullptr) {
          load8_bf16(bias + nb + 8 * q, bx);
        } else {
#pragma unroll
          for (int k = 0; k < 8; ++k) bx[k] = 0.f;
        }
        if constexpr (KIND == A8_EPI_LSRES) {
          float rx[8], gx[8];
          const __nv_bfloat16* res = reinterpret_cast<const __nv_bfloat16*>(e.res) + (size_t)m * e.ldres;
          load8_bf16(res + nb + 8 * q, rx);
          load8_bf16(reinterpret_cast<const __nv_bfloat16*>(e.gamma) + nb + 8 * q, gx);
#pragma unroll
          for (int k = 0; k < 8; ++k) o[8 * q + k] = rx[k] + bf16r(gx[k] * bf16r(v[8 * q + k] + bx[k]));
        } else {
#pragma unroll
          for (int k = 0; k < 8; ++k) v[8 * q + k] += bx[k];
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int n = nb + i;
      float x = v[i];
      if constexpr (KIND == A8_EPI_LSRES) {
        if (vec) continue;                           // done above
      }
      if (!vec && bias != nullptr && n < a.N) x += __bfloat162float(bias[n]);
      if constexpr (KIND == A8_EPI_BF16) {
        o[i] = x;
      } else if constexpr (KIND == A8_EPI_GELU) {
        const float t = bf16r(x);
        o[i] = 0.5f * t * (1.0f + erff(t * 0.70710678118654752f));
      } else {
        const __nv_bfloat16* res = reinterpret_cast<const __nv_bfloat16*>(e.res) + (size_t)m * e.ldres;
        const __nv_bfloat16* gam = reinterpret_cast<const __nv_bfloat16*>(e.gamma);
        if (n < a.N) {
          const float t = bf16r(x);
          o[i] = __bfloat162float(res[n]) + bf16r(__bfloat162float(gam[n]) * t);
        } else {
          o[i] = 0.f;
        }
      }
    }
    if (nb + 32 <= a.N && ((reinterpret_cast<uintptr_t>(y + nb) & 15) == 0)) {
      uint4* dst = reinterpret_cast<uint4*>(y + nb);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        dst[q] = make_uint4(pack_bf16(o[8 * q], o[8 * q + 1]), pack_bf16(o[8 * q + 2], o[8 * q + 3]),
                            pack_bf16(o[8 * q + 4], o[8 * q + 5]), pack_bf16(o[8 * q + 6], o[8 * q + 7]));
    } else {
      for (int i = 0; i < 32; ++i)
        if (nb + i < a.N) y[nb + i] = __float2bfloat16_rn(o[i]);
    }
  } else if constexpr (KIND == A8_EPI_RESID) {
    // rmsnorm's residual add (serve/fast_kernels.py:36-40): y = bf16(bf16(acc + bias) + res), and this tile's part
    // of the row's sum of squares of y for the next GEMM's operand normalisation
    const __nv_bfloat16* bias = reinterpret_cast<const __nv_bfloat16*>(e.bias);
    const __nv_bfloat16* res = reinterpret_cast<const __nv_bfloat16*>(e.res) + (size_t)m * e.ldres;
    __nv_bfloat16* y = reinterpret_cast<__nv_bfloat16*>(a.y) + (size_t)m * a.ldy;
    float o[32];
    const bool vec = nb + 32 <= a.N &&
                     ((reinterpret_cast<uintptr_t>(y + nb) | reinterpret_cast<uintptr_t>(res + nb) |
                       (bias != nullptr ? reinterpret_cast<uintptr_t>(bias + nb) : 0)) & 15) == 0;
    if (vec) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float rx[8], bx[8];
        load8_bf16(res + nb + 8 * q, rx);
        if (bias != nullptr) {
          load8_bf16(bias + nb + 8 * q, bx);
        } else {
#pragma unroll
          for (int k = 0; k < 8; ++k) bx[k] = 0.f;
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) o[8 * q + k] = bf16r(bf16r(v[8 * q + k] + bx[k]) + rx[k]);
      }
      uint4* dst = reinterpret_cast<uint4*>(y + nb);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        dst[q] = make_uint4(pack_bf16(o[8 * q], o[8 * q + 1]), pack_bf16(o[8 * q + 2], o[8 * q + 3]),
                            pack_bf16(o[8 * q + 4], o[8 * q + 5]), pack_bf16(o[8 * q + 6], o[8 * q + 7]));
    } else {
      for (int i = 0; i < 32; ++i) {
        const int n = nb + i;
        o[i] = 0.f;
        if (n < a.N) {
          const float b = bias != nullptr ? __bfloat162float(bias[n]) : 0.f;
          o[i] = bf16r(bf16r(v[i] + b) + __bfloat162float(res[n]));
        }
      }
      for (int i = 0; i < 32; ++i)
        if (nb + i < a.N) y[nb + i] = __float2bfloat16_rn(o[i]);
    }
    if (e.ssq_out != nullptr) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i) ss += o[i] * o[i];
      // the four 32-column segments of this token sit in lanes 4j .. 4j+3 (all present or all gone)
      const unsigned quad = 0xFu << (threadIdx.x & 28);
      ss += __shfl_xor_sync(quad, ss, 1);
      ss += __shfl_xor_sync(quad, ss, 2);
      if (seg == 0) e.ssq_out[(size_t)(n0 >> 7) * e.ssq_ld + m] = ss;
    }
  } else if constexpr (KIND == A8_EPI_F32_ROUND) {
    float* y = reinterpret_cast<float*>(a.y) + (size_t)m * a.ldy;
    if (nb + 32 <= a.N && ((reinterpret_cast<uintptr_t>(y + nb) & 15) == 0)) {
      float4* dst = reinterpret_cast<float4*>(y + nb);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        dst[q] = make_float4(bf16r(v[4 * q]), bf16r(v[4 * q + 1]), bf16r(v[4 * q + 2]), bf16r(v[4 * q + 3]));
    } else {
      for (int i = 0; i < 32; ++i)
        if (nb + i < a.N) y[nb + i] = bf16r(v[i]);
    }
  }
}

// SiLU-mul: the tile's rows 0..63 are gate rows g_c, rows 64..127 the matching up rows u_c (c = 64 * tile + i).
__device__ __forceinline__ void epilogue_silu(const GemmArgs& a, const float* stage, int tile, int mb, int mend,
                                              int tid) {
  const int j = tid >> 2, seg = tid & 3;
  const int m = mb + j;
  if (m >= mend) return;
  const float* g = stage + j * STAGE_PITCH + seg * 16;
  const float* u = g + 64;
  const int c0 = tile * 64 + seg * 16;
  const int I = a.N / 2;
  __nv_bfloat16* y = reinterpret_cast<__nv_bfloat16*>(a.y) + (size_t)m * a.ldy;
  float o[16];
  // silu(g) = g / (1 + exp(-g)) with the approximate exponential and divide the reference's Triton kernel compiles to
  // (tl.exp, fp32 '/'; serve/fast_kernels.py:531-533), rounded to bf16 before the product
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float gv = bf16r(g[i]);
    const float uv = bf16r(u[i]);
    const float gs = bf16r(__fdividef(gv, 1.0f + __expf(-gv)));
    o[i] = gs * uv;
  }
  if (c0 + 16 <= I && ((reinterpret_cast<uintptr_t>(y + c0) & 15) == 0)) {
    uint4* dst = reinterpret_cast<uint4*>(y + c0);
    dst[0] = make_uint4(pack_bf16(o[0], o[1]), pack_bf16(o[2], o[3]), pack_bf16(o[4], o[5]), pack_bf16(o[6], o[7]));
    dst[1] = make_uint4(pack_bf16(o[8], o[9]), pack_bf16(o[10], o[11]), pack_bf16(o[12], o[13]),
                        pack_bf16(o[14], o[15]));
  } else {
    for (int i = 0; i < 16; ++i)
      if (c0 + i < I) y[c0 + i] = __float2bfloat16_rn(o[i]);
  }
}

// RoPE: the fused row of token m is [q heads | k heads | v heads] x hd. rotate_half pairs dims (d, d + hd/2), which
// sit 32 (hd 64) or 64 (hd 128) tile rows apart: the partner of 32-row segment seg is seg ^ (hd / 64).
__device__ __forceinline__ void epilogue_rope(const GemmArgs& a, const float* stage, int n0, int mb, int mend,
                                              int tid) {
  const int j = tid >> 2, seg = tid & 3;
  const int m = mb + j;
  if (m >= mend) return;
  const A8Epilogue& e = a.epi;
  const int hd = e.hd, half = hd >> 1;
  const int nb = n0 + seg * 32;
  if (nb >= a.N) return;
  const int pseg = seg ^ (hd >> 6);
  const float* src = stage + j * STAGE_PITCH + seg * 32;
  const float* psrc = stage + j * STAGE_PITCH + pseg * 32;
  const __nv_bfloat16* bias = reinterpret_cast<const __nv_bfloat16*>(e.bias);
  const int head = nb / hd;                 // fused head index: q 0..nq-1, k nq..nq+nkv-1, v after
  const int d0 = nb - head * hd;            // first dim of this segment inside the head
  const int pos = e.pos[m];
  const int slot = e.slot != nullptr ? e.slot[m] : m;
  float o[32];
  if (head < e.nq + e.nkv) {
    const __nv_bfloat16* cs = reinterpret_cast<const __nv_bfloat16*>(e.cos) + (size_t)pos * hd + d0;
    const __nv_bfloat16* sn = reinterpret_cast<const __nv_bfloat16*>(e.sin) + (size_t)pos * hd + d0;
    const int pb = n0 + pseg * 32;          // partner rows
    const float sign = d0 < half ? -1.0f : 1.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {           // 8 dims at a time: one 16-byte load of each table row
      float c[8], s[8], bx[8], bp[8];
      load8_bf16(cs + 8 * q, c);
      load8_bf16(sn + 8 * q, s);
      if (bias != nullptr) {
        load8_bf16(bias + nb + 8 * q, bx);
        load8_bf16(bias + pb + 8 * q, bp);
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int i = 8 * q + k;
        float x = bf16r(src[i]);
        float xp = bf16r(psrc[i]);
        if (bias != nullptr) {
          x += bx[k];
          xp += bp[k];
        }
        o[i] = x * c[k] + sign * xp * s[k];
      }
    }
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float bx[8];
      if (bias != nullptr) load8_bf16(bias + nb + 8 * q, bx);
#pragma unroll
      for (int k = 0; k < 8; ++k) o[8 * q + k] = bf16r(src[8 * q + k]) + (bias != nullptr ? bx[k] : 0.f);
    }
  }
  __nv_bfloat16* dst;
  if (head < e.nq) {
    dst = reinterpret_cast<__nv_bfloat16*>(a.y) + (size_t)m * a.ldy + nb;
  } else {
    const bool is_k = head < e.nq + e.nkv;
    const int kh = is_k ? head - e.nq : head - e.nq - e.nkv;
    const int col = pos % e.ring;
    __nv_bfloat16* cache = reinterpret_cast<__nv_bfloat16*>(is_k ? e.kc : e.vc);
    dst = cache + (((size_t)slot * e.nkv + kh) * e.cache_len + col) * hd + d0;
  }
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q)
    d4[q] = make_uint4(pack_bf16(o[8 * q], o[8 * q + 1]), pack_bf16(o[8 * q + 2], o[8 * q + 3]),
                       pack_bf16(o[8 * q + 4], o[8 * q + 5]), pack_bf16(o[8 * q + 6], o[8 * q + 7]));
}

template <int KIND>
__device__ __forceinline__ void run_epilogue(const GemmArgs& a, const float* stage, int n0, int mb, int mend,
                                             int tid) {
  mend = min(mend, a.M);
  if constexpr (KIND == A8_EPI_SILU) {
    epilogue_silu(a, stage, n0 / 128, mb, mend, tid);
  } else if constexpr (KIND == A8_EPI_ROPE) {
    epilogue_rope(a, stage, n0, mb, mend, tid);
  } else {
    epilogue_chunk<KIND>(a, stage, n0, mb, mend, tid);
  }
}

// ------------------------------------------------------------------------------------------------ kernel
template <int KIND>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    k_gemm(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, const GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int stages = a.stages;
  const uint32_t stage_bytes = TILE_A_BYTES + a.ntok * BK * 2;
  // [pipeline slots][cluster split-K: receive buffer S x w x 128 fp32][reduced slice 32 x STAGE_PITCH][barriers]
  const int ntok32 = (a.ntok + 31) / 32 * 32;
  const int S = a.splits;
  const int w = ((ntok32 + S - 1) / S + 3) / 4 * 4;         // token columns each cluster rank reduces
  const int wp = w % 32 ? w : w + 4;                        // their row pitch in the receive buffer (bank spread)
  const uint32_t pipe_bytes = stages * stage_bytes;
  const uint32_t recv_bytes = S > 1 ? uint32_t(S * 128 * wp * 4) : 0u;
  const uint32_t slice_bytes = S > 1 ? uint32_t(32 * STAGE_PITCH * 4) : 0u;
  float* recv = reinterpret_cast<float*>(smem + pipe_bytes);
  float* slice = reinterpret_cast<float*>(smem + pipe_bytes + recv_bytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + pipe_bytes + recv_bytes + slice_bytes);
  uint64_t* empty = full + stages;
  uint64_t* accum = empty + stages;
  uint64_t* recv_bar = accum + 1;         // split-K: the peers' partials have all landed in recv
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_bar + 1);
  // operand normalisation: a stage's X tile normalised in place (normed[s]), per-token 1/rms, the norm weight
  const bool norm = a.epi.norm_w != nullptr;
  uint64_t* normed = recv_bar + 2;
  // (16-byte aligned: the norm weight is read as 16-byte vectors)
  float* rstd_s = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(normed + stages) + 15) & ~uintptr_t(15));
  uint32_t* normw_s = reinterpret_cast<uint32_t*>(rstd_s + 256);   // bf16 pairs

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile_n = blockIdx.x, tile_m = blockIdx.y, split = blockIdx.z;
  const int n0 = tile_n * 128, m0 = tile_m * a.ntok;
  const int kb0 = split * a.kb_per_split;
  const int nkb = min(a.kb_total, kb0 + a.kb_per_split) - kb0;

  if (tid == 0) {
    tma_prefetch(&tmW);
    tma_prefetch(&tmX);
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    mbar_init(recv_bar, 1);
    for (int s = 0; s < stages; ++s) mbar_init(&normed[s], NORM_WARPS);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, a.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch();
  if (S > 1) cluster_arrive_relaxed();          // this CTA's recv_bar exists (the peers wait for it before sending)

  auto tileA = [&](int s) { return smem + s * stage_bytes; };
  auto tileB = [&](int s) { return smem + s * stage_bytes + TILE_A_BYTES; };

  int issued = 0;                               // stage loads requested (producer lane)
  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pw = policy_evict_first(), px = policy_evict_last();
      const int pre = min(stages, nkb);
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], stage_bytes);
        tma_load_2d(tileA(i), &tmW, &full[i], (kb0 + i) * BK, n0, pw);
      }
      pdl_wait();                               // X is produced by the previous kernel
      for (int i = 0; i < pre; ++i) tma_load_2d(tileB(i), &tmX, &full[i], (kb0 + i) * BK, m0, px);
      issued = pre;
      // slot and phase by counters: no divisions between this lane's issues (i >= pre only runs when pre == stages)
      for (int i = pre, s = 0, ph = 0; i < nkb; ++i) {
        if (!mbar_wait(&empty[s], ph, ERR_TIMEOUT_EMPTY, KERNEL_ID_GEMM)) break;
        mbar_arrive_expect_tx(&full[s], stage_bytes);
        tma_load_2d(tileA(s), &tmW, &full[s], (kb0 + i) * BK, n0, pw);
        tma_load_2d(tileB(s), &tmX, &full[s], (kb0 + i) * BK, m0, px);
        issued = i + 1;
        if (++s == stages) {
          s = 0;
          ph ^= 1;
        }
      }
      // every requested stage has landed before the slots are reused as epilogue staging (immediate in normal
      // operation: the MMA issuer consumed them; bounded after an error)
      for (int i = max(0, issued - stages); i < issued; ++i)
        mbar_wait(&full[i % stages], (i / stages) & 1, ERR_TIMEOUT_FULL, KERNEL_ID_GEMM);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc(128, a.ntok, 1);
      // stage s's descriptors are stage 0's plus s stage sizes (the address field counts 16-byte units)
      const uint64_t da0 = umma_desc_sw128(tileA(0)), db0 = umma_desc_sw128(tileB(0));
      uint64_t* const bars = norm ? normed : full;
      for (int i = 0, s = 0, ph = 0; i < nkb; ++i) {
        if (!mbar_wait(&bars[s], ph, ERR_TIMEOUT_FULL, KERNEL_ID_GEMM)) break;
        tc_fence_after();
        const uint64_t off = (uint64_t)(s * (stage_bytes >> 4));
        const uint64_t da = da0 + off, db = db0 + off;
        umma_f16(tmem, da, db, idesc, i != 0);
#pragma unroll
        for (int k = 1; k < BK / 16; ++k) umma_f16(tmem, da + 2 * k, db + 2 * k, idesc, 1);
        umma_commit(&empty[s]);
        if (++s == stages) {
          s = 0;
          ph ^= 1;
        }
      }
      umma_commit(accum);
    }
  } else if (norm && warp >= NORM_WARP0 && warp < NORM_WARP0 + NORM_WARPS) {
    // RMSNorm of the X rows (serve/fast_kernels.py:41-45): row m of every stage's tile becomes
    // bf16(w * bf16(x * rstd[m])), rstd from the row's partial sums of squares added in tile order. The tile is
    // 128B-swizzled: 16-byte chunk pc of row m holds K elements 8 (pc ^ (m % 8)) .. +7 of the stage's 64.
    const int nt = tid - NORM_WARP0 * 32;
    const uint32_t* nw = reinterpret_cast<const uint32_t*>(a.epi.norm_w);
    for (int k = nt; k < a.K / 2; k += NORM_WARPS * 32) normw_s[k] = nw[k];
    pdl_wait();                                 // the partial sums are the previous kernel's output
    const int tiles = (a.K + 127) / 128;
    for (int j = nt; j < a.ntok; j += NORM_WARPS * 32) {
      const int m = m0 + j;
      float r = 0.f;
      if (m < a.M) {
        float ss = 0.f;
        for (int t = 0; t < tiles; ++t) ss += a.epi.ssq_in[(size_t)t * a.epi.ssq_ld + m];
        r = rsqrtf(ss / (float)a.K + a.epi.eps);
      }
      rstd_s[j] = r;
    }
    named_bar_sync(1, NORM_WARPS * 32);
    for (int i = 0, s = 0, ph = 0; i < nkb; ++i, s = s + 1 == stages ? 0 : s + 1, ph ^= s == 0) {
      if (!mbar_wait(&full[s], ph, ERR_TIMEOUT_FULL, KERNEL_ID_GEMM)) break;
      uint8_t* tb = tileB(s);
      const uint4* wk0 = reinterpret_cast<const uint4*>(normw_s + (kb0 + i) * (BK / 2));
      for (int c = nt; c < a.ntok * 8; c += NORM_WARPS * 32) {
        const int m = c >> 3, pc = c & 7;
        const uint4 wq = wk0[pc ^ (m & 7)];
        uint4* p = reinterpret_cast<uint4*>(tb + m * 128 + pc * 16);
        const uint4 u = *p;
        const float rs = rstd_s[m];
        // bf16(w * bf16(x * rs)): the product of two bf16 values is exact in fp32, so one bf16x2 multiply rounds it
        // exactly as the fp32 product rounded to bf16
        *p = make_uint4(bf16x2_mul(scale_bf16x2(u.x, rs), wq.x), bf16x2_mul(scale_bf16x2(u.y, rs), wq.y),
                        bf16x2_mul(scale_bf16x2(u.z, rs), wq.z), bf16x2_mul(scale_bf16x2(u.w, rs), wq.w));
      }
      fence_proxy_async_smem();                 // the tensor core reads these generic-proxy writes
      __syncwarp();
      if (lane == 0) mbar_arrive(&normed[s]);
    }
  }
  __syncwarp();
  pdl_wait();
  const bool ok = mbar_wait(accum, 0, ERR_TIMEOUT_ACCUM, KERNEL_ID_GEMM);
  __syncthreads();                              // the producer's drain is done before staging reuses the slots
  tc_fence_after();

  // Epilogue by all 16 warps. A warp reads the TMEM lanes of its quarter (warp % 4) and the four warps of a quarter
  // take turns over the 32-column chunks (part = warp / 4), so up to four chunks are in flight; each chunk is staged
  // transposed in the idle pipeline slots and finished by one 128-thread group (thread t: token t / 4, 32 rows).
  constexpr int CHUNK_FLOATS = 32 * STAGE_PITCH;
  const int quarter = warp & 3, part = warp >> 2, gtid = tid & 127;
  const int row = quarter * 32 + lane;
  const uint32_t trow = tmem + (uint32_t(quarter * 32) << 16);
  const int nchunk = (a.ntok + 31) / 32;
  const int par = min(GEMM_PARTS, (int)(pipe_bytes / (CHUNK_FLOATS * 4)));   // chunks staged at once

  if (a.splits == 1) {
    for (int c0 = 0; c0 < nchunk; c0 += par) {
      const int c = c0 + part;
      float* stage = reinterpret_cast<float*>(smem) + part * CHUNK_FLOATS;
      if (part < par && c < nchunk) {
        float v[32];
        tmem_ld32(trow + c * 32, v);
        if (!ok) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0.f;
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) stage[i * STAGE_PITCH + row] = v[i];
      }
      __syncthreads();
      // (a tile's last chunk may reach past its ntok columns into the next tile's tokens: those are not written)
      if (part < par && c < nchunk)
        run_epilogue<KIND>(a, stage, n0, m0 + c * 32, min(m0 + c * 32 + 32, m0 + a.ntok), gtid);
      __syncthreads();
    }
  } else {
    // The K splits of this tile form one cluster (blockIdx.z = rank). Token column col belongs to rank col / w (w a
    // multiple of 4): every CTA sends its fp32 partial of each column into the owner's receive buffer
    // recv[rank][row][col - owner w] with asynchronous 16-byte remote stores that count towards the owner's recv_bar,
    // then each owner waits for its (S - 1) * 128 * w * 4 bytes, adds its columns over the ranks in split order
    // (deterministic) from its own shared memory and runs the epilogue on them. The receive buffer is not part of the
    // pipeline slots: a peer may send while this CTA is still in its mainloop.
    const uint32_t recv_local = smem_u32(recv);
    const int owners = (ntok32 + w - 1) / w;
    const bool owner_here = split < owners;
    const int my_cols = owner_here ? min(w, ntok32 - split * w) : 0;   // the last owner's range may be shorter
    if (tid == 0 && owner_here) mbar_arrive_expect_tx(recv_bar, uint32_t((S - 1) * 128 * my_cols * 4));
    cluster_wait();                             // every peer's recv_bar is initialised
    for (int c = part; c < nchunk; c += GEMM_PARTS) {
      float v[32];
      tmem_ld32(trow + c * 32, v);
      if (!ok) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0.f;
      }
      int owner = (c * 32) / w, obeg = owner * w;   // owner of the chunk's first column, stepped along it
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        const int col = c * 32 + g * 4;
        while (col >= obeg + w) {
          ++owner;
          obeg += w;
        }
        const uint32_t off = uint32_t(((split * 128 + row) * wp + (col - obeg)) * 4);
        if (owner == split) {
          *reinterpret_cast<float4*>(recv + off / 4) = make_float4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
        } else {
          dsmem_st_async4(dsmem_addr(recv_local + off, owner), dsmem_addr(smem_u32(recv_bar), owner), v[4 * g],
                          v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
        }
      }
    }
    if (owner_here) mbar_wait(recv_bar, 0, ERR_TIMEOUT_OTHER, KERNEL_ID_GEMM);
    __syncthreads();                            // this CTA's own partial (plain stores) is visible to all its threads
    const int c0 = min(ntok32, split * w), c1 = min(ntok32, c0 + w);
    for (int cc = c0; cc < c1; cc += 32) {                   // the slice buffer and the epilogue take 32 columns
      const int ce = min(c1, cc + 32);
      for (int col = cc + 4 * part; col < ce; col += 4 * GEMM_PARTS) {
        const int j = col - c0;
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int p = 0; p < S; ++p) {
          const float4 t = *reinterpret_cast<const float4*>(recv + (p * 128 + row) * wp + j);
          s.x += t.x;
          s.y += t.y;
          s.z += t.z;
          s.w += t.w;
        }
        float* sl = slice + (col - cc) * STAGE_PITCH + row;
        sl[0] = s.x;
        sl[STAGE_PITCH] = s.y;
        sl[2 * STAGE_PITCH] = s.z;
        sl[3 * STAGE_PITCH] = s.w;
      }
      __syncthreads();
      if (part == 0) run_epilogue<KIND>(a, slice, n0, m0 + cc, min(m0 + ce, m0 + a.ntok), gtid);
      __syncthreads();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, a.tmem_cols);
}

// ------------------------------------------------------------------------------------------------ host
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

int encode_map_2d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                  uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                  CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return A8_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_stride_bytes & 15)) return A8_ERR_ALIGN;
  if ((uint64_t(box_inner) * elem_bytes) % 16) return A8_ERR_ALIGN;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? A8_OK : A8_ERR_CUDA;
}

int encode_map_3d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t d0, uint64_t d1,
                  uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1, uint32_t b2,
                  CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return A8_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (stride1_bytes & 15) || (stride2_bytes & 15)) return A8_ERR_ALIGN;
  if ((uint64_t(b0) * elem_bytes) % 16) return A8_ERR_ALIGN;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(m, dt, 3, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? A8_OK : A8_ERR_CUDA;
}

static int pick_ntok(int M) {
  const int tiles = (M + 255) / 256;
  int per = (M + tiles - 1) / tiles;
  return std::max(16, (per + 15) / 16 * 16);
}

static const void* gemm_fn(int kind) {
  switch (kind) {
    case A8_EPI_BF16: return (const void*)k_gemm<A8_EPI_BF16>;
    case A8_EPI_F32_ROUND: return (const void*)k_gemm<A8_EPI_F32_ROUND>;
    case A8_EPI_SILU: return (const void*)k_gemm<A8_EPI_SILU>;
    case A8_EPI_ROPE: return (const void*)k_gemm<A8_EPI_ROPE>;
    case A8_EPI_GELU: return (const void*)k_gemm<A8_EPI_GELU>;
    case A8_EPI_LSRES: return (const void*)k_gemm<A8_EPI_LSRES>;
    default: return (const void*)k_gemm<A8_EPI_RESID>;
  }
}

static void configure(int kind) {
  static bool done[8] = {false};
  if (done[kind]) return;
  cudaFuncSetAttribute(gemm_fn(kind), cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  cudaFuncSetAttribute(gemm_fn(kind), cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  done[kind] = true;
}

// How many clusters of S CTAs with this shared memory can be resident at once (0: none).
static int max_clusters(int kind, int smem, int S) {
  static std::mutex mu;
  static std::unordered_map<long long, int> cache;
  const long long key = ((long long)kind << 40) | ((long long)smem << 8) | S;
  {
    std::lock_guard<std::mutex> g(mu);
    auto f = cache.find(key);
    if (f != cache.end()) return f->second;
  }
  configure(kind);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, 1, S);
  cfg.blockDim = dim3(GEMM_THREADS);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 1;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = S;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_fn(kind), &cfg) != cudaSuccess) n = 0;
  cudaGetLastError();
  std::lock_guard<std::mutex> g(mu);
  cache[key] = n;
  return n;
}

static int num_sms() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
  }
  return sms;
}

// Shared memory of a (ntok, splits) configuration: pipeline slots, and for split-K the receive buffer of
// S x 128 x wp fp32 plus the reduced slice (as the kernel lays them out). Returns the stage count, or 0 if it does
// not fit in 227 KB.
static int size_config(int ntok, int S, int kb_per_split, int extra, int* smem) {
  const int stage_bytes = TILE_A_BYTES + ntok * BK * 2;
  const int ntok32 = (ntok + 31) / 32 * 32;
  const int w = ((ntok32 + S - 1) / S + 3) / 4 * 4;
  const int wp = w % 32 ? w : w + 4;
  const int reduce_bytes = S > 1 ? S * 128 * wp * 4 + 32 * STAGE_PITCH * 4 : 0;
  int stages = std::max(2, std::min(8, (200 * 1024 - reduce_bytes - extra) / stage_bytes));
  stages = std::min(stages, std::max(2, kb_per_split));
  *smem = stages * stage_bytes + reduce_bytes + 1024 + 256 + extra;
  return *smem <= 227 * 1024 ? stages : 0;
}

// Token tile and K splits of Y[M, N] = X[M, K] . W[N, K]^T. An explicit split count keeps the token tile of at most
// 256 balanced rows; otherwise every (token tile 32..256, splits 1..16) is scored by a launch-time model fitted to
// measured times of the tick's GEMM shapes on B200 -- waves of resident CTAs (or clusters) x (per K block cost
// growing with the tile + a fixed cost), plus the split-K exchange -- and the cheapest is kept (cached per shape).
static void choose(int kind, int N, int K, int M, int splits_req, int extra, int* ntok, int* splits) {
  const int kb_total = (K + BK - 1) / BK;
  if (splits_req > 0) {
    *ntok = pick_ntok(M);
    *splits = std::max(1, std::min(std::min(splits_req, kb_total), 16));
    return;
  }
  static std::mutex mu;
  static std::unordered_map<long long, long long> cache;
  const long long key = ((long long)(kind + 8 * (extra > 0)) << 56) | ((long long)N << 36) | ((long long)K << 18) | M;
  {
    std::lock_guard<std::mutex> g(mu);
    auto f = cache.find(key);
    if (f != cache.end()) {
      *ntok = int(f->second >> 8);
      *splits = int(f->second & 0xFF);
      return;
    }
  }
  const int n_tiles = (N + 127) / 128, sms = num_sms();
  double best = 1e30;
  // below 128 token rows (weight-bound decode steps): the balanced tile, and splits filling the SMs with at least
  // two K blocks each
  int bt = pick_ntok(M), bs = 1;
  {
    const int tiles = n_tiles * ((M + bt - 1) / bt);
    bs = tiles >= sms ? 1 : std::max(1, sms / tiles);
    bs = std::max(1, std::min(std::min(bs, std::max(1, kb_total / 2)), 16));
  }
  for (int nt = 32; nt <= 256 && M >= 128; nt += 16) {
    const int tt = (M + nt - 1) / nt;
    const int per = std::max(16, ((M + tt - 1) / tt + 15) / 16 * 16);
    if (per != nt) continue;                  // (the balanced tile of another candidate)
    const int tiles = n_tiles * tt;
    for (int s = 1; s <= std::min(16, kb_total); ++s) {
      const int kps = (kb_total + s - 1) / s, S = (kb_total + kps - 1) / kps;
      if (S != s) continue;
      int smem = 0;
      if (size_config(per, S, kps, extra, &smem) == 0) continue;
      const int cap = S == 1 ? sms : max_clusters(kind, smem, S);
      if (cap <= 0) continue;
      const int waves = (tiles + cap - 1) / cap;
      const double t = waves * (kps * (0.2 + 0.3 * per / 128.0) + 3.0) + (S > 1 ? 1.0 + 0.4 * S * per / 128.0 : 0.0);
      if (t < best - 1e-9) {
        best = t;
        bt = per;
        bs = S;
      }
    }
  }
  *ntok = bt;
  *splits = bs;
  std::lock_guard<std::mutex> g(mu);
  cache[key] = ((long long)bt << 8) | bs;
}

static bool cluster_fits(int kind, int smem, int S) { return max_clusters(kind, smem, S) > 0; }

int gemm_plan(GemmPlan* p, const void* x, int ldx, const void* w, int N, int K, int M, void* y, int ldy,
              const A8Epilogue* epi, int splits) {
  std::memset(p, 0, sizeof(*p));
  if (x == nullptr || w == nullptr || y == nullptr || epi == nullptr || N <= 0 || K <= 0 || M <= 0) return A8_ERR_ARG;
  if (epi->kind < A8_EPI_BF16 || epi->kind > A8_EPI_RESID) return A8_ERR_ARG;
  if (epi->kind == A8_EPI_RESID && (epi->res == nullptr || (epi->ssq_out != nullptr && epi->ssq_ld < M)))
    return A8_ERR_ARG;
  const bool norm = epi->norm_w != nullptr;
  if (norm && (epi->ssq_in == nullptr || epi->ssq_ld < M || K > NORM_MAX_K || K % BK != 0 || !(epi->eps >= 0.f)))
    return A8_ERR_ARG;
  if (norm && (reinterpret_cast<uintptr_t>(epi->norm_w) & 3)) return A8_ERR_ALIGN;   // read as bf16 pairs
  const int extra = norm ? NORM_SMEM : 0;
  if (epi->kind == A8_EPI_SILU && (N % 128) != 0) return A8_ERR_ARG;
  if (epi->kind == A8_EPI_ROPE && (epi->hd != 64 && epi->hd != 128)) return A8_ERR_ARG;
  if (epi->kind == A8_EPI_ROPE && (N != (epi->nq + 2 * epi->nkv) * epi->hd || epi->pos == nullptr ||
                                   epi->kc == nullptr || epi->vc == nullptr ||
                                   epi->cos == nullptr || epi->ring <= 0))
    return A8_ERR_ARG;
  if (epi->kind == A8_EPI_LSRES && (epi->res == nullptr || epi->gamma == nullptr)) return A8_ERR_ARG;
  GemmArgs& a = p->args;
  choose(epi->kind, N, K, M, splits, extra, &a.ntok, &a.splits);
  a.n_tiles = (N + 127) / 128;
  a.tok_tiles = (M + a.ntok - 1) / a.ntok;
  a.kb_total = (K + BK - 1) / BK;
  a.kb_per_split = (a.kb_total + a.splits - 1) / a.splits;
  a.splits = (a.kb_total + a.kb_per_split - 1) / a.kb_per_split;
  a.N = N;
  a.K = K;
  a.M = M;
  a.ldy = ldy;
  a.y = y;
  a.epi = *epi;
  a.tmem_cols = a.ntok <= 32 ? 32 : a.ntok <= 64 ? 64 : a.ntok <= 128 ? 128 : 256;
  const int stage_bytes = TILE_A_BYTES + a.ntok * BK * 2;
  const int budget = 200 * 1024;
  const int ntok32 = (a.ntok + 31) / 32 * 32;
  int smem = 0;
  for (;;) {
    // cluster split-K: receive buffer (S x 128 x wp fp32) + reduced slice beside the pipeline slots (as the kernel)
    const int w = ((ntok32 + a.splits - 1) / a.splits + 3) / 4 * 4;
    const int wp = w % 32 ? w : w + 4;
    const int reduce_bytes = a.splits > 1 ? a.splits * 128 * wp * 4 + 32 * STAGE_PITCH * 4 : 0;
    a.stages = std::max(2, std::min(8, (budget - reduce_bytes - extra) / stage_bytes));
    a.stages = std::min(a.stages, std::max(2, a.kb_per_split));
    smem = a.stages * stage_bytes + reduce_bytes + 1024 + 256 + extra;
    const bool fits = smem <= 227 * 1024 && (a.splits == 1 || cluster_fits(epi->kind, smem, a.splits));
    if (fits || a.splits == 1) break;
    const int s = std::max(1, a.splits / 2);         // a cluster that cannot be resident: halve it
    a.kb_per_split = (a.kb_total + s - 1) / s;
    a.splits = (a.kb_total + a.kb_per_split - 1) / a.kb_per_split;
  }
  int rc = encode_map_2d(&p->tmW, w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, N, (uint64_t)K * 2, BK, 128,
                         CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_map_2d(&p->tmX, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, M, (uint64_t)ldx * 2, BK, a.ntok,
                     CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  p->grid = dim3(a.n_tiles, a.tok_tiles, a.splits);
  p->smem_bytes = smem;
  p->kind = epi->kind;
  p->ok = true;
  return A8_OK;
}

template <int KIND>
static cudaError_t launch_kind(const GemmPlan* p, cudaStream_t s, bool pdl) {
  configure(KIND);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = p->grid;
  cfg.blockDim = dim3(GEMM_THREADS);
  cfg.dynamicSmemBytes = p->smem_bytes;
  cfg.stream = s;
  cudaLaunchAttribute at[2];
  int n = 0;
  if (pdl) {
    at[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[n++].val.programmaticStreamSerializationAllowed = 1;
  }
  if (p->args.splits > 1) {
    at[n].id = cudaLaunchAttributeClusterDimension;
    at[n].val.clusterDim.x = 1;
    at[n].val.clusterDim.y = 1;
    at[n++].val.clusterDim.z = p->args.splits;
  }
  cfg.attrs = at;
  cfg.numAttrs = n;
  ++g_launches;
  return cudaLaunchKernelEx(&cfg, k_gemm<KIND>, p->tmW, p->tmX, p->args);
}

int gemm_launch(const GemmPlan* p, cudaStream_t s, bool pdl) {
  if (!p->ok) return A8_ERR_ARG;
  cudaError_t e;
  switch (p->kind) {
    case A8_EPI_BF16: e = launch_kind<A8_EPI_BF16>(p, s, pdl); break;
    case A8_EPI_F32_ROUND: e = launch_kind<A8_EPI_F32_ROUND>(p, s, pdl); break;
    case A8_EPI_SILU: e = launch_kind<A8_EPI_SILU>(p, s, pdl); break;
    case A8_EPI_ROPE: e = launch_kind<A8_EPI_ROPE>(p, s, pdl); break;
    case A8_EPI_GELU: e = launch_kind<A8_EPI_GELU>(p, s, pdl); break;
    case A8_EPI_LSRES: e = launch_kind<A8_EPI_LSRES>(p, s, pdl); break;
    case A8_EPI_RESID: e = launch_kind<A8_EPI_RESID>(p, s, pdl); break;
    default: return A8_ERR_ARG;
  }
  return e == cudaSuccess ? A8_OK : A8_ERR_CUDA;
}

}  // namespace a8

using namespace a8;

extern "C" int a8_gemm(const void* x, int ldx, const void* w, int N, int K, int M, void* y, int ldy,
                       const A8Epilogue* epi, int splits, a8_stream_t stream) {
  GemmPlan p;
  int rc = gemm_plan(&p, x, ldx, w, N, K, M, y, ldy, epi, splits);
  if (rc) return rc;
  return gemm_launch(&p, reinterpret_cast<cudaStream_t>(stream), true);
}

extern "C" int a8_device_ok(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return 0;
  return prop.major == 10 && prop.minor == 0;
}

extern "C" int a8_get_error(int out[4]) {
  if (cudaDeviceSynchronize() != cudaSuccess) return A8_ERR_CUDA;
  if (cudaMemcpyFromSymbol(out, g_err, sizeof(int) * 4) != cudaSuccess) return A8_ERR_CUDA;
  return A8_OK;
}

extern "C" long long a8_launch_count(void) { return g_launches; }

extern "C" int a8_clear_error(void) {
  int z[4] = {0, 0, 0, 0};
  return cudaMemcpyToSymbol(g_err, z, sizeof(z)) == cudaSuccess ? A8_OK : A8_ERR_CUDA;
}
