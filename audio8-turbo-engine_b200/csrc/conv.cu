// Channels-last causal convolution / polyphase transposed convolution of the codec's conv decoder as a persistent,
// warp-specialized tcgen05 implicit GEMM (serve/fast_kernels.py:551-623 conv_cl, :695-729 snake_cat;
// serve/fast_engine.py:178-232 _CLConv).
//
//   y[b, t, n] = bias[n] + sum_j sum_c xin[b, t + j*dil, c] * W[n, j*Cin + c]  (+ res[b, t, n]),   t in [0, T)
//
// xin is the conv's input [rows, ctx + T, Cin] (fp16) with its carried context in rows [0, ctx). A transposed conv
// (stride s, kernel 2s, right crop s) is a 2-tap conv whose N = s * Cout holds every phase (n = p * Cout + c), so row
// (b, t) of y is output timesteps t*s .. t*s+s-1 of [rows, T*s, Cout].
//
// Work unit = 128 token rows (TB batch rows x TT timesteps) x ntile output channels. The A tile of K block (tap j,
// channel block c) is ONE 3-D TMA box {KC, TT, TB} at (c*KC, t0 + j*dil, b0) of xin -- the tap shift is a coordinate.
// One CTA per SM loops over work units:
//   warp 0      TMA producer: a ring of `stages` A+B slots (slab mode: the input slabs)
//   warp 1      MMA issuer (tcgen05.mma kind::f16, fp16 x fp16 -> fp32) into one of two TMEM accumulators
//   warp 2      slab mode: the weight tiles
//   warps 3-18  epilogue: while the MMA fills one accumulator, these drain the other (tcgen05.ld 16 columns at a
//               time; a lane quarter of TMEM is shared by four warps, which deal its 16-column chunks round robin).
//               19 warps put five on three of the SM's four register-file quarters: 96 registers a thread.
// The epilogue writes, per output: the raw fp16 y (the residual stream), and/or the NEXT conv's input rows
// snake(y) (x + inv * sin(alpha x)^2 on the fp16 y, stored fp16) straight into that conv's xin after its context --
// so no separate activation pass -- or, for conv_out, tanh(fp16 y) into fp32 audio.
#include "common.cuh"

namespace a8 {

constexpr int KERNEL_ID_CONV = 4;
constexpr int CONV_EPI_WARPS = 16;
constexpr int CONV_THREADS = 96 + 32 * CONV_EPI_WARPS;   // A producer, MMA, B producer, epilogue
constexpr int CONV_BAR_BYTES = 512;                        // mbarriers + the TMEM address, after the pipeline
constexpr int ETMA_WARP_BYTES = 4096;                      // TMA epilogue: residual[2] | raw | next input, 1 KB each
constexpr int ETMA_BYTES = CONV_EPI_WARPS * ETMA_WARP_BYTES + 128;   // every epilogue warp's staging + alignment

struct ConvArgs {
  int rows, T, Cin, N, taps, dil, ctx;
  int KC;                   // channels per K block: 64 (128-byte swizzle) or 32 (64-byte swizzle)
  int TT, TB;               // token tile: TB batch rows x TT timesteps (TT * TB == 128)
  int ntile, n_tiles, m_tiles;
  int kb_total, stages;
  // slab mode (TT = 128, one batch row a unit): the unit's input rows [t0, t0 + R) of one channel block are
  // loaded ONCE (a slab) and every tap reads it at row offset j*dil; weights stream through their own ring
  int slab, R, na, nb;
  int resident;             // slab mode, one output tile: all taps x cblocks weight tiles (nb of them) stay loaded
  int pair;                 // slab mode, streamed weights: CTA pairs (k_conv<KC, true>), half of each weight tile a CTA
  int wbox;                 // slab mode, streamed weights: one TMA box (and one ring slot) a channel block, every tap
  int etma;                 // 1x1 convs: residual in / outputs out by TMA boxes (k_conv<KC, false, true>)
  int sub;                  // 128-row sub-tiles a unit (slab mode: 2 share every weight tile; else 1)
  int hb;                   // slab rows a TMA box (a slab of R rows is ceil(R / hb) boxes)
  uint32_t a_slot;          // bytes of one slab slot
  uint32_t acc_cols;        // TMEM columns of one accumulator (power of two >= ntile)
  const float* bias;        // [N] (fp16 values as fp32) or null
  const __half* res;        // [b*res_bs + t*res_ts + n] or null
  long long res_bs, res_ts;
  __half* raw;              // [b*raw_bs + t*raw_ts + n] or null
  long long raw_bs, raw_ts;
  __half* nxt;              // [b*nxt_bs + nxt_off + t*N + n] or null: the next conv's input rows
  long long nxt_bs, nxt_off;
  int cout;                 // channels of an output timestep (N / phases): the activation's channel is n % cout
  const float* alpha;       // [cout] activation of nxt, or null (identity)
  const float* inv;
  float* audio;             // tanh mode: audio[b*audio_bs + t] = tanh(fp16(y[b, t, 0])), or null
  long long audio_bs;
};

// 32 lanes x 16 consecutive 32-bit columns
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// UMMA descriptor of a 128B-swizzled K-major tile starting at any 128-byte row of a tile that TMA wrote from a
// 1024-aligned base: the swizzle is a function of the absolute shared-memory address, so a row offset is a plain
// start-address offset (matrix base offset 0). Checked on the GPU for row offsets 0..54 (dilations 1, 3, 8, 9): a
// base offset of (addr >> 7) & 7 gives wrong products, 0 gives the exact ones.
__device__ __forceinline__ uint64_t umma_desc_sw128_row(uint32_t addr) {
  return ((uint64_t)((addr >> 4) & 0x3FFFu)) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
// the same for a 64B-swizzled tile (64-byte rows, 8-row groups 512 B apart)
__device__ __forceinline__ uint64_t umma_desc_sw64_row(uint32_t addr) {
  return ((uint64_t)((addr >> 4) & 0x3FFFu)) | (1ull << 16) | (32ull << 32) | (1ull << 46) | (4ull << 61);
}

// sin^2(t) for |t| < 2^21 without branches. sin^2 has period pi, so t = k pi + r with k = rint(t / pi) (round to
// nearest by adding 1.5 2^23) and r = t - k pi by a two-term split of pi (Cody-Waite reduction with fused
// multiply-adds); then sin^2(r) = u P(u), u = r^2, with P of degree 5 fitted to sin^2(sqrt u) / u over
// u in [0, (pi/2 + 0.1)^2] (iteratively reweighted least squares on 6000 Chebyshev nodes toward the minimax of the
// absolute error of u P; the 0.1 covers r past pi/2 when 1/pi's rounding moves k by one at large |t|). Emulated in fp32
// with fused multiply-adds against a float64 sin^2 (tests/test_sin2_poly.py), the result stays within 2.5e-7
// absolute for |t| < 2^21. Computed two at a time with packed fp32 instructions (each lane rounds as the scalar
// instruction would); no quadrant select.
constexpr float SIN2_RANGE = 2097152.f;
__device__ __forceinline__ float2 sin2_reduced2(float2 t) {
  const float2 big = ffma2(t, f2(0.318309873342514038f), f2(12582912.0f));   // 1 / pi
  const float2 k = fsub2(big, f2(12582912.0f));
  float2 r = ffma2(k, f2(-3.14159274101257324f), t);   // -(pi rounded to fp32)
  r = ffma2(k, f2(8.74227765734758577e-8f), r);        // -(pi minus that)
  const float2 u = fmul2(r, r);
  float2 p = ffma2(f2(-3.453945510e-06f), u, f2(1.381000038e-04f));
  p = ffma2(p, u, f2(-3.169148928e-03f));
  p = ffma2(p, u, f2(4.443938658e-02f));
  p = ffma2(p, u, f2(-3.333311677e-01f));
  p = ffma2(p, u, f2(9.999997020e-01f));
  return fmul2(u, p);
}

// The next conv's input of 16 consecutive outputs: ha = fp16(y + inv sin^2(alpha y)) from the fp16-rounded y (as
// fp32 in v) and the channels' alpha / inv staged in shared memory (16-byte aligned), two values a word. CHECK: also
// report whether every |alpha y| stayed inside sin2_reduced2's range.
template <bool CHECK>
__device__ __forceinline__ bool snake16(const float* v, const float* al_s, const float* iv_s, uint32_t* ha) {
  bool ok = true;
#pragma unroll
  for (int i = 0; i < 16; i += 4) {
    const float4 al = *reinterpret_cast<const float4*>(al_s + i);
    const float4 iv = *reinterpret_cast<const float4*>(iv_s + i);
    const float2 y0 = make_float2(v[i], v[i + 1]), y1 = make_float2(v[i + 2], v[i + 3]);
    const float2 t0 = fmul2(y0, make_float2(al.x, al.y)), t1 = fmul2(y1, make_float2(al.z, al.w));
    if (CHECK) ok &= fmaxf(fmaxf(fabsf(t0.x), fabsf(t0.y)), fmaxf(fabsf(t1.x), fabsf(t1.y))) < SIN2_RANGE;
    const float2 z0 = ffma2(make_float2(iv.x, iv.y), sin2_reduced2(t0), y0);
    const float2 z1 = ffma2(make_float2(iv.z, iv.w), sin2_reduced2(t1), y1);
    ha[i / 2] = pack_f16(z0.x, z0.y);
    ha[i / 2 + 1] = pack_f16(z1.x, z1.y);
  }
  return ok;
}

// The same with sinf, for a chunk where some |alpha y| left that range. Its arrays are its own (sinf's wide-argument
// path may keep them in local memory; the fast path's registers stay out of it).
__device__ __forceinline__ void snake16_exact(const float* v, const float* al_s, const float* iv_s, uint32_t* ha) {
  float y[16];
  uint32_t h[8];
#pragma unroll
  for (int i = 0; i < 16; ++i) y[i] = v[i];
#pragma unroll 1
  for (int i = 0; i < 16; i += 2) {
    const float s0 = sinf(y[i] * al_s[i]), s1 = sinf(y[i + 1] * al_s[i + 1]);
    h[i / 2] = pack_f16(y[i] + iv_s[i] * s0 * s0, y[i + 1] + iv_s[i + 1] * s1 * s1);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) ha[i] = h[i];
}

// PAIR: slab mode with streamed weights on CTA pairs (clusters of 2, tcgen05 cta_group::2). The two CTAs take two
// m-tiles of one n-tile as one 256-row MMA: each loads its own input slab and half of every weight tile (N / 2 rows)
// and both loads complete bytes on the first CTA's barriers; the first CTA's MMA warp issues for the pair and its
// commits arrive on both CTAs' barriers; each CTA's epilogue drains its own accumulator rows and arrives on the first
// CTA's accumulator-drained barrier. Half the MMA instructions, half the weight bytes a CTA.
// ETMA: 1x1 convs (no slab, one 128-step sub-tile, at least 32 steps a unit) and the single-CTA slab convs whose
// weights stream by channel-block boxes (the transposed convs): each epilogue warp moves its item's 32
// token rows x 16 channels by TMA through its own shared-memory staging -- the residual in (one item ahead), the raw
// output and the next conv's input out -- a box of whole lines instead of 32 scattered 32-byte sectors a warp access.
template <int KC, bool PAIR, bool ETMA>
__global__ void __launch_bounds__(CONV_THREADS, 1)
    k_conv(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
           const __grid_constant__ CUtensorMap tmR, const __grid_constant__ CUtensorMap tmO,
           const __grid_constant__ CUtensorMap tmN, const ConvArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int stages = a.stages;
  const uint32_t a_bytes = 128 * KC * 2, b_bytes = (PAIR ? a.ntile / 2 : a.ntile) * KC * 2;
  const uint32_t stage_bytes = a_bytes + b_bytes;
  // pipeline: `stages` slots of (A, B) -- or, in slab mode, na slab slots then nb weight slots
  const uint32_t bslot = a.wbox ? a.taps * b_bytes : b_bytes;   // a weight ring slot: one tap's tile, or every tap's
  const uint32_t pipe_bytes = a.slab ? a.na * a.a_slot + a.nb * bslot : stages * stage_bytes;
  const int nbar = a.slab ? a.na + (a.resident ? 1 : a.nb) : stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + pipe_bytes);
  uint64_t* empty = full + nbar;
  uint64_t* tfull = empty + nbar;         // [2] accumulator ready
  uint64_t* tempty = tfull + 2;           // [2] accumulator drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  uint32_t* s_amax = tmem_slot + 1;       // max |alpha| bits over the staged activation (NaN above every number)
  // the epilogue's per-column constants, staged once: bias [N], then alpha and inv [cout] (no global loads per tile)
  float* s_bias = reinterpret_cast<float*>(smem + pipe_bytes + CONV_BAR_BYTES);
  float* s_alpha = s_bias + (a.bias != nullptr ? (a.N + 3) / 4 * 4 : 0);
  float* s_inv = s_alpha + (a.cout + 3) / 4 * 4;
  uint64_t* rbar = reinterpret_cast<uint64_t*>(tmem_slot + 2);   // ETMA: [epilogue warp][2] residual boxes landed
  uint8_t* estage = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(s_inv + (a.cout + 3) / 4 * 4) + 127) &
                                               ~uintptr_t(127));

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tiles_t = a.T / (a.TT * a.sub);
  const int cblocks = a.Cin / KC;
  const int nkb = a.kb_total;
  const int total = a.m_tiles * a.n_tiles;
  // work items: tiles, or for a pair (m-tile pair, n-tile) -- the second m-tile past the last one is a phantom whose
  // rows lie beyond the input (zero-filled loads, nothing stored)
  const uint32_t rank = PAIR ? cluster_rank() : 0u;
  const int cid = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int ncl = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int iters = PAIR ? ((a.m_tiles + 1) / 2) * a.n_tiles : total;
  auto tile_of = [&](int q) { return PAIR ? ((q / a.n_tiles) * 2 + (int)rank) * a.n_tiles + q % a.n_tiles : q; };

  if (tid == 0) {
    tma_prefetch(&tmX);
    tma_prefetch(&tmW);
    for (int s = 0; s < nbar; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], PAIR ? 2 * CONV_EPI_WARPS : CONV_EPI_WARPS);
    }
    *s_amax = 0;
    if constexpr (ETMA)
      for (int i = 0; i < 2 * CONV_EPI_WARPS; ++i) mbar_init(&rbar[i], 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    if constexpr (PAIR)
      tmem_alloc_pair(tmem_slot, 2 * a.sub * a.acc_cols);
    else
      tmem_alloc(tmem_slot, 2 * a.sub * a.acc_cols);
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();     // the peer's barriers exist before anything signals them
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch();

  auto tileA = [&](int s) { return smem + s * stage_bytes; };
  auto tileB = [&](int s) { return smem + s * stage_bytes + a_bytes; };
  auto coords = [&](int tile, int* b0, int* t0, int* n0) {
    const int mt = tile / a.n_tiles, nt = tile % a.n_tiles;
    *b0 = (mt / tiles_t) * a.TB;
    *t0 = (mt % tiles_t) * a.TT * a.sub;
    *n0 = nt * a.ntile;
  };

  // Ring positions advance with counters (slot, phase) rather than divisions: the producer and MMA loops are single
  // threads whose every instruction sits between two tensor-core issues.
  auto advance = [](int& slot, uint32_t& phase, int n) {
    if (++slot == n) {
      slot = 0;
      phase ^= 1u;
    }
  };
  const uint64_t desc_hi = KC == 64 ? ((1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61))
                                    : ((1ull << 16) | (32ull << 32) | (1ull << 46) | (4ull << 61));
  // an operand descriptor is desc_hi plus the start address in 16-byte units (14 bits: shared memory < 256 KB), so an
  // offset into a tile -- a slot, a slab row, a 16-element K step -- is a plain add
  auto desc_at = [&](uint32_t addr) { return desc_hi | (uint64_t)((addr >> 4) & 0x3FFFu); };

  if (a.slab) {
    // ------------------------------------------------------------------ slab mode
    // A (warp 0): for each unit, for each channel block c, the slab of its input rows. B (warp 2): the weight tiles
    // of (channel block, tap) -- all of them loaded once and kept (a.resident), or streamed through a ring of nb
    // slots in the order the MMA uses them. The two producers never wait on each other.
    auto slotA = [&](int s) { return smem + s * a.a_slot; };
    auto slotB = [&](int s) { return smem + a.na * a.a_slot + s * bslot; };
    uint64_t *fullA = full, *emptyA = empty, *fullB = full + a.na, *emptyB = empty + a.na;
    if (warp == 0 && lane == 0) {
      const uint64_t pol_x = policy_evict_first();
      const int nbox = (a.R + a.hb - 1) / a.hb;
      const uint32_t box_bytes = a.hb * KC * 2, slab_bytes = nbox * box_bytes;
      int qa = 0, sa = 0;
      uint32_t pa = 0;
      bool ok = true;
      pdl_wait();                              // the input rows are the previous kernel's output
      for (int q = cid; q < iters && ok; q += ncl) {
        int b0, t0, n0;
        coords(tile_of(q), &b0, &t0, &n0);
        for (int c = 0; c < cblocks; ++c) {
          if (!(ok = mbar_wait(&emptyA[sa], pa ^ 1u, ERR_TIMEOUT_EMPTY, KERNEL_ID_CONV))) break;
          if constexpr (PAIR) {                  // both slabs count on the first CTA's barrier
            if (rank == 0) mbar_arrive_expect_tx(&fullA[sa], 2 * slab_bytes);
            const uint32_t mb = dsmem_addr(smem_u32(&fullA[sa]), 0);
            for (int x = 0; x < nbox; ++x)
              tma_load_3d_pair(slotA(sa) + x * box_bytes, &tmX, mb, c * KC, t0 + x * a.hb, b0, pol_x);
          } else {
            mbar_arrive_expect_tx(&fullA[sa], slab_bytes);
            for (int x = 0; x < nbox; ++x)       // rows past the end of the input read as zeros (and go unused)
              tma_load_3d(slotA(sa) + x * box_bytes, &tmX, &fullA[sa], c * KC, t0 + x * a.hb, b0, pol_x);
          }
          ++qa;
          advance(sa, pa, a.na);
        }
      }
      // every load issued has landed before the CTA can exit (also after a timeout); a pair's second CTA knows it
      // from the first, which waited for both slabs, at the closing cluster barrier
      if (!PAIR || rank == 0)
        for (int i = max(0, qa - a.na); i < qa; ++i)
          mbar_wait(&fullA[i % a.na], (i / a.na) & 1, ERR_TIMEOUT_FULL, KERNEL_ID_CONV);
    } else if (warp == 2 && lane == 0) {
      // weights are never written by a previous kernel: no wait for it
      const uint64_t pol_w = policy_evict_last();
      if (a.resident) {                        // one output tile (n0 = 0): every (c, j) tile, once
        mbar_arrive_expect_tx(&fullB[0], uint32_t(a.nb) * b_bytes);
        for (int c = 0; c < cblocks; ++c)
          for (int j = 0; j < a.taps; ++j)
            tma_load_2d(slotB(c * a.taps + j), &tmW, &fullB[0], j * a.Cin + c * KC, 0, pol_w);
        mbar_wait(&fullB[0], 0, ERR_TIMEOUT_FULL, KERNEL_ID_CONV);
      } else {
        int qb = 0, sb = 0;
        uint32_t pb = 0;
        bool ok = true;
        for (int q = cid; q < iters && ok; q += ncl) {
          int b0, t0, n0;
          coords(tile_of(q), &b0, &t0, &n0);
          for (int c = 0; c < cblocks && ok; ++c) {
            if (a.wbox) {                        // every tap's tile of channel block c in one box
              if (!(ok = mbar_wait(&emptyB[sb], pb ^ 1u, ERR_TIMEOUT_EMPTY, KERNEL_ID_CONV))) break;
              if constexpr (PAIR) {
                if (rank == 0) mbar_arrive_expect_tx(&fullB[sb], 2 * bslot);
                tma_load_3d_pair(slotB(sb), &tmW, dsmem_addr(smem_u32(&fullB[sb]), 0), c * KC,
                                 n0 + (int)rank * (a.ntile / 2), 0, pol_w);
              } else {
                mbar_arrive_expect_tx(&fullB[sb], bslot);
                tma_load_3d(slotB(sb), &tmW, &fullB[sb], c * KC, n0, 0, pol_w);
              }
              ++qb;
              advance(sb, pb, a.nb);
              continue;
            }
            for (int j = 0; j < a.taps; ++j) {
              if (!(ok = mbar_wait(&emptyB[sb], pb ^ 1u, ERR_TIMEOUT_EMPTY, KERNEL_ID_CONV))) break;
              if constexpr (PAIR) {              // this CTA's half of the tile's output channels
                if (rank == 0) mbar_arrive_expect_tx(&fullB[sb], 2 * b_bytes);
                tma_load_2d_pair(slotB(sb), &tmW, dsmem_addr(smem_u32(&fullB[sb]), 0), j * a.Cin + c * KC,
                                 n0 + (int)rank * (a.ntile / 2), pol_w);
              } else {
                mbar_arrive_expect_tx(&fullB[sb], b_bytes);
                tma_load_2d(slotB(sb), &tmW, &fullB[sb], j * a.Cin + c * KC, n0, pol_w);
              }
              ++qb;
              advance(sb, pb, a.nb);
            }
          }
        }
        if (!PAIR || rank == 0)
          for (int i = max(0, qb - a.nb); i < qb; ++i)
            mbar_wait(&fullB[i % a.nb], (i / a.nb) & 1, ERR_TIMEOUT_FULL, KERNEL_ID_CONV);
      }
    } else if (warp == 1 && (!PAIR || rank == 0)) {
      // the whole warp walks the loop (warp-uniform descriptors and ring positions); one elected lane issues the MMAs
      // and commits (from one lane alone, each commit + barrier wait between MMA groups cost ~20 ns an MMA more)
      const uint32_t idesc = umma_idesc(PAIR ? 256 : 128, a.ntile, 0);   // fp16 x fp16 -> fp32
      const uint64_t dA0 = desc_at(smem_u32(slotA(0))), dB0 = desc_at(smem_u32(slotB(0)));
      const uint32_t a_step = a.a_slot >> 4, b_step = b_bytes >> 4;   // one slot, in descriptor units
      const uint32_t row_step = (KC * 2) >> 4, tap_step = a.dil * row_step, sub_step = 128 * row_step;
      int sa = 0, sb = 0, it = 0;
      uint32_t pa = 0, pb = 0;
      bool ok = !a.resident || mbar_wait_all(&fullB[0], 0, ERR_TIMEOUT_FULL, KERNEL_ID_CONV);
      for (int q = cid; q < iters && ok; q += ncl, ++it) {
        const int acc = it & 1, use = it >> 1;
        if (!(ok = mbar_wait_all(&tempty[acc], (use & 1) ^ 1, ERR_TIMEOUT_ACCUM, KERNEL_ID_CONV))) break;
        tc_fence_after();
        const uint32_t d0 = tmem + acc * a.sub * a.acc_cols;
        uint64_t dBr = dB0;                      // resident weights: tile (c, j) sits at slot c * taps + j
        for (int c = 0; c < cblocks && ok; ++c) {
          if (!(ok = mbar_wait_all(&fullA[sa], pa, ERR_TIMEOUT_FULL, KERNEL_ID_CONV))) break;
          tc_fence_after();
          // Consecutive MMAs into one accumulator pipeline; switching accumulators between them serialises each
          // behind the last (measured from one thread, N 16-256: ~51 ns an MMA chained, ~131 ns alternating). With
          // resident weights each sub-tile therefore takes its whole (tap, K step) run in turn -- the same summation
          // order a sub-tile had -- and only streamed weight tiles are shared MMA by MMA across sub-tiles.
          if (a.resident) {
            if (elect_one()) {
              for (int s = 0; s < a.sub; ++s) {
                uint64_t da_j = dA0 + sa * a_step + s * sub_step, db = dBr;   // tile (c, j) at slot c * taps + j
                const uint32_t d = d0 + s * a.acc_cols;
                for (int j = 0; j < a.taps; ++j, da_j += tap_step, db += b_step) {
                  umma_f16(d, da_j, db, idesc, (c | j) != 0);
#pragma unroll
                  for (int k = 1; k < KC / 16; ++k) umma_f16(d, da_j + 2 * k, db + 2 * k, idesc, 1);
                }
              }
            }
            __syncwarp();
            dBr += a.taps * b_step;
          } else if (a.wbox) {                   // slot sb holds channel block c's tile for every tap
            if (!(ok = mbar_wait_all(&fullB[sb], pb, ERR_TIMEOUT_FULL, KERNEL_ID_CONV))) break;
            tc_fence_after();
            if (elect_one()) {
              uint64_t da_j = dA0 + sa * a_step, db = dB0 + sb * (bslot >> 4);
              for (int j = 0; j < a.taps; ++j, da_j += tap_step, db += b_step) {
                const uint32_t acc0 = (c | j) != 0;
                if constexpr (PAIR) {
                  umma_f16_pair(d0, da_j, db, idesc, acc0);
#pragma unroll
                  for (int k = 1; k < KC / 16; ++k) umma_f16_pair(d0, da_j + 2 * k, db + 2 * k, idesc, 1);
                } else {
                  umma_f16(d0, da_j, db, idesc, acc0);
#pragma unroll
                  for (int k = 1; k < KC / 16; ++k) umma_f16(d0, da_j + 2 * k, db + 2 * k, idesc, 1);
                }
              }
              if constexpr (PAIR)
                umma_commit_pair(&emptyB[sb]);
              else
                umma_commit(&emptyB[sb]);
            }
            __syncwarp();
            advance(sb, pb, a.nb);
          } else {
            uint64_t da_j = dA0 + sa * a_step;   // tap j reads the slab from row j * dil
            for (int j = 0; j < a.taps; ++j, da_j += tap_step) {
              if (!(ok = mbar_wait_all(&fullB[sb], pb, ERR_TIMEOUT_FULL, KERNEL_ID_CONV))) break;
              tc_fence_after();
              const uint64_t db = dB0 + sb * b_step;
              const uint32_t acc0 = (c | j) != 0;
              if (elect_one()) {
                if constexpr (PAIR) {            // (the host pairs CTAs only with one 128-step sub-tile)
                  umma_f16_pair(d0, da_j, db, idesc, acc0);
#pragma unroll
                  for (int k = 1; k < KC / 16; ++k) umma_f16_pair(d0, da_j + 2 * k, db + 2 * k, idesc, 1);
                  umma_commit_pair(&emptyB[sb]);
                } else {
                  umma_f16(d0, da_j, db, idesc, acc0);
#pragma unroll
                  for (int k = 1; k < KC / 16; ++k) umma_f16(d0, da_j + 2 * k, db + 2 * k, idesc, 1);
                  if (a.sub == 2) {              // the second 128-step sub-tile shares the weight tile
                    const uint64_t da2 = da_j + sub_step;
                    umma_f16(d0 + a.acc_cols, da2, db, idesc, acc0);
#pragma unroll
                    for (int k = 1; k < KC / 16; ++k) umma_f16(d0 + a.acc_cols, da2 + 2 * k, db + 2 * k, idesc, 1);
                  }
                  umma_commit(&emptyB[sb]);
                }
              }
              __syncwarp();
              advance(sb, pb, a.nb);
            }
          }
          if (elect_one()) {
            if constexpr (PAIR)
              umma_commit_pair(&emptyA[sa]);
            else
              umma_commit(&emptyA[sa]);
          }
          __syncwarp();
          advance(sa, pa, a.na);
        }
        if (elect_one()) {                       // (after a timeout too: the epilogue is not left waiting)
          if constexpr (PAIR)
            umma_commit_pair(&tfull[acc]);
          else
            umma_commit(&tfull[acc]);
        }
        __syncwarp();
      }
    }
  } else if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_last(), pol_x = policy_evict_first();
      // the first tile's weights do not depend on the previous kernel: start them before waiting for it
      const int first = blockIdx.x;
      int q = 0, sq = 0;                     // k blocks issued so far (all tiles); ring slot of the next
      uint32_t pq = 0;
      bool ok = true;
      if (first < total) {
        int b0, t0, n0;
        coords(first, &b0, &t0, &n0);
        const int pre = min(stages, nkb);
        for (int i = 0; i < pre; ++i) {
          mbar_arrive_expect_tx(&full[i], stage_bytes);
          tma_load_2d(tileB(i), &tmW, &full[i], (i / cblocks) * a.Cin + (i % cblocks) * KC, n0, pol_w);
        }
        pdl_wait();
        for (int i = 0; i < pre; ++i)
          tma_load_3d(tileA(i), &tmX, &full[i], (i % cblocks) * KC, t0 + (i / cblocks) * a.dil, b0, pol_x);
        q = pre;
        sq = pre == stages ? 0 : pre;
        pq = pre == stages ? 1u : 0u;
        for (int i = pre, c = pre % cblocks, j = pre / cblocks; i < nkb; ++i) {
          if (!(ok = mbar_wait(&empty[sq], pq ^ 1u, ERR_TIMEOUT_EMPTY, KERNEL_ID_CONV))) break;
          mbar_arrive_expect_tx(&full[sq], stage_bytes);
          tma_load_2d(tileB(sq), &tmW, &full[sq], j * a.Cin + c * KC, n0, pol_w);
          tma_load_3d(tileA(sq), &tmX, &full[sq], c * KC, t0 + j * a.dil, b0, pol_x);
          q = i + 1;
          advance(sq, pq, stages);
          if (++c == cblocks) {
            c = 0;
            ++j;
          }
        }
      } else {
        pdl_wait();
      }
      for (int tile = first + gridDim.x; tile < total && ok; tile += gridDim.x) {
        int b0, t0, n0;
        coords(tile, &b0, &t0, &n0);
        for (int i = 0, c = 0, j = 0; i < nkb; ++i, ++q) {
          if (!(ok = mbar_wait(&empty[sq], pq ^ 1u, ERR_TIMEOUT_EMPTY, KERNEL_ID_CONV))) break;
          mbar_arrive_expect_tx(&full[sq], stage_bytes);
          tma_load_2d(tileB(sq), &tmW, &full[sq], j * a.Cin + c * KC, n0, pol_w);
          tma_load_3d(tileA(sq), &tmX, &full[sq], c * KC, t0 + j * a.dil, b0, pol_x);
          advance(sq, pq, stages);
          if (++c == cblocks) {
            c = 0;
            ++j;
          }
        }
      }
      // every load issued has landed before the CTA can exit (also after a timeout)
      for (int i = max(0, q - stages); i < q; ++i)
        mbar_wait(&full[i % stages], (i / stages) & 1, ERR_TIMEOUT_FULL, KERNEL_ID_CONV);
    }
  } else if (warp == 1) {
    const uint32_t idesc = umma_idesc(128, a.ntile, 0);   // fp16 x fp16 -> fp32 (the warp walks, one lane issues)
    const uint64_t dA0 = desc_at(smem_u32(tileA(0))), dB0 = desc_at(smem_u32(tileB(0)));
    const uint32_t st_step = stage_bytes >> 4;
    int sq = 0, it = 0;
    uint32_t pq = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++it) {
      const int acc = it & 1, use = it >> 1;
      if (!(ok = mbar_wait_all(&tempty[acc], (use & 1) ^ 1, ERR_TIMEOUT_ACCUM, KERNEL_ID_CONV))) break;
      tc_fence_after();
      const uint32_t d = tmem + acc * a.acc_cols;
      for (int i = 0; i < nkb; ++i) {
        if (!(ok = mbar_wait_all(&full[sq], pq, ERR_TIMEOUT_FULL, KERNEL_ID_CONV))) break;
        tc_fence_after();
        const uint64_t da = dA0 + sq * st_step, db = dB0 + sq * st_step;
        if (elect_one()) {
          umma_f16(d, da, db, idesc, i != 0);
#pragma unroll
          for (int k = 1; k < KC / 16; ++k) umma_f16(d, da + 2 * k, db + 2 * k, idesc, 1);
          umma_commit(&empty[sq]);
        }
        __syncwarp();
        advance(sq, pq, stages);
      }
      if (elect_one()) umma_commit(&tfull[acc]);   // (after a timeout too: the epilogue is not left waiting)
      __syncwarp();
    }
  }
  if (warp >= 3) {
    // ---------------------------------------------------------------- epilogue warps
    const int ew = warp - 3;                  // 0 .. CONV_EPI_WARPS-1
    const int quarter = warp & 3;             // TMEM lanes [32 quarter, +32) are this warp's
    const int part = ew >> 2;                 // the warps on one quarter split the 16-column chunks round robin
    constexpr int PARTS = CONV_EPI_WARPS / 4;
    const int r = quarter * 32 + lane;        // token row of the tile
    const int rb = r / a.TT, rt = r - rb * a.TT;   // its batch row and timestep within a unit
    {                                         // weights, not written by the previous kernel: before its end
      const int et = tid - 96;
      if (a.bias != nullptr)
        for (int i = et; i < a.N; i += 32 * CONV_EPI_WARPS) s_bias[i] = a.bias[i];
      uint32_t amax = 0;
      if (a.alpha != nullptr)
        for (int i = et; i < a.cout; i += 32 * CONV_EPI_WARPS) {
          const float al = a.alpha[i];
          s_alpha[i] = al;
          s_inv[i] = a.inv[i];
          amax = max(amax, __float_as_uint(al) & 0x7FFFFFFFu);
        }
      amax = __reduce_max_sync(0xffffffffu, amax);
      if (lane == 0 && amax != 0) atomicMax(s_amax, amax);
      asm volatile("bar.sync 1, %0;" ::"n"(32 * CONV_EPI_WARPS) : "memory");   // the epilogue warps only
    }
    const bool act = a.nxt != nullptr && a.alpha != nullptr;
    // |y| <= 65504 for an fp16 y, so below |alpha| = 32 every |alpha y| is inside sin2_reduced2's range: no check
    const bool chk = act && *s_amax >= __float_as_uint(SIN2_RANGE / 65536.f);
    const bool cmod = a.cout != a.N;          // a transposed conv's phases share their channel's activation
    pdl_wait();                               // outputs may be buffers the previous kernel still reads
    const int nchunk = a.ntile >> 4;          // (outside the audio mode N and ntile are multiples of 16)
    const int W = a.sub * nchunk;             // epilogue items of a unit: (sub-tile, 16-column chunk) pairs
    if constexpr (ETMA) {
      uint8_t* wst = estage + ew * ETMA_WARP_BYTES;   // residual[2] | raw | next input
      uint64_t* rbw = rbar + 2 * ew;
      const uint64_t pol = policy_evict_first();
      const bool has_res = a.res != nullptr;
      const int row0 = quarter * 32;
      uint32_t rq = 0, rd = 0;                        // residual boxes requested / consumed by this warp
      int it = 0;
      for (int q = cid; q < iters; q += ncl, ++it) {
        const int acc = it & 1, use = it >> 1;
        int b0, t0, n0;
        coords(tile_of(q), &b0, &t0, &n0);
        const int bw = b0 + row0 / a.TT, tw = t0 + row0 % a.TT;   // the warp's box: 32 steps of one batch row
        const bool live = bw < a.rows;                 // (warp-uniform; rows past the input are clipped by TMA)
        int f = part - (it * W) % PARTS;
        if (f < 0) f += PARTS;
        auto request = [&](int item) {                 // residual box of an item into the next staging slot
          if (lane == 0) {
            uint64_t* bar = &rbw[rq & 1];
            mbar_arrive_expect_tx(bar, 1024);
            tma_load_3d(wst + (rq & 1) * 1024, &tmR, bar, n0 + item * 16, tw, bw, pol);
          }
          ++rq;
        };
        if (has_res && f < W) request(f);              // before the accumulator wait
        const bool ok = mbar_wait(&tfull[acc], use & 1, ERR_TIMEOUT_ACCUM, KERNEL_ID_CONV);
        if (!ok) break;                                // (recorded; the MMA has stopped too)
        tc_fence_after();
        const uint32_t tbase = tmem + acc * a.acc_cols + (uint32_t(row0) << 16);
        for (; f < W; f += PARTS) {
          // the next item's residual goes to the slot the previous item's came from (read into registers already)
          if (has_res && f + PARTS < W) request(f + PARTS);
          const int nb = n0 + f * 16;
          float v[16];
          tmem_ld16(tbase + f * 16, v);
          if (a.bias != nullptr) {
#pragma unroll
            for (int i = 0; i < 16; i += 4) {
              const float4 bv = *reinterpret_cast<const float4*>(s_bias + nb + i);
              const float2 p0 = fadd2(make_float2(v[i], v[i + 1]), make_float2(bv.x, bv.y));
              const float2 p1 = fadd2(make_float2(v[i + 2], v[i + 3]), make_float2(bv.z, bv.w));
              v[i] = p0.x;
              v[i + 1] = p0.y;
              v[i + 2] = p1.x;
              v[i + 3] = p1.y;
            }
          }
          if (has_res) {
            mbar_wait(&rbw[rd & 1], (rd >> 1) & 1, ERR_TIMEOUT_FULL, KERNEL_ID_CONV);
            const uint4* src = reinterpret_cast<const uint4*>(wst + (rd & 1) * 1024 + lane * 32);
            const uint4 u0 = src[0], u1 = src[1];
            ++rd;
            const uint32_t rc[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float2 qq = fadd2(make_float2(v[2 * i], v[2 * i + 1]), unpack_f16(rc[i]));
              v[2 * i] = qq.x;
              v[2 * i + 1] = qq.y;
            }
          }
          uint32_t hy[8], ha[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {               // fp16 y, and v becomes it (as fp32)
            hy[i] = pack_f16(v[2 * i], v[2 * i + 1]);
            const float2 qq = unpack_f16(hy[i]);
            v[2 * i] = qq.x;
            v[2 * i + 1] = qq.y;
          }
          if (act) {
            int c = nb;
            if (cmod)
              while (c >= a.cout) c -= a.cout;   // nb < N = phases x cout
            if (chk) {
              const bool good = snake16<true>(v, s_alpha + c, s_inv + c, ha);
              if (!__all_sync(0xffffffffu, good || !live)) snake16_exact(v, s_alpha + c, s_inv + c, ha);   // rare
            } else {
              snake16<false>(v, s_alpha + c, s_inv + c, ha);
            }
          }
          if (lane == 0) bulk_wait_read();            // this warp's last stores have read the staging
          __syncwarp();
          uint4* dr = reinterpret_cast<uint4*>(wst + 2048 + lane * 32);
          uint4* dn = reinterpret_cast<uint4*>(wst + 3072 + lane * 32);
          if (a.raw != nullptr) {
            dr[0] = make_uint4(hy[0], hy[1], hy[2], hy[3]);
            dr[1] = make_uint4(hy[4], hy[5], hy[6], hy[7]);
          }
          if (a.nxt != nullptr) {
            const uint32_t* o = act ? ha : hy;
            dn[0] = make_uint4(o[0], o[1], o[2], o[3]);
            dn[1] = make_uint4(o[4], o[5], o[6], o[7]);
          }
          fence_proxy_async_smem();                    // the staging writes, to the TMA engine
          __syncwarp();
          if (lane == 0) {
            if (a.raw != nullptr) tma_store_3d(&tmO, wst + 2048, nb, tw, bw);
            if (a.nxt != nullptr) tma_store_3d(&tmN, wst + 3072, nb, tw, bw);
            bulk_commit();
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
      }
      // residual boxes still in flight (after a timeout) land before the CTA ends; so do the stores
      for (; rd < rq; ++rd) mbar_wait(&rbw[rd & 1], (rd >> 1) & 1, ERR_TIMEOUT_FULL, KERNEL_ID_CONV);
      if (lane == 0) bulk_wait_all();
    } else {
      const long long res_sub = 128LL * a.res_ts, raw_sub = 128LL * a.raw_ts, nxt_sub = 128LL * a.N;
      int it = 0;
      for (int q = cid; q < iters; q += ncl, ++it) {
        const int acc = it & 1, use = it >> 1;
        int b0, t0, n0;
        coords(tile_of(q), &b0, &t0, &n0);
        const int b = b0 + rb;
        const bool live = b < a.rows;
        const long long ts = t0 + rt;
        // the unit's items are dealt round robin over the warps of this lane quarter, the deal continuing from unit to
        // unit (a warp left with fewer items of one unit takes more of the next)
        int f = part - (it * W) % PARTS;
        if (f < 0) f += PARTS;
        int s = f / nchunk, ch = f - s * nchunk;
        // this thread's elements of (sub-tile 0, chunk 0) of the unit; null where nothing is read or written
        const __half* resp = (a.res != nullptr && live) ? a.res + b * a.res_bs + ts * a.res_ts + n0 : nullptr;
        const bool ok = mbar_wait(&tfull[acc], use & 1, ERR_TIMEOUT_ACCUM, KERNEL_ID_CONV);
        if (!ok) break;                         // (recorded; the MMA has stopped too)
        tc_fence_after();
        const uint32_t tbase = tmem + acc * a.sub * a.acc_cols + (uint32_t(quarter * 32) << 16);
        if (a.audio != nullptr) {
          for (int sb = part; sb < a.sub; sb += PARTS) {
            float v[16];
            tmem_ld16(tbase + sb * a.acc_cols, v);
            if (live) {
              const float bias = a.bias != nullptr ? a.bias[0] : 0.f;
              a.audio[(size_t)b * a.audio_bs + t0 + sb * 128 + rt] = tanhf(f16r(v[0] + bias));
            }
          }
        } else {
          __half* rawp = (a.raw != nullptr && live) ? a.raw + b * a.raw_bs + ts * a.raw_ts + n0 : nullptr;
          __half* nxtp = (a.nxt != nullptr && live) ? a.nxt + b * a.nxt_bs + a.nxt_off + ts * a.N + n0 : nullptr;
          for (; f < W; f += PARTS) {
            int s2 = s, ch2 = ch + PARTS;       // the next item of this warp
            while (ch2 >= nchunk) {
              ch2 -= nchunk;
              ++s2;
            }
            const int nb = n0 + ch * 16;
            if (nb < a.N) {                     // warp-uniform: a unit's last tile may reach past N
              float v[16];
              tmem_ld16(tbase + s * a.acc_cols + ch * 16, v);
              if (a.bias != nullptr) {
#pragma unroll
                for (int i = 0; i < 16; i += 4) {
                  const float4 bv = *reinterpret_cast<const float4*>(s_bias + nb + i);
                  const float2 p0 = fadd2(make_float2(v[i], v[i + 1]), make_float2(bv.x, bv.y));
                  const float2 p1 = fadd2(make_float2(v[i + 2], v[i + 3]), make_float2(bv.z, bv.w));
                  v[i] = p0.x;
                  v[i + 1] = p0.y;
                  v[i + 2] = p1.x;
                  v[i + 3] = p1.y;
                }
              }
              if (resp != nullptr) {            // (the decoder's residual convs take the TMA-box epilogue)
                uint32_t rc[8];
                ld_global_v8(resp + s * res_sub + ch * 16, rc);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  const float2 q = fadd2(make_float2(v[2 * i], v[2 * i + 1]), unpack_f16(rc[i]));
                  v[2 * i] = q.x;
                  v[2 * i + 1] = q.y;
                }
              }
              uint32_t hy[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) {     // fp16 y, and v becomes it (as fp32)
                hy[i] = pack_f16(v[2 * i], v[2 * i + 1]);
                const float2 q = unpack_f16(hy[i]);
                v[2 * i] = q.x;
                v[2 * i + 1] = q.y;
              }
              if (rawp != nullptr) st_global_v8(rawp + s * raw_sub + ch * 16, hy);   // one 32-byte sector a thread
              if (act) {
                int c = nb;
                if (cmod)
                  while (c >= a.cout) c -= a.cout;   // nb < N = phases x cout
                uint32_t ha[8];
                if (chk) {
                  const bool good = snake16<true>(v, s_alpha + c, s_inv + c, ha);
                  if (!__all_sync(0xffffffffu, good || !live)) snake16_exact(v, s_alpha + c, s_inv + c, ha);   // rare
                } else {
                  snake16<false>(v, s_alpha + c, s_inv + c, ha);
                }
                if (nxtp != nullptr) st_global_v8(nxtp + s * nxt_sub + ch * 16, ha);
              } else if (nxtp != nullptr) {
                st_global_v8(nxtp + s * nxt_sub + ch * 16, hy);
              }
            }
            s = s2;
            ch = ch2;
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (PAIR)                   // the pair's MMA warp (first CTA) waits for both CTAs' drains
            mbar_arrive_cluster(dsmem_addr(smem_u32(&tempty[acc]), 0));
          else
            mbar_arrive(&tempty[acc]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) {
    cluster_sync();                       // no CTA leaves while its peer may still signal its barriers
    if (warp == 1) tmem_dealloc_pair(tmem, 2 * a.sub * a.acc_cols);
  } else {
    if (warp == 1) tmem_dealloc(tmem, 2 * a.sub * a.acc_cols);
  }
}

// ------------------------------------------------------------------------------------------------ context shift
// After a codec step: every conv's carried context becomes the last ctx rows its input had, xin[b, :ctx] =
// xin[b, T : T + ctx] (serve/fast_engine.py:230-231 state update). Rows move in chunks of T so a chunk never
// overlaps its source (ctx > T: the old context's tail moves down first). One block per (conv, batch row).
__global__ void k_ctx_shift(const A8CtxShift* __restrict__ tab, int rows) {
  pdl_launch();
  pdl_wait();
  const A8CtxShift e = tab[blockIdx.x];
  const int b = blockIdx.y;
  if (b >= rows) return;
  uint4* base = reinterpret_cast<uint4*>(reinterpret_cast<__half*>(e.xin) + (size_t)b * (e.ctx + e.T) * e.Cin);
  const int vec_row = e.Cin / 8;
  for (int r0 = 0; r0 < e.ctx; r0 += e.T) {
    const int nrow = min(e.T, e.ctx - r0);
    for (int i = threadIdx.x; i < nrow * vec_row; i += blockDim.x)
      base[(size_t)r0 * vec_row + i] = base[(size_t)(r0 + e.T) * vec_row + i];
    __syncthreads();
  }
}

// ------------------------------------------------------------------------------------------------ host
struct ConvPlan {
  CUtensorMap tmX, tmW;
  ConvArgs args;
  dim3 grid;
  int smem;
};

// xin: fp16 [rows, ctx + T, Cin]; w: fp16 [N, taps * Cin] (K-major). Outputs as in ConvArgs (set by the caller).
static int conv_plan_kc(ConvPlan* p, const void* xin, int rows, int T, int Cin, int ctx, const void* w, int N,
                        int taps, int dil, int kc) {
  if (xin == nullptr || w == nullptr || rows <= 0 || T <= 0 || Cin <= 0 || N <= 0 || taps <= 0) return A8_ERR_ARG;
  if (Cin % 32) return A8_ERR_ARG;
  if ((taps - 1) * dil > ctx) return A8_ERR_ARG;
  ConvArgs& a = p->args;
  a = ConvArgs{};
  a.rows = rows;
  a.T = T;
  a.Cin = Cin;
  a.N = N;
  a.taps = taps;
  a.dil = dil;
  a.ctx = ctx;
  a.KC = kc;
  a.TT = T >= 128 ? 128 : T;
  if (128 % a.TT || T % a.TT) return A8_ERR_ARG;
  a.TB = 128 / a.TT;
  const int nt = (N + 255) / 256;
  a.ntile = std::max(16, ((N + nt - 1) / nt + 15) / 16 * 16);
  a.n_tiles = (N + a.ntile - 1) / a.ntile;
  a.m_tiles = (T / a.TT) * ((rows + a.TB - 1) / a.TB);
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
  }
  // A k > 1 conv outside slab mode with too few work units for the SMs (the first conv at T = 4: 36 units of 256
  // columns) takes narrower output tiles: each SM then streams a smaller share of the weights
  if (taps > 1 && !(a.TT == 128 && ctx <= 128))
    while (a.ntile >= 128 && a.ntile % 32 == 0 && 2 * a.m_tiles * a.n_tiles <= sms) {
      a.ntile /= 2;
      a.n_tiles = (N + a.ntile - 1) / a.ntile;
    }
  a.kb_total = taps * (Cin / a.KC);
  a.acc_cols = a.ntile <= 32 ? 32 : a.ntile <= 64 ? 64 : a.ntile <= 128 ? 128 : 256;
  const int stage_bytes = 128 * a.KC * 2 + a.ntile * a.KC * 2;
  // shared memory for the pipeline: what is left of 227 KB after the alignment slack, the barriers and the
  // epilogue's staged column constants (bias [N], alpha and inv [cout <= N])
  const int n4 = (N + 3) / 4 * 4;
  const int budget = 227 * 1024 - 1024 - CONV_BAR_BYTES - 3 * n4 * 4;
  a.stages = std::max(2, std::min(8, budget / stage_bytes));
  a.cout = N;
  // slab mode: units of one batch row, 128 steps -- or two 128-step sub-tiles sharing each weight tile when T allows
  // and the output tile is at most 128 columns (the accumulator pairs stay double-buffered in 512 TMEM columns;
  // narrowing a wider tile to get there measured slower: twice the MMA instructions at half the width)
  a.sub = 1;
  a.slab = (a.TT == 128 && taps > 1 && ctx <= 128) ? 1 : 0;
  if (a.slab && T % 256 == 0 && a.ntile <= 128) a.sub = 2;
  a.m_tiles = (T / (a.TT * a.sub)) * ((rows + a.TB - 1) / a.TB);
  const int b_bytes = a.ntile * a.KC * 2;
  if (a.slab) {
    a.R = 128 * a.sub + ctx;
    a.hb = a.R <= 256 ? a.R : ((a.R + 1) / 2 + 7) / 8 * 8;   // boxes of <= 256 rows, 8-row aligned
    const int nbox = (a.R + a.hb - 1) / a.hb;
    a.a_slot = ((uint32_t)nbox * a.hb * a.KC * 2 + 1023) / 1024 * 1024;
    // weights resident when one output tile's (every tap and channel block) fit beside two slab slots; the
    // rest of the room deepens the slab ring (up to 4). Otherwise two slab slots and a ring of weight tiles.
    const int wres = taps * (Cin / a.KC) * b_bytes;
    if (a.n_tiles == 1 && wres + 2 * (int)a.a_slot <= budget) {
      a.resident = 1;
      a.nb = taps * (Cin / a.KC);
      a.na = std::min(4, (budget - wres) / (int)a.a_slot);
    } else {
      a.resident = 0;
      a.na = 2;
      // Streamed weights: CTA pairs, each CTA holding half of every weight tile (so the ring holds twice the MMA
      // work in the same bytes) and one 256-row MMA instruction doing both CTAs' rows. Measured on the k7 convs at
      // Cin 192 / 384: ~8 % faster; the 2-tap transposed conv is not (kept on single CTAs).
      a.pair = (a.sub == 1 && a.ntile % 32 == 0 && taps > 2) ? 1 : 0;
      const int bb = a.pair ? b_bytes / 2 : b_bytes, room = budget - a.na * (int)a.a_slot;
      // A TMA box costs ~270 ns of the SM's load engine whatever its size (measured: 96-row boxes stream 45 GB/s an
      // SM, 192-row ones 90, one 84 KB box of 7 taps 165), so when two slots fit, a slot holds one channel block's
      // tiles for every tap, loaded as one 3-D box; else a ring of one tap's tile a slot.
      if (a.sub == 1 && room >= 2 * taps * bb) {
        a.wbox = 1;
        a.nb = std::min(4, room / (taps * bb));
        a.na = std::min(4, (budget - a.nb * taps * bb) / (int)a.a_slot);   // what the weight slots leave: slabs
      } else {
        a.nb = std::min(a.pair ? 24 : 16, room / bb);
        if (a.nb < 2) return A8_ERR_SIZE;                    // (not reached with the decoder's shapes)
      }
    }
  }
  const CUtensorMapSwizzle sw = a.KC == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  int rc = encode_map_3d(&p->tmX, xin, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, Cin, ctx + T, rows, (uint64_t)Cin * 2,
                         (uint64_t)(ctx + T) * Cin * 2, a.KC, a.slab ? a.hb : a.TT, a.slab ? 1 : a.TB, sw);
  if (rc) return rc;
  if (a.wbox)   // W [N, taps * Cin] viewed as (channel within Cin, output row, tap): box {KC, rows, taps}, tap-major
    rc = encode_map_3d(&p->tmW, w, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, Cin, N, taps, (uint64_t)taps * Cin * 2,
                       (uint64_t)Cin * 2, a.KC, a.pair ? a.ntile / 2 : a.ntile, taps, sw);
  else
    rc = encode_map_2d(&p->tmW, w, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)taps * Cin, N,
                       (uint64_t)taps * Cin * 2, a.KC, a.pair ? a.ntile / 2 : a.ntile, sw);
  if (rc) return rc;
  const int total = a.m_tiles * a.n_tiles;
  if (a.pair) {
    const int pairs = (a.m_tiles + 1) / 2 * a.n_tiles;
    p->grid = dim3(2 * std::min(pairs, sms / 2));
  } else {
    p->grid = dim3(std::min(total, sms));
  }
  const int bslot = (a.pair ? b_bytes / 2 : b_bytes) * (a.wbox ? taps : 1);
  p->smem = (a.slab ? a.na * a.a_slot + a.nb * bslot : a.stages * stage_bytes) + 1024 + CONV_BAR_BYTES;
  return A8_OK;
}

int conv_plan(ConvPlan* p, const void* xin, int rows, int T, int Cin, int ctx, const void* w, int N, int taps,
              int dil) {
  int rc = conv_plan_kc(p, xin, rows, T, Cin, ctx, w, N, taps, dil, Cin % 64 == 0 ? 64 : 32);
  // Paired k7 convs stream a channel block's weights for every tap a slot: at K blocks of 64 the two rings hold two
  // blocks each, at 32 four (the same bytes, prefetched twice as far ahead of the MMAs). Measured on the Cin 192 / 384
  // k7 convs: 2-4 % faster at 32.
  if (rc == A8_OK && p->args.pair && p->args.wbox && p->args.KC == 64) {
    ConvPlan q;
    if (conv_plan_kc(&q, xin, rows, T, Cin, ctx, w, N, taps, dil, 32) == A8_OK && q.args.pair && q.args.wbox &&
        q.args.nb > p->args.nb && q.args.na > p->args.na)
      *p = q;
  }
  return rc;
}

// The outputs' alignment: 16-element row segments are stored as 32-byte vectors.
static int conv_check_outputs(const ConvArgs& a) {
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 31) == 0; };
  if (a.audio == nullptr && a.raw == nullptr && a.nxt == nullptr) return A8_ERR_ARG;
  if (a.audio == nullptr && a.N % 16) return A8_ERR_ARG;   // the epilogue stores 16-column segments
  if (a.N % 16 == 0) {
    if (a.raw != nullptr && (!al(a.raw) || a.raw_bs % 16 || a.raw_ts % 16)) return A8_ERR_ALIGN;
    if (a.res != nullptr && (!al(a.res) || a.res_bs % 16 || a.res_ts % 16)) return A8_ERR_ALIGN;
    if (a.nxt != nullptr && (!al(a.nxt) || a.nxt_bs % 16 || a.nxt_off % 16)) return A8_ERR_ALIGN;
    if (a.bias != nullptr && !al(a.bias)) return A8_ERR_ALIGN;
    if (a.alpha != nullptr && (a.cout % 16 || (reinterpret_cast<uintptr_t>(a.alpha) & 15) ||
                               (reinterpret_cast<uintptr_t>(a.inv) & 15)))
      return A8_ERR_ALIGN;
  }
  if (a.alpha != nullptr && (a.inv == nullptr || a.cout <= 0 || a.N % a.cout)) return A8_ERR_ARG;
  return A8_OK;
}

int conv_launch(const ConvPlan* p0, cudaStream_t s) {
  int rc = conv_check_outputs(p0->args);
  if (rc) return rc;
  ConvPlan q = *p0;
  ConvArgs& a = q.args;
  const int params = ((a.bias != nullptr ? (a.N + 3) / 4 * 4 : 0) + 2 * ((a.cout + 3) / 4 * 4)) * 4;
  // 1x1 convs with channel-contiguous rows and at least 32 steps a unit: the epilogue's I/O by TMA boxes (residual in,
  // outputs out), paid for with a shallower (A, B) pipeline; anything that does not fit keeps the per-lane epilogue
  // The same for slab convs whose weights stream by channel-block boxes on single CTAs (the transposed convs), paid
  // for with fewer weight slots.
  CUtensorMap tmR = {}, tmO = {}, tmN = {};
  a.etma = 0;
  const bool eshape = a.sub == 1 && a.TT >= 32 && a.TT % 32 == 0 && a.audio == nullptr && a.N % 16 == 0 &&
                      a.N % a.ntile == 0 && (a.res == nullptr || a.res_ts == a.N) &&
                      (a.raw == nullptr || a.raw_ts == a.N);
  const bool eplain = !a.slab && a.taps == 1, eslab = a.slab && a.wbox && !a.pair && !a.resident;
  if (eshape && (eplain || eslab)) {
    const int stage_bytes = 128 * a.KC * 2 + a.ntile * a.KC * 2;
    const int budget = 227 * 1024 - 1024 - CONV_BAR_BYTES - params - ETMA_BYTES;
    const int bslot = a.taps * a.ntile * a.KC * 2;
    const int st = eplain ? std::min(a.stages, budget / stage_bytes)
                          : std::min(a.nb, (budget - a.na * (int)a.a_slot) / bslot);
    const int nbar = eplain ? st : a.na + st;   // ring barriers + accumulator barriers + slots + residual barriers
    const auto FP16 = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const auto NOSW = CU_TENSOR_MAP_SWIZZLE_NONE;
    bool ok = st >= 2 && (2 * nbar + 4) * 8 + 8 + 2 * CONV_EPI_WARPS * 8 <= CONV_BAR_BYTES;
    if (ok && a.res != nullptr)
      ok = encode_map_3d(&tmR, a.res, FP16, 2, a.N, a.T, a.rows, (uint64_t)a.N * 2, (uint64_t)a.res_bs * 2, 16, 32, 1,
                         NOSW) == A8_OK;
    if (ok && a.raw != nullptr)
      ok = encode_map_3d(&tmO, a.raw, FP16, 2, a.N, a.T, a.rows, (uint64_t)a.N * 2, (uint64_t)a.raw_bs * 2, 16, 32, 1,
                         NOSW) == A8_OK;
    if (ok && a.nxt != nullptr)
      ok = encode_map_3d(&tmN, a.nxt + a.nxt_off, FP16, 2, a.N, a.T, a.rows, (uint64_t)a.N * 2,
                         (uint64_t)a.nxt_bs * 2, 16, 32, 1, NOSW) == A8_OK;
    if (ok) {
      a.etma = 1;
      if (eplain) {
        a.stages = st;
        q.smem = st * stage_bytes + 1024 + CONV_BAR_BYTES;
      } else {
        a.nb = st;
        q.smem = a.na * a.a_slot + st * bslot + 1024 + CONV_BAR_BYTES;
      }
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = q.grid;
  cfg.blockDim = dim3(CONV_THREADS);
  cfg.dynamicSmemBytes = q.smem + params + (a.etma ? ETMA_BYTES : 0);
  if (cfg.dynamicSmemBytes > 227 * 1024) return A8_ERR_SIZE;
  cfg.stream = s;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  at[1].id = cudaLaunchAttributeClusterDimension;   // CTA pairs: clusters of 2
  at[1].val.clusterDim.x = 2;
  at[1].val.clusterDim.y = 1;
  at[1].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = a.pair ? 2 : 1;
  ++g_launches;
  using Kern = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, ConvArgs);
  static bool attr[6] = {false, false, false, false, false, false};
  const int v = (a.KC == 64 ? 0 : 3) + (a.pair ? 1 : a.etma ? 2 : 0);
  const Kern table[6] = {k_conv<64, false, false>, k_conv<64, true, false>, k_conv<64, false, true>,
                         k_conv<32, false, false>, k_conv<32, true, false>, k_conv<32, false, true>};
  if (!attr[v]) {
    cudaFuncSetAttribute(table[v], cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    attr[v] = true;
  }
  const cudaError_t e = cudaLaunchKernelEx(&cfg, table[v], q.tmX, q.tmW, tmR, tmO, tmN, a);
  return e == cudaSuccess ? A8_OK : A8_ERR_CUDA;
}

int ctx_shift_launch(const A8CtxShift* tab_dev, int n, int rows, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n, rows);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  ++g_launches;
  return cudaLaunchKernelEx(&cfg, k_ctx_shift, tab_dev, rows) == cudaSuccess ? A8_OK : A8_ERR_CUDA;
}

}  // namespace a8

using namespace a8;

extern "C" int a8_conv(const A8ConvRun* r, a8_stream_t stream) {
  if (r == nullptr) return A8_ERR_ARG;
  ConvPlan p;
  int rc = conv_plan(&p, r->xin, r->rows, r->T, r->Cin, r->ctx, r->w, r->N, r->taps, r->dil);
  if (rc) return rc;
  ConvArgs& a = p.args;
  a.bias = reinterpret_cast<const float*>(r->bias);
  a.res = reinterpret_cast<const __half*>(r->res);
  a.res_bs = r->res_bs;
  a.res_ts = r->res_ts;
  a.raw = reinterpret_cast<__half*>(r->raw);
  a.raw_bs = r->raw_bs;
  a.raw_ts = r->raw_ts;
  a.nxt = reinterpret_cast<__half*>(r->nxt);
  a.nxt_bs = r->nxt_bs;
  a.nxt_off = r->nxt_off;
  a.cout = r->cout > 0 ? r->cout : r->N;
  a.alpha = r->alpha;
  a.inv = r->inv;
  a.audio = r->audio;
  a.audio_bs = r->audio_bs;
  return conv_launch(&p, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int a8_ctx_shift(const A8CtxShift* table, int n, int rows, a8_stream_t stream) {
  if (table == nullptr || n <= 0 || rows <= 0) return A8_ERR_ARG;
  return ctx_shift_launch(table, n, rows, reinterpret_cast<cudaStream_t>(stream));
}
