// Packed causal prefill attention on the tensor cores (serve/fast_kernels.py:296-358, _prefill_attn_kernel /
// PrefillPlan).
//
// An admission's packed rows come in query blocks (q0, n, slot, pos0) of at most 64 consecutive positions of one
// request: row q0 + r sits at position pos0 + r of cache row `slot` and attends keys [0, pos0 + r] there (its own K/V
// and the request's earlier ones were stored by the qkv GEMM epilogue). One CTA takes one block, one kv head and a
// pair of that kv head's query heads: a 128-row tcgen05 tile (64 rows x 2 heads; with an odd group the last head pairs
// with zero rows), so every 64-key K / V tile it loads serves 128 query vectors.
//   warp 0 / one lane : TMA producer: the Q tile once, then the block's K tiles (pass 1), K and V tiles (pass 2)
//                       through a ring of stages
//   warp 1 / one lane : MMA issuer: S = Q K^T (M 128, N 64, K 64) into one of two TMEM tiles; O += P V^T
//   warps 2-3         : each V tile [keys x hd] rewritten as the K-major [hd x keys] operand of P V
//   warps 4-7         : softmax, one query vector a thread (its TMEM lane)
// The softmax takes two passes over the keys with the exact row maximum, as the CPU oracle does: pass 1 finds each
// row's max of q.k over its causal keys; pass 2 forms p = exp(scale (s - max)), sums p in fp32 and gives bf16(p) to
// the tensor core (the reference rounds P to bf16 for its tl.dot too, serve/fast_kernels.py:325-330).
#include "common.cuh"

namespace a8 {

constexpr int KERNEL_ID_PATTN = 7;
constexpr int PATTN_THREADS = 256;
constexpr int PATTN_NST = 2;                      // K / V ring stages
constexpr int PATTN_TILE = 64 * 128;              // 64 rows x 128 bytes (64 bf16): one TMA box
constexpr int PATTN_Q_BYTES = 2 * PATTN_TILE;     // 128 query vectors
constexpr int PATTN_P_BYTES = 2 * PATTN_TILE;     // P tile: 128 query vectors x 64 keys
constexpr int PATTN_STAGE = 3 * PATTN_TILE;       // K, V, V^T
constexpr int PATTN_DATA = PATTN_Q_BYTES + 2 * PATTN_P_BYTES + PATTN_NST * PATTN_STAGE;
constexpr int PATTN_SMEM = PATTN_DATA + 1024 + 256;
constexpr uint32_t PATTN_TMEM_COLS = 256;         // S0 [0, 64), S1 [64, 128), O [128, 192)

struct PattnArgs {
  const int* blocks;      // [nblocks][4]: q0, n, slot, pos0 (n = 0: nothing)
  int nq, nkv, group;
  int cache_len;
  long long layer_base;   // TMA row index of this layer's [cache row 0, head 0, key 0]
  float scale_log2;
  __nv_bfloat16* out;
  int out_stride;
  int rows;               // packed rows: a block row past them is not written
};

__global__ void __launch_bounds__(PATTN_THREADS, 1)
    k_pattn(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
            const __grid_constant__ CUtensorMap tmV, const PattnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sP = smem + PATTN_Q_BYTES;                                   // [2][P tile]
  uint8_t* sKV = sP + 2 * PATTN_P_BYTES;                                // [NST][K | V | V^T]
  uint64_t* q_full = reinterpret_cast<uint64_t*>(smem + PATTN_DATA);
  uint64_t* kv_full = q_full + 1;
  uint64_t* kv_empty = kv_full + PATTN_NST;
  uint64_t* vt_full = kv_empty + PATTN_NST;
  uint64_t* s_full = vt_full + PATTN_NST;
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_free + 2;
  uint64_t* p_free = p_full + 2;
  uint64_t* o_full = p_free + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_full + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int blk = blockIdx.x, kvh = blockIdx.y, pair = blockIdx.z;
  pdl_launch();
  pdl_wait();                                     // q and the K / V are the previous kernel's output
  const int q0 = a.blocks[4 * blk], n = a.blocks[4 * blk + 1], slot = a.blocks[4 * blk + 2],
            pos0 = a.blocks[4 * blk + 3];
  const int hA = kvh * a.group + 2 * pair;        // the tile's two query heads (hB may be past the group: zeros)
  if (n <= 0 || 2 * pair >= a.group) return;      // (uniform over the CTA, before any barrier)
  const int hB = 2 * pair + 1 < a.group ? hA + 1 : -1;
  const int nt = (pos0 + n + 63) / 64;            // key tiles; item i < nt: pass 1, i >= nt: pass 2
  const int items = 2 * nt;
  const long long krow = a.layer_base + ((long long)slot * a.nkv + kvh) * a.cache_len;

  if (tid == 0) {
    tma_prefetch(&tmQ);
    tma_prefetch(&tmK);
    tma_prefetch(&tmV);
    mbar_init(q_full, 1);
    for (int s = 0; s < PATTN_NST; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&vt_full[s], 2);                  // the two V^T warps
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_free[b], 4);                   // the four softmax warps
      mbar_init(&p_full[b], 4);
      mbar_init(&p_free[b], 1);
    }
    mbar_init(o_full, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, PATTN_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto stK = [&](int s) { return sKV + s * PATTN_STAGE; };
  auto stV = [&](int s) { return sKV + s * PATTN_STAGE + PATTN_TILE; };
  auto stVT = [&](int s) { return sKV + s * PATTN_STAGE + 2 * PATTN_TILE; };

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol = policy_evict_last();
      mbar_arrive_expect_tx(q_full, PATTN_Q_BYTES);
      tma_load_2d(sQ, &tmQ, q_full, hA * 64, q0, pol);
      // with no second head the box starts past the row's last column: the TMA fills it with zeros
      tma_load_2d(sQ + PATTN_TILE, &tmQ, q_full, (hB >= 0 ? hB : a.nq) * 64, q0, pol);
      int issued = 0;
      for (int i = 0; i < items; ++i) {
        const int s = i % PATTN_NST;
        if (i >= PATTN_NST && !mbar_wait(&kv_empty[s], ((i / PATTN_NST) - 1) & 1, ERR_TIMEOUT_EMPTY,
                                         KERNEL_ID_PATTN))
          break;
        const bool pass2 = i >= nt;
        const int j = pass2 ? i - nt : i;
        mbar_arrive_expect_tx(&kv_full[s], pass2 ? 2 * PATTN_TILE : PATTN_TILE);
        tma_load_2d(stK(s), &tmK, &kv_full[s], 0, int(krow + 64 * j), pol);
        if (pass2) tma_load_2d(stV(s), &tmV, &kv_full[s], 0, int(krow + 64 * j), pol);
        issued = i + 1;
      }
      // every requested stage has landed before the CTA can finish (bounded after an error)
      for (int i = max(0, issued - PATTN_NST); i < issued; ++i)
        mbar_wait(&kv_full[i % PATTN_NST], (i / PATTN_NST) & 1, ERR_TIMEOUT_FULL, KERNEL_ID_PATTN);
      mbar_wait(q_full, 0, ERR_TIMEOUT_FULL, KERNEL_ID_PATTN);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc(128, 64, 1);
      const uint32_t tO = tmem + 128;
      bool ok = mbar_wait(q_full, 0, ERR_TIMEOUT_FULL, KERNEL_ID_PATTN);
      const uint64_t dq = umma_desc_sw128(sQ);
      // O += P_j V_j^T for the pass-2 item i (key tile j = i - nt)
      auto pv = [&](int i) -> bool {
        const int s = i % PATTN_NST, j = i - nt, pb = j & 1;
        if (!mbar_wait(&p_full[pb], (j >> 1) & 1, ERR_TIMEOUT_FULL, KERNEL_ID_PATTN)) return false;
        if (!mbar_wait(&vt_full[s], (i / PATTN_NST) & 1, ERR_TIMEOUT_FULL, KERNEL_ID_PATTN)) return false;
        tc_fence_after();
        const uint64_t dp = umma_desc_sw128(sP + pb * PATTN_P_BYTES), dv = umma_desc_sw128(stVT(s));
#pragma unroll
        for (int k = 0; k < 4; ++k) umma_f16(tO, dp + 2 * k, dv + 2 * k, idesc, (j | k) != 0);
        umma_commit(&p_free[pb]);
        umma_commit(&kv_empty[s]);
        return true;
      };
      for (int i = 0; ok && i < items; ++i) {
        const int s = i % PATTN_NST, b = i & 1;
        ok = mbar_wait(&kv_full[s], (i / PATTN_NST) & 1, ERR_TIMEOUT_FULL, KERNEL_ID_PATTN);
        if (ok && i >= 2) ok = mbar_wait(&s_free[b], ((i >> 1) - 1) & 1, ERR_TIMEOUT_OTHER, KERNEL_ID_PATTN);
        if (!ok) break;
        tc_fence_after();
        const uint64_t dk = umma_desc_sw128(stK(s));
#pragma unroll
        for (int k = 0; k < 4; ++k) umma_f16(tmem + b * 64, dq + 2 * k, dk + 2 * k, idesc, k != 0);
        umma_commit(&s_full[b]);
        if (i < nt) {
          // pass 1 uses K only: the stage is free once S is; its V^T barrier still completes a phase (below)
          if (!(ok = mbar_wait(&vt_full[s], (i / PATTN_NST) & 1, ERR_TIMEOUT_FULL, KERNEL_ID_PATTN))) break;
          umma_commit(&kv_empty[s]);
        } else if (i > nt) {
          ok = pv(i - 1);                         // the previous tile's P V overlaps this tile's softmax
        }
      }
      if (ok) ok = pv(items - 1);
      umma_commit(o_full);
    }
  } else if (warp < 4) {
    // V^T: V tile row = key (128 bytes of hd, 128B-swizzled) -> V^T row = hd index (128 bytes of keys, swizzled)
    const int t = tid - 64;                       // 0 .. 63: the V^T row (hd index d) this thread writes
    for (int i = 0; i < items; ++i) {
      const int s = i % PATTN_NST;
      if (!mbar_wait(&kv_full[s], (i / PATTN_NST) & 1, ERR_TIMEOUT_FULL, KERNEL_ID_PATTN)) break;
      if (i >= nt) {
        const uint8_t* v = stV(s);
        uint8_t* vt = stVT(s);
        const int d = t, dc = d >> 3, dl = d & 7;
#pragma unroll
        for (int c = 0; c < 8; ++c) {             // keys 8c .. 8c+7
          uint32_t w[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int k0 = 8 * c + 2 * q;
            const uint16_t lo = *reinterpret_cast<const uint16_t*>(v + sw128(k0, dc) + 2 * dl);
            const uint16_t hi = *reinterpret_cast<const uint16_t*>(v + sw128(k0 + 1, dc) + 2 * dl);
            w[q] = uint32_t(lo) | (uint32_t(hi) << 16);
          }
          *reinterpret_cast<uint4*>(vt + sw128(d, c)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        fence_proxy_async_smem();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&vt_full[s]);
    }
  } else {
    // softmax: thread q = TMEM lane q = query vector q of the tile (head hA for q < 64, hB above), row q0 + (q % 64)
    const int q = tid - 128, r = q & 63;
    const int head = q < 64 ? hA : hB;
    const bool live = r < n && head >= 0 && q0 + r < a.rows;
    const int pos = pos0 + r;
    const uint32_t trow = tmem + (uint32_t((warp & 3) * 32) << 16);
    float mx = -INFINITY, l = 0.f;
    bool ok = true;
    for (int i = 0; i < items; ++i) {
      const int b = i & 1;
      const bool pass2 = i >= nt;
      const int j = pass2 ? i - nt : i;
      if (!(ok = mbar_wait(&s_full[b], (i >> 1) & 1, ERR_TIMEOUT_FULL, KERNEL_ID_PATTN))) break;
      tc_fence_after();
      float sv[64];
      tmem_ld32(trow + b * 64, sv);
      tmem_ld32(trow + b * 64 + 32, sv + 32);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[b]);
      const int kmax = pos - 64 * j;              // keys c <= kmax of this tile are causal for this row
      if (!pass2) {
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (c <= kmax) mx = fmaxf(mx, sv[c]);
        continue;
      }
      const int pb = j & 1;
      uint32_t pk[32];
#pragma unroll
      for (int c = 0; c < 64; c += 2) {
        const float p0 = (live && c <= kmax) ? exp2f((sv[c] - mx) * a.scale_log2) : 0.f;
        const float p1 = (live && c + 1 <= kmax) ? exp2f((sv[c + 1] - mx) * a.scale_log2) : 0.f;
        l += p0;
        l += p1;
        pk[c >> 1] = pack_bf16(p0, p1);
      }
      if (j >= 2 && !(ok = mbar_wait(&p_free[pb], ((j >> 1) - 1) & 1, ERR_TIMEOUT_OTHER, KERNEL_ID_PATTN))) break;
      uint8_t* prow = sP + pb * PATTN_P_BYTES;
#pragma unroll
      for (int c = 0; c < 8; ++c)                 // keys 8c .. 8c+7 of query vector q (128B swizzle)
        *reinterpret_cast<uint4*>(prow + sw128(q, c)) =
            make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[pb]);
    }
    if (ok) ok = mbar_wait(o_full, 0, ERR_TIMEOUT_ACCUM, KERNEL_ID_PATTN);
    tc_fence_after();
    float o[64];
    tmem_ld32(trow + 128, o);
    tmem_ld32(trow + 160, o + 32);
    if (ok && live) {
      const float inv = 1.0f / l;
      __nv_bfloat16* dst = a.out + (size_t)(q0 + r) * a.out_stride + head * 64;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(dst + 8 * c) =
            make_uint4(pack_bf16(o[8 * c] * inv, o[8 * c + 1] * inv), pack_bf16(o[8 * c + 2] * inv, o[8 * c + 3] * inv),
                       pack_bf16(o[8 * c + 4] * inv, o[8 * c + 5] * inv),
                       pack_bf16(o[8 * c + 6] * inv, o[8 * c + 7] * inv));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, PATTN_TMEM_COLS);
}

// Q map: bf16 [rows, q_stride] viewed as rows of nq * 64 columns, 64 x 64 boxes (128B swizzle).
int pattn_launch(const void* q, int q_stride, int rows, const CUtensorMap& mk, const CUtensorMap& mv,
                 const PattnArgs& a, int nblocks, cudaStream_t s) {
  CUtensorMap mq;
  int rc = encode_map_2d(&mq, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)a.nq * 64, (uint64_t)rows,
                         (uint64_t)q_stride * 2, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_pattn, cudaFuncAttributeMaxDynamicSharedMemorySize, PATTN_SMEM);
    attr = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nblocks, a.nkv, (a.group + 1) / 2);
  cfg.blockDim = dim3(PATTN_THREADS);
  cfg.dynamicSmemBytes = PATTN_SMEM;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  ++g_launches;
  return cudaLaunchKernelEx(&cfg, k_pattn, mq, mk, mv, a) == cudaSuccess ? A8_OK : A8_ERR_CUDA;
}

}  // namespace a8

using namespace a8;

extern "C" int a8_prefill_attention(const void* q, int q_stride, const void* kc, const void* vc, int layers,
                                    int cache_rows, int nq, int nkv, int hd, int cache_len, int layer,
                                    const int* blocks, int nblocks, int rows, float scale, void* out, int out_stride,
                                    a8_stream_t stream) {
  if (q == nullptr || kc == nullptr || vc == nullptr || blocks == nullptr || out == nullptr || rows <= 0 ||
      nblocks <= 0)
    return A8_ERR_ARG;
  if (hd != 64 || nkv <= 0 || nq % nkv != 0 || nq / nkv > 8 || layer < 0 || layer >= layers || q_stride < nq * hd ||
      out_stride < nq * hd)
    return A8_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(q) & 15) || (q_stride % 8) || (reinterpret_cast<uintptr_t>(out) & 15) ||
      (out_stride % 8))
    return A8_ERR_ALIGN;
  const long long total = (long long)layers * cache_rows * nkv * cache_len;
  if (total >= (1ll << 31)) return A8_ERR_SIZE;
  CUtensorMap mk, mv;
  int rc = attn_maps(&mk, &mv, kc, vc, total, hd);
  if (rc) return rc;
  PattnArgs a = {};
  a.blocks = blocks;
  a.nq = nq;
  a.nkv = nkv;
  a.group = nq / nkv;
  a.cache_len = cache_len;
  a.layer_base = (long long)layer * cache_rows * nkv * cache_len;
  a.scale_log2 = (scale > 0 ? scale : 1.0f / sqrtf((float)hd)) * 1.4426950408889634f;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.out_stride = out_stride;
  a.rows = rows;
  return pattn_launch(q, q_stride, rows, mk, mv, a, nblocks, reinterpret_cast<cudaStream_t>(stream));
}
