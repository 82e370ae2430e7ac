// Split-K GQA attention for one query token per row over a per-row number of cached keys.
//
// Serves every attention of the tick and of admission (serve/fast_kernels.py:193-358):
//   decode (slow AR, fast AR, codec ring): row r attends keys [0, lens[r]) of cache row rowmap[r] (or r)
//   packed causal prefill: row i attends [0, pos_i] of its request's cache row (lens = pos + 1, rowmap = slot),
//   the K/V of every packed token having been stored by the qkv GEMM epilogue beforehand.
//
// Grid (rows, kv heads, S): block (r, h, s) takes the s-th of S equal 64-key-aligned parts of row r's keys (the
// reference's per-row split, serve/fast_kernels.py:207-209); S is chosen per call so that rows x heads x S fills the
// 148 SMs twice over (1 when the rows alone do). Inside a block a producer warp streams the part's 64-key K / V tiles
// by TMA (128-byte swizzle) through a ring of NST stages (full / empty mbarriers); four compute warps each take 16 keys
// of every tile: S = Q K^T and O += P V with mma.sync m16n8k16 (the GROUP query heads of the kv head padded to 16
// rows), online softmax with quad shuffles. The warps merge through shared memory; with S > 1 every block leaves
// (max, sum, acc) in the workspace and the last block of (r, h) (atomic ticket) merges them in split order.
#include <algorithm>

#include <atomic>

#include "common.cuh"

namespace a8 {

constexpr int KERNEL_ID_ATTN = 2;
constexpr int ATTN_MAX_SPLITS = 16;

struct AttnArgs {
  const __nv_bfloat16* q;
  int q_stride;           // elements between query rows
  int nq, nkv;
  const int* lens;        // keys of row r: min(lens[r] + lens_add, lens_max)
  int lens_add, lens_max;
  const int* rowmap;      // may be null (cache row = query row)
  int cache_rows_per_layer_head;   // rows of the 2-D TMA view per (cache row, head): cache_len
  long long layer_base;   // TMA row index of this layer's [cache row 0, head 0, key 0]
  int nsplit;             // S
  float scale_log2;       // softmax scale * log2(e)
  __nv_bfloat16* out;
  int out_stride;
  float* ws;              // [rows * nkv * S][16][HD] accumulators, then [..][16][2] (max, sum)
  int* counters;          // [rows * nkv]
  int rows;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Byte offset of (key row, 16-byte chunk c) inside a TMA tile of 64 rows x 128 bytes with the 128-byte swizzle.
__device__ __forceinline__ uint32_t sw128(int row, int c) { return row * 128 + ((c ^ (row & 7)) << 4); }

template <int HD, int NST>
struct AttnSmem {
  static constexpr int BOXES = HD / 64;            // 64-column boxes per 64-key tile
  static constexpr int BOX_BYTES = 64 * 128;
  static constexpr int STAGE_BYTES = 2 * BOXES * BOX_BYTES;   // K then V
  static constexpr int MERGE_BYTES = 4 * 16 * HD * 4 + 4 * 16 * 2 * 4;
  static constexpr int DATA_BYTES = NST * STAGE_BYTES > MERGE_BYTES ? NST * STAGE_BYTES : MERGE_BYTES;
  static constexpr int TOTAL = DATA_BYTES + 1024 + 2 * NST * 8;
};

template <int HD, int GROUP, int NST>
__global__ void __launch_bounds__(160)
    k_attn(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV, const AttnArgs a) {
  using SM = AttnSmem<HD, NST>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + SM::DATA_BYTES);
  uint64_t* empty = full + NST;
  __shared__ int s_last;

  const int r = blockIdx.x, h = blockIdx.y, sp = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_launch();
  pdl_wait();
  const int L = min(a.lens[r] + a.lens_add, a.lens_max);
  if (L <= 0) return;
  const int per = ((L + a.nsplit - 1) / a.nsplit + 63) / 64 * 64;   // keys of one split, 64-aligned
  const int nsplit = (L + per - 1) / per;                            // splits that hold keys
  if (sp >= nsplit) return;
  const int lo = sp * per;
  const int hi = min(L, lo + per);
  const int nblk = (hi - lo + 63) / 64;
  const int crow = a.rowmap != nullptr ? a.rowmap[r] : r;
  const long long base = a.layer_base + ((long long)crow * a.nkv + h) * a.cache_rows_per_layer_head + lo;

  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);                 // the four compute warps release a stage
    }
    fence_mbar_init();
  }
  __syncthreads();

  float o[HD / 8][4];
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;   // rows lane/4 and lane/4 + 8

  if (warp == 4) {
    // ---- producer: the part's 64-key tiles through the ring ----
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int issued = 0;
      for (int b = 0; b < nblk; ++b) {
        const int s = b % NST;
        if (b >= NST && !mbar_wait(&empty[s], ((b / NST) - 1) & 1, ERR_TIMEOUT_EMPTY, KERNEL_ID_ATTN)) break;
        uint8_t* st = smem + s * SM::STAGE_BYTES;
        mbar_arrive_expect_tx(&full[s], SM::STAGE_BYTES);
#pragma unroll
        for (int x = 0; x < SM::BOXES; ++x) {
          tma_load_2d(st + x * SM::BOX_BYTES, &tmK, &full[s], x * 64, (int)(base + b * 64), pol);
          tma_load_2d(st + (SM::BOXES + x) * SM::BOX_BYTES, &tmV, &full[s], x * 64, (int)(base + b * 64), pol);
        }
        issued = b + 1;
      }
      // every requested tile has landed before the stages are reused for the merge (bounded after an error)
      for (int b = max(0, issued - NST); b < issued; ++b)
        mbar_wait(&full[b % NST], (b / NST) & 1, ERR_TIMEOUT_FULL, KERNEL_ID_ATTN);
    }
  } else {
    // ---- compute warps: Q fragments (the GROUP query heads of kv head h, padded to 16 rows with zeros) ----
    constexpr int KS = HD / 16;
    uint32_t qa[KS][4];
    {
      const int g0 = lane >> 2, g1 = g0 + 8, c = 2 * (lane & 3);
      const __nv_bfloat16* qr = a.q + (size_t)r * a.q_stride + (size_t)h * GROUP * HD;
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        const int d = kk * 16 + c;
        qa[kk][0] = g0 < GROUP ? *reinterpret_cast<const uint32_t*>(qr + g0 * HD + d) : 0u;
        qa[kk][1] = g1 < GROUP ? *reinterpret_cast<const uint32_t*>(qr + g1 * HD + d) : 0u;
        qa[kk][2] = g0 < GROUP ? *reinterpret_cast<const uint32_t*>(qr + g0 * HD + d + 8) : 0u;
        qa[kk][3] = g1 < GROUP ? *reinterpret_cast<const uint32_t*>(qr + g1 * HD + d + 8) : 0u;
      }
    }
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    const int krow0 = warp * 16;                 // this warp's 16 keys of every 64-key tile
    for (int b = 0; b < nblk; ++b) {
      const int s = b % NST;
      if (!mbar_wait(&full[s], (b / NST) & 1, ERR_TIMEOUT_FULL, KERNEL_ID_ATTN)) break;
      const int kbase = lo + b * 64 + krow0;
      if (kbase < hi) {
        const uint32_t sK = smem_u32(smem + s * SM::STAGE_BYTES);
        const uint32_t sV = sK + SM::BOXES * SM::BOX_BYTES;
        float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
          const int ch = 2 * kk + ((lane >> 3) & 1);          // 16-byte chunk of the head dim
          const int kr = krow0 + ((lane >> 4) << 3) + (lane & 7);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(sK + (ch >> 3) * SM::BOX_BYTES + sw128(kr, ch & 7), b0, b1, b2, b3);
          mma_bf16(sc[0], qa[kk], b0, b1);
          mma_bf16(sc[1], qa[kk], b2, b3);
        }
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const bool valid = kbase + t * 8 + 2 * (lane & 3) + e < hi;
            sc[t][e] = valid ? sc[t][e] * a.scale_log2 : -INFINITY;
            sc[t][2 + e] = valid ? sc[t][2 + e] * a.scale_log2 : -INFINITY;
            mx0 = fmaxf(mx0, sc[t][e]);
            mx1 = fmaxf(mx1, sc[t][2 + e]);
          }
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffff, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffff, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffff, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffff, mx1, 2));
        const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
        const float al0 = exp2f(m0 - n0), al1 = exp2f(m1 - n1);
        m0 = n0;
        m1 = n1;
        float p[2][4];
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          p[t][0] = exp2f(sc[t][0] - n0);
          p[t][1] = exp2f(sc[t][1] - n0);
          p[t][2] = exp2f(sc[t][2] - n1);
          p[t][3] = exp2f(sc[t][3] - n1);
        }
        l0 = l0 * al0 + p[0][0] + p[0][1] + p[1][0] + p[1][1];
        l1 = l1 * al1 + p[0][2] + p[0][3] + p[1][2] + p[1][3];
#pragma unroll
        for (int i = 0; i < HD / 8; ++i) {
          o[i][0] *= al0;
          o[i][1] *= al0;
          o[i][2] *= al1;
          o[i][3] *= al1;
        }
        uint32_t pa[4] = {pack_bf16(p[0][0], p[0][1]), pack_bf16(p[0][2], p[0][3]), pack_bf16(p[1][0], p[1][1]),
                          pack_bf16(p[1][2], p[1][3])};
#pragma unroll
        for (int nt = 0; nt < HD / 8; nt += 2) {
          const int ch = nt + (lane >> 4);
          const int kr = krow0 + (((lane >> 3) & 1) << 3) + (lane & 7);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(sV + (ch >> 3) * SM::BOX_BYTES + sw128(kr, ch & 7), b0, b1, b2, b3);
          mma_bf16(o[nt], pa, b0, b1);
          mma_bf16(o[nt + 1], pa, b2, b3);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    l0 += __shfl_xor_sync(0xffffffff, l0, 1);
    l0 += __shfl_xor_sync(0xffffffff, l0, 2);
    l1 += __shfl_xor_sync(0xffffffff, l1, 1);
    l1 += __shfl_xor_sync(0xffffffff, l1, 2);
  }

  // ---- merge the four compute warps through shared memory (the producer drained every tile) ----
  __syncthreads();
  float* sO = reinterpret_cast<float*>(smem);                 // [4][16][HD]
  float* sML = sO + 4 * 16 * HD;                              // [4][16][2]
  if (warp < 4) {
    const int g0 = lane >> 2, c = 2 * (lane & 3);
    float* ow = sO + warp * 16 * HD;
#pragma unroll
    for (int nt = 0; nt < HD / 8; ++nt) {
      ow[g0 * HD + nt * 8 + c] = o[nt][0];
      ow[g0 * HD + nt * 8 + c + 1] = o[nt][1];
      ow[(g0 + 8) * HD + nt * 8 + c] = o[nt][2];
      ow[(g0 + 8) * HD + nt * 8 + c + 1] = o[nt][3];
    }
    if ((lane & 3) == 0) {
      sML[(warp * 16 + g0) * 2] = m0;
      sML[(warp * 16 + g0) * 2 + 1] = l0;
      sML[(warp * 16 + g0 + 8) * 2] = m1;
      sML[(warp * 16 + g0 + 8) * 2 + 1] = l1;
    }
  }
  __syncthreads();
  const int slot_id = r * a.nkv + h;
  for (int idx = tid; idx < GROUP * HD; idx += blockDim.x) {
    const int g = idx / HD, d = idx % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, sML[(w * 16 + g) * 2]);
    float num = 0.f, den = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float mw = sML[(w * 16 + g) * 2];
      const float f = mw == -INFINITY ? 0.f : exp2f(mw - M);
      num += f * sO[(w * 16 + g) * HD + d];
      den += f * sML[(w * 16 + g) * 2 + 1];
    }
    if (nsplit == 1) {
      a.out[(size_t)r * a.out_stride + (h * GROUP + g) * HD + d] = __float2bfloat16_rn(num / den);
    } else {
      float* acc = a.ws + ((size_t)slot_id * a.nsplit + sp) * 16 * HD;
      acc[g * HD + d] = num;
      if (d == 0) {
        float* ml = a.ws + (size_t)a.rows * a.nkv * a.nsplit * 16 * HD + ((size_t)slot_id * a.nsplit + sp) * 32;
        ml[g * 2] = M;
        ml[g * 2 + 1] = den;
      }
    }
  }
  if (nsplit == 1) return;
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(&a.counters[slot_id], 1) == nsplit - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const float* mlb = a.ws + (size_t)a.rows * a.nkv * a.nsplit * 16 * HD + (size_t)slot_id * a.nsplit * 32;
  for (int idx = tid; idx < GROUP * HD; idx += blockDim.x) {
    const int g = idx / HD, d = idx % HD;
    float mv[ATTN_MAX_SPLITS], lv[ATTN_MAX_SPLITS], av[ATTN_MAX_SPLITS];
    float M = -INFINITY;
#pragma unroll
    for (int s2 = 0; s2 < ATTN_MAX_SPLITS; ++s2) {
      if (s2 < nsplit) {
        mv[s2] = __ldcg(mlb + s2 * 32 + g * 2);
        lv[s2] = __ldcg(mlb + s2 * 32 + g * 2 + 1);
        av[s2] = __ldcg(a.ws + ((size_t)slot_id * a.nsplit + s2) * 16 * HD + g * HD + d);
        M = fmaxf(M, mv[s2]);
      }
    }
    float num = 0.f, den = 0.f;
#pragma unroll
    for (int s2 = 0; s2 < ATTN_MAX_SPLITS; ++s2) {
      if (s2 < nsplit) {
        const float f = exp2f(mv[s2] - M);
        num += f * av[s2];
        den += f * lv[s2];
      }
    }
    a.out[(size_t)r * a.out_stride + (h * GROUP + g) * HD + d] = __float2bfloat16_rn(num / den);
  }
  if (tid == 0) a.counters[slot_id] = 0;
}

// ------------------------------------------------------------------------------------------------ host
template <int HD, int GROUP, int NST>
static int launch_attn(const CUtensorMap& mk, const CUtensorMap& mv, const AttnArgs& a, cudaStream_t s) {
  using SM = AttnSmem<HD, NST>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_attn<HD, GROUP, NST>, cudaFuncAttributeMaxDynamicSharedMemorySize, SM::TOTAL);
    attr = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.rows, a.nkv, a.nsplit);
  cfg.blockDim = dim3(160);
  cfg.dynamicSmemBytes = SM::TOTAL;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  ++g_launches;
  return cudaLaunchKernelEx(&cfg, k_attn<HD, GROUP, NST>, mk, mv, a) == cudaSuccess ? A8_OK : A8_ERR_CUDA;
}

// Splits of each row: enough (row, head, split) blocks to fill the 148 SMs twice, at least 64 keys a split.
int attn_splits(int rows, int nkv, int max_len) {
  const int want = (2 * 148 + rows * nkv - 1) / (rows * nkv);
  const int cap = (max_len + 63) / 64;
  return std::max(1, std::min(std::min(want, cap), ATTN_MAX_SPLITS));
}

// kc / vc: bf16 [layers * cache_rows, nkv, cache_len, hd] viewed as rows of hd
int attn_maps(CUtensorMap* mk, CUtensorMap* mv, const void* kc, const void* vc, long long total_rows, int hd) {
  int rc = encode_map_2d(mk, kc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, hd, total_rows, (uint64_t)hd * 2, 64, 64,
                         CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  return encode_map_2d(mv, vc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, hd, total_rows, (uint64_t)hd * 2, 64, 64,
                       CU_TENSOR_MAP_SWIZZLE_128B);
}

long long attn_ws_floats(int rows, int nkv, int nsplit, int hd) {
  return (long long)rows * nkv * nsplit * (16 * hd + 32);
}

int attn_launch(const CUtensorMap& mk, const CUtensorMap& mv, AttnArgs a, int hd, int group, cudaStream_t s) {
  if (hd == 64 && group == 7) return launch_attn<64, 7, 4>(mk, mv, a, s);
  if (hd == 64 && group == 1) return launch_attn<64, 1, 4>(mk, mv, a, s);
  if (hd == 128 && group == 1) return launch_attn<128, 1, 2>(mk, mv, a, s);
  if (hd == 128 && group == 7) return launch_attn<128, 7, 2>(mk, mv, a, s);
  return A8_ERR_ARG;
}

}  // namespace a8

using namespace a8;

extern "C" int a8_attention_workspace(int rows, int nkv, int hd, int max_len, long long* ws_floats,
                                      int* n_counters) {
  if (rows <= 0 || nkv <= 0 || (hd != 64 && hd != 128) || max_len <= 0) return A8_ERR_ARG;
  // the split count grows as the rows shrink: size for the largest need over every call of up to `rows` rows
  long long need = 0;
  int tickets = 0;
  for (int r = 1; r <= rows; ++r) {
    const int S = attn_splits(r, nkv, max_len);
    if (S > 1) {
      need = std::max(need, attn_ws_floats(r, nkv, S, hd));
      tickets = r * nkv;
    }
  }
  if (ws_floats) *ws_floats = need;
  if (n_counters) *n_counters = tickets;
  return A8_OK;
}

// a8_attention's argument checks, shared with a8_attention_noalloc (which runs them before it touches its array).
static int attn_check(const void* q, int q_stride, const void* kc, const void* vc, int layers, int cache_rows,
                      int nq, int nkv, int hd, int cache_len, int layer, const int* lens, int rows, int max_len,
                      const void* out) {
  if (q == nullptr || kc == nullptr || vc == nullptr || lens == nullptr || out == nullptr || rows <= 0) return A8_ERR_ARG;
  if (nkv <= 0 || nq % nkv != 0 || layer < 0 || layer >= layers || max_len <= 0 || max_len > cache_len)
    return A8_ERR_ARG;
  if (hd != 64 && hd != 128) return A8_ERR_ARG;
  const int group = nq / nkv;
  if (!((hd == 64 && (group == 7 || group == 1)) || (hd == 128 && (group == 7 || group == 1)))) return A8_ERR_ARG;
  if ((q_stride % 2) || (reinterpret_cast<uintptr_t>(q) & 3)) return A8_ERR_ALIGN;
  if ((long long)layers * cache_rows * nkv * cache_len >= (1ll << 31)) return A8_ERR_SIZE;
  if ((reinterpret_cast<uintptr_t>(kc) & 15) || (reinterpret_cast<uintptr_t>(vc) & 15)) return A8_ERR_ALIGN;
  return A8_OK;
}

extern "C" int a8_attention(const void* q, int q_stride, const void* kc, const void* vc, int layers, int cache_rows,
                            int nq, int nkv, int hd, int cache_len, int layer, const int* lens, const int* rowmap,
                            int rows, int max_len, float scale, void* out, int out_stride, float* ws,
                            long long ws_floats, int* counters, int n_counters, a8_stream_t stream) {
  int rc = attn_check(q, q_stride, kc, vc, layers, cache_rows, nq, nkv, hd, cache_len, layer, lens, rows, max_len,
                      out);
  if (rc) return rc;
  const int group = nq / nkv;
  const int S = attn_splits(rows, nkv, max_len);
  if (S > 1) {
    if (ws == nullptr || counters == nullptr || ws_floats < attn_ws_floats(rows, nkv, S, hd) ||
        n_counters < rows * nkv)
      return A8_ERR_SIZE;
  }
  CUtensorMap mk, mv;
  const long long total = (long long)layers * cache_rows * nkv * cache_len;
  rc = attn_maps(&mk, &mv, kc, vc, total, hd);
  if (rc) return rc;
  AttnArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q);
  a.q_stride = q_stride;
  a.nq = nq;
  a.nkv = nkv;
  a.lens = lens;
  a.lens_add = 0;
  a.lens_max = max_len;
  a.rowmap = rowmap;
  a.cache_rows_per_layer_head = cache_len;
  a.layer_base = (long long)layer * cache_rows * nkv * cache_len;
  a.nsplit = S;
  a.scale_log2 = (scale > 0 ? scale : 1.0f / sqrtf((float)hd)) * 1.4426950408889634f;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.out_stride = out_stride;
  a.ws = ws;
  a.counters = counters;
  a.rows = rows;
  return attn_launch(mk, mv, a, hd, group, reinterpret_cast<cudaStream_t>(stream));
}

// ------------------------------------------------------------------------------------------------ allocation-free
// a8_attention for callers that cannot allocate device memory: the split workspace (partials and tickets) lives in
// a fixed array of this library instead of caller memory. The array is a host-side stand-in in host code; its device
// address comes from cudaGetSymbolAddress, taken once per device with that device current, on the first call there.
// The array is sized for the largest need of any valid call (A8_ATTENTION_NOALLOC_FLOATS in the header).
namespace a8 {
static __device__ __align__(256) float g_attn_noalloc[A8_ATTENTION_NOALLOC_FLOATS];
// Device address of g_attn_noalloc per device ordinal. Threads that race on a first call store the same value; the
// address belongs to the device's primary context and is stale after cudaDeviceReset (not re-queried).
static std::atomic<float*> g_attn_noalloc_dev[64];
}  // namespace a8

extern "C" int a8_attention_noalloc(const void* q, int q_stride, const void* kc, const void* vc, int layers,
                                    int cache_rows, int nq, int nkv, int hd, int cache_len, int layer, const int* lens,
                                    const int* rowmap, int rows, int max_len, float scale, void* out, int out_stride,
                                    a8_stream_t stream) {
  // every check runs before the shared array is touched: a rejected call leaves another call's tickets alone
  int rc = attn_check(q, q_stride, kc, vc, layers, cache_rows, nq, nkv, hd, cache_len, layer, lens, rows, max_len,
                      out);
  if (rc) return rc;
  const int S = attn_splits(rows, nkv, max_len);
  const long long partials = S > 1 ? attn_ws_floats(rows, nkv, S, hd) : 0;
  const long long tickets = S > 1 ? (long long)rows * nkv : 0;
  if (partials + tickets > A8_ATTENTION_NOALLOC_FLOATS) return A8_ERR_SIZE;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return A8_ERR_DEVICE;
  float* ws = g_attn_noalloc_dev[dev].load(std::memory_order_relaxed);
  if (ws == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_attn_noalloc) != cudaSuccess || p == nullptr) return A8_ERR_CUDA;
    ws = reinterpret_cast<float*>(p);
    g_attn_noalloc_dev[dev].store(ws, std::memory_order_relaxed);
  }
  int* counters = reinterpret_cast<int*>(ws + partials);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // the tickets must start at zero: the array keeps whatever the previous call left
  if (tickets > 0 && cudaMemsetAsync(counters, 0, tickets * sizeof(int), s) != cudaSuccess) return A8_ERR_CUDA;
  return a8_attention(q, q_stride, kc, vc, layers, cache_rows, nq, nkv, hd, cache_len, layer, lens, rowmap, rows,
                      max_len, scale, out, out_stride, S > 1 ? ws : nullptr, partials, S > 1 ? counters : nullptr,
                      (int)tickets, stream);
}
