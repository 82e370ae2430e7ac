// Split-K GQA attention for one query token per row over a per-row number of cached keys.
//
// Serves every attention of the tick and of admission (serve/fast_kernels.py:193-358):
//   decode (slow AR, fast AR, codec ring): row r attends keys [0, lens[r]) of cache row rowmap[r] (or r)
//   packed causal prefill: row i attends [0, pos_i] of its request's cache row (lens = pos + 1, rowmap = slot),
//   the K/V of every packed token having been stored by the qkv GEMM epilogue beforehand.
//
// Grid (rows, kv heads, splits): block (r, h, s) takes keys [s*CHUNK, min(L, (s+1)*CHUNK)); blocks past the row's
// length exit at once, so the grid is fixed (graph-safe) while the work follows each row's length. K and V arrive by
// TMA in 64-key boxes (128-byte swizzle) on one mbarrier per box. Four warps take 16-key units round-robin: S = Q K^T
// and O += P V with mma.sync m16n8k16 (the GROUP query heads of the kv head padded to 16 rows), online softmax with
// quad shuffles, then the warps merge through shared memory. With several splits each block leaves (max, sum, acc)
// in the workspace and the last block of (r, h) (atomic ticket) merges them in split order.
#include "common.cuh"

namespace a8 {

constexpr int KERNEL_ID_ATTN = 2;

struct AttnArgs {
  const __nv_bfloat16* q;
  int q_stride;           // elements between query rows
  int nq, nkv;
  const int* lens;        // keys of row r: min(lens[r] + lens_add, lens_max)
  int lens_add, lens_max;
  const int* rowmap;      // may be null (cache row = query row)
  int cache_rows_per_layer_head;   // rows of the 2-D TMA view per (cache row, head): cache_len
  long long layer_base;   // TMA row index of this layer's [cache row 0, head 0, key 0]
  int max_splits;
  float scale_log2;       // softmax scale * log2(e)
  __nv_bfloat16* out;
  int out_stride;
  float* ws;              // [rows * nkv * max_splits][16][HD] accumulators, then [..][16][2] (max, sum)
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

template <int HD, int CHUNK>
struct AttnSmem {
  static constexpr int BOXES = HD / 64;            // 64-column boxes per 64-key block
  static constexpr int BLOCKS = CHUNK / 64;        // 64-key blocks per split
  static constexpr int BOX_BYTES = 64 * 128;
  static constexpr int KV_BYTES = BLOCKS * BOXES * BOX_BYTES;
  static constexpr int TOTAL = 2 * KV_BYTES + 1024 + 64 * BLOCKS;
};

template <int HD, int GROUP, int CHUNK>
__global__ void __launch_bounds__(128)
    k_attn(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV, const AttnArgs a) {
  using SM = AttnSmem<HD, CHUNK>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = smem + SM::KV_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 2 * SM::KV_BYTES);
  __shared__ int s_last;

  const int r = blockIdx.x, h = blockIdx.y, sp = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_launch();
  pdl_wait();
  const int L = min(a.lens[r] + a.lens_add, a.lens_max);
  const int nsplit = (L + CHUNK - 1) / CHUNK;
  if (sp >= nsplit || L <= 0) return;
  const int lo = sp * CHUNK;
  const int hi = min(L, lo + CHUNK);
  const int nkeys = hi - lo;
  const int nblk = (nkeys + 63) / 64;
  const int crow = a.rowmap != nullptr ? a.rowmap[r] : r;
  const long long base = a.layer_base + ((long long)crow * a.nkv + h) * a.cache_rows_per_layer_head + lo;

  if (tid == 0) {
    for (int b = 0; b < SM::BLOCKS; ++b) mbar_init(&bars[b], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    const uint64_t pol = policy_evict_first();
    for (int b = 0; b < nblk; ++b) {
      mbar_arrive_expect_tx(&bars[b], 2 * SM::BOXES * SM::BOX_BYTES);
      for (int x = 0; x < SM::BOXES; ++x) {
        tma_load_2d(sK + (b * SM::BOXES + x) * SM::BOX_BYTES, &tmK, &bars[b], x * 64, (int)(base + b * 64), pol);
        tma_load_2d(sV + (b * SM::BOXES + x) * SM::BOX_BYTES, &tmV, &bars[b], x * 64, (int)(base + b * 64), pol);
      }
    }
  }

  // Q fragments (rows = the GROUP query heads of kv head h, padded to 16 with zeros)
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

  float o[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;   // rows lane/4 and lane/4 + 8
  const int nunits = (nkeys + 15) / 16;
  int waited = -1;
  bool ok = true;
  const uint32_t sKa = smem_u32(sK), sVa = smem_u32(sV);

  for (int u = warp; u < nunits; u += 4) {
    const int blk = u >> 2;
    if (blk > waited) {
      for (int b = waited + 1; b <= blk; ++b)
        ok = ok && mbar_wait(&bars[b], 0, ERR_TIMEOUT_FULL, KERNEL_ID_ATTN);
      waited = blk;
    }
    if (!ok) break;
    const int krow0 = (u & 3) * 16;             // first key row of the unit inside its 64-key block
    // S = Q K^T for 16 keys (two n8 tiles)
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
      const int ch = 2 * kk + ((lane >> 3) & 1);          // 16-byte chunk of the head dim
      const int kr = krow0 + ((lane >> 4) << 3) + (lane & 7);
      const uint32_t addr = sKa + (blk * SM::BOXES + (ch >> 3)) * SM::BOX_BYTES + sw128(kr, ch & 7);
      uint32_t b0, b1, b2, b3;
      ldsm_x4(addr, b0, b1, b2, b3);
      mma_bf16(s[0], qa[kk], b0, b1);
      mma_bf16(s[1], qa[kk], b2, b3);
    }
    // online softmax over the unit (scale folded into log2 units)
    const int kbase = lo + blk * 64 + krow0;
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = kbase + t * 8 + 2 * (lane & 3) + e;
        const bool valid = key < hi;
        s[t][e] = valid ? s[t][e] * a.scale_log2 : -INFINITY;
        s[t][2 + e] = valid ? s[t][2 + e] * a.scale_log2 : -INFINITY;
        mx0 = fmaxf(mx0, s[t][e]);
        mx1 = fmaxf(mx1, s[t][2 + e]);
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
      p[t][0] = exp2f(s[t][0] - n0);
      p[t][1] = exp2f(s[t][1] - n0);
      p[t][2] = exp2f(s[t][2] - n1);
      p[t][3] = exp2f(s[t][3] - n1);
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
    // O += P V: V rows = keys, transposed fragments by ldmatrix.trans, two head-dim n8 tiles per load
#pragma unroll
    for (int nt = 0; nt < HD / 8; nt += 2) {
      const int ch = nt + (lane >> 4);
      const int kr = krow0 + (((lane >> 3) & 1) << 3) + (lane & 7);
      const uint32_t addr = sVa + (blk * SM::BOXES + (ch >> 3)) * SM::BOX_BYTES + sw128(kr, ch & 7);
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(addr, b0, b1, b2, b3);
      mma_bf16(o[nt], pa, b0, b1);
      mma_bf16(o[nt + 1], pa, b2, b3);
    }
  }
  l0 += __shfl_xor_sync(0xffffffff, l0, 1);
  l0 += __shfl_xor_sync(0xffffffff, l0, 2);
  l1 += __shfl_xor_sync(0xffffffff, l1, 1);
  l1 += __shfl_xor_sync(0xffffffff, l1, 2);

  // ---- merge the four warps through shared memory (the K/V tiles are no longer read) ----
  // every box this block requested has landed (immediate in normal operation; bounded after an error) before the
  // tiles' memory is reused
  for (int b = 0; b < nblk; ++b) mbar_wait(&bars[b], 0, ERR_TIMEOUT_FULL, KERNEL_ID_ATTN);
  __syncthreads();
  float* sO = reinterpret_cast<float*>(smem);                 // [4][16][HD]
  float* sML = sO + 4 * 16 * HD;                              // [4][16][2]
  {
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
  const int slot_id = (r * a.nkv + h);
  for (int idx = tid; idx < GROUP * HD; idx += 128) {
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
      float* acc = a.ws + ((size_t)slot_id * a.max_splits + sp) * 16 * HD;
      acc[g * HD + d] = num;
      if (d == 0) {
        float* ml = a.ws + (size_t)a.rows * a.nkv * a.max_splits * 16 * HD +
                    ((size_t)slot_id * a.max_splits + sp) * 32;
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
  const float* mlb = a.ws + (size_t)a.rows * a.nkv * a.max_splits * 16 * HD + (size_t)slot_id * a.max_splits * 32;
  for (int idx = tid; idx < GROUP * HD; idx += 128) {
    const int g = idx / HD, d = idx % HD;
    float M = -INFINITY;
    for (int s2 = 0; s2 < nsplit; ++s2) M = fmaxf(M, __ldcg(mlb + s2 * 32 + g * 2));
    float num = 0.f, den = 0.f;
    for (int s2 = 0; s2 < nsplit; ++s2) {
      const float f = exp2f(__ldcg(mlb + s2 * 32 + g * 2) - M);
      num += f * __ldcg(a.ws + ((size_t)slot_id * a.max_splits + s2) * 16 * HD + g * HD + d);
      den += f * __ldcg(mlb + s2 * 32 + g * 2 + 1);
    }
    a.out[(size_t)r * a.out_stride + (h * GROUP + g) * HD + d] = __float2bfloat16_rn(num / den);
  }
  if (tid == 0) a.counters[slot_id] = 0;
}

// ------------------------------------------------------------------------------------------------ host
template <int HD, int GROUP, int CHUNK>
static int launch_attn(const CUtensorMap& mk, const CUtensorMap& mv, const AttnArgs& a, cudaStream_t s) {
  using SM = AttnSmem<HD, CHUNK>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_attn<HD, GROUP, CHUNK>, cudaFuncAttributeMaxDynamicSharedMemorySize, SM::TOTAL);
    attr = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.rows, a.nkv, a.max_splits);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = SM::TOTAL;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  ++g_launches;
  return cudaLaunchKernelEx(&cfg, k_attn<HD, GROUP, CHUNK>, mk, mv, a) == cudaSuccess ? A8_OK : A8_ERR_CUDA;
}

int attn_chunk(int hd) { return hd == 64 ? 256 : 128; }

// kc / vc: bf16 [layers * cache_rows, nkv, cache_len, hd] viewed as rows of hd
int attn_maps(CUtensorMap* mk, CUtensorMap* mv, const void* kc, const void* vc, long long total_rows, int hd) {
  int rc = encode_map_2d(mk, kc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, hd, total_rows, (uint64_t)hd * 2, 64, 64,
                         CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  return encode_map_2d(mv, vc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, hd, total_rows, (uint64_t)hd * 2, 64, 64,
                       CU_TENSOR_MAP_SWIZZLE_128B);
}

long long attn_ws_floats(int rows, int nkv, int max_splits, int hd) {
  return (long long)rows * nkv * max_splits * (16 * hd + 32);
}

int attn_launch(const CUtensorMap& mk, const CUtensorMap& mv, AttnArgs a, int hd, int group, cudaStream_t s) {
  if (hd == 64 && group == 7) return launch_attn<64, 7, 256>(mk, mv, a, s);
  if (hd == 64 && group == 1) return launch_attn<64, 1, 256>(mk, mv, a, s);
  if (hd == 128 && group == 1) return launch_attn<128, 1, 128>(mk, mv, a, s);
  if (hd == 128 && group == 7) return launch_attn<128, 7, 128>(mk, mv, a, s);
  return A8_ERR_ARG;
}

}  // namespace a8

using namespace a8;

extern "C" int a8_attention_workspace(int rows, int nkv, int hd, int max_len, long long* ws_floats,
                                      int* n_counters) {
  if (rows <= 0 || nkv <= 0 || (hd != 64 && hd != 128) || max_len <= 0) return A8_ERR_ARG;
  const int ms = (max_len + attn_chunk(hd) - 1) / attn_chunk(hd);
  if (ws_floats) *ws_floats = ms > 1 ? attn_ws_floats(rows, nkv, ms, hd) : 0;
  if (n_counters) *n_counters = ms > 1 ? rows * nkv : 0;
  return A8_OK;
}

extern "C" int a8_attention(const void* q, int q_stride, const void* kc, const void* vc, int layers, int cache_rows,
                            int nq, int nkv, int hd, int cache_len, int layer, const int* lens, const int* rowmap,
                            int rows, int max_len, float scale, void* out, int out_stride, float* ws,
                            long long ws_floats, int* counters, int n_counters, a8_stream_t stream) {
  if (q == nullptr || kc == nullptr || vc == nullptr || lens == nullptr || out == nullptr || rows <= 0) return A8_ERR_ARG;
  if (nkv <= 0 || nq % nkv != 0 || layer < 0 || layer >= layers || max_len <= 0 || max_len > cache_len)
    return A8_ERR_ARG;
  const int group = nq / nkv;
  const int chunk = attn_chunk(hd);
  const int ms = (max_len + chunk - 1) / chunk;
  if ((q_stride % 2) || (reinterpret_cast<uintptr_t>(q) & 3)) return A8_ERR_ALIGN;
  if (ms > 1) {
    if (ws == nullptr || counters == nullptr || ws_floats < attn_ws_floats(rows, nkv, ms, hd) ||
        n_counters < rows * nkv)
      return A8_ERR_SIZE;
  }
  CUtensorMap mk, mv;
  const long long total = (long long)layers * cache_rows * nkv * cache_len;
  if (total >= (1ll << 31)) return A8_ERR_SIZE;
  int rc = attn_maps(&mk, &mv, kc, vc, total, hd);
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
  a.max_splits = ms;
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
// address comes from cudaGetSymbolAddress, taken once per device with that device current, on the first call.
namespace a8 {
static __device__ __align__(256) float g_attn_noalloc[A8_ATTENTION_NOALLOC_FLOATS];
static float* g_attn_noalloc_dev[64];   // device address of g_attn_noalloc, per device ordinal
}  // namespace a8

extern "C" int a8_attention_noalloc(const void* q, int q_stride, const void* kc, const void* vc, int layers,
                                    int cache_rows, int nq, int nkv, int hd, int cache_len, int layer, const int* lens,
                                    const int* rowmap, int rows, int max_len, float scale, void* out, int out_stride,
                                    a8_stream_t stream) {
  if (rows <= 0 || nkv <= 0 || (hd != 64 && hd != 128) || max_len <= 0) return A8_ERR_ARG;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return A8_ERR_DEVICE;
  if (g_attn_noalloc_dev[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_attn_noalloc) != cudaSuccess || p == nullptr) return A8_ERR_CUDA;
    g_attn_noalloc_dev[dev] = reinterpret_cast<float*>(p);
  }
  const int chunk = attn_chunk(hd);
  const int ms = (max_len + chunk - 1) / chunk;
  const long long partials = ms > 1 ? attn_ws_floats(rows, nkv, ms, hd) : 0;
  const long long tickets = ms > 1 ? (long long)rows * nkv : 0;
  if (partials + tickets > A8_ATTENTION_NOALLOC_FLOATS) return A8_ERR_SIZE;
  float* ws = g_attn_noalloc_dev[dev];
  int* counters = reinterpret_cast<int*>(ws + partials);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // the tickets must start at zero: the array keeps whatever the previous call left
  if (tickets > 0 && cudaMemsetAsync(counters, 0, tickets * sizeof(int), s) != cudaSuccess) return A8_ERR_CUDA;
  return a8_attention(q, q_stride, kc, vc, layers, cache_rows, nq, nkv, hd, cache_len, layer, lens, rowmap, rows,
                      max_len, scale, out, out_stride, ms > 1 ? ws : nullptr, partials, ms > 1 ? counters : nullptr,
                      (int)tickets, stream);
}
