// Per-row sampling with the engine's state updates fused in (serve/fast_engine.py:141-172, :719-769, :820-835).
//
// One block of 512 threads per row. The draw follows the checkpoint's sampler step for step:
//   top-k of the logits (ties: lower index first), each candidate's cumulative probability under the UNTEMPERED
//   softmax of ALL logits, drop candidates whose cumulative probability passes top_p (the best always stays),
//   softmax(v / temperature), exponential race argmax(p_i / E_i), E_i ~ Exp(1).
// E_i = -log(u_i) with u_i from Philox4x32-10 keyed by the engine seed and counted by (i / 4, row, tick, stream),
// word i % 4, u = ((w >> 8) + 0.5) * 2^-24 -- so a CPU restatement reproduces every draw bit for bit.
// Top-k: a radix select (8 bits a pass; two passes when every logit is a bf16 value, else four) on order-preserving
// keys finds the k-th largest value; the candidates are compacted in index order and sorted by a bitonic network on
// (value desc, index asc) -- by one warp for up to 64 of them -- and for k <= 64 each race is one warp's.
#include "common.cuh"

namespace a8 {

constexpr int SAMPLE_THREADS = 512;
constexpr int KERNEL_ID_SAMPLE = 3;

enum SampleMode { SM_CODEBOOK = 0, SM_SEMANTIC = 1, SM_PREFILL = 2, SM_PLAIN = 3 };

struct SampleArgs {
  const float* logits;
  int ld, V;
  int mode;
  int do_sample, k;
  float p, t;            // regular draw
  float p2, t2;          // RAS redraw (semantic mode, do_sample)
  unsigned long long seed;
  const long long* tick_id;
  int stream1, stream2;
  // codebook mode: codes[row, cb_index] = draw; x_next[row] = fast_emb[draw]
  int64_t* codes;
  int ncb, cb_index;
  const __nv_bfloat16* fast_emb;
  __nv_bfloat16* x_next;
  int ldx;
  int H;
  // semantic / prefill mode
  const int64_t* tok_in;
  int64_t* tok;
  int64_t* prev;
  int ras_w;
  int* nstep;
  int* cpos;
  int S;
  const __nv_bfloat16* h_src;
  int ldh;
  __nv_bfloat16* hid;
  int64_t* frame_prev;
  const int64_t* sil_frame;
  long long eos, sb;
  int nsem;
  const int* st;         // prefill: slot of each row
  const int* cpos_new;   // prefill: position after the prompt
  const int* frame0;     // prefill: int32 [rows, ncb] the codec frame each slot decodes first (or null)
  int B;                 // prefill: slots; a row aimed at slot >= B (a graph's padding) writes nothing
  int64_t* out_tok;      // plain mode: the drawn index
};

// ------------------------------------------------------------------------------------------------ Philox4x32-10
__device__ __forceinline__ void philox(uint32_t c[4], uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(0xD2511F53u, c[0]), lo0 = 0xD2511F53u * c[0];
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c[2]), lo1 = 0xCD9E8D57u * c[2];
    const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0;
    c[1] = lo1;
    c[2] = n2;
    c[3] = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}
__device__ __forceinline__ float exp_noise(unsigned long long seed, int stream, long long tick, int row, int i) {
  uint32_t c[4] = {uint32_t(i >> 2), uint32_t(row), uint32_t(tick), uint32_t(stream)};
  philox(c, uint32_t(seed), uint32_t(seed >> 32));
  const uint32_t w = c[i & 3];
  const float u = ((float)(w >> 8) + 0.5f) * 5.9604644775390625e-08f;
  return -logf(u);
}

// ------------------------------------------------------------------------------------------------ block helpers
__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffff, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  v = l < (SAMPLE_THREADS / 32) ? red[l] : -INFINITY;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffff, v, o));
  return v;
}
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  v = l < (SAMPLE_THREADS / 32) ? red[l] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  return v;
}
// (value, index) argmax, first index on ties
__device__ __forceinline__ void block_argmax(float& v, int& i, float* redv, int* redi) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffff, v, o);
    const int oi = __shfl_xor_sync(0xffffffff, i, o);
    if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) { redv[w] = v; redi[w] = i; }
  __syncthreads();
  v = l < (SAMPLE_THREADS / 32) ? redv[l] : -INFINITY;
  i = l < (SAMPLE_THREADS / 32) ? redi[l] : 0x7FFFFFFF;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffff, v, o);
    const int oi = __shfl_xor_sync(0xffffffff, i, o);
    if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
  }
}
// exclusive scan of per-thread counts; returns the thread's offset, *total = sum
__device__ __forceinline__ int block_excl_scan(int v, int* red, int* total) {
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffff, x, o);
    if (l >= o) x += y;
  }
  __syncthreads();
  if (l == 31) red[w] = x;
  __syncthreads();
  int pre = 0, tot = 0;
  for (int j = 0; j < SAMPLE_THREADS / 32; ++j) {
    if (j < w) pre += red[j];
    tot += red[j];
  }
  *total = tot;
  return pre + x - v;
}

__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float unkey(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// One exponential-race draw over the sorted candidates (s_v, s_cum): returns the winning position.
__device__ int race(const float* s_v, const float* s_cum, int k, float p, float t, unsigned long long seed, int stream,
                    long long tick, int row, float* red, int* redi) {
  const float z0 = s_v[0] / t;
  float part = 0.f;
  for (int i = threadIdx.x; i < k; i += SAMPLE_THREADS) {
    const bool keep = (i == 0) || !(p < 1.0f && s_cum[i] > p);
    if (keep) part += expf(s_v[i] / t - z0);
  }
  const float sum = block_sum(part, red);
  float best = -INFINITY;
  int bi = 0x7FFFFFFF;
  for (int i = threadIdx.x; i < k; i += SAMPLE_THREADS) {
    const bool keep = (i == 0) || !(p < 1.0f && s_cum[i] > p);
    const float pr = keep ? expf(s_v[i] / t - z0) / sum : 0.f;
    const float sc = pr / exp_noise(seed, stream, tick, row, i);
    if (sc > best || (sc == best && i < bi)) { best = sc; bi = i; }
  }
  block_argmax(best, bi, red, redi);
  return bi;
}

// The same draw by one warp, for k <= 64 (two candidates a lane, warp shuffles only). The softmax normaliser is a
// common factor of every score, so the winner does not depend on the order of its sum.
__device__ int race_warp(const float* s_v, const float* s_cum, int k, float p, float t, unsigned long long seed,
                         int stream, long long tick, int row) {
  const int lane = threadIdx.x & 31;
  const float z0 = s_v[0] / t;
  float e[2];
  float part = 0.f;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int i = lane + 32 * h;
    const bool keep = i < k && ((i == 0) || !(p < 1.0f && s_cum[i] > p));
    e[h] = keep ? expf(s_v[i] / t - z0) : 0.f;
    part += e[h];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffff, part, o);
  float best = -INFINITY;
  int bi = 0x7FFFFFFF;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int i = lane + 32 * h;
    if (i < k) {
      const float sc = (e[h] / part) / exp_noise(seed, stream, tick, row, i);
      if (sc > best || (sc == best && i < bi)) { best = sc; bi = i; }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffff, best, o);
    const int oi = __shfl_xor_sync(0xffffffff, bi, o);
    if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
  }
  return bi;
}

// Descending bitonic sort of s_c[0, 64) by one warp (two entries a lane), 64-bit keys.
__device__ void sort64_warp(unsigned long long* s_c) {
  const int lane = threadIdx.x & 31;
  unsigned long long x[2] = {s_c[2 * lane], s_c[2 * lane + 1]};
#pragma unroll
  for (int size = 2; size <= 64; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int pidx = 2 * lane + h;
        const bool desc = (pidx & size) == 0;
        unsigned long long y;
        if (stride == 1) {
          y = x[h ^ 1];
        } else {
          y = __shfl_xor_sync(0xffffffff, x[h], stride >> 1);
        }
        const bool lower = (pidx & stride) == 0;         // this entry is the lower index of its pair
        const bool keep_max = desc == lower;
        if (stride != 1) x[h] = keep_max ? (x[h] > y ? x[h] : y) : (x[h] < y ? x[h] : y);
        else if (h == 0) {                               // both entries of the pair live in this lane
          const unsigned long long hi = x[0] > x[1] ? x[0] : x[1], lo = x[0] > x[1] ? x[1] : x[0];
          x[0] = keep_max ? hi : lo;
          x[1] = keep_max ? lo : hi;
        }
      }
    }
  }
  s_c[2 * lane] = x[0];
  s_c[2 * lane + 1] = x[1];
}

__global__ void __launch_bounds__(SAMPLE_THREADS) k_sample(const SampleArgs a) {
  extern __shared__ uint8_t smem_raw[];
  float* s_x = reinterpret_cast<float*>(smem_raw);                       // [V]
  const int vpad = (a.V + 3) & ~3;
  float* s_v = s_x + vpad;                                                // [kpad]
  float* s_cum = s_v + ((a.k + 3) & ~3);
  int* s_idx = reinterpret_cast<int*>(s_cum + ((a.k + 3) & ~3));
  int kp2 = 1;
  while (kp2 < a.k) kp2 <<= 1;
  unsigned long long* s_c = reinterpret_cast<unsigned long long*>(
      (reinterpret_cast<uintptr_t>(s_idx + ((a.k + 3) & ~3)) + 7) & ~uintptr_t(7));   // [max(kp2, 64)]
  __shared__ float red[32];
  __shared__ int redi[32];
  __shared__ int hist[256];
  __shared__ int s_sel[4];

  pdl_launch();
  pdl_wait();
  const int row = blockIdx.x, tid = threadIdx.x;
  // a prefill graph's padding request (slot B, the scratch row) draws nothing (uniform over the block)
  if (a.mode == SM_PREFILL && (a.st[row] < 0 || a.st[row] >= a.B)) return;
  const int V = a.V;
  const float* lg = a.logits + (size_t)row * a.ld;
  for (int i = tid; i < V; i += SAMPLE_THREADS) s_x[i] = lg[i];
  __syncthreads();
  const long long tick = a.tick_id != nullptr ? *a.tick_id : 0;

  int j1, j2 = -1;
  if (!a.do_sample) {
    float best = -INFINITY;
    int bi = 0x7FFFFFFF;
    for (int i = tid; i < V; i += SAMPLE_THREADS)
      if (s_x[i] > best) { best = s_x[i]; bi = i; }
    block_argmax(best, bi, red, redi);
    j1 = bi;
  } else {
    const int k = a.k;
    // log-sum-exp of all logits; whether every logit is a bf16 value (its low 16 bits zero: the head GEMM's logits)
    float mx = -INFINITY;
    uint32_t low = 0;
    for (int i = tid; i < V; i += SAMPLE_THREADS) {
      mx = fmaxf(mx, s_x[i]);
      low |= __float_as_uint(s_x[i]) & 0xFFFFu;
    }
    const bool bf16_keys = !__syncthreads_or(low != 0u);
    mx = block_max(mx, red);
    float se = 0.f;
    for (int i = tid; i < V; i += SAMPLE_THREADS) se += expf(s_x[i] - mx);
    const float lse = mx + logf(block_sum(se, red));
    // radix select of the k-th largest key (bf16 values: the high 16 bits of a key decide, two passes)
    uint32_t prefix = 0, mask = 0;
    int remain = k;
    const int last_shift = bf16_keys ? 16 : 0;
    for (int shift = 24; shift >= last_shift; shift -= 8) {
      for (int b = tid; b < 256; b += SAMPLE_THREADS) hist[b] = 0;
      __syncthreads();
      // logits crowd into few bins of the high bytes: lanes of a warp with the same bin add once, together
      for (int it = 0; it < (V + SAMPLE_THREADS - 1) / SAMPLE_THREADS; ++it) {
        const int i = it * SAMPLE_THREADS + tid;
        const uint32_t key = i < V ? fkey(s_x[i]) : 0u;
        const int bin = (i < V && (key & mask) == prefix) ? int((key >> shift) & 255) : -1;
        const unsigned peers = __match_any_sync(0xffffffffu, bin);
        if (bin >= 0 && (tid & 31) == __ffs(peers) - 1) atomicAdd(&hist[bin], __popc(peers));
      }
      __syncthreads();
      // the bin holding the remain-th largest key, scanning from bin 255 down: warp 0, lane l owns bins
      // 255 - 8l .. 248 - 8l; a warp prefix sum of the lane totals finds the one lane whose bins reach `remain`,
      // which walks its 8 (matching elements always number at least `remain`, so exactly one lane does)
      if (tid < 32) {
        int c[8], loc = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          c[q] = hist[255 - (tid * 8 + q)];
          loc += c[q];
        }
        int inc = loc;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, inc, o);
          if (tid >= o) inc += y;
        }
        const int pre = inc - loc;
        if (pre < remain && remain <= inc) {
          int acc = pre, q = 0;
          for (; q < 7; ++q) {
            if (acc + c[q] >= remain) break;
            acc += c[q];
          }
          s_sel[0] = 255 - (tid * 8 + q);
          s_sel[1] = acc;
        }
      }
      __syncthreads();
      prefix |= uint32_t(s_sel[0]) << shift;
      mask |= 255u << shift;
      remain -= s_sel[1];
      __syncthreads();
    }
    // key of the k-th largest; take `remain` of the ties, lowest index first. With bf16 values the low half of a key
    // follows from its sign: 0 for a positive value, 0xFFFF for a negative one (the key of a negative value is ~u)
    const uint32_t T = bf16_keys ? (prefix | ((prefix & 0x80000000u) ? 0u : 0xFFFFu)) : prefix;
    // compaction in index order: thread owns a contiguous index range
    const int per = (V + SAMPLE_THREADS - 1) / SAMPLE_THREADS;
    const int i0 = tid * per, i1 = min(V, i0 + per);
    int ngt = 0, neq = 0;
    for (int i = i0; i < i1; ++i) {
      const uint32_t key = fkey(s_x[i]);
      ngt += key > T;
      neq += key == T;
    }
    int tot_gt, tot_eq;
    const int off_gt = block_excl_scan(ngt, redi, &tot_gt);
    const int off_eq = block_excl_scan(neq, redi, &tot_eq);
    for (int i = tid; i < kp2; i += SAMPLE_THREADS) s_c[i] = 0ull;
    __syncthreads();
    {
      int pg = off_gt, pe = off_eq;
      for (int i = i0; i < i1; ++i) {
        const uint32_t key = fkey(s_x[i]);
        if (key > T) {
          s_c[pg++] = (uint64_t(key) << 32) | uint32_t(~uint32_t(i));
        } else if (key == T) {
          if (pe < remain) s_c[tot_gt + pe] = (uint64_t(key) << 32) | uint32_t(~uint32_t(i));
          ++pe;
        }
      }
    }
    __syncthreads();
    // bitonic sort, descending (one warp for up to 64 candidates)
    if (kp2 <= 64) {
      if (tid < 32) {
        if (kp2 < 64)
          for (int i = kp2 + tid; i < 64; i += 32) s_c[i] = 0ull;
        __syncwarp();
        sort64_warp(s_c);
      }
      __syncthreads();
    }
    for (int size = 2; size <= kp2 && kp2 > 64; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int i = tid; i < kp2; i += SAMPLE_THREADS) {
          const int jx = i ^ stride;
          if (jx > i) {
            const bool desc = (i & size) == 0;
            const unsigned long long x = s_c[i], y = s_c[jx];
            if (desc ? (x < y) : (x > y)) { s_c[i] = y; s_c[jx] = x; }
          }
        }
        __syncthreads();
      }
    }
    // values, indices, cumulative probability (sequential per chunk of threads: a block scan)
    for (int i = tid; i < k; i += SAMPLE_THREADS) {
      s_v[i] = unkey(uint32_t(s_c[i] >> 32));
      s_idx[i] = int(~uint32_t(s_c[i] & 0xFFFFFFFFu));
    }
    __syncthreads();
    if (tid < 32) {
      float run = 0.f;
      for (int base = 0; base < k; base += 32) {
        const int i = base + tid;
        float x = i < k ? expf(s_v[i] - lse) : 0.f;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_up_sync(0xffffffff, x, o);
          if (tid >= o) x += y;
        }
        if (i < k) s_cum[i] = run + x;
        run += __shfl_sync(0xffffffff, x, 31);
      }
    }
    __syncthreads();
    if (k <= 64) {
      // the regular draw by warp 0, the RAS redraw by warp 1, side by side
      __shared__ int s_pick[2];
      if (tid < 32) {
        const int c1 = race_warp(s_v, s_cum, k, a.p, a.t, a.seed, a.stream1, tick, row);
        if (tid == 0) s_pick[0] = c1;
      } else if (tid < 64 && a.mode == SM_SEMANTIC) {
        const int c2 = race_warp(s_v, s_cum, k, a.p2, a.t2, a.seed, a.stream2, tick, row);
        if (tid == 32) s_pick[1] = c2;
      }
      __syncthreads();
      j1 = s_idx[s_pick[0]];
      if (a.mode == SM_SEMANTIC) j2 = s_idx[s_pick[1]];
    } else {
      const int c1 = race(s_v, s_cum, k, a.p, a.t, a.seed, a.stream1, tick, row, red, redi);
      j1 = s_idx[c1];
      if (a.mode == SM_SEMANTIC) {
        const int c2 = race(s_v, s_cum, k, a.p2, a.t2, a.seed, a.stream2, tick, row, red, redi);
        j2 = s_idx[c2];
      }
    }
  }

  // ---------------------------------------------------------------- outputs / state
  if (a.mode == SM_CODEBOOK) {
    if (tid == 0) a.codes[(size_t)row * a.ncb + a.cb_index] = j1;
    if (a.x_next != nullptr)
      for (int c = tid * 8; c < a.H; c += SAMPLE_THREADS * 8)
        *reinterpret_cast<uint4*>(a.x_next + (size_t)row * a.ldx + c) =
            *reinterpret_cast<const uint4*>(a.fast_emb + (size_t)j1 * a.H + c);
  } else if (a.mode == SM_PLAIN) {
    if (tid == 0) a.out_tok[row] = j1;
  } else if (a.mode == SM_SEMANTIC) {
    const long long t_in = a.tok_in[row];
    if (tid == 0) {
      int64_t* pv = a.prev + (size_t)row * a.ras_w;
      if (a.nstep[row] > 0) {               // the consumed token joins the RAS window (not a row's first token)
        for (int i = 0; i + 1 < a.ras_w; ++i) pv[i] = pv[i + 1];
        pv[a.ras_w - 1] = t_in;
      }
      const long long nrm = j1 == a.nsem ? a.eos : j1 + a.sb;
      long long nt = nrm;
      if (a.do_sample) {
        const long long high = j2 == a.nsem ? a.eos : j2 + a.sb;
        bool rep = false;
        for (int i = 0; i < a.ras_w; ++i) rep |= pv[i] == nrm;
        rep &= nrm != a.eos;
        nt = rep ? high : nrm;
      }
      if (t_in == a.eos) nt = t_in;         // EOS sticks
      a.tok[row] = nt;
      const int cp = a.cpos[row] + 1;
      a.cpos[row] = cp < a.S - 1 ? cp : a.S - 1;
      a.nstep[row] = a.nstep[row] + 1;
    }
    for (int c = tid * 8; c < a.H; c += SAMPLE_THREADS * 8)
      *reinterpret_cast<uint4*>(a.hid + (size_t)row * a.H + c) =
          *reinterpret_cast<const uint4*>(a.h_src + (size_t)row * a.ldh + c);
    if (tid < a.ncb)
      a.frame_prev[(size_t)row * a.ncb + tid] =
          t_in == a.eos ? a.sil_frame[tid] : a.codes[(size_t)row * a.ncb + tid];
  } else {  // SM_PREFILL
    const int slot = a.st[row];
    if (slot < 0 || slot >= a.B) return;       // a graph's padding request (the scratch slot): no state to write
    if (tid == 0) {
      a.tok[slot] = j1 == a.nsem ? a.eos : j1 + a.sb;
      a.cpos[slot] = a.cpos_new[row];
      a.nstep[slot] = 0;
    }
    if (tid < a.ras_w) a.prev[(size_t)slot * a.ras_w + tid] = 0;
    if (a.frame0 != nullptr && tid < a.ncb)
      a.frame_prev[(size_t)slot * a.ncb + tid] = a.frame0[(size_t)row * a.ncb + tid];
    for (int c = tid * 8; c < a.H; c += SAMPLE_THREADS * 8)
      *reinterpret_cast<uint4*>(a.hid + (size_t)slot * a.H + c) =
          *reinterpret_cast<const uint4*>(a.h_src + (size_t)row * a.ldh + c);
  }
}

int sample_smem(int V, int k) {
  int kp2 = 1;
  while (kp2 < k) kp2 <<= 1;
  if (kp2 < 64) kp2 = 64;                  // the one-warp sort pads the candidates to 64
  return ((V + 3) & ~3) * 4 + 3 * ((k + 3) & ~3) * 4 + 8 + kp2 * 8;
}

int sample_launch(const SampleArgs& a, int rows, cudaStream_t s) {
  const int smem = sample_smem(a.V, a.do_sample ? a.k : 1);
  if (smem > 200 * 1024) return A8_ERR_SIZE;
  static int configured = 0;
  if (smem > 48 * 1024 && configured < smem) {
    cudaFuncSetAttribute(k_sample, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    configured = 200 * 1024;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rows);
  cfg.blockDim = dim3(SAMPLE_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  ++g_launches;
  return cudaLaunchKernelEx(&cfg, k_sample, a) == cudaSuccess ? A8_OK : A8_ERR_CUDA;
}

}  // namespace a8

using namespace a8;

// Plain draw per row (tests and tools): out[row] = the sampled (or argmax) index into the row's V logits.
// Replaces _Sampler.__call__ (serve/fast_engine.py:168-172) with explicit Philox noise (seed, stream, tick).
extern "C" int a8_sample(const float* logits, int ld, int V, int rows, int do_sample, int top_k, float top_p,
                         float temperature, unsigned long long seed, int stream_id, const long long* tick_id,
                         int64_t* out, a8_stream_t stream) {
  if (logits == nullptr || out == nullptr || rows <= 0 || V <= 0 || V > 16384) return A8_ERR_ARG;
  SampleArgs a = {};
  a.logits = logits;
  a.ld = ld;
  a.V = V;
  a.mode = SM_PLAIN;
  a.do_sample = do_sample;
  a.k = (top_k > 0 && top_k < V) ? top_k : V;
  a.p = top_p;
  a.t = fmaxf(temperature, 1e-5f);
  a.seed = seed;
  a.tick_id = tick_id;
  a.stream1 = stream_id;
  a.out_tok = out;
  return sample_launch(a, rows, reinterpret_cast<cudaStream_t>(stream));
}
