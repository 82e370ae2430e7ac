// Per-slot streaming rate conversion + PCM16 of the codec's audio (replaces the worker's per-request
// soxr.ResampleStream(native_sr, out_sr).resample_chunk(y, last) and _pcm16, serve/engine_worker.py:443-461, :423-424).
//
// One CTA a slot row. The row's kept history (hist_len samples) and this tick's frame are staged in shared memory
// behind a zero tail (the inputs past the end of a flushed stream). Output n uses phase p = (n down + half) % up;
// phases repeat every `up` outputs, so thread t of a CTA of `period` threads (a multiple of up) owns outputs
// n_out + t + i period, all of one phase: each tap is read once from the (L2-resident) table and applied to up to
// RS_PT outputs whose input windows sit period * down / up samples apart. The table streams through shared memory
// in chunks of RS_KC taps (all phases), double-buffered with cp.async, so the tap loop reads only shared memory.
// When few rows run (a bucket smaller than a wave of CTAs), a row's chunks are dealt round-robin over a cluster of
// `splits` CTAs; each adds its partial sums into the rank-0 CTA's shared memory (DSMEM) and rank 0 finishes the row.
// Every CTA of a cluster reads the row's state before the first cluster barrier and takes the same branch, so each
// cluster barrier is reached by all of them.
#include "common.cuh"

namespace a8 {

constexpr int KERNEL_ID_RESAMPLE = 5;
constexpr int RS_PT = 8;           // outputs a thread at most
constexpr int RS_KC = 32;          // taps a staged table chunk (the table's taps are a multiple of it)
enum { RS_SKIP = 1, RS_DONE = 2 };

__device__ __forceinline__ void cp_async16(float* dst, const float* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ long long floor_div(long long a, long long b) {
  const long long q = a / b;
  return (a % b != 0 && ((a < 0) != (b < 0))) ? q - 1 : q;
}

__global__ void k_resample_reset(A8Resample d, const int* __restrict__ slots, const int* __restrict__ caps,
                                 int drop_first) {
  pdl_launch();
  pdl_wait();
  const int s = slots[blockIdx.x];
  if (s < 0 || s >= d.rows) {
    if (threadIdx.x == 0) set_error(ERR_BOUNDS, KERNEL_ID_RESAMPLE, s);
    return;
  }
  float* h = d.hist + (size_t)s * d.hist_len;
  for (int i = threadIdx.x; i < d.hist_len; i += blockDim.x) h[i] = 0.f;
  if (threadIdx.x == 0) {
    d.n_in[s] = 0;
    d.n_out[s] = 0;
    d.left[s] = caps[blockIdx.x];
    d.flags[s] = drop_first ? RS_SKIP : 0;
  }
}

__global__ void __launch_bounds__(512) k_resample(A8Resample d, const float* __restrict__ audio, int ld_audio,
                                                   const int64_t* __restrict__ tok_in, long long eos,
                                                   int16_t* __restrict__ pcm, float* __restrict__ f32, int ld_out,
                                                   int* __restrict__ counts, int splits) {
  // table chunks [2][RS_KC up] | buf [hist_len + frame + zpad] | partial sums [splits - 1][RS_PT][period] (rank 0)
  extern __shared__ __align__(16) float smem_rs[];
  __shared__ long long s_nin, s_nout;
  __shared__ int s_flags, s_left;
  pdl_launch();
  pdl_wait();
  const int r = blockIdx.x / splits;
  const int z = splits > 1 ? (int)cluster_rank() : 0;
  if (threadIdx.x == 0) {
    s_flags = d.flags[r];
    s_nin = d.n_in[r];
    s_nout = d.n_out[r];
    s_left = d.left[r];
  }
  __syncthreads();
  if (splits > 1) cluster_sync();             // every CTA of the row has its state before rank 0 may change it
  const int flags = s_flags;
  const bool ended = tok_in[r] == eos;
  if (flags & RS_DONE) {                      // no stream in this row: nothing in, nothing out
    if (threadIdx.x == 0 && z == 0) counts[r] = 0;
    return;
  }
  if (flags & RS_SKIP) {                      // the silence frame a fresh row decodes first: dropped
    if (threadIdx.x == 0 && z == 0) {
      d.flags[r] = ended ? RS_DONE : 0;
      counts[r] = 0;
    }
    return;
  }
  const int H = d.hist_len, F = d.frame, Z = d.zpad, CH = RS_KC * d.up;
  const int nch = (d.taps / RS_KC - z + splits - 1) / splits;   // this CTA's chunks: z, z + splits, ...
  float* tabs = smem_rs;
  float* buf = smem_rs + 2 * CH;               // buf[i] = input sample n_in - hist_len + i
  float* part = buf + H + F + Z;               // rank 0: the other CTAs' partial sums
  auto issue = [&](int j) {                    // this CTA's j-th chunk -> tabs[j & 1] (every thread's share)
    const float* src = d.table + (size_t)(z + j * splits) * CH;
    float* dst = tabs + (j & 1) * CH;
    for (int i = threadIdx.x * 4; i < CH; i += blockDim.x * 4) cp_async16(dst + i, src + i);
    cp_async_commit();
  };
  if (nch > 0) issue(0);
  const float* hist = d.hist + (size_t)r * H;
  const float* x = audio + (size_t)r * ld_audio;
  if (((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(hist)) & 15) == 0 && (F & 3) == 0) {
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x)
      reinterpret_cast<float4*>(buf)[i] = reinterpret_cast<const float4*>(hist)[i];
    for (int i = threadIdx.x; i < F / 4; i += blockDim.x)
      reinterpret_cast<float4*>(buf + H)[i] = reinterpret_cast<const float4*>(x)[i];
  } else {
    for (int i = threadIdx.x; i < H; i += blockDim.x) buf[i] = hist[i];
    for (int i = threadIdx.x; i < F; i += blockDim.x) buf[H + i] = x[i];
  }
  for (int i = threadIdx.x; i < Z; i += blockDim.x) buf[H + F + i] = 0.f;

  const long long up = d.up, down = d.down, half = d.half;
  const long long nin = s_nin, nout = s_nout, N = nin + F;
  const int left = s_left - 1;
  const bool last = ended || left <= 0;
  long long n_end = last ? (N * up + down - 1) / down : floor_div(N * up - 1 - half, down) + 1;
  if (n_end < nout) n_end = nout;
  long long cnt = n_end - nout;
  if (cnt > d.out_max) {
    if (threadIdx.x == 0) set_error(ERR_BOUNDS, KERNEL_ID_RESAMPLE, (int)cnt);
    cnt = d.out_max;
  }
  const long long base = nin - H;             // input index of buf[0]
  const int t = threadIdx.x;
  const long long q0 = (nout + t) * down + half;
  const long long m0 = q0 / up;
  const int p = (int)(q0 - m0 * up);
  const long long stride = (long long)d.period * down / up;
  int nloc = 0;                                // outputs of this thread: nout + t + i period < nout + cnt
  if (t < cnt) nloc = (int)min((long long)RS_PT, (cnt - 1 - t) / d.period + 1);
  const long long lo = m0 - (d.taps - 1) - base, hi = m0 + (nloc - 1) * stride - base;
  if (nloc > 0 && (lo < 0 || hi >= H + F + Z)) {
    set_error(ERR_BOUNDS, KERNEL_ID_RESAMPLE, (int)(lo < 0 ? lo : hi));
    nloc = 0;
  }
  float acc[RS_PT];
#pragma unroll
  for (int i = 0; i < RS_PT; ++i) acc[i] = 0.f;
  const float* xb = buf + (nloc > 0 ? m0 - base : 0);
  const int st = (int)stride, up_i = d.up;
  // lane l walks a chunk's taps from (m0 - base - l) mod 32 on: its x words then sit in bank (l - kk) mod 32 at step
  // kk (buf starts on a 32-word boundary), so a warp's x loads are conflict-free; table words are in bank p mod 32
  const int rot = (int)((m0 - base - (threadIdx.x & 31)) & (RS_KC - 1));
  __syncthreads();                             // buf staged (also when this CTA has no chunk)
  for (int c = 0; c < nch; ++c) {              // every thread takes every barrier
    if (c + 1 < nch) {
      issue(c + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();                           // chunk c visible to all
    if (nloc > 0) {
      const float* tc = tabs + (c & 1) * CH + p;
      const float* xc = xb - (z + c * splits) * RS_KC;
#pragma unroll 8
      for (int kk = 0; kk < RS_KC; ++kk) {
        const int kr = (kk + rot) & (RS_KC - 1);
        const float cf = tc[kr * up_i];
        const float* xr = xc - kr;
#pragma unroll
        for (int i = 0; i < RS_PT; ++i)
          if (i < nloc) acc[i] = fmaf(cf, xr[i * st], acc[i]);
      }
    }
    __syncthreads();                           // tabs[c & 1] free for chunk c + 2
  }
  if (splits > 1) {                            // partial sums -> rank 0's shared memory, then rank 0 adds them
    if (z > 0 && nloc > 0) {
      const uint32_t dst = dsmem_addr(smem_u32(part + (size_t)(z - 1) * RS_PT * d.period), 0);
#pragma unroll
      for (int i = 0; i < RS_PT; ++i)
        if (i < nloc) dsmem_st(dst + 4u * (i * d.period + t), acc[i]);
    }
    cluster_sync();
    if (z > 0) return;
    for (int q = 1; q < splits; ++q) {
      const float* pq = part + (size_t)(q - 1) * RS_PT * d.period;
#pragma unroll
      for (int i = 0; i < RS_PT; ++i)
        if (i < nloc) acc[i] += pq[i * d.period + t];
    }
  }
  if (nloc > 0) {
    int16_t* po = pcm + (size_t)r * ld_out;
    float* fo = f32 != nullptr ? f32 + (size_t)r * ld_out : nullptr;
#pragma unroll
    for (int i = 0; i < RS_PT; ++i) {
      if (i < nloc) {
        const int o = t + i * d.period;
        const float y = acc[i];
        po[o] = (int16_t)(int)(fminf(fmaxf(y, -1.f), 1.f) * 32767.f);
        if (fo != nullptr) fo[o] = y;
      }
    }
  }
  float* hw = d.hist + (size_t)r * H;         // keep the last H inputs (buf is read-only since the staging)
  for (int i = threadIdx.x; i < H; i += blockDim.x) hw[i] = buf[F + i];
  if (threadIdx.x == 0) {
    d.n_in[r] = N;
    d.n_out[r] = nout + cnt;
    d.left[r] = left;
    d.flags[r] = last ? RS_DONE : 0;
    counts[r] = (int)cnt;
  }
}

static int rs_launch_cfg(cudaLaunchConfig_t& cfg, cudaLaunchAttribute* at, dim3 grid, dim3 block, size_t smem,
                         a8_stream_t stream, int cluster = 1) {
  cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  at[1].id = cudaLaunchAttributeClusterDimension;
  at[1].val.clusterDim.x = cluster;
  at[1].val.clusterDim.y = 1;
  at[1].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = cluster > 1 ? 2 : 1;
  return 0;
}

static bool rs_desc_ok(const A8Resample& d) {
  if (d.table == nullptr || d.hist == nullptr || d.n_in == nullptr || d.n_out == nullptr || d.left == nullptr ||
      d.flags == nullptr)
    return false;
  if (d.up <= 0 || d.down <= 0 || d.taps <= 0 || d.frame <= 0 || d.rows <= 0 || d.out_max <= 0) return false;
  if (d.period <= 0 || d.period > 512 || d.period % d.up != 0 || d.taps % RS_KC != 0) return false;
  if ((long long)d.period * RS_PT < d.out_max) return false;
  // the history covers every tap of a pending output; the zero tail covers a flush's look-ahead
  if (d.hist_len < d.taps + d.down / d.up + 2) return false;
  if ((long long)d.zpad < d.half / d.up + d.down / d.up + 2) return false;
  if (d.half < 0 || d.half >= (long long)d.taps * d.up) return false;
  return true;
}

}  // namespace a8

using namespace a8;

extern "C" int a8_resample_reset(const A8Resample* d, const int* slots, const int* caps, int n, int drop_first,
                                 a8_stream_t stream) {
  if (d == nullptr || slots == nullptr || caps == nullptr || n < 0 || !rs_desc_ok(*d)) return A8_ERR_ARG;
  if (n == 0) return A8_OK;
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute at[2];
  rs_launch_cfg(cfg, at, dim3(n), dim3(128), 0, stream);
  ++g_launches;
  return cudaLaunchKernelEx(&cfg, k_resample_reset, *d, slots, caps, drop_first) == cudaSuccess ? A8_OK
                                                                                               : A8_ERR_CUDA;
}

extern "C" int a8_resample_step(const A8Resample* d, const float* audio, int ld_audio, const int64_t* tok_in,
                                long long eos, int b, int16_t* pcm, float* f32, int ld_out, int* counts,
                                a8_stream_t stream) {
  if (d == nullptr || audio == nullptr || tok_in == nullptr || pcm == nullptr || counts == nullptr ||
      !rs_desc_ok(*d))
    return A8_ERR_ARG;
  if (b < 0 || b > d->rows || ld_audio < d->frame || ld_out < d->out_max) return A8_ERR_ARG;
  if (b == 0) return A8_OK;
  const size_t base = sizeof(float) * (2ull * RS_KC * d->up + d->hist_len + d->frame + d->zpad);
  // splits: the most CTAs a row (1, 2 or 4, at most one a table chunk) that still fit one wave of the whole grid
  int splits = 1;
  for (int S : {4, 2}) {
    if (S > d->taps / RS_KC) continue;
    const size_t smem = base + sizeof(float) * (size_t)(S - 1) * RS_PT * d->period;
    const int per_sm = (int)std::min<size_t>(2048 / d->period, (227 * 1024) / (smem + 1024));
    if ((long long)b * S <= (long long)num_sms() * per_sm) {
      splits = S;
      break;
    }
  }
  const size_t smem = base + sizeof(float) * (size_t)(splits - 1) * RS_PT * d->period;
  if (smem > 200 * 1024) return A8_ERR_SIZE;
  static size_t smem_set = 0;
  if (smem > 48 * 1024 && smem > smem_set) {
    if (cudaFuncSetAttribute(k_resample, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return A8_ERR_CUDA;
    smem_set = smem;
  }
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute at[2];
  rs_launch_cfg(cfg, at, dim3(b * splits), dim3(d->period), smem, stream, splits);
  ++g_launches;
  return cudaLaunchKernelEx(&cfg, k_resample, *d, audio, ld_audio, tok_in, eos, pcm, f32, ld_out, counts, splits) ==
                 cudaSuccess
             ? A8_OK
             : A8_ERR_CUDA;
}
