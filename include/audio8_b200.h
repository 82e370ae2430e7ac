/* audio8_b200.h -- C ABI of the B200 (sm_100a) Audio8 decode-tick library, libaudio8_b200.so.
 *
 * Plain pointers (device memory unless stated), sizes and a CUDA stream; every function returns 0 (A8_OK) or an
 * A8_ERR_* code and never throws. All launches are asynchronous on the given stream and capture-safe (no host
 * synchronisation, no allocation), so a caller may record them into a CUDA graph.
 *
 * Each entry point replaces a piece of the reference engine (serve/fast_kernels.py, serve/fast_engine.py of
 * lvt1693/audio8-turbo-engine); the comment above it names the reference interface (file:line).
 *
 * Device-side waits are bounded: a wait that runs out records an error code readable with a8_get_error() and the
 * kernel returns; a8_get_error() is the only call here that synchronises with the device.
 */
#ifndef AUDIO8_B200_H
#define AUDIO8_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* a8_stream_t; /* a cudaStream_t */

enum {
  A8_OK = 0,
  A8_ERR_ARG = 1,    /* bad argument (null pointer, unsupported shape) */
  A8_ERR_CUDA = 2,   /* a CUDA runtime / driver call failed */
  A8_ERR_ALIGN = 3,  /* a pointer or stride breaks a 16-byte TMA alignment rule */
  A8_ERR_SIZE = 4,   /* a workspace or a table is too small for the request */
  A8_ERR_DEVICE = 5  /* no sm_100 device current */
};

/* ---------------------------------------------------------------------------------------------- status */
/* 1 when the current device is a compute-capability 10.0 GPU (B200), else 0. */
int a8_device_ok(void);
/* Device error record of the bounded waits: out[0] code (0 = none), out[1] kernel id, out[2] block, out[3] extra.
 * Synchronises the device. */
int a8_get_error(int out[4]);
int a8_clear_error(void);
/* Kernels this library has launched (or recorded into a graph) in this process; a host-side count, no device sync.
 * No counterpart in the reference (a benchmark aid). */
long long a8_launch_count(void);

/* ---------------------------------------------------------------------------------------------- GEMM */
/* Epilogue kinds of a8_gemm. Y = X[M,K] . W[N,K]^T accumulated in fp32 on the tensor cores (tcgen05, TMEM). */
enum {
  A8_EPI_BF16 = 0,      /* y bf16 [M, ldy]:   bf16(acc (+ bias))                                           */
  A8_EPI_F32_ROUND = 1, /* y fp32 [M, ldy]:   float(bf16(acc)) -- the reference's bf16 logits as fp32      */
  A8_EPI_SILU = 2,      /* W rows interleaved per 64 (gate 0-63, up 64-127 of every 128): y bf16 [M, N/2]:
                           bf16(bf16(silu(bf16 g)) * bf16 u)                                               */
  A8_EPI_ROPE = 3,      /* fused qkv epilogue: bias, RoPE (rotate_half, fp32, one rounding), q -> y [M, nq, hd],
                           k / v -> caches at [slot, head, pos % ring]                                      */
  A8_EPI_GELU = 4,      /* y bf16: bf16(gelu_erf(bf16(acc + bias)))                                        */
  A8_EPI_LSRES = 5,     /* y bf16: bf16(res + bf16(gamma * bf16(acc + bias)))  (ConvNeXt layer scale)      */
  A8_EPI_RESID = 6      /* y bf16: bf16(bf16(acc + bias) + res), the residual add of rmsnorm
                           (serve/fast_kernels.py:36-40; y may equal res); with ssq_out, each 128-column tile t
                           also writes ssq_out[t * ssq_ld + m] = sum of y[m, 128 t .. 128 t + 127]^2 (fp32)       */
};

typedef struct A8Epilogue {
  int kind;
  const void* bias;  /* bf16 [N] or NULL */
  /* A8_EPI_ROPE */
  const void* cos;   /* bf16 [npos, hd] rotate_half table (cos of both halves) */
  const void* sin;   /* bf16 [npos, hd] */
  const int* pos;    /* int32 [M] rope position of each token row */
  const int* slot;   /* int32 [M] cache row of each token row */
  void* kc;          /* bf16 [rows, nkv, cache_len, hd] */
  void* vc;
  int nq, nkv, hd, ring, cache_len;
  /* A8_EPI_LSRES, A8_EPI_RESID */
  const void* gamma; /* bf16 [N] */
  const void* res;   /* bf16 [M, ldres] (may equal y) */
  int ldres;
  /* A8_EPI_RESID: per-row sums of squares of y, one partial per 128-column tile (NULL: none) */
  float* ssq_out;
  int ssq_ld;        /* row stride of the partials (>= M) */
  /* Operand normalisation, any kind (NULL norm_w: none): before the MMA reads it, every X row is replaced by
   * bf16(norm_w * bf16(x * rsqrt(ss / K + eps))), ss = the sum over t < ceil(K / 128) of ssq_in[t * ssq_ld + m]
   * in t order -- the RMSNorm of serve/fast_kernels.py:41-45 on rows whose sums of squares an A8_EPI_RESID GEMM
   * wrote. K <= 1024. */
  const void* norm_w; /* bf16 [K] */
  const float* ssq_in;
  float eps;
} A8Epilogue;

/* y = epilogue(x[M, K] . w[N, K]^T). x row stride ldx, w dense; bf16. Replaces GemmDispatch / linear_triton
 * (serve/fast_kernels.py:364-520) and, through the epilogues, bias_rope_store (:139-187) and silu_mul (:526-545).
 * splits: K splits of a 128-row weight tile (0 = automatic, at most 16); the splits of a tile run as one thread-block
 * cluster and add their partial sums through distributed shared memory, in split order (no global scratch). */
int a8_gemm(const void* x, int ldx, const void* w, int N, int K, int M, void* y, int ldy, const A8Epilogue* epi,
            int splits, a8_stream_t stream);

/* ---------------------------------------------------------------------------------------------- attention */
/* Workspace of a8_attention / a8_stack_forward's attention for calls of up to `rows` query rows whose key count is at
 * most max_len (fewer rows are split into more parts, so this is the largest need over 1..rows rows). */
int a8_attention_workspace(int rows, int nkv, int hd, int max_len, long long* ws_floats, int* n_counters);

/* out[r, h, :] = softmax(q[r, h] . K[c, h / group, :L_r] * scale) V[c, h / group, :L_r], c = rowmap[r] (or r),
 * L_r = min(lens[r], max_len); caches bf16 [layers, cache_rows, nkv, cache_len, hd], hd 64 or 128.
 * Replaces DecodeAttention (serve/fast_kernels.py:193-290) and, with lens = pos + 1 and rowmap = the request's
 * slot, prefill_attention (:296-358). scale <= 0: hd^-0.5. */
int a8_attention(const void* q, int q_stride, const void* kc, const void* vc, int layers, int cache_rows, int nq,
                 int nkv, int hd, int cache_len, int layer, const int* lens, const int* rowmap, int rows, int max_len,
                 float scale, void* out, int out_stride, float* ws, long long ws_floats, int* counters, int n_counters,
                 a8_stream_t stream);

/* Packed causal prefill attention on the tensor cores (replaces prefill_attention / PrefillPlan,
 * serve/fast_kernels.py:296-358): blocks int32 [nblocks][4] = (q0, n, slot, pos0), each up to 64 consecutive packed
 * rows of one request -- row q0 + r is at position pos0 + r of cache row `slot` and attends keys [0, pos0 + r] of it
 * (stored beforehand); a block with n = 0 is skipped. q / out bf16 [rows, stride] rows of nq * hd (16-byte aligned
 * rows), caches as a8_attention; hd 64, nq / nkv <= 8. Softmax with the exact row maximum in two passes over the keys,
 * P rounded to bf16 for P.V, as the reference's kernel feeds its tl.dot. scale <= 0: hd^-0.5. */
int a8_prefill_attention(const void* q, int q_stride, const void* kc, const void* vc, int layers, int cache_rows,
                         int nq, int nkv, int hd, int cache_len, int layer, const int* blocks, int nblocks, int rows,
                         float scale, void* out, int out_stride, a8_stream_t stream);

/* Size of the library-owned workspace of a8_attention_noalloc, in 4-byte words (5 MiB): the largest need of any valid
 * call (hd 128 at rows * nkv = 295: 590 split parts x 2080 words + 295 tickets = 1,227,495 words). */
#define A8_ATTENTION_NOALLOC_FLOATS (5 << 18)

/* a8_attention without caller-provided scratch. No counterpart in the reference: it exists for callers that cannot
 * allocate device memory -- a host-language binding that is handed only the device pointers of its inputs and outputs
 * and has no CUDA allocator of its own, or a serving process whose memory pool already owns the whole device -- and
 * so cannot supply the workspace a8_attention needs when a row's keys span several splits.
 * The split partials and tickets live in one array inside this library (5 MiB, held on every device that loads the
 * library until the process exits). A call needs rows * nkv * S * (16 hd + 32) + rows * nkv words of it when its rows
 * are split in S > 1 parts (S = min(16, ceil(max_len / 64), ceil(296 / (rows * nkv)))). rows * nkv * S is at most 590,
 * so the need is at most 623,335 words at hd 64 and 1,227,495 at hd 128: every call the arguments allow fits, and
 * A8_ERR_SIZE is only a guard. Arguments are checked before the array is touched.
 * The first call on a device looks up the array's device address (cudaGetSymbolAddress, with that device current):
 * make that first call before any stream capture; the address is not re-queried after cudaDeviceReset. Every call
 * shares the array and it keeps the last call's contents; the tickets are cleared (cudaMemsetAsync on the given
 * stream) at each call. Calls that overlap on the GPU (other streams, other threads, the same device) race on the
 * array. Allocates nothing. */
int a8_attention_noalloc(const void* q, int q_stride, const void* kc, const void* vc, int layers, int cache_rows,
                         int nq, int nkv, int hd, int cache_len, int layer, const int* lens, const int* rowmap,
                         int rows, int max_len, float scale, void* out, int out_stride, a8_stream_t stream);

/* ---------------------------------------------------------------------------------------------- row kernels */
/* y = bf16(w * bf16(h * rsqrt(mean(h^2) + eps))), h = bf16(x + res) stored back into res (res may be NULL: h = x).
 * N <= 1024, a multiple of 8. Replaces rmsnorm (serve/fast_kernels.py:30-69). */
int a8_rmsnorm(const void* x, int ldx, void* res, int ldr, const void* w, void* y, int ldy, int rows, int N, float eps,
               a8_stream_t stream);
/* x[r] = emb[sem[r]] + bf16(sum_k cbemb[codes[r, k] + cbk k]) (serve/fast_engine.py:715-717). */
int a8_embed_frame(const int64_t* sem, const int64_t* codes, int ncb, int cbk, const void* emb, const void* cbemb,
                   void* x, int ldx, int rows, int H, int vocab, a8_stream_t stream);
/* Packed prompt rows (serve/fast_engine.py:941-945): ids int32 [rows][2 + ncb] = (sem, audio, code_0 ..): x[r] =
 * emb[sem] on text rows, bf16(emb[sem] + bf16(sum_k cbemb[code_k + cbk k])) on audio rows. */
int a8_embed_prompt(const int* ids, int ncb, int cbk, const void* emb, const void* cbemb, void* x, int ldx, int rows,
                    int H, int vocab, a8_stream_t stream);
/* Tick start (serve/fast_engine.py:742-749, :705): tok_in = tok, codes[:, 0] = clamp(tok - sb), fast AR rows
 * x2[2r] = hid[r], x2[2r+1] = fast_emb[codes[r, 0]]; tick_id[0] = ctr[0]++ (ctr may be NULL). */
int a8_tick_start(const int64_t* tok, int64_t* tok_in, int64_t* codes, int ncb, long long sb, int cbk, const void* hid,
                  const void* fast_emb, void* x2, int rows, int H, long long* ctr, long long* tick_id,
                  a8_stream_t stream);
/* y[r] = src[idx[r]] (bf16 rows of H). */
int a8_gather_rows(const void* src, int lds, const int* idx, void* y, int ldy, int rows, int H, a8_stream_t stream);

/* ---------------------------------------------------------------------------------------------- codec */
/* One launch of the decoder conv (serve/fast_kernels.py:551-623 conv_cl, serve/fast_engine.py:218-232 _CLConv):
 *   y[b, t, n] = bias[n] + sum_{j < taps} sum_c xin[b, t + j*dil, c] * w[n, j*Cin + c]  (+ res[b*res_bs + t*res_ts + n])
 * for t in [0, T), accumulated in fp32 on the tensor cores and rounded to fp16 once. xin fp16 [rows, ctx + T, Cin]
 * holds the conv's carried context in rows [0, ctx) (Cin a multiple of 32, (taps-1)*dil <= ctx; T with
 * T % min(T,128) == 0 and 128 % min(T,128) == 0). w fp16 [N, taps*Cin]; a transposed conv of stride s is 2 taps with
 * N = s*Cout, n = p*Cout + c, so row t holds output timesteps t*s + p. Outputs, any of:
 *   raw   fp16 y at raw[b*raw_bs + t*raw_ts + n]
 *   nxt   the NEXT conv's input rows, act(y) at nxt[b*nxt_bs + nxt_off + t*N + n], act(v) = v + inv[c] sin(alpha[c] v)^2
 *         on the fp16 y (c = n % cout; alpha NULL: identity) -- the snake of serve/fast_kernels.py:578-583, :709-713
 *   audio conv_out: audio[b*audio_bs + t] = tanh(fp16(y[b, t, 0])) (fp32)
 * With N a multiple of 16, raw / res / nxt / bias are 32-byte aligned with strides multiples of 16 elements. */
typedef struct A8ConvRun {
  const void* xin;
  int rows, T, Cin, ctx;
  const void* w;
  int N, taps, dil;
  const float* bias;      /* [N] (the fp16 bias as fp32) or NULL */
  const void* res;        /* fp16 or NULL */
  long long res_bs, res_ts;
  void* raw;              /* fp16 or NULL */
  long long raw_bs, raw_ts;
  void* nxt;              /* fp16 or NULL */
  long long nxt_bs, nxt_off;
  int cout;               /* channels of an output timestep (0: N) */
  const float* alpha;     /* [cout] or NULL */
  const float* inv;       /* [cout]: 1 / (alpha + 1e-9) */
  float* audio;           /* or NULL */
  long long audio_bs;
} A8ConvRun;
int a8_conv(const A8ConvRun* r, a8_stream_t stream);

/* A conv's carried context for the next frame (serve/fast_engine.py:230-231): xin[b, :ctx] = xin[b, T : T + ctx] for
 * rows [0, rows) of each table entry (the table in device memory; one launch for all of a step's convs). */
typedef struct A8CtxShift {
  void* xin;              /* fp16 [rows, ctx + T, Cin] */
  int ctx, T, Cin;
} A8CtxShift;
int a8_ctx_shift(const A8CtxShift* table, int n, int rows, a8_stream_t stream);

/* A conv's input rows from a tensor (serve/fast_kernels.py:695-729 snake_cat without the context, which lives in
 * xin): xin[b, ctx + t, c] = fp16(act(x[b, t, c])) for x fp16 (x_bf16 = 0) or bf16 rows of C at batch stride x_bs
 * elements, act as in a8_conv (alpha NULL: identity). C a multiple of 8. */
int a8_conv_input(const void* x, int x_bf16, long long x_bs, int T, int C, void* xin, int ctx, const float* alpha,
                  const float* inv, int rows, a8_stream_t stream);
/* Upsample stage middle (serve/fast_engine.py:484-489): bf16 causal depthwise conv (K taps <= 8, carried tail
 * st [rows, K-1, C] at st_bs elements a row, every product and sum rounded to bf16 in tap order, bias first) and
 * LayerNorm(eps) over C (C a multiple of 128, <= 4096): z = bf16(LN(dwconv([st ; u]))), st = last K-1 input rows. */
int a8_ups_dwln(const void* u, int T, int C, void* st, long long st_bs, int K, const void* dww, const void* dwb,
                const void* lnw, const void* lnb, float eps, void* z, int rows, a8_stream_t stream);
/* Codec input (serve/fast_engine.py:472-477): x[r] = bf16(t_sem[clamp(codes[r,0])] + sum_k t_res[k, clamp(codes[r,k+1])])
 * (fp32 tables [v_sem, C] and [ncb-1, v_res, C]); pos_c[r] = min(pos[r], max_pos-1), lens[r] = min(pos[r]+1, window),
 * pos[r] += 1. */
int a8_codec_embed(const int64_t* codes, int ncb, const float* t_sem, int v_sem, const float* t_res, int v_res, int C,
                   void* x, int* pos, int* pos_c, int* lens, int max_pos, int window, int rows, a8_stream_t stream);

/* ---------------------------------------------------------------------------------------------- sampling */
/* out[r] = draw over logits[r, :V] (fp32): top-k (ties: lower index first), top-p on the untempered softmax (the best
 * candidate always kept), temperature, exponential race with E = -log(u), u from Philox4x32-10(key = seed,
 * counter = (i / 4, r, tick_id[0] (0 if NULL), stream_id)); do_sample = 0: argmax (first index).
 * Replaces _Sampler (serve/fast_engine.py:141-172). */
int a8_sample(const float* logits, int ld, int V, int rows, int do_sample, int top_k, float top_p, float temperature,
              unsigned long long seed, int stream_id, const long long* tick_id, int64_t* out, a8_stream_t stream);

/* ---------------------------------------------------------------------------------------------- stacks */
typedef struct A8Scratch {
  void* h;              /* bf16 [rows, dim]: normed activations; after a stack forward, its final-normed output */
  void* q;              /* bf16 [rows, nq * hd] */
  void* o;              /* bf16 [rows, nq * hd] */
  void* a;              /* bf16 [rows, dim] */
  void* mlp;            /* bf16 [rows, inter] */
  float* attn_ws;       /* attention split partials (a8_attention_workspace) */
  long long attn_ws_floats;
  int* attn_counters;   /* zeroed once */
  int n_attn_counters;
  float* ssq;           /* [8, ssq_ld]: per-row sums of squares of the residual stream, one partial per 128 columns */
  int ssq_ld;           /* rows the partials hold (>= the rows of any call) */
} A8Scratch;

/* A transformer stack on packed weights (serve/fast_engine.py:82-115): q / k rows of wqkv permuted per head for
 * rotate_half, w13 = gate and up rows interleaved per 64 (rows 128t..128t+63 = w1[64t..], +64..+127 = w3[64t..]),
 * LayerScale folded into wo / w2 where the model has one. */
typedef struct A8StackDesc {
  int layers, dim, nq, nkv, hd, inter;
  float eps;
  const void* wqkv;     /* bf16 [layers, (nq + 2 nkv) hd, dim] */
  const void* bqkv;     /* bf16 [layers, (nq + 2 nkv) hd] or NULL */
  const void* wo;       /* bf16 [layers, dim, nq hd] */
  const void* w13;      /* bf16 [layers, 2 inter, dim] */
  const void* w2;       /* bf16 [layers, dim, inter] */
  const void* ln1;      /* bf16 [layers, dim] */
  const void* ln2;      /* bf16 [layers, dim] */
  const void* norm;     /* bf16 [dim] */
  const void* cos;      /* bf16 [npos, hd] */
  const void* sin;      /* bf16 [npos, hd] */
  void* kc;             /* bf16 [layers, cache_rows, nkv, cache_len, hd] */
  void* vc;
  int cache_rows, cache_len, ring;   /* ring 0: positions stored at pos, else at pos % ring */
} A8StackDesc;

typedef struct A8StackRun {
  void* x;              /* bf16 [rows, ldx] input rows, consumed as the residual stream (updated in place) */
  int ldx;
  int rows;
  const int* pos;       /* int32 [rows] RoPE position */
  const int* slot;      /* int32 [rows] cache row the K/V go to (NULL: the row index) */
  const int* lens;      /* int32 [rows] keys attended (NULL: pos + 1) */
  int lens_max;         /* clamp of the keys attended (0: cache_len) */
  const int* rowmap;    /* int32 [rows] cache row attended (NULL: the row index) */
  int max_len;          /* bound of any row's keys (0: cache_len); sets the split count */
  A8Scratch scratch;    /* output in scratch.h */
  const int* blocks;    /* packed causal prefill (hd 64): int32 [nblocks][4] query blocks as a8_prefill_attention
                           (pos / slot must agree); NULL: every row by the decode attention */
  int nblocks;
} A8StackRun;

/* _Stack.forward (serve/fast_engine.py:117-138): decode rows or packed causal prefill rows. */
int a8_stack_forward(const A8StackDesc* d, const A8StackRun* r, a8_stream_t stream);

/* ---------------------------------------------------------------------------------------------- streaming codec */
/* One conv of the decoder program. Its input rows xin (context first, persistent across frames) are written by the
 * previous op's epilogue with this op's activation; the first op's by a8_conv_input from the upsample output; the last
 * op writes audio. */
typedef struct A8ConvOp {
  const void* w;          /* fp16 [N, taps * Cin] */
  const float* bias;      /* [N] (the fp16 bias as fp32) or NULL */
  const float* alpha;     /* the snake in front of this conv: alpha [Cin] or NULL (no activation) */
  const float* inv;       /* 1 / (alpha + 1e-9) [Cin] */
  void* xin;              /* fp16 [slot rows, ctx + T, Cin] */
  int Cin, N, taps, dil, ctx;
  int T;                  /* input timesteps a frame */
  int raw;                /* act buffer receiving the raw output (a later residual), or -1 */
  int res;                /* act buffer added to the output, or -1 */
} A8ConvOp;

/* One upsample stage ([transposed conv k = s = 2 as a GEMM, causal ConvNeXt block], serve/fast_engine.py:479-491). */
typedef struct A8Upsample {
  const void* tw;         /* bf16 [2C, C]: rows [0, C) phase 0, [C, 2C) phase 1 */
  const void* tb;         /* bf16 [2C] */
  const void* dww;        /* bf16 [K, C] depthwise taps */
  const void* dwb;        /* bf16 [C] */
  void* st;               /* bf16 carried tail [slot rows, K - 1, C] at st_bs elements a row */
  long long st_bs;
  int K;
  float eps;
  const void* lnw;        /* bf16 [C] */
  const void* lnb;
  const void* w1;         /* bf16 [mlp, C] */
  const void* b1;
  const void* w2;         /* bf16 [C, mlp] */
  const void* b2;
  const void* gamma;      /* bf16 [C] */
  int mlp;
} A8Upsample;

#define A8_MAX_UPS 4
#define A8_MAX_CONV_OPS 40

typedef struct A8Vocoder {
  int B;                  /* slot rows */
  int ncb, C, v_sem, v_res, max_pos, window, up;
  const float* t_sem;     /* fp32 [v_sem, C] code table of the semantic codebook (out_proj folded in) */
  const float* t_res;     /* fp32 [ncb - 1, v_res, C] */
  int* pos;               /* [B] frames decoded per row */
  int* pos_c;             /* [B] scratch: this frame's RoPE position */
  int* lens;              /* [B] scratch: keys attended */
  void* x;                /* bf16 [B, C] scratch: the transformer's input rows */
  A8StackDesc post;       /* window transformer (ring = window) */
  A8Scratch scratch;      /* for B rows */
  int n_ups;
  A8Upsample ups[A8_MAX_UPS];
  void* ubuf[4];          /* bf16 scratch: [B * 2^n_ups, C] x3 and [B * 2^n_ups, mlp] */
  int n_ops;
  A8ConvOp ops[A8_MAX_CONV_OPS];
  void* act[2];           /* fp16 scratch for raw outputs: each the largest [B, T, N] of the program */
  const A8CtxShift* ctx_table; /* device table of the ops with a context (a8_ctx_shift after the step) */
  int n_ctx;
  int conv_ctas;          /* persistent CTAs of each decoder conv (0: one per SM); fewer leave SMs to the tick's
                             other stream */
  float* audio;           /* fp32 [B, up] */
} A8Vocoder;

/* StreamingVocoder.step (serve/fast_engine.py:470-494): one codec frame for rows [0, b): codes [b, ncb] (int64, row
 * stride ncb) -> audio [b, up]; every row's carried state advances one frame. */
int a8_voc_step(const A8Vocoder* v, const int64_t* codes, int b, a8_stream_t stream);
/* The conv decoder part of the step alone (serve/fast_engine.py:301-309 _CLDecoder.__call__): u bf16 [b, T0, C]
 * (T0 = ops[0].T) -> audio [b, up]; every conv context advances one frame. */
int a8_voc_decode(const A8Vocoder* v, const void* u, int b, a8_stream_t stream);

/* A piece of per-slot state: for every slot, nchunks chunks of chunk_bytes at base + slot * slot_stride +
 * k * chunk_stride (addresses and sizes multiples of 4 bytes; 16 for the vector path); in a snapshot it sits at
 * blob_off (the blob 16-byte aligned). */
typedef struct A8StateSeg {
  void* base;
  long long slot_stride, chunk_bytes, chunk_stride;
  int nchunks;
  long long blob_off;
} A8StateSeg;

enum { A8_STATE_CLEAR = 0, A8_STATE_LOAD = 1, A8_STATE_SNAPSHOT = 2 };

/* The vocoder's row-state arena (serve/fast_engine.py:368-393 _arena_init, :453-468 snapshot / load_many / clear /
 * clear_many) as one launch over a segment table in device memory: CLEAR zeroes the state of slots[0..nslots),
 * LOAD copies the snapshot blob into each of them, SNAPSHOT copies slot slots[0] into the blob. */
int a8_state_rows(const A8StateSeg* segs, int nseg, const int* slots, int nslots, int op, void* blob,
                  a8_stream_t stream);

/* ---------------------------------------------------------------------------------------------- resampler */
/* Per-slot streaming rate conversion of the codec's audio (native rate -> out rate, e.g. 44.1 -> 16 kHz) and PCM16,
 * replacing the worker's post-processing per request (serve/engine_worker.py:443-449 soxr.ResampleStream(native_sr,
 * out_sr, 1, dtype="float32"), :460-461 resample_chunk(y, last=final), :423-424 _pcm16). A linear-phase FIR h of
 * odd length L = 2 half + 1 at the up-sampled rate: output n = sum_k table[k][p] x[m - k] with q = n down + half,
 * m = q / up, p = q % up and x beyond the input zero; the output is delay-compensated (output 0 is centred on input
 * 0) and a stream of N inputs yields ceil(N up / down) outputs in all. */
typedef struct A8Resample {
  const float* table;     /* [taps, up]: table[k][p] = up * h[p + k up] (0 past L) */
  float* hist;            /* [rows, hist_len] the last hist_len input samples of each slot */
  long long* n_in;        /* [rows] input samples taken so far */
  long long* n_out;       /* [rows] output samples given so far */
  int* left;              /* [rows] frames the slot still takes (its frame cap) */
  int* flags;             /* [rows] bit 0: drop the next frame (the silence frame); bit 1: stream ended */
  int up, down, taps, hist_len, zpad, frame, rows, out_max, period;
  long long half;
} A8Resample;

/* Start a stream in each of slots[0, n) (int32, device): history zeroed, counters 0, `caps[i]` (int32, device)
 * frames, the first frame dropped when drop_first (the frame a fresh slot decodes from the silence frame). */
int a8_resample_reset(const A8Resample* d, const int* slots, const int* caps, int n, int drop_first,
                      a8_stream_t stream);

/* One frame for slot rows [0, b): audio fp32 [b, ld_audio] (frame samples a row), tok_in int64 [b] = the token each
 * row consumed this tick. A live row takes its frame; when it consumed `eos` or used its last capped frame the frame
 * is its last and the stream is flushed (zeros past the end). counts[r] = outputs written this step: pcm int16
 * [b, ld_out] (clip to [-1, 1], x 32767, truncated) and, when f32 is not NULL, the fp32 samples [b, ld_out]. Rows
 * whose stream ended, and a dropped frame, give 0 outputs. */
int a8_resample_step(const A8Resample* d, const float* audio, int ld_audio, const int64_t* tok_in, long long eos,
                     int b, int16_t* pcm, float* f32, int ld_out, int* counts, a8_stream_t stream);

/* ---------------------------------------------------------------------------------------------- engine */
typedef struct A8Engine {
  int B, S, H, ncb, cbk, nsem, vocab, ras_w;
  long long eos, sb;
  int do_sample, top_k;
  float top_p, temperature, ras_top_p, ras_temperature;
  unsigned long long seed;
  A8StackDesc slow, fast;
  const void* emb;        /* bf16 [vocab, H] */
  const void* cbemb;      /* bf16 [ncb cbk, H] */
  const void* head;       /* bf16 [nsem + 1, H]: semantic rows then EOS */
  const void* fast_emb;   /* bf16 [cbk, H] */
  const void* fast_out;   /* bf16 [cbk, H] */
  /* slot state (fixed addresses; rows >= B are scratch) */
  int64_t* tok;           /* [B + 1] */
  void* hid;              /* bf16 [B + 1, H] */
  int* cpos;              /* [B + 1] */
  int64_t* prev;          /* [B + 1, ras_w] */
  int* nstep;             /* [B + 1] */
  int64_t* tok_in;        /* [B] */
  int64_t* frame_prev;    /* [B, ncb] */
  const int64_t* sil_frame; /* [ncb] */
  long long* tick_ctr;    /* [1] ticks run so far (the sampling noise's tick counter) */
  long long* tick_id;     /* [1] */
  /* tick scratch */
  void* x_fast2;          /* bf16 [2B, H] */
  void* x_fast;           /* bf16 [B, H] */
  void* x_slow;           /* bf16 [B, H] */
  int64_t* codes;         /* [B, ncb] */
  float* logits;          /* [B, ld_logits] */
  int ld_logits;
  const int* f_pos;       /* int32 [ncb, 2B]: row i all equal to i */
  const int* f_pos0;      /* int32 [2B]: r % 2 */
  const int* f_slot0;     /* int32 [2B]: r / 2 */
  A8Scratch scratch;      /* for 2B rows */
  const A8Vocoder* voc;   /* host descriptor of the codec (NULL: the tick makes no audio) */
  a8_stream_t side;       /* the codec's stream (not the tick's) */
  float* rec_logits;      /* NULL, or fp32 [ncb - 1, B, ld_logits]: codebook i's logits (i = 1 .. ncb-1) are written
                             to slice i - 1 instead of `logits` and drawn from there, so they stay readable after the
                             tick (a diagnostic; no extra work) */
} A8Engine;

/* One frame for slot rows [0, b): fast AR (2-token pass + ncb - 2 passes, each sampled), slow AR step, semantic
 * draw with RAS, state update; with a codec, audio[:b] = the codec step of the previous tick's frame_prev, run on the
 * side stream (forked from and joined back into `stream`). Replaces FastEngine._tick (serve/fast_engine.py:737-769).
 * The first call with a codec on a device creates the fork / join events: make it outside stream capture. */
int a8_tick(const A8Engine* e, int b, a8_stream_t stream);

/* The slow AR half of the tick for rows [0, b), reading tok_in and codes as left by the tick's first half: input
 * embedding, 24-layer step at positions cpos, semantic head, draw with RAS, state update
 * (serve/fast_engine.py:750-769). */
int a8_slow_step(const A8Engine* e, int b, a8_stream_t stream);

/* Admission tail for n requests (serve/fast_engine.py:1124-1133 and _pf_body :828-835): h_last bf16 [n, H] = each
 * request's final-normed last prompt row; first token drawn without the RAS window (noise stream 18 at the current
 * tick count), written with hid, cpos = cpos_new into slots[i]; prev and nstep of those slots cleared; with frame0
 * (int32 [n, ncb], or NULL) frame_prev[slots[i]] = frame0[i], the frame the slot's codec decodes first (:1138-1156).
 * A request aimed at slot B or beyond (a prefill graph's padding) draws and writes nothing. */
int a8_prefill_finish(const A8Engine* e, const void* h_last, int n, const int* slots, const int* cpos_new,
                      const int* frame0, a8_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* AUDIO8_B200_H */
