// The decode tick and the transformer stack forward, as sequences of the library's kernels on caller-owned memory.
// Mirrors serve/fast_engine.py: _Stack.forward (:117-138), FastEngine._fast_codes (:702-713), _embed (:715-717),
// _head (:719-721), _sample_sem (:726-735), _tick (:737-769), _pf_body (:820-835).
#include "common.cuh"

namespace a8 {

int attn_maps(CUtensorMap* mk, CUtensorMap* mv, const void* kc, const void* vc, long long total_rows, int hd);
int attn_launch(const CUtensorMap& mk, const CUtensorMap& mv, AttnArgs a, int hd, int group, cudaStream_t s);
int attn_splits(int rows, int nkv, int max_len);
long long attn_ws_floats(int rows, int nkv, int nsplit, int hd);
int sample_launch(const SampleArgs& a, int rows, cudaStream_t s);
int pattn_launch(const void* q, int q_stride, int rows, const CUtensorMap& mk, const CUtensorMap& mv,
                 const PattnArgs& a, int nblocks, cudaStream_t s);

#define A8_TRY(x)              \
  do {                         \
    int _rc = (x);             \
    if (_rc != A8_OK) return _rc; \
  } while (0)

static inline size_t bstride(const A8StackDesc& d, int which) {
  const size_t qkv = (size_t)(d.nq + 2 * d.nkv) * d.hd;
  switch (which) {
    case 0: return qkv * d.dim;                    // wqkv
    case 1: return qkv;                            // bqkv
    case 2: return (size_t)d.dim * d.nq * d.hd;    // wo
    case 3: return (size_t)2 * d.inter * d.dim;    // w13
    case 4: return (size_t)d.dim * d.inter;        // w2
    default: return (size_t)d.dim;                 // ln1 / ln2
  }
}
template <class T>
static inline const T* at(const void* base, size_t elems) {
  return reinterpret_cast<const T*>(base) + elems;
}

static int gemm(const void* x, int ldx, const void* w, int N, int K, int M, void* y, int ldy, const A8Epilogue& e,
                const A8Scratch& sc, cudaStream_t s) {
  GemmPlan p;
  (void)sc;
  A8_TRY(gemm_plan(&p, x, ldx, w, N, K, M, y, ldy, &e, 0));
  return gemm_launch(&p, s, true);
}

// _Stack.forward (serve/fast_engine.py:117-138). With the residual stream's sums of squares in scratch (the usual
// case: dim <= 1024), each layer is six launches -- qkv GEMM (the RMSNorm of the residual stream in its operand
// producer, bias + RoPE + KV store in its epilogue), attention, o GEMM, residual add + RMSNorm, w13 GEMM (SiLU * up in
// the epilogue), w2 GEMM (residual add + the rows' sums of squares in its epilogue) -- plus one RMSNorm launch at each
// end of the stack: the first layer's input and the final-normed output in scratch.h. The w13 GEMM keeps the separate
// RMSNorm: its 76 weight tiles would each normalise the same rows (measured slower than the launch it saves).
// Otherwise every norm is its own launch (seven a layer), with the same arithmetic.
int stack_forward(const A8StackDesc& d, const A8StackRun& r, cudaStream_t s) {
  const int R = r.rows, D = d.dim, QW = d.nq * d.hd, NQKV = (d.nq + 2 * d.nkv) * d.hd;
  const A8Scratch& sc = r.scratch;
  __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(sc.h);
  __nv_bfloat16* q = reinterpret_cast<__nv_bfloat16*>(sc.q);
  __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(sc.o);
  __nv_bfloat16* a = reinterpret_cast<__nv_bfloat16*>(sc.a);
  __nv_bfloat16* m = reinterpret_cast<__nv_bfloat16*>(sc.mlp);
  void* res = r.x;
  const bool fuse = sc.ssq != nullptr && sc.ssq_ld >= R && D <= 1024 && D % 64 == 0;
  a8_stream_t st = reinterpret_cast<a8_stream_t>(s);
  A8_TRY(a8_rmsnorm(r.x, r.ldx, nullptr, 0, d.ln1, h, D, R, D, d.eps, st));
  CUtensorMap mk, mv;
  const long long total = (long long)d.layers * d.cache_rows * d.nkv * d.cache_len;
  A8_TRY(attn_maps(&mk, &mv, d.kc, d.vc, total, d.hd));
  const int max_len = r.max_len > 0 ? r.max_len : d.cache_len;
  // packed prefill rows with a query-block table go to the tensor-core prefill attention
  const bool packed = r.blocks != nullptr && r.nblocks > 0 && d.hd == 64 && d.nq / d.nkv <= 8;
  const int ms = packed ? 1 : attn_splits(R, d.nkv, max_len);
  if (ms > 1 && (sc.attn_ws == nullptr || sc.attn_ws_floats < attn_ws_floats(R, d.nkv, ms, d.hd) ||
                 sc.attn_counters == nullptr || sc.n_attn_counters < R * d.nkv))
    return A8_ERR_SIZE;
  // an operand normalised in the GEMM's producer: the residual rows with norm weight w (RMSNorm of the stream)
  auto normed = [&](A8Epilogue& e, const void* w) {
    e.norm_w = w;
    e.ssq_in = sc.ssq;
    e.ssq_ld = sc.ssq_ld;
    e.eps = d.eps;
  };
  // the residual add of rmsnorm in the epilogue, in place on the stream, with the rows' sums of squares
  A8Epilogue resid = {};
  resid.kind = A8_EPI_RESID;
  resid.res = res;
  resid.ldres = r.ldx;
  resid.ssq_out = sc.ssq;
  resid.ssq_ld = sc.ssq_ld;
  for (int l = 0; l < d.layers; ++l) {
    const bool in_h = !fuse || l == 0;          // the layer's normed input is already in h
    A8Epilogue e = {};
    e.kind = A8_EPI_ROPE;
    e.bias = d.bqkv != nullptr ? at<__nv_bfloat16>(d.bqkv, l * bstride(d, 1)) : nullptr;
    e.cos = d.cos;
    e.sin = d.sin;
    e.pos = r.pos;
    e.slot = r.slot;
    e.kc = reinterpret_cast<__nv_bfloat16*>(d.kc) + (size_t)l * d.cache_rows * d.nkv * d.cache_len * d.hd;
    e.vc = reinterpret_cast<__nv_bfloat16*>(d.vc) + (size_t)l * d.cache_rows * d.nkv * d.cache_len * d.hd;
    e.nq = d.nq;
    e.nkv = d.nkv;
    e.hd = d.hd;
    e.ring = d.ring > 0 ? d.ring : (1 << 30);
    e.cache_len = d.cache_len;
    if (!in_h) normed(e, at<__nv_bfloat16>(d.ln1, l * bstride(d, 5)));
    A8_TRY(gemm(in_h ? (const void*)h : r.x, in_h ? D : r.ldx, at<__nv_bfloat16>(d.wqkv, l * bstride(d, 0)), NQKV, D,
                R, q, QW, e, sc, s));
    AttnArgs aa = {};
    aa.q = q;
    aa.q_stride = QW;
    aa.nq = d.nq;
    aa.nkv = d.nkv;
    aa.lens = r.lens != nullptr ? r.lens : r.pos;
    aa.lens_add = r.lens != nullptr ? 0 : 1;
    aa.lens_max = r.lens_max > 0 ? r.lens_max : d.cache_len;
    aa.rowmap = r.rowmap;
    aa.cache_rows_per_layer_head = d.cache_len;
    aa.layer_base = (long long)l * d.cache_rows * d.nkv * d.cache_len;
    aa.nsplit = ms;
    aa.scale_log2 = (1.0f / sqrtf((float)d.hd)) * 1.4426950408889634f;
    aa.out = o;
    aa.out_stride = QW;
    aa.ws = sc.attn_ws;
    aa.counters = sc.attn_counters;
    aa.rows = R;
    if (packed) {
      PattnArgs pa = {};
      pa.blocks = r.blocks;
      pa.nq = d.nq;
      pa.nkv = d.nkv;
      pa.group = d.nq / d.nkv;
      pa.cache_len = d.cache_len;
      pa.layer_base = aa.layer_base;
      pa.scale_log2 = aa.scale_log2;
      pa.out = o;
      pa.out_stride = QW;
      pa.rows = R;
      A8_TRY(pattn_launch(q, QW, R, mk, mv, pa, r.nblocks, s));
    } else {
      A8_TRY(attn_launch(mk, mv, aa, d.hd, d.nq / d.nkv, s));
    }
    A8Epilogue plain = {};
    plain.kind = A8_EPI_BF16;
    A8Epilogue silu = {};
    silu.kind = A8_EPI_SILU;
    const void* w13 = at<__nv_bfloat16>(d.w13, l * bstride(d, 3));
    const void* w2 = at<__nv_bfloat16>(d.w2, l * bstride(d, 4));
    if (fuse) {
      A8_TRY(gemm(o, QW, at<__nv_bfloat16>(d.wo, l * bstride(d, 2)), D, QW, R, a, D, plain, sc, s));
      A8_TRY(a8_rmsnorm(a, D, res, r.ldx, at<__nv_bfloat16>(d.ln2, l * bstride(d, 5)), h, D, R, D, d.eps, st));
      A8_TRY(gemm(h, D, w13, 2 * d.inter, D, R, m, d.inter, silu, sc, s));
      A8_TRY(gemm(m, d.inter, w2, D, d.inter, R, res, r.ldx, resid, sc, s));
    } else {
      A8_TRY(gemm(o, QW, at<__nv_bfloat16>(d.wo, l * bstride(d, 2)), D, QW, R, a, D, plain, sc, s));
      A8_TRY(a8_rmsnorm(a, D, res, r.ldx, at<__nv_bfloat16>(d.ln2, l * bstride(d, 5)), h, D, R, D, d.eps, st));
      A8_TRY(gemm(h, D, w13, 2 * d.inter, D, R, m, d.inter, silu, sc, s));
      A8_TRY(gemm(m, d.inter, w2, D, d.inter, R, a, D, plain, sc, s));
      // the next layer's normed input (or, after the last layer, the stack's final-normed output) goes to h
      const void* nxt = l + 1 < d.layers ? at<__nv_bfloat16>(d.ln1, (l + 1) * bstride(d, 5)) : d.norm;
      A8_TRY(a8_rmsnorm(a, D, res, r.ldx, nxt, h, D, R, D, d.eps, st));
    }
  }
  if (fuse) A8_TRY(a8_rmsnorm(r.x, r.ldx, nullptr, 0, d.norm, h, D, R, D, d.eps, st));   // the final norm
  return A8_OK;
}

}  // namespace a8

using namespace a8;

namespace a8 {

static SampleArgs sample_base(const A8Engine& e) {
  SampleArgs sa = {};
  sa.do_sample = e.do_sample;
  sa.p = e.top_p;
  sa.t = fmaxf(e.temperature, 1e-5f);
  sa.seed = e.seed;
  sa.tick_id = e.tick_id;
  sa.H = e.H;
  sa.ncb = e.ncb;
  sa.eos = e.eos;
  sa.sb = e.sb;
  sa.nsem = e.nsem;
  sa.ras_w = e.ras_w;
  return sa;
}

static int fast_logits_and_draw(const A8Engine& e, const void* h, int ldh, int b, int i, bool next, cudaStream_t s) {
  A8Epilogue lg = {};
  lg.kind = A8_EPI_F32_ROUND;
  float* logits = e.rec_logits != nullptr ? e.rec_logits + (size_t)(i - 1) * e.B * e.ld_logits : e.logits;
  A8_TRY(gemm(h, ldh, e.fast_out, e.cbk, e.H, b, logits, e.ld_logits, lg, e.scratch, s));
  SampleArgs sa = sample_base(e);
  sa.logits = logits;
  sa.ld = e.ld_logits;
  sa.V = e.cbk;
  sa.k = (e.top_k > 0 && e.top_k < e.cbk) ? e.top_k : e.cbk;
  sa.mode = SM_CODEBOOK;
  sa.stream1 = i;                      // codebook i's noise stream
  sa.codes = e.codes;
  sa.cb_index = i;
  sa.fast_emb = reinterpret_cast<const __nv_bfloat16*>(e.fast_emb);
  sa.x_next = next ? reinterpret_cast<__nv_bfloat16*>(e.x_fast) : nullptr;
  sa.ldx = e.H;
  return sample_launch(sa, b, s);
}

int fast_ar(const A8Engine& e, int b, cudaStream_t s) {
  const int H = e.H;
  // positions 0 and 1 in one 2-token pass (cache row = row / 2)
  A8StackRun r = {};
  r.x = e.x_fast2;
  r.ldx = H;
  r.rows = 2 * b;
  r.pos = e.f_pos0;
  r.slot = e.f_slot0;
  r.rowmap = e.f_slot0;
  r.max_len = 2;
  r.scratch = e.scratch;
  A8_TRY(stack_forward(e.fast, r, s));
  const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(e.scratch.h);
  A8_TRY(fast_logits_and_draw(e, h + H, 2 * H, b, 1, true, s));
  for (int i = 2; i < e.ncb; ++i) {
    A8StackRun ri = {};
    ri.x = e.x_fast;
    ri.ldx = H;
    ri.rows = b;
    ri.pos = e.f_pos + (size_t)i * 2 * e.B;
    ri.max_len = i + 1;
    ri.scratch = e.scratch;
    A8_TRY(stack_forward(e.fast, ri, s));
    A8_TRY(fast_logits_and_draw(e, e.scratch.h, H, b, i, i + 1 < e.ncb, s));
  }
  return A8_OK;
}

int slow_step(const A8Engine& e, int b, cudaStream_t s) {
  const int H = e.H;
  A8_TRY(a8_embed_frame(e.tok_in, e.codes, e.ncb, e.cbk, e.emb, e.cbemb, e.x_slow, H, b, H, e.vocab,
                        reinterpret_cast<a8_stream_t>(s)));
  A8StackRun rs = {};
  rs.x = e.x_slow;
  rs.ldx = H;
  rs.rows = b;
  rs.pos = e.cpos;
  rs.max_len = e.S;
  rs.scratch = e.scratch;
  A8_TRY(stack_forward(e.slow, rs, s));
  A8Epilogue lg = {};
  lg.kind = A8_EPI_F32_ROUND;
  A8_TRY(gemm(e.scratch.h, H, e.head, e.nsem + 1, H, b, e.logits, e.ld_logits, lg, e.scratch, s));
  SampleArgs sa = sample_base(e);
  sa.logits = e.logits;
  sa.ld = e.ld_logits;
  sa.V = e.nsem + 1;
  sa.k = (e.top_k > 0 && e.top_k < sa.V) ? e.top_k : sa.V;
  sa.mode = SM_SEMANTIC;
  sa.p2 = e.ras_top_p;
  sa.t2 = fmaxf(e.ras_temperature, 1e-5f);
  sa.stream1 = 16;
  sa.stream2 = 17;
  sa.codes = e.codes;
  sa.tok_in = e.tok_in;
  sa.tok = e.tok;
  sa.prev = e.prev;
  sa.nstep = e.nstep;
  sa.cpos = e.cpos;
  sa.S = e.S;
  sa.h_src = reinterpret_cast<const __nv_bfloat16*>(e.scratch.h);
  sa.ldh = H;
  sa.hid = reinterpret_cast<__nv_bfloat16*>(e.hid);
  sa.frame_prev = e.frame_prev;
  sa.sil_frame = e.sil_frame;
  return sample_launch(sa, b, s);
}

// Events of the tick's fork / join with the codec's stream, one set per device (created at the first tick with a
// codec, which must run outside stream capture; a captured graph keeps only the dependencies they express).
struct TickEvents {
  cudaEvent_t fork = nullptr, read = nullptr, join = nullptr;
};
static int tick_events(TickEvents** out) {
  static TickEvents ev[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return A8_ERR_CUDA;
  TickEvents& t = ev[dev];
  if (t.fork == nullptr) {
    if (cudaEventCreateWithFlags(&t.fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&t.read, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&t.join, cudaEventDisableTiming) != cudaSuccess)
      return A8_ERR_CUDA;
  }
  *out = &t;
  return A8_OK;
}

// FastEngine._tick (serve/fast_engine.py:737-769): the codec decodes the PREVIOUS tick's frame (frame_prev) on the
// side stream while this stream runs the fast AR and the slow step; the semantic draw, which rewrites frame_prev,
// waits until the codec has read it, and the tick ends when both streams have.
int tick(const A8Engine& e, int b, cudaStream_t s) {
  A8_TRY(a8_tick_start(e.tok, e.tok_in, e.codes, e.ncb, e.sb, e.cbk, e.hid, e.fast_emb, e.x_fast2, b, e.H,
                       e.tick_ctr, e.tick_id, reinterpret_cast<a8_stream_t>(s)));
  TickEvents* ev = nullptr;
  const bool codec = e.voc != nullptr;
  cudaStream_t side = reinterpret_cast<cudaStream_t>(e.side);
  if (codec) {
    if (side == nullptr || side == s) return A8_ERR_ARG;
    A8_TRY(tick_events(&ev));
    if (cudaEventRecord(ev->fork, s) != cudaSuccess || cudaStreamWaitEvent(side, ev->fork, 0) != cudaSuccess)
      return A8_ERR_CUDA;
    A8_TRY(voc_step(*e.voc, e.frame_prev, b, side, ev->read));
    if (cudaEventRecord(ev->join, side) != cudaSuccess) return A8_ERR_CUDA;
  }
  A8_TRY(fast_ar(e, b, s));
  if (codec && cudaStreamWaitEvent(s, ev->read, 0) != cudaSuccess) return A8_ERR_CUDA;
  A8_TRY(slow_step(e, b, s));
  if (codec && cudaStreamWaitEvent(s, ev->join, 0) != cudaSuccess) return A8_ERR_CUDA;
  return A8_OK;
}

// Admission tail (serve/fast_engine.py:1124-1133, :828-835): logits of each request's last prompt row -> its first
// token (no RAS window), hidden, position; RAS window and step count cleared.
int prefill_finish(const A8Engine& e, const void* h_last, int n, const int* slots, const int* cpos_new,
                   const int* frame0, cudaStream_t s) {
  A8Epilogue lg = {};
  lg.kind = A8_EPI_F32_ROUND;
  A8_TRY(gemm(h_last, e.H, e.head, e.nsem + 1, e.H, n, e.logits, e.ld_logits, lg, e.scratch, s));
  SampleArgs sa = sample_base(e);
  sa.logits = e.logits;
  sa.ld = e.ld_logits;
  sa.V = e.nsem + 1;
  sa.k = (e.top_k > 0 && e.top_k < sa.V) ? e.top_k : sa.V;
  sa.mode = SM_PREFILL;
  sa.stream1 = 18;
  sa.tok = e.tok;
  sa.prev = e.prev;
  sa.nstep = e.nstep;
  sa.cpos = e.cpos;
  sa.h_src = reinterpret_cast<const __nv_bfloat16*>(h_last);
  sa.ldh = e.H;
  sa.hid = reinterpret_cast<__nv_bfloat16*>(e.hid);
  sa.st = slots;
  sa.cpos_new = cpos_new;
  sa.frame0 = frame0;
  sa.frame_prev = e.frame_prev;
  sa.B = e.B;
  sa.tick_id = e.tick_ctr;            // draws between ticks use the count of ticks run so far
  return sample_launch(sa, n, s);
}

}  // namespace a8

extern "C" int a8_tick(const A8Engine* e, int b, a8_stream_t stream) {
  if (e == nullptr || b <= 0 || b > e->B) return A8_ERR_ARG;
  return tick(*e, b, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int a8_slow_step(const A8Engine* e, int b, a8_stream_t stream) {
  if (e == nullptr || b <= 0 || b > e->B) return A8_ERR_ARG;
  return slow_step(*e, b, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int a8_prefill_finish(const A8Engine* e, const void* h_last, int n, const int* slots, const int* cpos_new,
                                 const int* frame0, a8_stream_t stream) {
  if (e == nullptr || h_last == nullptr || slots == nullptr || cpos_new == nullptr || n <= 0) return A8_ERR_ARG;
  return prefill_finish(*e, h_last, n, slots, cpos_new, frame0, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int a8_stack_forward(const A8StackDesc* d, const A8StackRun* r, a8_stream_t stream) {
  if (d == nullptr || r == nullptr || r->x == nullptr || r->pos == nullptr || r->rows <= 0) return A8_ERR_ARG;
  if (d->layers <= 0 || d->dim <= 0 || d->dim > 1024 || d->nkv <= 0 || d->nq % d->nkv) return A8_ERR_ARG;
  return stack_forward(*d, *r, reinterpret_cast<cudaStream_t>(stream));
}
