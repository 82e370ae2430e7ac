"""Kernel parity on the GPU, through the C ABI, against the CPU oracle (oracle/ref_cpu.py) on seeded inputs.

Tolerances: results stored in bf16 may differ from the oracle by the rounding of a differently ordered fp32 sum:
a GEMM output within 1 bf16 ulp almost everywhere (checked as max relative error <= 1e-2 and >= 97% bit-equal),
attention (bf16 softmax weights in the tensor-core P.V) within 1e-2 relative; the sampler is bit-exact.
"""
import ctypes as C

import pytest
import torch

from oracle import ref_cpu as R

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


@pytest.fixture(scope="module")
def L(a8):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    a8.load()
    a8._lib.call("a8_clear_error")
    return a8._lib


@pytest.fixture(scope="module")
def ws():
    return (torch.zeros(1 << 25, dtype=torch.float32, device="cuda"), torch.zeros(1 << 15, dtype=torch.int32,
                                                                                  device="cuda"))


def rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp(min=1e-6))


def frac_equal(a, b):
    return float((a.float().cpu() == b.float().cpu()).float().mean())


def gemm(L, ws, x, w, y, epi, splits=0, ldy=None):
    M, K = x.shape
    N = w.shape[0]
    L.call("a8_gemm", L.ptr(x), x.stride(0), L.ptr(w), N, K, M, L.ptr(y), ldy or y.stride(0), C.byref(epi), splits,
           L.stream_handle())
    torch.cuda.synchronize()
    assert L.device_error()[0] == 0, L.device_error()


def rnd(g, *shape, scale=1.0):
    return (torch.randn(*shape, generator=g) * scale).to(BF)


@pytest.mark.parametrize("M,N,K,splits", [(1, 1152, 896, 0), (3, 896, 896, 1), (17, 896, 4864, 0),
                                          (64, 4160, 896, 0), (192, 9728, 896, 0), (300, 896, 4864, 0),
                                          (64, 896, 4864, 5), (2048, 1024, 1024, 0), (130, 4097, 896, 3),
                                          # several token tiles whose width is not a multiple of 32 (a tile's last
                                          # 32-column chunk reaches into the next tile's tokens)
                                          (280, 896, 896, 2), (280, 896, 4864, 0), (223, 1152, 896, 0),
                                          (1000, 896, 896, 0), (1024, 4097, 896, 0), (720, 896, 4864, 0)])
def test_gemm_bf16(L, ws, M, N, K, splits):
    g = torch.Generator().manual_seed(M * 7 + N)
    x, w = rnd(g, M, K), rnd(g, N, K, scale=K ** -0.5)
    ref = R.linear(x.float(), w.float())
    y = torch.zeros(M, N, dtype=BF, device="cuda")
    gemm(L, ws, x.cuda(), w.cuda(), y, L.A8Epilogue(kind=L.EPI_BF16), splits)
    assert rel(y, ref) < 1e-2 and frac_equal(y, ref) > 0.97, (rel(y, ref), frac_equal(y, ref))


def test_gemm_bias_gelu_lsres_f32(L, ws):
    g = torch.Generator().manual_seed(11)
    M, N, K = 37, 4096, 1024
    x, w, b = rnd(g, M, K), rnd(g, N, K, scale=K ** -0.5), rnd(g, N, scale=0.1)
    acc = x.float() @ w.float().t()
    # bias
    y = torch.zeros(M, N, dtype=BF, device="cuda")
    bc = b.cuda()
    gemm(L, ws, x.cuda(), w.cuda(), y, L.A8Epilogue(kind=L.EPI_BF16, bias=L.ptr(bc)))
    ref = R.bf(acc + b.float())
    assert rel(y, ref) < 1e-2 and frac_equal(y, ref) > 0.97
    # gelu(bf16(acc + b)) (ConvNeXt pwconv1)
    gemm(L, ws, x.cuda(), w.cuda(), y, L.A8Epilogue(kind=L.EPI_GELU, bias=L.ptr(bc)))
    ref = R.bf(torch.nn.functional.gelu(R.bf(acc + b.float())))
    assert rel(y, ref) < 1e-2 and frac_equal(y, ref) > 0.97
    # layer-scale residual: bf16(res + bf16(gamma * bf16(acc + b)))
    gam, res = rnd(g, N, scale=0.2).cuda(), rnd(g, M, N).cuda()
    gemm(L, ws, x.cuda(), w.cuda(), y, L.A8Epilogue(kind=L.EPI_LSRES, bias=L.ptr(bc), gamma=L.ptr(gam),
                                                   res=L.ptr(res), ldres=N))
    ref = R.bf(res.float().cpu() + R.bf(gam.float().cpu() * R.bf(acc + b.float())))
    assert rel(y, ref) < 1e-2 and frac_equal(y, ref) > 0.97
    # fp32 copy of the bf16-rounded result (logits), odd N with a padded row stride
    N2 = 4097
    w2 = rnd(g, N2, K, scale=K ** -0.5)
    lg = torch.full((M, 4100), 7.0, device="cuda")
    gemm(L, ws, x.cuda(), w2.cuda(), lg, L.A8Epilogue(kind=L.EPI_F32_ROUND), ldy=4100)
    ref = R.linear(x.float(), w2.float())
    assert rel(lg[:, :N2], ref) < 1e-2 and frac_equal(lg[:, :N2], ref) > 0.97
    assert bool((lg[:, N2:] == 7.0).all())                       # nothing written past N


@pytest.mark.parametrize("M,D,splits", [(1, 896, 0), (64, 896, 0), (192, 896, 0), (223, 1024, 0), (384, 896, 3),
                                         (1000, 896, 0), (2048, 1024, 0)])
def test_gemm_resid_then_normed_operand(L, ws, M, D, splits):
    """The fused RMSNorm of the stacks: an A8_EPI_RESID GEMM adds its output to the residual stream in place and
    writes per-row sums of squares per 128 columns; the next GEMM normalises that stream in its operand producer.
    Against the oracle's linear + rmsnorm(residual) + linear (serve/fast_kernels.py:30-46)."""
    from audio8_b200.engine import interleave_w13
    g = torch.Generator().manual_seed(M + D)
    K1, I, eps = 896, 1024, 1e-6
    x, w = rnd(g, M, K1), rnd(g, D, K1, scale=K1 ** -0.5)
    res = rnd(g, M, D)
    lnw = (1.0 + 0.1 * torch.randn(D, generator=g)).to(BF)
    w1, w3 = rnd(g, I, D, scale=D ** -0.5), rnd(g, I, D, scale=D ** -0.5)
    # oracle
    a_o = R.linear(x.float(), w.float())
    h_o, r_o = R.rmsnorm(a_o, lnw.float(), eps, residual=res.float())
    y_o = R.silu_mul(torch.cat([R.linear(h_o, w1.float()), R.linear(h_o, w3.float())], -1))
    # device: residual add + partial sums of squares, then the normalised operand of the SiLU GEMM
    RS = res.cuda().contiguous()
    ssq = torch.full((8, M + 5), float("nan"), device="cuda")
    e1 = L.A8Epilogue(kind=L.EPI_RESID, res=L.ptr(RS), ldres=D, ssq_out=L.ptr(ssq), ssq_ld=M + 5)
    gemm(L, ws, x.cuda(), w.cuda(), RS, e1, splits)
    assert rel(RS, r_o) < 1e-2 and frac_equal(RS, r_o) > 0.97
    t = -(-D // 128)
    ss_ref = (RS.float().cpu() ** 2).view(M, t, 128).sum(-1).t()
    assert torch.allclose(ssq[:t, :M].cpu(), ss_ref, rtol=1e-5, atol=1e-5)
    LN = lnw.cuda()
    e2 = L.A8Epilogue(kind=L.EPI_SILU, norm_w=L.ptr(LN), ssq_in=L.ptr(ssq), ssq_ld=M + 5, eps=eps)
    y = torch.zeros(M, I, dtype=BF, device="cuda")
    gemm(L, ws, RS, interleave_w13(w1, w3).cuda(), y, e2, ldy=I)
    # the engine's own residual (bit-level differences in RS propagate), so compare against the oracle norm of RS
    h_e = R.rmsnorm(RS.float().cpu(), lnw.float(), eps)
    y_e = R.silu_mul(torch.cat([R.linear(h_e, w1.float()), R.linear(h_e, w3.float())], -1))
    assert rel(y, y_e) < 1e-2 and frac_equal(y, y_e) > 0.97, (rel(y, y_e), frac_equal(y, y_e))
    assert rel(y, y_o) < 2e-2


@pytest.mark.parametrize("layout", ["mixed", "long"])
def test_prefill_attention_blocks(L, layout):
    """a8_prefill_attention (tcgen05, query blocks of up to 64 rows) against the oracle's packed causal attention
    (serve/fast_kernels.py:296-332): requests continuing after a prefix already in their cache row, blocks shorter
    than 64 rows, a one-row request, a padding block (n = 0), GQA 14 / 2 at hd 64, layer 1 of 2."""
    g = torch.Generator().manual_seed(3 if layout == "mixed" else 4)
    nq, nkv, hd, S, layers, rows_c = 14, 2, 64, 2048, 2, 5
    reqs = [(1, 0, 70), (3, 150, 20), (0, 64, 133), (2, 500, 1), (4, 7, 64)] if layout == "mixed" else \
        [(2, 1900, 140), (0, 0, 300)]
    R_ = sum(n for _, _, n in reqs)
    q = rnd(g, R_, nq * hd)
    kc, vc = rnd(g, layers, rows_c, nkv, S, hd), rnd(g, layers, rows_c, nkv, S, hd)
    blocks, r0 = [], 0
    for slot, p0, n in reqs:
        blocks += [(r0 + a, min(64, n - a), slot, p0 + a) for a in range(0, n, 64)]
        r0 += n
    table = torch.tensor(blocks + [(0, 0, 0, 0)], dtype=torch.int32)
    ref = R.prefill_attention(q.float().view(R_, nq, hd), kc[1].float(), vc[1].float(), blocks)
    Q, KC, VC, T = q.cuda(), kc.cuda(), vc.cuda(), table.cuda()
    out = torch.full((R_, nq * hd), float("nan"), dtype=BF, device="cuda")
    L.call("a8_prefill_attention", L.ptr(Q), nq * hd, L.ptr(KC), L.ptr(VC), layers, rows_c, nq, nkv, hd, S, 1,
           L.ptr(T), T.shape[0], R_, 0.0, L.ptr(out), nq * hd, L.stream_handle())
    torch.cuda.synchronize()
    assert L.device_error()[0] == 0, L.device_error()
    assert not torch.isnan(out.float()).any()
    e = rel(out.view(R_, nq, hd), ref)
    assert e < 1e-2, e
    assert frac_equal(out.view(R_, nq, hd), ref) > 0.9


@pytest.mark.parametrize("M", [1, 64, 200, 223, 450])
def test_gemm_silu(L, ws, M):
    from audio8_b200.engine import interleave_w13
    g = torch.Generator().manual_seed(M)
    K, I = 896, 4864
    x = rnd(g, M, K)
    w1, w3 = rnd(g, I, K, scale=K ** -0.5), rnd(g, I, K, scale=K ** -0.5)
    ref = R.silu_mul(torch.cat([R.linear(x.float(), w1.float()), R.linear(x.float(), w3.float())], -1))
    y = torch.zeros(M, I, dtype=BF, device="cuda")
    gemm(L, ws, x.cuda(), interleave_w13(w1, w3).cuda(), y, L.A8Epilogue(kind=L.EPI_SILU), ldy=I)
    assert rel(y, ref) < 1e-2 and frac_equal(y, ref) > 0.97


@pytest.mark.parametrize("shape", ["slow", "codec"])
def test_gemm_rope_store(L, ws, shape):
    g = torch.Generator().manual_seed(5)
    if shape == "slow":
        nq, nkv, hd, D, ring, rows, clen, base, has_b = 14, 2, 64, 896, 1 << 30, 6, 300, 1e6, True
    else:
        nq, nkv, hd, D, ring, rows, clen, base, has_b = 8, 8, 128, 1024, 128, 5, 128, 1e4, False
    M = 9
    N = (nq + 2 * nkv) * hd
    x, w = rnd(g, M, D), rnd(g, N, D, scale=D ** -0.5)
    b = rnd(g, N, scale=0.3) if has_b else None
    npos = 700 if ring < clen * 2 else clen
    cos, sin = R.rope_tables(base, hd, npos)
    # distinct cache cells (two tokens writing one cell would make the stored value depend on write order)
    col = torch.randperm(min(clen, ring), generator=g)[:M]
    pos = (col + min(clen, ring) * torch.randint(0, npos // min(clen, ring), (M,), generator=g)).to(torch.int32)
    slot = torch.randint(0, rows, (M,), generator=g, dtype=torch.int32)
    slot[1] = slot[0]
    kc_o = torch.zeros(rows, nkv, clen, hd)
    vc_o = torch.zeros_like(kc_o)
    q_o = R.bias_rope_store(R.linear(x.float(), w.float()), b.float() if b is not None else None, cos, sin, pos, slot,
                            kc_o, vc_o, nq, nkv, hd, ring)
    kc = torch.zeros(rows, nkv, clen, hd, dtype=BF, device="cuda")
    vc = torch.zeros_like(kc)
    q = torch.zeros(M, nq * hd, dtype=BF, device="cuda")
    Cs, Sn, P, S = cos.to(BF).cuda(), sin.to(BF).cuda(), pos.cuda(), slot.cuda()
    bb = b.cuda() if b is not None else None
    e = L.A8Epilogue(kind=L.EPI_ROPE, bias=L.ptr(bb), cos=L.ptr(Cs), sin=L.ptr(Sn), pos=L.ptr(P), slot=L.ptr(S),
                     kc=L.ptr(kc), vc=L.ptr(vc), nq=nq, nkv=nkv, hd=hd, ring=ring, cache_len=clen)
    gemm(L, ws, x.cuda(), w.cuda(), q, e)
    assert rel(q.view(M, nq, hd), q_o) < 1e-2 and frac_equal(q.view(M, nq, hd), q_o) > 0.97
    assert rel(kc, kc_o) < 1e-2 and frac_equal(kc, kc_o) > 0.97
    assert rel(vc, vc_o) < 1e-2 and frac_equal(vc, vc_o) > 0.97


def attention(L, ws, q, kc, vc, lens, rowmap=None, max_len=None):
    layers, rows, nkv, clen, hd = kc.shape
    b, nq, _ = q.shape
    out = torch.zeros(b, nq * hd, dtype=BF, device="cuda")
    ln = lens.int().cuda()
    rm = rowmap.int().cuda() if rowmap is not None else None
    L.call("a8_attention", L.ptr(q), nq * hd, L.ptr(kc), L.ptr(vc), layers, rows, nq, nkv, hd, clen, layers - 1,
           L.ptr(ln), L.ptr(rm), b, max_len or clen, 0.0, L.ptr(out), nq * hd, L.ptr(ws[0]), ws[0].numel(),
           L.ptr(ws[1]), ws[1].numel(), L.stream_handle())
    torch.cuda.synchronize()
    assert L.device_error()[0] == 0, L.device_error()
    return out.view(b, nq, hd)


def test_attention_gqa_ragged(L, ws):
    g = torch.Generator().manual_seed(3)
    nq, nkv, hd, S = 14, 2, 64, 2048
    lens = torch.tensor([1, 2, 15, 16, 17, 63, 64, 65, 255, 256, 257, 700, 1500, 2047, 2048, 999])
    b = len(lens)
    q = rnd(g, b, nq, hd)
    kc, vc = rnd(g, 2, b + 2, nkv, S, hd), rnd(g, 2, b + 2, nkv, S, hd)
    out = attention(L, ws, q.cuda(), kc.cuda(), vc.cuda(), lens)
    ref = R.decode_attention(q.float(), kc[1].float(), vc[1].float(), lens)
    assert rel(out, ref) < 1e-2
    rowmap = torch.randint(0, b + 2, (b,), generator=g)
    out = attention(L, ws, q.cuda(), kc.cuda(), vc.cuda(), lens, rowmap)
    ref = R.decode_attention(q.float(), kc[1].float(), vc[1].float(), lens, rowmap=rowmap)
    assert rel(out, ref) < 1e-2


@pytest.mark.parametrize("nq,nkv", [(14, 2), (8, 8)])
def test_attention_short_window(L, ws, nq, nkv):
    """Windows of at most 32 keys (the fast AR's 2..10 positions): against the oracle, with and without a row map (two
    query rows a cache row, as the fast AR's first pass), and the result independent of the max_len bound given."""
    g = torch.Generator().manual_seed(11 + nq)
    hd, clen = 64, 40
    lens = torch.tensor([1, 2, 3, 5, 9, 10, 10, 16, 31, 32, 7, 1])
    b = len(lens)
    q = rnd(g, b, nq, hd)
    kc, vc = rnd(g, 2, b + 3, nkv, clen, hd), rnd(g, 2, b + 3, nkv, clen, hd)
    out = attention(L, ws, q.cuda(), kc.cuda(), vc.cuda(), lens, max_len=32)
    assert rel(out, R.decode_attention(q.float(), kc[1].float(), vc[1].float(), lens)) < 1e-2
    wide = attention(L, ws, q.cuda(), kc.cuda(), vc.cuda(), lens, max_len=clen)
    assert rel(out, wide) < 1e-2
    rowmap = torch.arange(b) // 2                        # the fast AR's first pass: two query rows a cache row
    out = attention(L, ws, q.cuda(), kc.cuda(), vc.cuda(), lens, rowmap, max_len=32)
    assert rel(out, R.decode_attention(q.float(), kc[1].float(), vc[1].float(), lens, rowmap=rowmap)) < 1e-2


def test_attention_mha_ring(L, ws):
    g = torch.Generator().manual_seed(4)
    q = rnd(g, 7, 8, 128)
    kc, vc = rnd(g, 1, 7, 8, 128, 128), rnd(g, 1, 7, 8, 128, 128)
    lens = torch.tensor([1, 2, 33, 64, 100, 127, 128])
    out = attention(L, ws, q.cuda(), kc.cuda(), vc.cuda(), lens, max_len=128)
    assert rel(out, R.decode_attention(q.float(), kc[0].float(), vc[0].float(), lens)) < 1e-2


def test_attention_as_packed_prefill(L, ws):
    """The packed causal prefill is decode attention with lens = pos + 1 and rowmap = the request's slot."""
    g = torch.Generator().manual_seed(6)
    nq, nkv, hd = 14, 2, 64
    d = dict(ns=[70, 5, 130], starts=[30, 0, 12], slots=[2, 0, 1])
    R_ = sum(d["ns"])
    q = rnd(g, R_, nq, hd)
    kc, vc = rnd(g, 1, 3, nkv, 256, hd), rnd(g, 1, 3, nkv, 256, hd)
    pos = torch.cat([torch.arange(a, a + n) for a, n in zip(d["starts"], d["ns"])])
    slot = torch.cat([torch.full((n,), s) for n, s in zip(d["ns"], d["slots"])])
    out = attention(L, ws, q.cuda(), kc.cuda(), vc.cuda(), pos + 1, slot, max_len=int(pos.max()) + 1)
    blocks, r0 = [], 0
    for n, s, a in zip(d["ns"], d["slots"], d["starts"]):
        for off in range(0, n, 64):
            blocks.append((r0 + off, min(64, n - off), s, a + off))
        r0 += n
    ref = R.prefill_attention(q.float(), kc[0].float(), vc[0].float(), blocks)
    assert rel(out, ref) < 1e-2


@pytest.mark.parametrize("N", [896, 1024])
def test_rmsnorm(L, N):
    g = torch.Generator().manual_seed(N)
    rows = 37
    x, r, w = rnd(g, rows, N, scale=2.0), rnd(g, rows, N, scale=3.0), (torch.rand(N, generator=g) + 0.5).to(BF)
    X, Rz, W = x.cuda(), r.cuda().clone(), w.cuda()
    y = torch.zeros(rows, N, dtype=BF, device="cuda")
    L.call("a8_rmsnorm", L.ptr(X), N, L.ptr(Rz), N, L.ptr(W), L.ptr(y), N, rows, N, 1e-6, L.stream_handle())
    torch.cuda.synchronize()
    yo, ro = R.rmsnorm(x.float(), w.float(), 1e-6, residual=r.float())
    assert torch.equal(Rz.cpu(), ro.to(BF))
    assert frac_equal(y, yo) > 0.99 and rel(y, yo) < 1e-2
    L.call("a8_rmsnorm", L.ptr(X), N, None, 0, L.ptr(W), L.ptr(y), N, rows, N, 1e-6, L.stream_handle())
    torch.cuda.synchronize()
    yo = R.rmsnorm(x.float(), w.float(), 1e-6)
    assert frac_equal(y, yo) > 0.99 and rel(y, yo) < 1e-2


def test_embed_frame(L):
    g = torch.Generator().manual_seed(9)
    V, H, ncb, cbk, b = 4000, 896, 10, 64, 13
    emb, cbemb = rnd(g, V, H, scale=0.1), rnd(g, ncb * cbk, H, scale=0.05)
    sem = torch.randint(0, V, (b,), generator=g)
    codes = torch.randint(0, cbk, (b, ncb), generator=g)
    x = torch.zeros(b, H, dtype=BF, device="cuda")
    d = [t.cuda() for t in (sem, codes, emb, cbemb)]        # kept alive until the kernel has run
    L.call("a8_embed_frame", L.ptr(d[0]), L.ptr(d[1]), ncb, cbk, L.ptr(d[2]), L.ptr(d[3]), L.ptr(x), H, b, H, V,
           L.stream_handle())
    torch.cuda.synchronize()
    off = (torch.arange(ncb) * cbk).view(1, -1)
    ref = R.bf(emb.float()[sem] + R.bf(cbemb.float()[codes + off].sum(1)))
    assert frac_equal(x, ref) > 0.99 and rel(x, ref) < 1e-2


@pytest.mark.parametrize("V,k,p,t", [(4097, 50, 0.95, 0.8), (4096, 50, 1.0, 1.0), (4097, 0, 0.9, 0.7),
                                     (4096, 7, 0.3, 1.3)])
def test_sampler_exact(L, V, k, p, t):
    g = torch.Generator().manual_seed(V + k)
    rows = 33
    lg = R.bf(torch.randn(rows, V, generator=g) * 3.0)
    lg[3, 100:110] = lg[3].max()                                   # a tie group at the top
    out = torch.empty(rows, dtype=torch.int64, device="cuda")
    tick = torch.tensor([5], dtype=torch.int64, device="cuda")
    LG = lg.cuda()
    L.call("a8_sample", L.ptr(LG), V, V, rows, 1, k, p, t, 1234, 17, L.ptr(tick), L.ptr(out),
           L.stream_handle())
    torch.cuda.synchronize()
    kk = k if 0 < k < V else V
    v, idx, cum = R.topk_filter(lg, kk)
    ref = R.draw(v, idx, cum, p, t, R.philox_exp(1234, 17, 5, list(range(rows)), kk))
    assert torch.equal(out.cpu(), ref)
    L.call("a8_sample", L.ptr(LG), V, V, rows, 0, k, p, t, 0, 0, None, L.ptr(out), L.stream_handle())
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), lg.argmax(-1))
