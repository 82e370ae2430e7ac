"""Codec decoder kernels on the GPU, through the C ABI, against the CPU oracle (oracle/ref_cpu.py Conv / Vocoder).

Tolerances: the convs accumulate in fp32 in a different order than the oracle's matmul and round to fp16 once, so an
output may differ by one fp16 rounding: checked on the GPU's own input rows as max relative error <= 4e-3 and >= 95%
bit-equal, and end to end (the oracle's own activation) as max relative error <= 4e-3 -- the fp16 snake rows differ
from the oracle's by rare one-ulp sin() differences (<= 1 %, another library's sin), and each such input flip moves
many outputs by an ulp. The carried context is those activated rows. The bf16 op-by-op depthwise conv is the
oracle's exact sequence; LayerNorm statistics (fp32, another summation order) may move a result by one bf16 ulp.
"""
import ctypes as C
from types import SimpleNamespace

import pytest
import torch

from oracle import ref_cpu as R

pytestmark = pytest.mark.gpu
F16, BF = torch.float16, torch.bfloat16


@pytest.fixture(scope="module")
def L(a8):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    a8.load()
    a8._lib.call("a8_clear_error")
    return a8._lib


def rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp(min=1e-6))


def frac_equal(a, b):
    return float((a.float().cpu() == b.float().cpu()).float().mean())


def sync_ok(L):
    torch.cuda.synchronize()
    err = L.device_error()
    assert err[0] == 0, err


def make_conv(g, Cin, Cout, k=7, dil=1, trans=False, stride=1, snake=True, Bmax=64):
    """An oracle Conv over a seeded torch conv module; its context starts random (a stream already running)."""
    if trans:
        m = torch.nn.ConvTranspose1d(Cin, Cout, 2 * stride, stride=stride)
    else:
        m = torch.nn.Conv1d(Cin, Cout, k, dilation=dil)
    with torch.no_grad():
        m.weight.copy_(torch.randn(m.weight.shape, generator=g) * (Cin * m.weight.shape[-1]) ** -0.5)
        m.bias.copy_(torch.randn(m.bias.shape, generator=g) * 0.1)
    sm = SimpleNamespace(alpha=torch.rand(1, Cin, 1, generator=g) * 1.5 + 0.2) if snake else None
    c = R.Conv(SimpleNamespace(conv=m), Bmax, snake_mod=sm, trans=trans)
    if c.state is not None:
        c.state.copy_(R.hf(torch.randn(c.state.shape, generator=g)))
    return c


def device_conv(c, T, Bmax=64):
    """Device form of an oracle Conv: W2d[p*Cout + co, j*Cin + ci] = W[p, j, ci, co] (fp16), bias, snake terms, and
    its input rows xin [Bmax, ctx + T, Cin] with the oracle's current context in rows [0, ctx)."""
    ph, taps, Cin, Cout = c.W.shape
    w = c.W.permute(0, 3, 1, 2).reshape(ph * Cout, taps * Cin).to(F16).cuda().contiguous()
    d = SimpleNamespace(w=w, N=ph * Cout, T=T, bias=None, alpha=None, inv=None)
    if c.bias is not None:
        d.bias = c.bias.repeat(ph).to(F16).float().cuda()         # the fp16 bias, held as fp32
    if c.a is not None:
        d.alpha, d.inv = c.a.float().cuda().contiguous(), c.ib.float().cuda().contiguous()
    d.xin = torch.zeros(Bmax, c.ctx + T, Cin, dtype=F16, device="cuda")
    if c.state is not None:
        d.xin[:, :c.ctx] = c.state.to(F16).cuda()
    d.table = None
    if c.ctx > 0:                                          # a one-entry context-shift table in device memory
        from audio8_b200._lib import A8CtxShift
        entry = A8CtxShift(xin=d.xin.data_ptr(), ctx=c.ctx, T=T, Cin=Cin)
        d.table = torch.frombuffer(bytearray(bytes(entry)), dtype=torch.uint8).cuda()
    return d


def conv_run(L, c, d, b, **out):
    r = L.A8ConvRun(xin=L.ptr(d.xin), rows=b, T=d.T, Cin=c.Cin, ctx=c.ctx, w=L.ptr(d.w), N=d.N, taps=c.taps,
                    dil=c.dil, bias=L.ptr(d.bias))
    for k, v in out.items():
        setattr(r, k, v)
    L.call("a8_conv", C.byref(r), L.stream_handle())


def feed(L, c, d, x, b):
    """The conv's input rows from x [b, T, Cin] (fp16 or bf16), activated with its snake."""
    L.call("a8_conv_input", L.ptr(x), int(x.dtype == BF), d.T * c.Cin, d.T, c.Cin, L.ptr(d.xin), c.ctx,
           L.ptr(d.alpha), L.ptr(d.inv), b, L.stream_handle())


def shift(L, d, b):
    if d.table is not None:
        L.call("a8_ctx_shift", L.ptr(d.table), 1, b, L.stream_handle())


def run_conv(L, c, d, x, b, res=None):
    """input rows + conv (raw fp16 out) + context shift on the GPU for rows [0, b) of x [b, T, Cin]."""
    T = d.T
    feed(L, c, d, x, b)
    out = torch.empty(b, T * c.ph, c.Cout, dtype=F16, device="cuda")
    kw = dict(raw=L.ptr(out), raw_bs=T * d.N, raw_ts=d.N)
    if res is not None:
        kw.update(res=L.ptr(res), res_bs=T * d.N, res_ts=d.N)
    conv_run(L, c, d, b, **kw)
    shift(L, d, b)
    sync_ok(L)
    return out


CONV_CASES = [
    # name, Cin, Cout, k, dil, trans, stride, snake, T, rows, in_bf16
    ("dec_in", 256, 192, 7, 1, False, 1, False, 4, 5, True),
    ("unit_c1_dil3", 96, 96, 7, 3, False, 1, True, 32, 3, False),
    ("unit_c1_dil9_ctx_gt_T", 64, 64, 7, 9, False, 1, True, 32, 4, False),
    ("unit_c1_dil9", 64, 64, 7, 9, False, 1, True, 1024, 2, False),
    ("trans_s2", 192, 96, 0, 1, True, 2, True, 64, 3, False),
    ("trans_s8", 256, 128, 0, 1, True, 8, True, 4, 33, False),
    ("k7_wide", 384, 384, 7, 1, False, 1, True, 256, 2, False),
    ("many_tiles", 192, 192, 7, 3, False, 1, True, 1024, 40, False),
    # streamed weights on CTA pairs with an odd number of 128-step tiles (the last pair's second tile is beyond the rows)
    ("pair_odd_tiles", 192, 192, 7, 1, False, 1, True, 128, 3, False),
]


@pytest.mark.parametrize("name,Cin,Cout,k,dil,trans,stride,snake,T,rows,in_bf16", CONV_CASES,
                         ids=[c[0] for c in CONV_CASES])
def test_conv_vs_oracle(L, name, Cin, Cout, k, dil, trans, stride, snake, T, rows, in_bf16):
    g = torch.Generator().manual_seed(Cin * 31 + T + rows)
    c = make_conv(g, Cin, Cout, k, dil, trans, stride, snake)
    d = device_conv(c, T)
    for step in range(3):                                  # later steps read the context the earlier ones left
        xr = torch.randn(rows, T, Cin, generator=g)
        x = R.bf(xr) if in_bf16 else R.hf(xr)
        want = c(R.hf(x), rows)
        xin_before = d.xin[:rows, :c.ctx].float().cpu()
        got = run_conv(L, c, d, x.to(BF if in_bf16 else F16).cuda(), rows).view(rows, T * c.ph, c.Cout)
        assert rel(got, want) <= 4e-3, (name, step)
        # the activation: fp16 snake rows within one-ulp sin() differences of the oracle's (another library's sin)
        act = d.xin[:rows, c.ctx:].float().cpu()
        act_o = R.hf(R.snake(R.hf(x), c.a, c.ib)) if c.a is not None else R.hf(x)
        assert rel(act, act_o) <= 1e-3 and float((act != act_o).float().mean()) <= 0.01, (name, step)
        # the conv arithmetic alone: the oracle's sum on the GPU's own input rows
        xin = torch.cat([xin_before, act], 1)
        y = torch.zeros(rows, T, c.ph, c.Cout)
        for p in range(c.ph):
            y[:, :, p] = sum(xin[:, j * c.dil:j * c.dil + T] @ c.W[p, j] for j in range(c.taps))
        y = y.reshape(rows, T * c.ph, c.Cout)
        if c.bias is not None:
            y = y + c.bias
        y = R.hf(y)
        assert rel(got, y) <= 4e-3 and frac_equal(got, y) >= 0.95, (name, step)
        st = d.xin[:rows, :c.ctx].float().cpu()
        # the carried context is exactly the last ctx rows of (old context ; this step's activated rows): the shift
        # moves bytes
        assert torch.equal(st, torch.cat([xin_before, act], 1)[:, -c.ctx:]), (name, step)
        # against the oracle's own state: one-ulp sin() differences (the host's vectorised fp32 sin and CUDA's sinf
        # disagree on a few values in a hundred, more or fewer with the host array's alignment)
        flips = int((st != c.state[:rows]).sum())
        assert flips <= max(2, st.numel() // 40) and rel(st, c.state[:rows]) <= 1e-3, (name, step, flips)


def test_conv_1x1_residual(L):
    """A residual unit's 1x1 conv: snake on its input rows (no context), + bias + the unit's input."""
    g = torch.Generator().manual_seed(5)
    c = make_conv(g, 192, 192, k=1, snake=True)
    rows, T = 2, 256
    d = device_conv(c, T)
    x = R.hf(torch.randn(rows, T, 192, generator=g))
    res = R.hf(torch.randn(rows, T, 192, generator=g))
    want = c(x, rows, res=res)
    got = run_conv(L, c, d, x.to(F16).cuda(), rows, res=res.to(F16).cuda())
    assert rel(got, want) <= 4e-3 and frac_equal(got, want) >= 0.95


def test_conv_fused_next_input(L):
    """A transposed conv's epilogue writes the next conv's input rows already activated with THAT conv's snake
    (phases interleaved into timesteps), the next conv reads them after its context, and a residual 1x1 closes the
    unit: the chain equals the oracle's tc -> c1 -> c2(+res), and the raw tc output is kept for the residual."""
    g = torch.Generator().manual_seed(8)
    rows, T = 3, 32
    tc = make_conv(g, 192, 96, trans=True, stride=4, snake=True)
    c1 = make_conv(g, 96, 96, k=7, dil=3, snake=True)
    c2 = make_conv(g, 96, 96, k=1, snake=True)
    dtc, d1, d2 = device_conv(tc, T), device_conv(c1, 4 * T), device_conv(c2, 4 * T)
    raw = torch.empty(rows, 4 * T, 96, dtype=F16, device="cuda")
    out = torch.empty(rows, 4 * T, 96, dtype=F16, device="cuda")
    for step in range(2):
        x = R.hf(torch.randn(rows, T, 192, generator=g))
        y0 = tc(x, rows)
        want = c2(c1(y0, rows), rows, res=y0)
        feed(L, tc, dtc, x.to(F16).cuda(), rows)
        conv_run(L, tc, dtc, rows, raw=L.ptr(raw), raw_bs=T * dtc.N, raw_ts=dtc.N, nxt=L.ptr(d1.xin),
                 nxt_bs=(c1.ctx + 4 * T) * 96, nxt_off=c1.ctx * 96, cout=96, alpha=L.ptr(d1.alpha),
                 inv=L.ptr(d1.inv))
        conv_run(L, c1, d1, rows, nxt=L.ptr(d2.xin), nxt_bs=4 * T * 96, nxt_off=0, cout=96, alpha=L.ptr(d2.alpha),
                 inv=L.ptr(d2.inv))
        conv_run(L, c2, d2, rows, raw=L.ptr(out), raw_bs=4 * T * 96, raw_ts=96, res=L.ptr(raw), res_bs=4 * T * 96,
                 res_ts=96)
        shift(L, dtc, rows)
        shift(L, d1, rows)
        sync_ok(L)
        assert rel(raw, y0) <= 4e-3 and frac_equal(raw, y0) >= 0.95, step
        assert rel(out, want) <= 1e-2 and frac_equal(out, want) >= 0.9, step
        assert frac_equal(d1.xin[:rows, :c1.ctx], c1.state[:rows]) >= 0.97, step


def test_conv_out_tanh(L):
    """conv_out (Cout 1) + tanh into fp32 audio."""
    g = torch.Generator().manual_seed(6)
    c = make_conv(g, 96, 1, k=7, snake=True)
    rows, T = 3, 128
    d = device_conv(c, T)
    audio = torch.empty(rows, T, dtype=torch.float32, device="cuda")
    for _ in range(2):
        x = R.hf(torch.randn(rows, T, 96, generator=g))
        want = torch.tanh(c(x, rows)[..., 0])
        feed(L, c, d, x.to(F16).cuda(), rows)
        conv_run(L, c, d, rows, audio=audio.data_ptr(), audio_bs=T)
        shift(L, d, rows)
        sync_ok(L)
        assert float((audio.cpu() - want).abs().max()) <= 2e-3


@pytest.mark.parametrize("T,rows", [(2, 3), (4, 5)])
def test_ups_dwln(L, T, rows):
    """Upsample stage middle: bf16 7-tap causal depthwise conv with its carried tail, then LayerNorm."""
    g = torch.Generator().manual_seed(T * 10 + rows)
    C_, K, eps = 1024, 7, 1e-6
    u = R.bf(torch.randn(rows, T, C_, generator=g))
    st = R.bf(torch.randn(rows, K - 1, C_, generator=g))
    dww, dwb = R.bf(torch.randn(K, C_, generator=g) * 0.3), R.bf(torch.randn(C_, generator=g) * 0.1)
    lnw, lnb = R.bf(1 + 0.1 * torch.randn(C_, generator=g)), R.bf(0.1 * torch.randn(C_, generator=g))
    xin = torch.cat([st, u], 1)
    y = R.bf(dwb + R.bf(xin[:, 0:T] * dww[0]))
    for j in range(1, K):
        y = R.bf(y + R.bf(xin[:, j:j + T] * dww[j]))
    want = R.bf(torch.nn.functional.layer_norm(y, (C_,), lnw, lnb, eps))
    want_st = xin[:, T:]
    ud, std, wd, bd, lwd, lbd = (t.to(BF).cuda().contiguous() for t in (u, st, dww, dwb, lnw, lnb))
    z = torch.empty(rows, T, C_, dtype=BF, device="cuda")
    L.call("a8_ups_dwln", L.ptr(ud), T, C_, L.ptr(std), (K - 1) * C_, K, L.ptr(wd), L.ptr(bd), L.ptr(lwd),
           L.ptr(lbd), eps, L.ptr(z), rows, L.stream_handle())
    sync_ok(L)
    assert torch.equal(std.float().cpu(), want_st)
    assert rel(z, want) <= 1e-2 and frac_equal(z, want) >= 0.97


def test_codec_embed(L):
    """Code tables with the codec's clamps, and the window transformer's positions."""
    g = torch.Generator().manual_seed(7)
    C_, vs, vr, ncb, rows = 1024, 4096, 1024, 10, 6
    t_sem = torch.randn(vs, C_, generator=g)
    t_res = torch.randn(ncb - 1, vr, C_, generator=g)
    codes = torch.randint(0, 4096, (rows, ncb), generator=g)
    codes[0, 0], codes[1, 3], codes[2, 9], codes[3, 0] = -5, 4000, -1, 5000      # out of range: clamped
    voc = SimpleNamespace(t_sem=t_sem, t_res=t_res, v_sem=vs, v_res=vr)
    want = R.bf(R.Vocoder.embed(voc, codes))
    pos = torch.tensor([0, 5, 127, 128, 8191, 9000], dtype=torch.int32)
    max_pos, win = 8192, 128
    pd = pos.cuda()
    pos_c, lens = torch.empty_like(pd), torch.empty_like(pd)
    x = torch.empty(rows, C_, dtype=BF, device="cuda")
    cd, sd, rd = codes.cuda(), t_sem.cuda(), t_res.cuda()
    L.call("a8_codec_embed", L.ptr(cd), ncb, L.ptr(sd), vs, L.ptr(rd), vr, C_, L.ptr(x),
           L.ptr(pd), L.ptr(pos_c), L.ptr(lens), max_pos, win, rows, L.stream_handle())
    sync_ok(L)
    assert rel(x, want) <= 1e-2 and frac_equal(x, want) >= 0.99
    assert torch.equal(pos_c.cpu(), pos.clamp(max=max_pos - 1))
    assert torch.equal(lens.cpu(), (pos + 1).clamp(max=win))
    assert torch.equal(pd.cpu(), pos + 1)
