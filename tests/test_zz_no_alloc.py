"""a8_attention_noalloc: the attention entry point for callers that cannot allocate device memory (a binding handed
only the device pointers of its inputs and outputs, a serving process whose memory pool owns the whole device). Its
split workspace lives in an array of the library, so the caller passes inputs and outputs only.

Checked through the C ABI against a8_attention (caller-owned workspace) and against the CPU oracle's attention, on
calls in a row whose rows span several splits, so the library's array is used and its leftovers from one call must
not leak into the next: the slow AR's GQA shape (hd 64, 14 / 2 heads) and the codec's MHA shape (hd 128, 8 / 8 heads)
at the row count with the largest workspace need.
This file is collected last (test_zz_*): it passes alone in a fresh process and after every other test.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


@pytest.fixture(scope="module")
def L(a8):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    a8.load()
    return a8._lib


def _case(seed, b, lens_hi, nq=14, nkv=2, hd=64):
    g = torch.Generator().manual_seed(seed)
    S, layers = 2048, 2
    q = (torch.randn(b, nq, hd, generator=g)).to(BF).cuda()
    kc = (torch.randn(layers, b + 1, nkv, S, hd, generator=g)).to(BF).cuda()
    vc = (torch.randn(layers, b + 1, nkv, S, hd, generator=g)).to(BF).cuda()
    lens = torch.randint(1, lens_hi + 1, (b,), generator=g, dtype=torch.int32)
    lens[0] = lens_hi
    return q, kc, vc, lens.cuda(), (nq, nkv, hd, S, layers)


def _run(L, fn, q, kc, vc, lens, dims, ws=None):
    nq, nkv, hd, S, layers = dims
    b = q.shape[0]
    out = torch.full((b, nq * hd), float("nan"), dtype=BF, device="cuda")
    args = [L.ptr(q), nq * hd, L.ptr(kc), L.ptr(vc), layers, b + 1, nq, nkv, hd, S, 1, L.ptr(lens), None, b, S, 0.0,
            L.ptr(out), nq * hd]
    if fn == "a8_attention":
        args += [L.ptr(ws[0]), ws[0].numel(), L.ptr(ws[1]), ws[1].numel()]
    L.call(fn, *args, L.stream_handle())
    torch.cuda.synchronize()
    return out


def test_noalloc_attention_matches_workspace_version_twice(L, a8):
    import ctypes as C
    ws_floats = C.c_longlong()
    n_cnt = C.c_int()
    from oracle.ref_cpu import decode_attention
    # calls in a row, different shapes and lengths; 36 rows x 8 heads at hd 128 = 2 splits, the largest need of the
    # library array (36 x 8 x 2 x 2080 partial words + 288 tickets)
    for seed, b, hi, nq, nkv, hd in ((11, 48, 2048, 14, 2, 64), (12, 37, 1300, 14, 2, 64), (13, 36, 900, 8, 8, 128),
                                     (14, 36, 2048, 8, 8, 128)):
        q, kc, vc, lens, dims = _case(seed, b, hi, nq, nkv, hd)
        L.check(L.load().a8_attention_workspace(b, dims[1], dims[2], dims[3], C.byref(ws_floats), C.byref(n_cnt)))
        ws = (torch.zeros(max(1, ws_floats.value), device="cuda"),
              torch.zeros(max(1, n_cnt.value), dtype=torch.int32, device="cuda"))
        ref = _run(L, "a8_attention", q, kc, vc, lens, dims, ws)
        got = _run(L, "a8_attention_noalloc", q, kc, vc, lens, dims)
        assert a8.device_error()[0] == 0
        assert not torch.isnan(got.float()).any()
        rel = float((got.float() - ref.float()).abs().max() / ref.float().abs().max())
        assert rel < 1e-2, rel
        orc = decode_attention(q.cpu().view(b, nq, hd), kc[1].cpu(), vc[1].cpu(), lens.cpu())
        rel_o = float((got.float().cpu().view(b, nq, hd) - orc).abs().max() / orc.abs().max())
        assert rel_o < 1e-2, rel_o
