"""The CPU oracle (oracle/ref_cpu.py) against golden outputs of the reference itself (tests/golden/*.pt, made by
tests/golden/make_golden.py from serve/fast_kernels.py and serve/fast_engine.py run on the CPU)."""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import ref_cpu as R

F = torch.float32


def rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).abs().max() / b.abs().max().clamp(min=1e-6))


def ulps_bf16(a, b):
    """Max distance in bf16 ulps between two bf16-valued tensors."""
    ai = a.to(torch.bfloat16).view(torch.int16).to(torch.int32)
    bi = b.to(torch.bfloat16).view(torch.int16).to(torch.int32)
    ai = torch.where(ai < 0, -(ai & 0x7FFF), ai)
    bi = torch.where(bi < 0, -(bi & 0x7FFF), bi)
    return int((ai - bi).abs().max())


@pytest.fixture(scope="module")
def K():
    return golden("kernels")


def test_rmsnorm(K):
    for N in (896, 1024):
        d = K[f"rmsnorm{N}"]
        x, r, w = d["x"].float(), d["r"].float(), d["w"].float()
        assert ulps_bf16(R.rmsnorm(x, w, 1e-6), d["y"]) <= 1
        y, ro = R.rmsnorm(x, w, 1e-6, residual=r)
        assert torch.equal(ro.to(torch.bfloat16), d["res_out"])       # the rounded residual add is exact
        assert ulps_bf16(y, d["y_res"]) <= 1


@pytest.mark.parametrize("name", ["slow", "codec"])
def test_bias_rope_store(K, name):
    d = K[f"rope_{name}"]
    kc = torch.zeros_like(d["kc"], dtype=F)
    vc = torch.zeros_like(kc)
    q = R.bias_rope_store(d["qkv"].float(), d["bias"], d["cos"].float(), d["sin"].float(), d["pos"], d["slot"], kc, vc,
                          d["nq"], d["nkv"], d["hd"], d["ring"])
    assert ulps_bf16(q, d["q"]) <= 1
    assert ulps_bf16(kc, d["kc"]) <= 1
    assert torch.equal(vc.to(torch.bfloat16), d["vc"])               # v: bias add, one rounding


def test_decode_attention(K):
    d = K["decode_attn"]
    o = R.decode_attention(d["q"].float(), d["kc"].float(), d["vc"].float(), d["lens"])
    for ns in (1, 3):
        assert rel(o, d[f"out_ns{ns}"]) < 1.5e-2
    om = R.decode_attention(d["q"].float(), d["kc"].float(), d["vc"].float(), d["lens"], rowmap=d["rowmap"])
    assert rel(om, d["out_map"]) < 1.5e-2
    m = K["decode_attn_mha"]
    assert rel(R.decode_attention(m["q"].float(), m["kc"].float(), m["vc"].float(), m["lens"]), m["out"]) < 1.5e-2


def test_prefill_attention(K):
    d = K["prefill_attn"]
    o = R.prefill_attention(d["q"].float(), d["kc"].float(), d["vc"].float(), d["blocks"])
    assert rel(o, d["out"]) < 1.5e-2


def test_silu_mul(K):
    d = K["silu_mul"]
    assert ulps_bf16(R.silu_mul(d["gu"].float()), d["y"]) <= 1


@pytest.mark.parametrize("name", ["k7d3", "trans4", "pw_snake", "k7_out"])
def test_conv(K, name):
    """_CLConv arithmetic (snake on fp16 input, implicit-GEMM conv / polyphase transposed conv, bias, residual);
    the reference accumulates each BK slice in fp16 (serve/fast_kernels.py:585-588), the oracle in fp32."""
    d = K["conv"][name]
    x = d["x"].float()
    a = d["a"]
    ib = 1.0 / (a + 1e-9)
    xa = R.hf(R.snake(x, a, ib))
    xin = torch.cat([d["st"].float(), xa], 1) if d["st"] is not None else xa
    if d["xin"] is not None:
        assert (xin - d["xin"].float()).abs().max() <= 2e-3 * xin.abs().max()
    W = d["W"].float()
    b, T, ph = x.shape[0], d["T"], d["ph"]
    y = torch.zeros(b, T, ph, W.shape[-1])
    for p in range(ph):
        for j in range(d["taps"]):
            y[:, :, p] += xin[:, j * d["dil"]:j * d["dil"] + T] @ W[p, j]
    y = y.reshape(b, T * ph, -1)
    if d["bias"] is not None:
        y = y + d["bias"].float()
    if d["res"] is not None:
        y = y + d["res"].float()
    assert rel(R.hf(y), d["y"]) < 5e-3


def test_sampler_filter_and_draw():
    S = golden("sampler")
    for name in ("sem", "cb"):
        d = S[name]
        v, idx, cum = R.topk_filter(d["logits"], d["k"])
        assert torch.equal(v, d["v"])                                # same sorted values
        for r in range(v.shape[0]):                                  # same index set within each tie group
            for val in torch.unique(v[r]):
                m = v[r] == val
                if val == v[r, -1]:
                    # the tie group at the k-th place may be cut anywhere (torch.topk leaves it unspecified; the
                    # oracle keeps the lowest indices): every kept index must hold that value
                    assert bool((d["logits"][r, idx[r][m]] == val).all())
                    assert bool((d["logits"][r, d["idx"][r][m]] == val).all())
                else:
                    assert set(idx[r][m].tolist()) == set(d["idx"][r][m].tolist())
        assert (cum - d["cum"]).abs().max() < 1e-5
        for key, ref in d["draws"].items():
            p, t = (float(s[1:]) for s in key.split("_"))
            got = R.draw(v, d["idx"], cum, p, t, d["E"])               # the reference's tie order, same noise
            assert torch.equal(got, ref), key
        assert torch.equal(d["logits"].argmax(-1), d["greedy"])


def test_philox_known_answer():
    """Philox4x32-10 known-answer vectors (Random123, kat_vectors: philox4x32_10)."""
    z = R.philox4x32([0], [0], [0], [0], 0, 0)
    assert [int(w[0]) for w in z] == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    f = R.philox4x32([0xFFFFFFFF], [0xFFFFFFFF], [0xFFFFFFFF], [0xFFFFFFFF], 0xFFFFFFFF, 0xFFFFFFFF)
    assert [int(w[0]) for w in f] == [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]
    p = R.philox4x32([0x243F6A88], [0x85A308D3], [0x13198A2E], [0x03707344], 0xA4093822, 0x299F31D0)
    assert [int(w[0]) for w in p] == [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]


def test_host_pieces():
    H = golden("host")
    pm = H["pf_meta"]
    for c in pm["cases"]:
        m = R.pf_meta_host(pm["NT"], pm["NR"], pm["BM"], pm["SCR"], c["nt"], c["slots"], c["ns"], c["starts"])
        assert np.array_equal(m, c["meta"].numpy())
    p = H["permute"]
    assert torch.equal(R.permute_qk(p["w"], 14, 2, 64), p["pw"])
    assert torch.equal(R.permute_qk(p["b"], 14, 2, 64), p["pb"])
    c, s = R.rope_tables(1e6, 64, 2048)
    assert torch.equal(c, H["rope"]["cos"].float()) and torch.equal(s, H["rope"]["sin"].float())
    c, s = R.rope_tables(1e4, 128, 300)
    assert torch.equal(c, H["rope"]["cos_codec"].float()) and torch.equal(s, H["rope"]["sin_codec"].float())


def test_buckets_and_nsplit():
    b = R.default_buckets(32)
    assert b == [1, 2, 4, 6, 8, 12, 16, 20, 24, 28, 32]
    assert R.bucket_for(b, 5) == 6 and R.bucket_for(b, 33) == 32 and R.bucket_for(b, 1) == 1
    assert R.default_buckets(200)[-1] == 200 and 192 in R.default_buckets(200)
    assert [R.ref_nsplit(x) for x in (1, 8, 64, 192)] == [16, 11, 2, 1]


@pytest.mark.slow
def test_stack(tiny_model):
    """Two slow layers: packed causal prefill of two requests, then a decode step with rowmap and split-K."""
    d = golden("stack")
    c = tiny_model.config
    st = R.Stack(tiny_model.layers, tiny_model.norm, c.n_head, c.n_local_heads, c.head_dim, c.norm_eps, c.rope_base,
                 cache_rows=4, cache_len=256, max_pos=256)
    h = st.forward(d["x"].float(), d["pos"], d["slot"], blocks=d["blocks"])
    assert rel(h, d["h_pf"]) < 2e-2
    hd = st.forward(d["xd"].float(), d["dpos"], d["dslot"], d["dpos"] + 1, rowmap=True)
    assert rel(hd, d["h_dec"]) < 2e-2
    assert rel(st.kc, d["kc"]) < 2e-2 and rel(st.vc, d["vc"]) < 2e-2


def snr_db(a, ref):
    a, ref = a.double().flatten(), ref.double().flatten()
    return float(10 * torch.log10((ref ** 2).sum() / ((a - ref) ** 2).sum().clamp(min=1e-30)))


@pytest.mark.slow
def test_vocoder_step(tiny_model):
    """StreamingVocoder.step: table sum, 2-layer window transformer, two upsample stages, full-size DAC decoder with
    carried conv state, 2 frames for 2 rows (reference run: its fp16 convs accumulate each BK slice in fp16)."""
    d = golden("vocoder")
    codec = tiny_model.load_codec("cpu", torch.float32)
    v = R.Vocoder(codec, 2)
    for t in range(d["codes"].shape[0]):
        w = v.step(d["codes"][t], 2)
        assert snr_db(w, d["wav"][t]) > 40, (t, snr_db(w, d["wav"][t]))
    assert torch.equal(v.pos[:2], d["pos"][:2])


def _ulp(v):
    e = max(-126, int(np.floor(np.log2(max(abs(float(v)), 1e-30)))))
    return 2.0 ** (e - 7)


@pytest.mark.slow
def test_engine_admit_and_ticks(tiny_model):
    """FastEngine (bf16 model, greedy): admission (prefix KV per voice, packed prefill, first token) and 3 ticks with
    the codec one frame behind. Each row is compared until its first difference, which must be a near-tie (within 2
    bf16 ulps) of the oracle's own logits for that draw -- random weights give nearly flat logits. Until then: codes,
    tokens and bookkeeping equal, logits within 2e-2, audio SNR > 40 dB."""
    from types import SimpleNamespace
    from oracle.standin import StubTokenizer
    d = golden("engine")
    gp = dict(do_sample=False, temperature=0.8, top_k=50, top_p=0.95, max_new_tokens=64)
    ora = R.OracleEngine(tiny_model, StubTokenizer(), gp, max_slots=3, max_seq=512)
    item = SimpleNamespace(ref_code=d["ref_code"], ref_text=d["ref_text"])
    reqs = [dict(text=d["text"], item=item, key="v0"), dict(text=d["text2"], item=item, key="v0")]
    ora.record = {}
    assert ora.admit([0, 2], reqs) == d["lens"]
    assert rel(ora.record["prefill_logits"][0], d["prefill_logits"][0]) < 2e-2
    assert torch.equal(ora.tok, d["state0"]["tok"]) and torch.equal(ora.cpos, d["state0"]["cpos"])
    live, ties = [True, True, True], []
    for t in range(d["tok_in"].shape[0]):
        ora.record = {}
        codes = ora.tick(3)
        for r in range(3):
            if not live[r]:
                continue
            assert snr_db(ora.audio[r], d["audio"][t][r]) > 40, (t, r)
            ref_codes = d["frame_prev"][t][r]
            if int(d["tok_in"][t][r]) != ora.eos and not torch.equal(codes[r], ref_codes):
                k = int((codes[r] != ref_codes).nonzero()[0])
                lg = ora.record["fast_logits"][k - 1][r]
                gap = float(lg[int(codes[r, k])] - lg[int(ref_codes[k])])
                assert gap <= 2 * _ulp(lg[int(codes[r, k])]), (t, r, k, gap)
                ties.append((t, r, k))
                live[r] = False
                continue
            assert rel(ora.record["logits"][-1][r], d["logits"][t][r]) < 2e-2, (t, r)
            for key in ("tok_in", "frame_prev", "cpos", "nstep", "prev"):
                assert torch.equal(getattr(ora, key)[r], d[key][t][r]), (t, r, key)
            if int(ora.tok[r]) != int(d["tok"][t][r]):
                j = lambda tok: ora.nsem if int(tok) == ora.eos else int(tok) - ora.sb
                lg = ora.record["logits"][-1][r]
                assert float(lg[j(ora.tok[r])] - lg[j(d["tok"][t][r])]) <= 2 * _ulp(lg[j(ora.tok[r])]), (t, r)
                ties.append((t, r, 0))
                live[r] = False
    assert sum(live) >= 1, ties
