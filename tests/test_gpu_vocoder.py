"""The streaming codec (StreamingVocoder drop-in, one a8_voc_step per frame) on the GPU against the CPU oracle
(oracle/ref_cpu.py Vocoder) on the stand-in codec (real widths, 2 transformer layers).

Bars: the window transformer's output within 2e-2 max-relative and >= 98% bit-equal; each row's audio stream at
SNR >= 40 dB (each frame >= 38 dB) against the oracle running its own carried state; the conv decoder alone, fed the
same frames, at SNR >= 50 dB. The stand-in's random weights make the codec very sensitive: the oracle against itself
with one bf16 ulp added to 1% of its transformer output already measures 39-44 dB, so the full-step bar sits at that
floor while the decoder bar is tight. The arena (clear / snapshot / load) is exact: rows loaded from a snapshot decode
bit-identical audio to the row it was taken from.
"""
import pytest
import torch

from oracle import ref_cpu as R

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


@pytest.fixture(scope="module")
def dev(a8):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    a8.load()
    return torch.device("cuda", 0)


def rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp(min=1e-6))


def snr_db(got, want):
    got, want = got.double().cpu(), want.double().cpu()
    return float(10 * torch.log10(want.pow(2).sum() / (got - want).pow(2).sum().clamp(min=1e-30)))


def random_codes(g, b, cfg, wild=False):
    c = torch.randint(0, cfg.codec_res_size, (b, cfg.num_codebooks), generator=g)
    c[:, 0] = torch.randint(0, cfg.codebook_size, (b,), generator=g)
    if wild:                                     # out-of-range codes: the codec clamps them
        c[0, 0], c[-1, 5] = cfg.codebook_size + 7, -3
    return c


def oracle_step(voc, codes, b):
    """Vocoder.step with its intermediates: (table input, transformer output, audio)."""
    x = voc.embed(codes)
    pos = voc.pos[:b]
    h = voc.post.forward(R.bf(x), pos.clamp(max=voc.max_pos - 1), torch.arange(b, dtype=torch.int32),
                         (pos + 1).clamp(max=voc.WINDOW), rowmap=False)
    u = voc.upsample(h.unsqueeze(1), b)
    wav = voc.decode(u, b)
    voc.pos[:b] += 1
    return R.bf(x), h, wav


def test_vocoder_frames_match_oracle(a8, dev, tiny_model):
    from audio8_b200.codec import StreamingVocoder
    cfg = tiny_model.config
    b, frames = 3, 4
    voc = StreamingVocoder(tiny_model.load_codec(device="cpu"), 4, dev)
    ora = R.Vocoder(tiny_model.load_codec(device="cpu"), 4)
    g = torch.Generator().manual_seed(11)
    got, want = [], []
    for f in range(frames):
        codes = random_codes(g, b, cfg, wild=(f == 1))
        wav = voc.step(codes.to(dev), b).clone()
        torch.cuda.synchronize()
        assert a8.device_error()[0] == 0
        _, h_o, wav_o = oracle_step(ora, codes, b)
        h = voc.scratch.h[:b].float().cpu()                           # the transformer's final-normed output
        assert rel(h, h_o) <= 2e-2 and float((h == h_o).float().mean()) >= 0.98, f
        assert torch.equal(voc.pos[:b].cpu(), ora.pos[:b])
        got.append(wav.cpu())
        want.append(wav_o)
        for r in range(b):
            s = snr_db(wav[r], wav_o[r])
            print(f"frame {f} row {r}: SNR {s:.1f} dB")
            assert s >= 38.0, (f, r, s)
    # the whole stream of each row (one bf16 flip at 1% of the transformer output alone costs the stand-in 39-44 dB)
    for r in range(b):
        s = snr_db(torch.stack([w[r] for w in got]), torch.stack([w[r] for w in want]))
        print(f"row {r}: SNR over {frames} frames {s:.1f} dB")
        assert s >= 40.0, (r, s)


def gpu_decode(voc, u, b):
    """The decoder's conv program alone (a8_voc_decode) on u [b, T, C]."""
    wav = voc.decode(u.to(voc.dev), b)
    torch.cuda.synchronize()
    return wav.cpu().clone()


def test_vocoder_decoder_matches_oracle(a8, dev, tiny_model):
    """The conv decoder (29 convs, carried contexts) fed the same upsampled frames as the oracle's: SNR >= 50 dB."""
    from audio8_b200.codec import StreamingVocoder
    cfg = tiny_model.config
    b = 3
    voc = StreamingVocoder(tiny_model.load_codec(device="cpu"), 4, dev)
    ora = R.Vocoder(tiny_model.load_codec(device="cpu"), 4)
    g = torch.Generator().manual_seed(13)
    for f in range(3):
        u = R.bf(torch.randn(b, 4, cfg.codec_dim, generator=g))
        wav = gpu_decode(voc, u, b)
        wav_o = ora.decode(u, b)
        assert a8.device_error()[0] == 0
        for r in range(b):
            s = snr_db(wav[r], wav_o[r])
            print(f"decoder frame {f} row {r}: SNR {s:.1f} dB")
            assert s >= 50.0, (f, r, s)


def test_vocoder_arena_snapshot_load_clear(a8, dev, tiny_model):
    from audio8_b200.codec import StreamingVocoder
    cfg = tiny_model.config
    voc = StreamingVocoder(tiny_model.load_codec(device="cpu"), 4, dev)
    g = torch.Generator().manual_seed(12)
    for _ in range(2):
        voc.step(random_codes(g, 4, cfg).to(dev), 4)
    snap = voc.snapshot(1)
    host = [t.cpu().pin_memory() for t in snap]          # as prime_speakers keeps it
    voc.clear_many([0])
    voc.load_many([2, 3], host)
    torch.cuda.synchronize()
    for t, nch, n, cs, ss in voc._states():
        flat = t.view(-1)
        for ch in range(nch):
            row = lambda s: flat[s * ss + ch * cs: s * ss + ch * cs + n]
            assert not row(0).float().abs().sum(), "cleared row not zero"
            assert torch.equal(row(2), row(1)) and torch.equal(row(3), row(1))
    codes = random_codes(g, 4, cfg)
    codes[2:] = codes[1]
    wav = voc.step(codes.to(dev), 4).clone()
    torch.cuda.synchronize()
    assert torch.equal(wav[2], wav[1]) and torch.equal(wav[3], wav[1])
    assert a8.device_error()[0] == 0
