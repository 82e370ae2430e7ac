"""Stand-in for the Audio8 checkpoint (test infrastructure, never shipped).

The reference engine (serve/fast_engine.py) wraps a Hugging Face ``trust_remote_code`` model
(``ArkttsModel`` + ``ArkttsCodec``) whose code and weights are not part of the reference repository.
This module builds a module tree with exactly the attribute names and shapes that
``FastEngine.__init__`` (serve/fast_engine.py:575-645) and ``StreamingVocoder.__init__``
(serve/fast_engine.py:318-366) read, filled with seeded random weights, so that the reference engine,
the CPU oracle (oracle/ref_cpu.py) and the CUDA engine can all be driven from the same weights.

Shapes follow the reference where it pins them (serve/fast_engine.py:1-35, :302, :318-366;
work/ru_sweep.py:42): slow AR 24 x Qwen2 block (896 wide, GQA 14/2, head_dim 64, FFN 4864, qkv bias),
fast AR 4 blocks of the same shape, a 1024-wide 8-layer window-128 codec transformer, two x2
upsample stages (ConvTranspose k2 s2 + ConvNeXt), and a DAC decoder 1024 -> 1536 -> 768 -> 384 ->
192 -> 96 with strides 8, 8, 4, 2.  Values the reference does not pin (codec heads, FFN width,
special token ids, RAS parameters) are synthetic choices listed in ``StandinConfig``.

Every tensor is drawn from one ``torch.Generator`` in a fixed order on the CPU, so the same seed gives
bit-identical weights on any x86 host with the same torch build.
"""
from __future__ import annotations

import math
import zlib
from dataclasses import dataclass, field
from types import SimpleNamespace
from typing import List

import torch
from torch import nn


@dataclass
class StandinConfig:
    # slow AR (serve/fast_engine.py:576-595 reads these names)
    dim: int = 896
    fast_dim: int = 896
    norm_fastlayer_input: bool = True
    max_seq_len: int = 2048
    n_layer: int = 24
    n_head: int = 14
    n_local_heads: int = 2
    head_dim: int = 64
    intermediate_size: int = 4864
    fast_n_layer: int = 4
    fast_n_head: int = 14
    fast_n_local_heads: int = 2
    fast_head_dim: int = 64
    norm_eps: float = 1e-6
    rope_base: float = 1e6
    num_codebooks: int = 10
    codebook_size: int = 4096
    vocab_size: int = 155776
    # synthetic ids (the checkpoint's are not in the reference); se - sb + 1 == 4096
    eos_token_id: int = 151645
    semantic_begin_id: int = 151680
    semantic_end_id: int = 155775
    ras_top_p: float = 0.95
    ras_temperature: float = 1.0
    ras_window_size: int = 10
    codec_sample_rate: int = 44100
    codec_frame_size: int = 2048
    # codec (width 1024 per serve/fast_engine.py:326-335; the rest assumed)
    codec_dim: int = 1024
    codec_n_layer: int = 8
    codec_n_head: int = 8
    codec_head_dim: int = 128
    codec_ffn: int = 4096
    codec_rope_base: float = 10000.0
    codec_cb_dim: int = 8
    codec_res_size: int = 1024
    codec_n_res: int = 9
    ups_kernel: int = 7
    ups_mlp: int = 4096
    dec_channels: List[int] = field(default_factory=lambda: [1536, 768, 384, 192, 96])
    dec_strides: List[int] = field(default_factory=lambda: [8, 8, 4, 2])
    dec_dilations: List[int] = field(default_factory=lambda: [1, 3, 9])
    dec_kernel: int = 7


def tiny_config(**over) -> StandinConfig:
    """Real widths, fewer layers: for tests that need the whole engine on a CPU in seconds."""
    c = StandinConfig(n_layer=2, fast_n_layer=1, codec_n_layer=2)
    for k, v in over.items():
        setattr(c, k, v)
    return c


class _Filler:
    """Seeded fills, in call order."""

    def __init__(self, seed: int):
        self.g = torch.Generator().manual_seed(int(seed))

    def normal(self, t: torch.Tensor, std: float, mean: float = 0.0):
        with torch.no_grad():
            t.copy_(torch.randn(t.shape, generator=self.g) * std + mean)

    def uniform(self, t: torch.Tensor, lo: float, hi: float):
        with torch.no_grad():
            t.copy_(torch.rand(t.shape, generator=self.g) * (hi - lo) + lo)


class RMSNorm(nn.Module):
    def __init__(self, n, eps):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(n))
        self.eps = eps


class _Attention(nn.Module):
    def __init__(self, dim, nq, nkv, hd, bias):
        super().__init__()
        self.n_head, self.n_local_heads, self.head_dim = nq, nkv, hd
        self.wqkv = nn.Linear(dim, (nq + 2 * nkv) * hd, bias=bias)
        self.wo = nn.Linear(nq * hd, dim, bias=False)


class _FFN(nn.Module):
    def __init__(self, dim, inter):
        super().__init__()
        self.w1 = nn.Linear(dim, inter, bias=False)
        self.w3 = nn.Linear(dim, inter, bias=False)
        self.w2 = nn.Linear(inter, dim, bias=False)


class _LayerScale(nn.Module):
    def __init__(self, n):
        super().__init__()
        self.gamma = nn.Parameter(torch.empty(n))


class Block(nn.Module):
    def __init__(self, dim, nq, nkv, hd, inter, eps, bias, layer_scale=False):
        super().__init__()
        self.attention = _Attention(dim, nq, nkv, hd, bias)
        self.feed_forward = _FFN(dim, inter)
        self.attention_norm = RMSNorm(dim, eps)
        self.ffn_norm = RMSNorm(dim, eps)
        if layer_scale:
            self.attention_layer_scale = _LayerScale(dim)
            self.ffn_layer_scale = _LayerScale(dim)


class _ConvWrap(nn.Module):
    """The codec wraps every conv as ``.conv`` (serve/fast_engine.py:184)."""

    def __init__(self, conv):
        super().__init__()
        self.conv = conv


class Snake(nn.Module):
    def __init__(self, c):
        super().__init__()
        self.alpha = nn.Parameter(torch.empty(1, c, 1))


class _Seq(nn.Module):
    def __init__(self, mods):
        super().__init__()
        self.block = nn.ModuleList(mods)


class _VQ(nn.Module):
    def __init__(self, v, d, out):
        super().__init__()
        self.codebook = nn.Embedding(v, d)
        self.out_proj = nn.Conv1d(d, out, 1)


class _DWConv(nn.Module):
    def __init__(self, c, k):
        super().__init__()
        self.conv = nn.Conv1d(c, c, k, groups=c)
        self.kernel_size = k


class _ConvNeXt(nn.Module):
    def __init__(self, c, k, mlp):
        super().__init__()
        self.dwconv = _DWConv(c, k)
        self.norm = nn.LayerNorm(c, eps=1e-6)
        self.pwconv1 = nn.Linear(c, mlp)
        self.pwconv2 = nn.Linear(mlp, c)
        self.gamma = nn.Parameter(torch.empty(c))


class StandinCodec(nn.Module):
    def __init__(self, cfg: StandinConfig):
        super().__init__()
        C = cfg.codec_dim
        self.sample_rate = cfg.codec_sample_rate
        q = nn.Module()
        q.semantic_quantizer = nn.Module()
        q.semantic_quantizer.quantizers = nn.ModuleList([_VQ(cfg.codebook_size, cfg.codec_cb_dim, C)])
        q.quantizer = nn.Module()
        q.quantizer.quantizers = nn.ModuleList(
            [_VQ(cfg.codec_res_size, cfg.codec_cb_dim, C) for _ in range(cfg.codec_n_res)])
        pm = nn.Module()
        pm.input_proj = nn.Identity()
        pm.output_proj = nn.Identity()
        pm.layers = nn.ModuleList([Block(C, cfg.codec_n_head, cfg.codec_n_head, cfg.codec_head_dim, cfg.codec_ffn,
                                         cfg.norm_eps, bias=False, layer_scale=True)
                                   for _ in range(cfg.codec_n_layer)])
        pm.norm = RMSNorm(C, cfg.norm_eps)
        pm.rope_base = cfg.codec_rope_base
        q.post_module = pm
        q.upsample = nn.ModuleList([
            nn.ModuleList([_ConvWrap(nn.ConvTranspose1d(C, C, 2, stride=2)), _ConvNeXt(C, cfg.ups_kernel, cfg.ups_mlp)])
            for _ in range(2)])
        self.quantizer = q
        ch, k = cfg.dec_channels, cfg.dec_kernel
        mods = [_ConvWrap(nn.Conv1d(C, ch[0], k))]
        for i, s in enumerate(cfg.dec_strides):
            cin, cout = ch[i], ch[i + 1]
            blk = [Snake(cin), _ConvWrap(nn.ConvTranspose1d(cin, cout, 2 * s, stride=s))]
            for d in cfg.dec_dilations:
                blk.append(_Seq([Snake(cout), _ConvWrap(nn.Conv1d(cout, cout, k, dilation=d)), Snake(cout),
                                 _ConvWrap(nn.Conv1d(cout, cout, 1))]))
            mods.append(_Seq(blk))
        mods += [Snake(ch[-1]), _ConvWrap(nn.Conv1d(ch[-1], 1, k)), nn.Tanh()]
        self.decoder = nn.Module()
        self.decoder.model = nn.ModuleList(mods)


class StandinModel(nn.Module):
    """The attribute tree FastEngine reads (serve/fast_engine.py:575-639)."""

    def __init__(self, cfg: StandinConfig):
        super().__init__()
        self.config = SimpleNamespace(**cfg.__dict__)
        self.cfg = cfg
        H = cfg.dim
        mk = lambda: Block(H, cfg.n_head, cfg.n_local_heads, cfg.head_dim, cfg.intermediate_size, cfg.norm_eps, True)
        self.layers = nn.ModuleList([mk() for _ in range(cfg.n_layer)])
        self.norm = RMSNorm(H, cfg.norm_eps)
        self.fast_layers = nn.ModuleList([
            Block(H, cfg.fast_n_head, cfg.fast_n_local_heads, cfg.fast_head_dim, cfg.intermediate_size, cfg.norm_eps,
                  True) for _ in range(cfg.fast_n_layer)])
        self.fast_norm = RMSNorm(H, cfg.norm_eps)
        self.embeddings = nn.Embedding(cfg.vocab_size, H)
        self.codebook_embeddings = nn.Embedding(cfg.num_codebooks * cfg.codebook_size, H)
        self.fast_embeddings = nn.Embedding(cfg.codebook_size, H)
        self.fast_output = nn.Linear(H, cfg.codebook_size, bias=False)
        # the codec's fp32 master lives outside the module tree: model.to(bfloat16) (how the serving stack loads the
        # checkpoint) leaves it fp32, and load_codec() hands out copies in the requested dtype, like a checkpoint reload
        object.__setattr__(self, "codec_master", StandinCodec(cfg))
        g = zlib.crc32(b"silence")
        self._sil = torch.tensor([(g >> (3 * k)) % (cfg.codebook_size if k == 0 else cfg.codec_res_size)
                                  for k in range(cfg.num_codebooks)], dtype=torch.long)

    @property
    def device(self):
        return self.embeddings.weight.device

    def load_codec(self, device=None, dtype=torch.float32):
        """ArkttsModel.load_codec: a fresh codec on (device, dtype) from the fp32 master (serve/fast_engine.py:628-632)."""
        import copy
        return copy.deepcopy(self.codec_master).to(device=device if device is not None else self.device, dtype=dtype)

    def encode_audio(self, wav, lens=None):
        """A fixed code frame for every 2048 samples (the stand-in has no encoder; the engine only encodes silence,
        serve/fast_engine.py:637-639)."""
        T = max(1, math.ceil(wav.shape[-1] / self.cfg.codec_frame_size))
        codes = self._sil.to(wav.device).view(1, -1, 1).expand(wav.shape[0], -1, T).contiguous()
        return codes, torch.full((wav.shape[0],), T, dtype=torch.long, device=wav.device)


def _init_block(f: _Filler, blk: Block, cfg_dim, inter, n_layers, bias_std=0.1, ls=None):
    a, ff = blk.attention, blk.feed_forward
    f.normal(a.wqkv.weight, 1.0 / math.sqrt(cfg_dim))
    if a.wqkv.bias is not None:
        f.normal(a.wqkv.bias, bias_std)
    f.normal(a.wo.weight, 0.5 / math.sqrt(a.wo.weight.shape[1] * n_layers))
    f.normal(ff.w1.weight, 1.0 / math.sqrt(cfg_dim))
    f.normal(ff.w3.weight, 1.0 / math.sqrt(cfg_dim))
    f.normal(ff.w2.weight, 0.5 / math.sqrt(inter * n_layers))
    f.normal(blk.attention_norm.weight, 0.1, 1.0)
    f.normal(blk.ffn_norm.weight, 0.1, 1.0)
    if ls is not None:
        f.normal(blk.attention_layer_scale.gamma, 0.02, ls)
        f.normal(blk.ffn_layer_scale.gamma, 0.02, ls)


def build_standin(seed: int = 0, cfg: StandinConfig = None, device="cpu") -> StandinModel:
    """The stand-in model with seeded weights (fp32 master copy on the CPU, then moved)."""
    cfg = cfg or StandinConfig()
    with torch.device("meta"):
        m = StandinModel(cfg)
    m = m.to_empty(device="cpu")
    object.__setattr__(m, "codec_master", m.codec_master.to_empty(device="cpu"))
    g = zlib.crc32(b"silence")
    m._sil = torch.tensor([(g >> (3 * k)) % (cfg.codebook_size if k == 0 else cfg.codec_res_size)
                           for k in range(cfg.num_codebooks)], dtype=torch.long)
    f = _Filler(seed)
    H = cfg.dim
    for blk in m.layers:
        _init_block(f, blk, H, cfg.intermediate_size, cfg.n_layer)
    f.normal(m.norm.weight, 0.1, 1.0)
    for blk in m.fast_layers:
        _init_block(f, blk, H, cfg.intermediate_size, cfg.fast_n_layer)
    f.normal(m.fast_norm.weight, 0.1, 1.0)
    # head logits = normed hidden (|h| ~ sqrt(896)) . embedding row: std 0.1 -> logits std ~3
    f.normal(m.embeddings.weight, 0.1)
    f.normal(m.codebook_embeddings.weight, 0.05)
    f.normal(m.fast_embeddings.weight, 0.1)
    f.normal(m.fast_output.weight, 0.1)
    c = m.codec_master
    q = c.quantizer
    for vq in list(q.semantic_quantizer.quantizers) + list(q.quantizer.quantizers):
        f.normal(vq.codebook.weight, 1.0)
        f.normal(vq.out_proj.weight, 0.5 / math.sqrt(cfg.codec_cb_dim))
        f.normal(vq.out_proj.bias, 0.05)
    C = cfg.codec_dim
    for blk in q.post_module.layers:
        _init_block(f, blk, C, cfg.codec_ffn, cfg.codec_n_layer, ls=0.1)
    f.normal(q.post_module.norm.weight, 0.1, 1.0)
    for tc, cnx in q.upsample:
        f.normal(tc.conv.weight, 1.0 / math.sqrt(C))
        f.normal(tc.conv.bias, 0.05)
        f.normal(cnx.dwconv.conv.weight, 1.0 / math.sqrt(cfg.ups_kernel))
        f.normal(cnx.dwconv.conv.bias, 0.05)
        f.normal(cnx.norm.weight, 0.1, 1.0)
        f.normal(cnx.norm.bias, 0.05)
        f.normal(cnx.pwconv1.weight, 1.0 / math.sqrt(C))
        f.normal(cnx.pwconv1.bias, 0.05)
        f.normal(cnx.pwconv2.weight, 1.0 / math.sqrt(cfg.ups_mlp))
        f.normal(cnx.pwconv2.bias, 0.05)
        f.normal(cnx.gamma, 0.02, 0.2)
    mods = list(c.decoder.model)
    k = cfg.dec_kernel
    f.normal(mods[0].conv.weight, 1.0 / math.sqrt(C * k))
    f.normal(mods[0].conv.bias, 0.05)
    for blk in mods[1:5]:
        bm = list(blk.block)
        f.uniform(bm[0].alpha, 0.5, 1.5)
        w = bm[1].conv.weight                                   # [Cin, Cout, 2s]
        f.normal(w, 1.0 / math.sqrt(w.shape[0] * 2))
        f.normal(bm[1].conv.bias, 0.05)
        for ru in bm[2:]:
            s1, c1, s2, c2 = ru.block
            f.uniform(s1.alpha, 0.5, 1.5)
            f.normal(c1.conv.weight, 1.0 / math.sqrt(c1.conv.weight.shape[1] * k))
            f.normal(c1.conv.bias, 0.05)
            f.uniform(s2.alpha, 0.5, 1.5)
            f.normal(c2.conv.weight, 0.3 / math.sqrt(c2.conv.weight.shape[1]))
            f.normal(c2.conv.bias, 0.05)
    f.uniform(mods[5].alpha, 0.5, 1.5)
    f.normal(mods[6].conv.weight, 0.3 / math.sqrt(cfg.dec_channels[-1] * k))
    f.normal(mods[6].conv.bias, 0.02)
    m.requires_grad_(False)
    if device != "cpu":
        m.to(device)
    return m


class StubTokenizer:
    """Deterministic stand-in for the checkpoint tokenizer: the prompt template pieces
    (serve/fast_engine.py:906-915) map to fixed id lists; other text is split on whitespace, integers are taken as
    ids and any other word is hashed into [0, 151643)."""

    FIXED = {
        "<|im_start|>system\n": [151644, 8948, 198],
        "convert the provided text to speech reference to the following:\n\nText:\n": [14166, 279, 3897, 1467, 311,
                                                                                         8806, 5785, 311, 279, 2701, 25],
        "\n\nSpeech:\n": [271, 55625, 510],
        "<|im_end|>\n": [151645, 198],
        "<|im_start|>user\n": [151644, 872, 198],
        "<|im_start|>assistant\n<|voice|>": [151644, 77091, 198, 151673],
        "convert the provided text to speech": [14166, 279, 3897, 1467, 311, 8806],
    }

    def encode(self, s, add_special_tokens=False):
        if s in self.FIXED:
            return list(self.FIXED[s])
        out = []
        for w in str(s).split():
            out.append(int(w) if w.isdigit() else zlib.crc32(w.encode()) % 151643)
        return out
