"""ctypes binding of libaudio8_b200.so (include/audio8_b200.h).

The library is built in-tree (``__graft_entry__.build()``) next to this file. There is no fallback: importing a
compute entry point on a machine without the library, or calling one without a B200, raises.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libaudio8_b200.so")

c_void_p, c_int, c_float, c_ll, c_ull = C.c_void_p, C.c_int, C.c_float, C.c_longlong, C.c_ulonglong

ERRORS = {0: "ok", 1: "bad argument", 2: "CUDA call failed", 3: "TMA alignment rule broken", 4: "workspace too small",
          5: "no sm_100 device"}

EPI_BF16, EPI_F32_ROUND, EPI_SILU, EPI_ROPE, EPI_GELU, EPI_LSRES, EPI_RESID = range(7)


class A8Epilogue(C.Structure):
    _fields_ = [("kind", c_int), ("bias", c_void_p), ("cos", c_void_p), ("sin", c_void_p), ("pos", c_void_p),
                ("slot", c_void_p), ("kc", c_void_p), ("vc", c_void_p), ("nq", c_int), ("nkv", c_int), ("hd", c_int),
                ("ring", c_int), ("cache_len", c_int), ("gamma", c_void_p), ("res", c_void_p), ("ldres", c_int),
                ("ssq_out", c_void_p), ("ssq_ld", c_int), ("norm_w", c_void_p), ("ssq_in", c_void_p),
                ("eps", c_float)]


class A8Scratch(C.Structure):
    _fields_ = [("h", c_void_p), ("q", c_void_p), ("o", c_void_p), ("a", c_void_p), ("mlp", c_void_p),
                ("attn_ws", c_void_p), ("attn_ws_floats", c_ll), ("attn_counters", c_void_p),
                ("n_attn_counters", c_int), ("ssq", c_void_p), ("ssq_ld", c_int)]


class A8StackDesc(C.Structure):
    _fields_ = [("layers", c_int), ("dim", c_int), ("nq", c_int), ("nkv", c_int), ("hd", c_int), ("inter", c_int),
                ("eps", c_float), ("wqkv", c_void_p), ("bqkv", c_void_p), ("wo", c_void_p), ("w13", c_void_p),
                ("w2", c_void_p), ("ln1", c_void_p), ("ln2", c_void_p), ("norm", c_void_p), ("cos", c_void_p),
                ("sin", c_void_p), ("kc", c_void_p), ("vc", c_void_p), ("cache_rows", c_int), ("cache_len", c_int),
                ("ring", c_int)]


class A8StackRun(C.Structure):
    _fields_ = [("x", c_void_p), ("ldx", c_int), ("rows", c_int), ("pos", c_void_p), ("slot", c_void_p),
                ("lens", c_void_p), ("lens_max", c_int), ("rowmap", c_void_p), ("max_len", c_int),
                ("scratch", A8Scratch), ("blocks", c_void_p), ("nblocks", c_int)]


MAX_UPS, MAX_CONV_OPS = 4, 40
STATE_CLEAR, STATE_LOAD, STATE_SNAPSHOT = 0, 1, 2


class A8ConvRun(C.Structure):
    _fields_ = [("xin", c_void_p), ("rows", c_int), ("T", c_int), ("Cin", c_int), ("ctx", c_int), ("w", c_void_p),
                ("N", c_int), ("taps", c_int), ("dil", c_int), ("bias", c_void_p), ("res", c_void_p),
                ("res_bs", c_ll), ("res_ts", c_ll), ("raw", c_void_p), ("raw_bs", c_ll), ("raw_ts", c_ll),
                ("nxt", c_void_p), ("nxt_bs", c_ll), ("nxt_off", c_ll), ("cout", c_int), ("alpha", c_void_p),
                ("inv", c_void_p), ("audio", c_void_p), ("audio_bs", c_ll)]


class A8CtxShift(C.Structure):
    _fields_ = [("xin", c_void_p), ("ctx", c_int), ("T", c_int), ("Cin", c_int)]


class A8ConvOp(C.Structure):
    _fields_ = [("w", c_void_p), ("bias", c_void_p), ("alpha", c_void_p), ("inv", c_void_p), ("xin", c_void_p),
                ("Cin", c_int), ("N", c_int), ("taps", c_int), ("dil", c_int), ("ctx", c_int), ("T", c_int),
                ("raw", c_int), ("res", c_int)]


class A8Upsample(C.Structure):
    _fields_ = [("tw", c_void_p), ("tb", c_void_p), ("dww", c_void_p), ("dwb", c_void_p), ("st", c_void_p),
                ("st_bs", c_ll), ("K", c_int), ("eps", c_float), ("lnw", c_void_p), ("lnb", c_void_p),
                ("w1", c_void_p), ("b1", c_void_p), ("w2", c_void_p), ("b2", c_void_p), ("gamma", c_void_p),
                ("mlp", c_int)]


class A8Vocoder(C.Structure):
    _fields_ = [("B", c_int), ("ncb", c_int), ("C", c_int), ("v_sem", c_int), ("v_res", c_int), ("max_pos", c_int),
                ("window", c_int), ("up", c_int), ("t_sem", c_void_p), ("t_res", c_void_p), ("pos", c_void_p),
                ("pos_c", c_void_p), ("lens", c_void_p), ("x", c_void_p), ("post", A8StackDesc),
                ("scratch", A8Scratch), ("n_ups", c_int), ("ups", A8Upsample * MAX_UPS), ("ubuf", c_void_p * 4),
                ("n_ops", c_int), ("ops", A8ConvOp * MAX_CONV_OPS), ("act", c_void_p * 2), ("ctx_table", c_void_p),
                ("n_ctx", c_int), ("conv_ctas", c_int), ("audio", c_void_p)]


class A8StateSeg(C.Structure):
    _fields_ = [("base", c_void_p), ("slot_stride", c_ll), ("chunk_bytes", c_ll), ("chunk_stride", c_ll),
                ("nchunks", c_int), ("blob_off", c_ll)]


class A8Engine(C.Structure):
    _fields_ = [("B", c_int), ("S", c_int), ("H", c_int), ("ncb", c_int), ("cbk", c_int), ("nsem", c_int),
                ("vocab", c_int), ("ras_w", c_int), ("eos", c_ll), ("sb", c_ll), ("do_sample", c_int),
                ("top_k", c_int), ("top_p", c_float), ("temperature", c_float), ("ras_top_p", c_float),
                ("ras_temperature", c_float), ("seed", c_ull), ("slow", A8StackDesc), ("fast", A8StackDesc),
                ("emb", c_void_p), ("cbemb", c_void_p), ("head", c_void_p), ("fast_emb", c_void_p),
                ("fast_out", c_void_p), ("tok", c_void_p), ("hid", c_void_p), ("cpos", c_void_p),
                ("prev", c_void_p), ("nstep", c_void_p), ("tok_in", c_void_p), ("frame_prev", c_void_p),
                ("sil_frame", c_void_p), ("tick_ctr", c_void_p), ("tick_id", c_void_p), ("x_fast2", c_void_p),
                ("x_fast", c_void_p), ("x_slow", c_void_p), ("codes", c_void_p), ("logits", c_void_p),
                ("ld_logits", c_int), ("f_pos", c_void_p), ("f_pos0", c_void_p), ("f_slot0", c_void_p),
                ("scratch", A8Scratch), ("voc", C.POINTER(A8Vocoder)), ("side", c_void_p),
                ("rec_logits", c_void_p)]


class A8Resample(C.Structure):
    _fields_ = [("table", c_void_p), ("hist", c_void_p), ("n_in", c_void_p), ("n_out", c_void_p), ("left", c_void_p),
                ("flags", c_void_p), ("up", c_int), ("down", c_int), ("taps", c_int), ("hist_len", c_int),
                ("zpad", c_int), ("frame", c_int), ("rows", c_int), ("out_max", c_int), ("period", c_int),
                ("half", c_ll)]


# name -> (restype, argtypes)
SIGNATURES = {
    "a8_device_ok": (c_int, []),
    "a8_get_error": (c_int, [C.POINTER(c_int)]),
    "a8_clear_error": (c_int, []),
    "a8_launch_count": (c_ll, []),
    "a8_gemm": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_void_p, c_int, C.POINTER(A8Epilogue),
                        c_int, c_void_p]),
    "a8_attention_workspace": (c_int, [c_int, c_int, c_int, c_int, C.POINTER(c_ll), C.POINTER(c_int)]),
    "a8_attention": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                             c_void_p, c_void_p, c_int, c_int, c_float, c_void_p, c_int, c_void_p, c_ll, c_void_p,
                             c_int, c_void_p]),
    "a8_prefill_attention": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
                                     c_int, c_void_p, c_int, c_int, c_float, c_void_p, c_int, c_void_p]),
    "a8_attention_noalloc": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
                                     c_int, c_void_p, c_void_p, c_int, c_int, c_float, c_void_p, c_int, c_void_p]),
    "a8_rmsnorm": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_float,
                           c_void_p]),
    "a8_embed_frame": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                               c_int, c_void_p]),
    "a8_tick_start": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_ll, c_int, c_void_p, c_void_p, c_void_p, c_int,
                              c_int, c_void_p, c_void_p, c_void_p]),
    "a8_gather_rows": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "a8_sample": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_float, c_float, c_ull, c_int, c_void_p,
                          c_void_p, c_void_p]),
    "a8_conv": (c_int, [C.POINTER(A8ConvRun), c_void_p]),
    "a8_ctx_shift": (c_int, [c_void_p, c_int, c_int, c_void_p]),
    "a8_conv_input": (c_int, [c_void_p, c_int, c_ll, c_int, c_int, c_void_p, c_int, c_void_p, c_void_p, c_int,
                              c_void_p]),
    "a8_ups_dwln": (c_int, [c_void_p, c_int, c_int, c_void_p, c_ll, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                            c_float, c_void_p, c_int, c_void_p]),
    "a8_codec_embed": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p,
                               c_void_p, c_int, c_int, c_int, c_void_p]),
    "a8_voc_step": (c_int, [C.POINTER(A8Vocoder), c_void_p, c_int, c_void_p]),
    "a8_voc_decode": (c_int, [C.POINTER(A8Vocoder), c_void_p, c_int, c_void_p]),
    "a8_state_rows": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "a8_resample_reset": (c_int, [C.POINTER(A8Resample), c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "a8_resample_step": (c_int, [C.POINTER(A8Resample), c_void_p, c_int, c_void_p, c_ll, c_int, c_void_p, c_void_p,
                                 c_int, c_void_p, c_void_p]),
    "a8_stack_forward": (c_int, [C.POINTER(A8StackDesc), C.POINTER(A8StackRun), c_void_p]),
    "a8_tick": (c_int, [C.POINTER(A8Engine), c_int, c_void_p]),
    "a8_slow_step": (c_int, [C.POINTER(A8Engine), c_int, c_void_p]),
    "a8_prefill_finish": (c_int, [C.POINTER(A8Engine), c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
    "a8_embed_prompt": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                c_void_p]),
}

_lib = None


class A8Error(RuntimeError):
    pass


def load():
    """The loaded library (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise A8Error(f"{LIB_PATH} is missing: build it with __graft_entry__.build() (there is no CPU fallback)")
        lib = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(rc, what="a8"):
    if rc != 0:
        raise A8Error(f"{what}: {ERRORS.get(rc, rc)}")


def call(name, *args):
    """Call an entry point and raise on a non-zero status."""
    check(getattr(load(), name)(*args), name)


def device_error():
    """The device-side error record (synchronises): (code, kernel, block, extra)."""
    out = (c_int * 4)()
    check(load().a8_get_error(out), "a8_get_error")
    return tuple(out)


def ptr(t):
    """Device address of a tensor (or None)."""
    return None if t is None else C.c_void_p(t.data_ptr())


def stream_handle(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)
