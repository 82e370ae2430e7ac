#!/usr/bin/env python3
"""Benchmark of the Audio8 decode tick on B200 (one JSON line on stdout, rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload cfg2|cfg1|cfg3|streams]

Workload cfg2 (the default): the full tick at 192 rows -- slow AR step, fast AR, streaming
codec -- replayed from one CUDA graph; value = frames/s, e2e = the same with each tick's inputs copied in from pinned
host memory and its audio, tokens and frames copied back; roofline = the codec conv with the largest time. The same
line then carries `serving`: --serve-streams closed-loop users a GPU (default 1408, 1536 slots) for --serve-seconds (default 30)
through the serving loop, with P95 RTF / TTFA and whether the real-time bars held (every rank runs its own replica).

Workloads cfg3 / streams (configs[3], [4] under torchrun): the serving loop (serving.ContinuousBatcher) over an engine of
1024 slots on a Poisson trace (40 req/s a GPU for 60 s; with N GPUs one global trace at 40N req/s split by
least-loaded assignment) or on --streams closed-loop users; value = real-time streams a GPU, with P95 RTF and TTFA.

Workload cfg1: the slow-AR decode step alone, bf16, bucket of 64 slots, each slot's KV
length drawn uniform in [200, 1500] from seed 1, one new token a slot, the stand-in model's full shapes (24 layers,
896 wide, GQA 14/2, FFN 4864, semantic head of 4097 rows). A step = input embedding + 24 layers + head + semantic draw
+ state update, replayed from one CUDA graph; every slot's position is restored before each step so the workload is
the same at every step. Data: synthetic (seeded random weights and KV; no checkpoint or dataset is involved).

--impl reference times the reference's own CPU implementation of the path: the reference has none (Triton only),
so it is the CPU restatement oracle/ref_cpu.py on all host threads, on a bounded sample of the same workload.
Multi-GPU (torchrun, N > 1): one independent replica per GPU (streams shard across replicas; nothing is exchanged),
value = all ranks' frames / the slowest rank's time.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

B_CFG1 = 64
L_LO, L_HI = 200, 1500
METRIC = "tick frames/s"
UNIT = "frames/s"


def _peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class Clocks:
    """nvidia-smi samples (SM clock, throttle reasons) while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.rows, self.proc, self.n0 = index, [], None, 0

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.time()                     # the timed region starts once samples are flowing (<= 3 s)
            while not self.rows and time.time() - t0 < 3.0 and self.proc.poll() is None:
                time.sleep(0.01)
        except (OSError, FileNotFoundError):
            self.proc = None
        self.n0 = len(self.rows)                 # samples taken before the region are not counted (if others came)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.t.join(timeout=2)

    def summary(self):
        rows = [r for r in self.rows[self.n0:] if len(r) >= 9] or [r for r in self.rows if len(r) >= 9]
        if not rows:
            return None
        sm = sorted(float(r[1]) for r in rows)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows)}


def cfg1_lengths():
    import torch
    g = torch.Generator().manual_seed(1)
    return torch.randint(L_LO, L_HI + 1, (B_CFG1,), generator=g)


def cfg1_bytes_flops(lens, layers=24):
    """Algorithmic HBM bytes and FLOPs of one cfg1 step (no padding rows or columns counted)."""
    b = len(lens)
    sl = int(lens.sum())
    w_layer = (1152 * 896 + 1152) * 2 + 896 * 896 * 2 + 9728 * 896 * 2 + 896 * 4864 * 2 + 2 * 896 * 2
    weights = layers * w_layer + 4097 * 896 * 2
    kv = layers * 2 * 2 * 64 * 2 * sl                       # K and V, 2 kv heads, hd 64, bf16
    kv_write = layers * 2 * 2 * 64 * 2 * b
    flops = 2 * b * (layers * 14_909_440 + 4097 * 896) + layers * 4 * 14 * 64 * sl
    return weights + kv + kv_write, flops, kv // layers


def cpu_sample(steps, threads=None):
    """The CPU restatement of the cfg1 step (all host threads): frames/s over a bounded number of steps."""
    import torch
    from oracle import ref_cpu as R
    from oracle.standin import StandinConfig, build_standin
    torch.set_num_threads(threads or os.cpu_count())
    m = build_standin(0, StandinConfig(fast_n_layer=1, codec_n_layer=1))
    c = m.config
    lens = cfg1_lengths()
    st = R.Stack(m.layers, m.norm, c.n_head, c.n_local_heads, c.head_dim, c.norm_eps, c.rope_base,
                 cache_rows=B_CFG1 + 1, cache_len=int(lens.max()) + 1, max_pos=int(lens.max()) + 1)
    g = torch.Generator().manual_seed(3)
    st.kc.copy_(R.bf(torch.randn(st.kc.shape, generator=g)))
    st.vc.copy_(R.bf(torch.randn(st.vc.shape, generator=g)))
    emb = R.bf(m.embeddings.weight.detach().float())
    head = torch.cat([emb[c.semantic_begin_id:c.semantic_end_id + 1], emb[c.eos_token_id:c.eos_token_id + 1]])
    x = R.bf(torch.randn(B_CFG1, c.dim, generator=g) * 0.1)
    pos = (lens - 1).to(torch.int32)
    ar = torch.arange(B_CFG1, dtype=torch.int32)
    t0 = time.perf_counter()
    for _ in range(steps):
        h = st.forward(x.clone(), pos, ar, pos + 1, rowmap=False)
        R.linear(h, head).argmax(-1)
    dt = time.perf_counter() - t0
    return B_CFG1 * steps / dt, torch.get_num_threads(), dt


def run_reference(args):
    if args.workload == "cfg2":
        return run_reference_cfg2(args)
    if args.workload in ("cfg3", "streams"):
        return run_reference_serving(args)
    value, cores, dt = cpu_sample(max(1, args.steps))
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": 0, "ms_per_step": round(1000 * dt / max(1, args.steps), 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (bf16 rounding points)",
            "data": "synthetic", "config": cfg_dict(1),
            "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": f"{args.steps} cfg1 steps (64 rows, KV U[200,1500], 24 layers + head)"},
            "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_reference_serving(args):
    """The CPU path as a stream count: its full-tick throughput (cfg2 sample) x frame length x 0.7 -- the streams it
    could keep at RTF 0.7 if its throughput held at any row count (an upper bound; a trace is not replayed on it)."""
    steps = max(1, min(args.steps, 2))
    fps, cores, dt = cpu_sample_cfg2(args.cpu_rows, steps)
    value = fps * (2048 / 44100) * 0.7
    line = {"impl": "reference", "metric": SERVE_METRIC, "value": round(value, 3), "unit": "streams",
            "n_gpus": args.gpus, "steps": steps, "warmup": 0, "ms_per_step": round(1000 * dt / steps, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 (bf16 / fp16 rounding points)", "data": "synthetic", "config": serve_dict(args, 1),
            "cpu_baseline": {"value": round(value, 3), "unit": "streams", "cores": cores, "kind": "port",
                             "sample": f"{steps} full tick(s) of {args.cpu_rows} rows on the CPU restatement "
                                       f"({fps:.2f} frames/s), as streams at RTF 0.7"},
            "e2e": {"value": round(value, 3), "unit": "streams", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_reference_cfg2(args):
    steps = max(1, min(args.steps, 2))
    value, cores, dt = cpu_sample_cfg2(args.cpu_rows, steps)
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus,
            "steps": steps, "warmup": 0, "ms_per_step": round(1000 * dt / steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 (bf16 / fp16 rounding points)", "data": "synthetic",
            "config": cfg2_dict(1),
            "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": f"{steps} cfg2 tick(s) of {args.cpu_rows} of the 192 rows (full tick with "
                                       f"codec) on the CPU restatement"},
            "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def cfg_dict(world):
    return {"workload": "cfg1: slow-AR decode step, bf16, 64 slots, KV length U[200,1500] (seed 1), 1 token a slot",
            "model": "Audio8 stand-in (seeded random weights, reference shapes)", "global_batch": B_CFG1 * world,
            "seq_len": f"{L_LO}-{L_HI}", "parallelism": f"replicas x{world}",
            "l2": "inputs larger than L2 (716 MB weights + ~670 MB KV a step)"}


def run_ours(args, rank, world, local):
    import ctypes as C

    import torch
    import torch.distributed as dist

    import __graft_entry__ as G
    from oracle.standin import StandinConfig, StubTokenizer, build_standin
    G.build()
    a8 = G.load_package()
    L = a8._lib
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    model = build_standin(0, StandinConfig(codec_n_layer=1))
    gp = dict(do_sample=True, temperature=0.8, top_k=50, top_p=0.95)
    eng = a8.FastEngine(model, StubTokenizer(), gp, max_slots=B_CFG1, max_seq=2048, buckets=[B_CFG1],
                        seq_from_env=False, seed=1234 + rank)
    del model
    b = B_CFG1
    lens = cfg1_lengths()
    g = torch.Generator(device=dev).manual_seed(3 + rank)
    for t in (eng.slow.kc, eng.slow.vc):
        t[:, :b].normal_(generator=g)
    cpos0 = (lens - 1).to(torch.int32).to(dev)
    eng.cpos[:b].copy_(cpos0)
    tok0 = (eng.sb + torch.randint(0, 4096, (b,), generator=g, device=dev)).long()
    codes0 = torch.randint(0, 4096, (b, eng.ncg), generator=g, device=dev)
    eng.tok_in.copy_(tok0)
    eng.codes.copy_(codes0)
    eng.hid[:b].normal_(generator=g)
    eng.nstep[:b].fill_(5)

    def step():
        eng.cpos[:b].copy_(cpos0)
        eng.slow_step(b)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
        step()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    n0 = L.load().a8_launch_count()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    launches = L.load().a8_launch_count() - n0
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        torch.cuda.synchronize()
        e0.record()
        for _ in range(args.steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.barrier()
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t)
    value = world * b * args.steps / (ms / 1000.0)
    err = a8.device_error()
    assert err[0] == 0, err

    # end to end through the public API: the step's inputs from pinned host memory, the drawn tokens back
    h_tok = tok0.cpu().pin_memory()
    h_codes = codes0.cpu().pin_memory()
    h_out = torch.empty(b, dtype=torch.int64).pin_memory()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record()
    for _ in range(args.steps):
        eng.tok_in.copy_(h_tok, non_blocking=True)
        eng.codes.copy_(h_codes, non_blocking=True)
        graph.replay()
        h_out.copy_(eng.tok[:b], non_blocking=True)
    e3.record()
    torch.cuda.synchronize()
    ms_e2e = e2.elapsed_time(e3)
    t = torch.tensor([ms_e2e], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_e2e = float(t)
    e2e = {"value": round(world * b * args.steps / (ms_e2e / 1000.0), 3), "unit": UNIT,
           "h2d_bytes_per_step": h_tok.numel() * 8 + h_codes.numel() * 8, "d2h_bytes_per_step": h_out.numel() * 8}

    roof = roofline(eng, L, lens, dev, args)
    line = None
    if rank == 0:
        nbytes, flops, _ = cfg1_bytes_flops(lens)
        line = {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": cfg_dict(world), "roofline": roof, "e2e": e2e, "gpu_launches": int(launches) * args.steps,
                "clocks": clk.summary(),
                "step_roofline": {"bound": "hbm", "algorithmic_bytes": nbytes, "flops": flops,
                                  "achieved_gbs": round(nbytes / (ms / args.steps / 1000.0) / 1e9, 1)}}
        if world == 1 and not args.no_cpu:
            v, cores, dt = cpu_sample(args.cpu_steps)
            line["cpu_baseline"] = {"value": round(v, 3), "unit": UNIT, "cores": cores, "kind": "port",
                                    "sample": f"{args.cpu_steps} cfg1 steps on the CPU oracle ({dt:.1f} s)"}
    if world > 1:
        dist.barrier()
    del graph
    return line


def roofline(eng, L, lens, dev, args):
    """Per-launch timing of the step's dominant kernels, each recorded for its 24 layers into a graph and timed with
    CUDA events on the stream it runs on: split-K decode attention (HBM: the KV it reads) and the w13 GEMM
    (HBM: its weights). Returns the one with the larger total time, with its achieved fraction of the peak."""
    import ctypes as C

    import torch
    hbm, _, kind = _peaks()
    b = B_CFG1
    st = eng.slow
    lens_d = lens.to(torch.int32).to(dev)
    sc = eng.scratch
    out = {}

    def timed(fn, n_launch):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        a, z = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = max(3, args.steps // 2)
        a.record()
        for _ in range(reps):
            g.replay()
        z.record()
        torch.cuda.synchronize()
        return a.elapsed_time(z) / (reps * n_launch) / 1000.0     # seconds per launch

    def attn_all():
        for l in range(st.layers):
            L.call("a8_attention", L.ptr(sc.q), 896, L.ptr(st.kc), L.ptr(st.vc), st.layers, st.cache_rows, 14, 2, 64,
                   st.cache_len, l, L.ptr(lens_d), None, b, st.cache_len, 0.0, L.ptr(sc.o), 896, L.ptr(sc.attn_ws),
                   sc.attn_ws.numel(), L.ptr(sc.attn_counters), sc.attn_counters.numel(), L.stream_handle())

    def w13_all():
        e = L.A8Epilogue(kind=L.EPI_SILU)
        for l in range(st.layers):
            L.call("a8_gemm", L.ptr(sc.h), 896, C.c_void_p(st.w13[l].data_ptr()), 2 * st.inter, 896, b, L.ptr(sc.mlp),
                   st.inter, C.byref(e), 0, L.stream_handle())

    t_attn = timed(attn_all, st.layers)
    kv_bytes = 2 * 2 * 64 * 2 * int(lens.sum()) + b * 14 * 64 * 2 * 2
    t_w13 = timed(w13_all, st.layers)
    w13_bytes = 2 * st.inter * 896 * 2 + b * (896 + st.inter) * 2
    cand = {"attention": (t_attn, kv_bytes), "w13_gemm": (t_w13, w13_bytes)}
    name = max(cand, key=lambda k: cand[k][0])
    t, nbytes = cand[name]
    achieved = nbytes / t / 1e9
    traffic = None
    tp = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(tp):
        tr = json.load(open(tp)).get(name)
        if tr:
            traffic = int(tr["bytes_per_unit"] * (int(lens.sum()) if name == "attention" else 1))
    return {"kernel": name, "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
            "frac": round(achieved / hbm, 4), "peak_kind": kind, "traffic": traffic,
            "algorithmic_bytes_per_launch": nbytes, "us_per_launch": round(t * 1e6, 2),
            "others": {k: {"us_per_launch": round(v[0] * 1e6, 2), "gbs": round(v[1] / v[0] / 1e9, 1)}
                       for k, v in cand.items() if k != name}}


# ---------------------------------------------------------------------------------------------------- cfg2
B_CFG2 = 192
L2_LO, L2_HI = 100, 2000


def cfg2_lengths(b=B_CFG2):
    import torch
    g = torch.Generator().manual_seed(2)
    return torch.randint(L2_LO, L2_HI + 1, (b,), generator=g)


def cfg2_dict(world):
    return {"workload": "cfg2: full tick, bf16, 192 rows: fast AR (2-token pass + 8 passes), slow AR step (KV length "
                        "U[100,2000], seed 2), streaming codec (window-128 transformer, 2 upsample stages, 29-conv "
                        "decoder, 2048 samples a row) on its side stream; codes uniform random",
            "model": "Audio8 stand-in (seeded random weights, reference shapes)", "global_batch": B_CFG2 * world,
            "seq_len": f"{L2_LO}-{L2_HI}", "parallelism": f"replicas x{world}",
            "l2": "inputs larger than L2 (~0.9 GB of weights + ~1.5 GB of slow KV read a tick)"}


def cpu_sample_cfg2(rows, ticks, threads=None):
    """The CPU restatement of the cfg2 tick (all host threads) on `rows` of the 192: frames/s."""
    import torch
    from oracle import ref_cpu as R
    from oracle.standin import StandinConfig, StubTokenizer, build_standin
    torch.set_num_threads(threads or os.cpu_count())
    m = build_standin(0, StandinConfig())
    gp = dict(do_sample=True, temperature=0.8, top_k=50, top_p=0.95)
    ora = R.OracleEngine(m, StubTokenizer(), gp, max_slots=rows, max_seq=2048, seed=1234)
    del m
    lens = cfg2_lengths()[:rows]
    g = torch.Generator().manual_seed(3)
    for t in (ora.slow.kc, ora.slow.vc):
        t[:, :rows].copy_(R.bf(torch.randn(t[:, :rows].shape, generator=g)))
    ora.cpos[:rows] = (lens - 1).to(torch.int32)
    ora.tok[:rows] = ora.sb + torch.randint(0, 4096, (rows,), generator=g)
    ora.hid[:rows] = R.bf(torch.randn(rows, ora.H, generator=g))
    ora.frame_prev[:rows] = torch.randint(0, 4096, (rows, ora.ncg), generator=g)
    ora.nstep[:rows] = 5
    t0 = time.perf_counter()
    for _ in range(ticks):
        ora.cpos[:rows] = (lens - 1).to(torch.int32)
        ora.tick(rows)
    dt = time.perf_counter() - t0
    return rows * ticks / dt, torch.get_num_threads(), dt


def conv_flops(voc, b):
    """Algorithmic FLOPs of each decoder conv of one codec step at b rows (output channels unpadded)."""
    out = []
    for c, T, *_ in voc.ops:
        out.append(2 * b * T * (c.ph * c.Cout) * c.taps * c.Cin)
    return out


def run_ours_cfg2(args, rank, world, local):
    import torch
    import torch.distributed as dist

    import __graft_entry__ as G
    from oracle.standin import StandinConfig, StubTokenizer, build_standin
    G.build()
    a8 = G.load_package()
    L = a8._lib
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    model = build_standin(0, StandinConfig())
    gp = dict(do_sample=True, temperature=0.8, top_k=50, top_p=0.95)
    b = B_CFG2
    eng = a8.FastEngine(model, StubTokenizer(), gp, max_slots=b, max_seq=2048, buckets=[b], seq_from_env=False,
                        seed=1234 + rank)
    del model
    lens = cfg2_lengths()
    g = torch.Generator(device=dev).manual_seed(3 + rank)
    for t in (eng.slow.kc, eng.slow.vc, eng.voc.post.kc, eng.voc.post.vc):
        t.normal_(generator=g)
    eng.voc.pos.fill_(1000)                               # steady state: every row attends a full 128-frame window
    cpos0 = (lens - 1).to(torch.int32).to(dev)
    eng.cpos[:b].copy_(cpos0)
    tok0 = (eng.sb + torch.randint(0, 4096, (b,), generator=g, device=dev)).long()
    frame0 = torch.randint(0, 4096, (b, eng.ncg), generator=g, device=dev)
    eng.tok[:b].copy_(tok0)
    eng.frame_prev.copy_(frame0)
    eng.hid[:b].normal_(generator=g)
    eng.nstep[:b].fill_(5)

    def step():
        eng.cpos[:b].copy_(cpos0)
        eng.tick(b)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
        step()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    n0 = L.load().a8_launch_count()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    launches = L.load().a8_launch_count() - n0
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        torch.cuda.synchronize()
        e0.record()
        for _ in range(args.steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.barrier()
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t)
    value = world * b * args.steps / (ms / 1000.0)
    err = a8.device_error()
    assert err[0] == 0, err

    # end to end as the serving loop drives it: each tick's input state (tokens, the frame to decode) from pinned host
    # memory, then the tick, then its audio, consumed tokens and frames read back
    h_tok, h_frame = tok0.cpu().pin_memory(), frame0.cpu().pin_memory()
    h_audio = torch.empty(b, eng.up, dtype=torch.float32).pin_memory()
    h_tin = torch.empty(b, dtype=torch.int64).pin_memory()
    h_fp = torch.empty(b, eng.ncg, dtype=torch.int64).pin_memory()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record()
    for _ in range(args.steps):
        eng.tok[:b].copy_(h_tok, non_blocking=True)
        eng.frame_prev.copy_(h_frame, non_blocking=True)
        graph.replay()
        h_audio.copy_(eng.audio[:b], non_blocking=True)
        h_tin.copy_(eng.tok_in[:b], non_blocking=True)
        h_fp.copy_(eng.frame_prev[:b], non_blocking=True)
    e3.record()
    torch.cuda.synchronize()
    ms_e2e = e2.elapsed_time(e3)
    t = torch.tensor([ms_e2e], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_e2e = float(t)
    e2e = {"value": round(world * b * args.steps / (ms_e2e / 1000.0), 3), "unit": UNIT,
           "h2d_bytes_per_step": h_tok.numel() * 8 + h_frame.numel() * 8,
           "d2h_bytes_per_step": h_audio.numel() * 4 + h_tin.numel() * 8 + h_fp.numel() * 8}
    del graph
    roof, convs = conv_roofline(eng, L, dev, b, args)
    line = None
    if rank == 0:
        tick_ms = ms / args.steps
        line = {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(tick_ms, 4), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (codec convs fp16)", "data": "synthetic",
                "config": cfg2_dict(world), "roofline": roof, "e2e": e2e, "gpu_launches": int(launches) * args.steps,
                "clocks": clk.summary(),
                "realtime": {"frame_ms": round(1000 * eng.up / eng.sr, 3), "rtf_at_192": round(
                    tick_ms / (1000 * eng.up / eng.sr), 4)},
                "codec_convs": convs}
        if world == 1 and not args.no_cpu:
            rows = args.cpu_rows
            v, cores, dt = cpu_sample_cfg2(rows, args.cpu_steps)
            line["cpu_baseline"] = {"value": round(v, 3), "unit": UNIT, "cores": cores, "kind": "port",
                                    "sample": f"{args.cpu_steps} cfg2 tick(s) of {rows} of the 192 rows on the CPU "
                                              f"oracle ({dt:.1f} s)"}
    if world > 1:
        dist.barrier()
    return line


def _conv_traffic(top, b):
    """DRAM bytes a launch of this conv shape moved in the committed ncu capture (profiles/traffic.json), or None."""
    tp = os.path.join(REPO, "profiles", "traffic.json")
    if not os.path.exists(tp):
        return None
    key = f"cin{top['Cin']}_n{top['N']}_k{top['taps']}_t{top['T']}_rows{b}"
    e = json.load(open(tp)).get("k_conv", {}).get(key)
    return int(e["bytes_per_unit"]) if e else None


def conv_roofline(eng, L, dev, b, args):
    """Each decoder conv of the codec step timed alone (CUDA events around each launch on its stream, L2 flushed
    between launches); the roofline line is the conv with the largest total time (tensor-bound: its algorithmic
    FLOPs / duration against the measured bf16 peak; fp16 and bf16 run at the same tensor-core rate)."""
    import ctypes as C

    import torch
    _, tf, kind = _peaks()
    voc = eng.voc
    flops = conv_flops(voc, b)
    # L2 flushed between launches by reading 256 MB (a read leaves no dirty lines whose write-back would be charged to
    # the timed launch)
    flush = torch.ones(64 << 20, dtype=torch.float32, device=dev)
    fsum = torch.empty((), device=dev)
    reps = max(3, min(10, args.steps))
    res = []
    for i, (c, T, *_) in enumerate(voc.ops):
        run = voc.conv_run(i, b)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps + 2)]
        for k, (a, z) in enumerate(ev):
            torch.sum(flush, dim=0, out=fsum)
            a.record()
            L.call("a8_conv", C.byref(run), L.stream_handle())
            z.record()
        torch.cuda.synchronize()
        t = sum(a.elapsed_time(z) for a, z in ev[2:]) / reps / 1000.0
        res.append({"op": i, "Cin": c.Cin, "N": c.N, "taps": c.taps, "T": T, "us": round(t * 1e6, 2),
                    "tflops": round(flops[i] / t / 1e12, 1)})
    assert L.device_error()[0] == 0
    top = max(res, key=lambda x: x["us"])
    achieved = flops[top["op"]] / (top["us"] * 1e-6) / 1e12
    total_us = sum(x["us"] for x in res)
    roof = {"kernel": f"k_conv (decoder op {top['op']}: Cin {top['Cin']}, N {top['N']}, taps {top['taps']}, "
                      f"T {top['T']}, {b} rows)", "bound": "tensor", "achieved": round(achieved, 1), "peak": tf,
            "unit": "TFLOP/s", "frac": round(achieved / tf, 4), "peak_kind": f"{kind} (burst bf16)",
            "traffic": _conv_traffic(top, b), "algorithmic_flops_per_launch": flops[top["op"]], "us_per_launch": top["us"],
            "all_convs": {"us_total": round(total_us, 1), "tflops": round(sum(flops) / (total_us * 1e-6) / 1e12, 1)}}
    return roof, res


SERVE_METRIC = "real-time streams/GPU at P95 RTF<0.7"
SERVE_BUCKETS = [1, 2, 4, 6, 8, 12, 16, 20, 24, 28, 32, 40, 48, 56, 64, 72, 80, 88, 96, 104, 112, 120, 128, 144, 160,
                 176, 192, 224, 256, 288, 320, 384, 448, 512, 576, 640, 704, 768, 832, 896, 960, 992, 1024, 1056, 1088,
                 1120, 1152, 1184, 1216, 1248, 1280, 1312, 1344, 1376, 1408, 1440, 1472, 1504, 1536, 1600, 1664, 1728,
                 1792]


def serve_dict(args, world):
    if args.workload == "streams":
        w = (f"closed loop: {args.streams} streams a GPU, each asking for its next utterance when one ends, for "
             f"{args.seconds:g} s")
    else:
        w = (f"cfg{3 if world == 1 else 4}: Poisson arrivals at {args.rate * world:g} req/s for {args.seconds:g} s"
             + (f", assigned to {world} replicas by least-loaded slot count" if world > 1 else ""))
    return {"workload": w + "; prompts U[20,200] random ids, one of 8 cached voices (150-frame prefixes), output "
                            "geometric mean 300 frames capped 1024; ragged packed prefill into running ticks, "
                            f"max_slots {args.slots}; audio out "
                            + (f"int16 at {args.out_sr} Hz (GPU resampler + PCM16)" if args.out_sr
                               else "fp32 at 44.1 kHz"),
            "model": "Audio8 stand-in (seeded random weights, reference shapes)", "parallelism": f"replicas x{world}",
            "timing": "wall clock, as the reference's serving numbers (RTF = wall time / audio length, TTFA "
                      "included); the first tick of a row (its silence frame) is not audio"}


def run_serving(args, rank, world, local):
    """BASELINE configs[3] (1 GPU) and [4] (one replica a GPU): the trace through serving.ContinuousBatcher."""
    import numpy as np
    import torch
    import torch.distributed as dist

    import __graft_entry__ as G
    from oracle.standin import StandinConfig, StubTokenizer, build_standin
    G.build()
    a8 = G.load_package()
    import importlib
    S = importlib.import_module(a8.__name__ + ".serving")
    torch.cuda.set_device(local)
    model = build_standin(0, StandinConfig())
    ncb = int(model.config.num_codebooks)
    gp = dict(do_sample=True, temperature=0.8, top_k=50, top_p=0.95)
    t0 = time.perf_counter()
    eng = a8.FastEngine(model, StubTokenizer(), gp, max_slots=args.slots, max_seq=2048,
                        buckets=[b for b in SERVE_BUCKETS if b <= args.slots], seq_from_env=False, seed=1234 + rank)
    del model
    eng.capture(log=lambda *a: None)
    t_build = time.perf_counter() - t0
    if args.workload == "streams":
        loop = S.ClosedLoop(args.streams, args.seconds, seed=11 + rank, ncb=ncb)
        reqs, follow, voices = loop.initial, loop.follow, loop.voices
    else:
        reqs, voices = S.poisson_trace(args.rate * world, args.seconds, seed=11, ncb=ncb)
        if world > 1:
            k = S.assign_least_loaded(reqs, world)
            reqs = [r for r, kk in zip(reqs, k) if kk == rank]
        follow = None
    S.warm_voices(eng, voices)
    # warm the admission path (first-call host work) on throwaway requests, then start from clean slots
    warm = [S.Request(rid=-1 - i, arrival=0.0, text=" ".join(["7"] * 20), item=voices[i % len(voices)][1],
                      key=voices[i % len(voices)][0], cap=4) for i in range(min(64, args.slots))]
    bat = S.ContinuousBatcher(eng, admit_every=args.admit_every, admit_batch=args.admit_batch,
                              max_admit=args.max_admit, copy_audio=not args.out_sr, out_sr=args.out_sr or None)
    bat.run(warm)
    torch.cuda.synchronize()
    eng.reset_state()
    if world > 1:
        dist.barrier()
    with Clocks(local) as clk:
        st = bat.run(reqs, follow=follow)
    err = a8.device_error()
    assert err[0] == 0, err
    done = st.finished()
    mine = {"ttfa": [r.t_first - r.arrival for r in done],
            "rtf": [(r.t_done - r.arrival) / (r.frames * st.frame_s) for r in done],
            "frames": sum(r.frames for r in done), "wall": st.wall, "streams": st.busy_time / max(1e-9, st.wall),
            "ticks": st.ticks, "summary": st.summary(), "launches": None}
    allr = [mine]
    if world > 1:
        allr = [None] * world
        dist.all_gather_object(allr, mine)
    if rank != 0:
        return None
    ttfa = np.concatenate([np.array(a["ttfa"]) for a in allr]) * 1000
    rtf = np.concatenate([np.array(a["rtf"]) for a in allr])
    p95_rtf, p95_ttfa = float(np.percentile(rtf, 95)), float(np.percentile(ttfa, 95))
    wall = max(a["wall"] for a in allr)
    streams = sum(a["streams"] for a in allr)
    ok = p95_rtf < 0.7 and p95_ttfa < 800
    frames = sum(a["frames"] for a in allr)
    # closed loop: the offered streams count when P95 RTF < 0.7 and P95 TTFA < 800 ms hold, else 0; open-loop trace:
    # the time-averaged concurrent streams it sustained (with meets_target saying whether the bars held)
    value = (args.streams * world if ok else 0.0) if args.workload == "streams" else streams
    line = {"metric": SERVE_METRIC, "value": round(value, 1), "unit": "streams", "n_gpus": world,
            "steps": sum(a["ticks"] for a in allr), "warmup": len(warm), "ms_per_step": round(
                1000 * wall / max(1, max(a["ticks"] for a in allr)), 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (codec convs fp16)",
            "data": "synthetic", "config": serve_dict(args, world),
            "meets_target": ok, "mean_streams": round(streams, 1), "rtf_p95": round(p95_rtf, 4), "rtf_p50": round(float(np.percentile(rtf, 50)), 4),
            "ttfa_ms_p95": round(p95_ttfa, 1), "ttfa_ms_p50": round(float(np.percentile(ttfa, 50)), 1),
            "frames_per_s": round(frames / wall, 1), "finished": int(len(rtf)),
            "per_rank": [a["summary"] for a in allr], "build_s": round(t_build, 1), "clocks": clk.summary(),
            "e2e": {"value": round(value, 1), "unit": "streams", "h2d_bytes_per_step": None,
                    "d2h_bytes_per_step": eng.B * (8 + (4 + 2 * bat.rs.out_max if bat.rs is not None
                                                        else 4 * eng.up)),
                    "note": "the trace is end to end by itself: prompts in, every tick's tokens and audio read back "
                            "to pinned host memory" + (f" (int16 at {args.out_sr} Hz, converted on the GPU)"
                                                       if args.out_sr else " (fp32 at the codec rate)")}}
    return line


def cfg2_engine(rank=0):
    """The cfg2 workload's engine and state (as run_ours_cfg2 sets it up); returns (eng, step) with step() one tick."""
    import torch

    import __graft_entry__ as G
    from oracle.standin import StandinConfig, StubTokenizer, build_standin
    G.build()
    a8 = G.load_package()
    dev = torch.device("cuda", torch.cuda.current_device())
    model = build_standin(0, StandinConfig())
    gp = dict(do_sample=True, temperature=0.8, top_k=50, top_p=0.95)
    b = B_CFG2
    eng = a8.FastEngine(model, StubTokenizer(), gp, max_slots=b, max_seq=2048, buckets=[b], seq_from_env=False,
                        seed=1234 + rank)
    del model
    lens = cfg2_lengths()
    g = torch.Generator(device=dev).manual_seed(3 + rank)
    for t in (eng.slow.kc, eng.slow.vc, eng.voc.post.kc, eng.voc.post.vc):
        t.normal_(generator=g)
    eng.voc.pos.fill_(1000)
    cpos0 = (lens - 1).to(torch.int32).to(dev)
    eng.cpos[:b].copy_(cpos0)
    eng.tok[:b].copy_((eng.sb + torch.randint(0, 4096, (b,), generator=g, device=dev)).long())
    eng.frame_prev.copy_(torch.randint(0, 4096, (b, eng.ncg), generator=g, device=dev))
    eng.hid[:b].normal_(generator=g)
    eng.nstep[:b].fill_(5)

    def step():
        eng.cpos[:b].copy_(cpos0)
        eng.tick(b)
    return a8, eng, step


def run_profile(args):
    """One eager cfg2 tick (after two warm-up ticks), or one decoder conv launch at 192 rows, inside
    cudaProfilerStart/Stop -- the region an `ncu --profile-from-start off` capture sees."""
    import ctypes as C

    import torch
    what = args.profile
    if what == "resample":
        return profile_resample()
    if what == "admit":
        return profile_admit()
    if what == "sample":
        return profile_sample()
    a8, eng, step = cfg2_engine()
    L = a8._lib
    if what == "tick":
        fn = step
    elif what.startswith("conv:"):
        i = int(what.split(":")[1])
        run = eng.voc.conv_run(i, B_CFG2)
        fn = lambda: L.call("a8_conv", C.byref(run), L.stream_handle())
    else:
        raise SystemExit(f"--profile {what}: expected tick, conv:I or resample")
    for _ in range(2):
        step()
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    fn()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    err = a8.device_error()
    assert err[0] == 0, err
    print(json.dumps({"profile": what, "ok": True}), flush=True)


def profile_admit(n=8):
    """One admission chunk of n config-0 requests (100-frame voice prefix, 64 text ids) into an engine of the full
    stand-in, its voice's prefix K/V cached by a first admission: the packed prefill's kernels (prompt embedding, the
    24 layers with the tensor-core causal attention, head and first-token draw) between cudaProfilerStart/Stop."""
    from types import SimpleNamespace

    import torch

    import __graft_entry__ as G
    from oracle.standin import StandinConfig, StubTokenizer, build_standin
    G.build()
    a8 = G.load_package()
    model = build_standin(0, StandinConfig())
    eng = a8.FastEngine(model, StubTokenizer(), dict(do_sample=True, temperature=0.8, top_k=50, top_p=0.95),
                        max_slots=2 * n, max_seq=2048, buckets=[n], seq_from_env=False, seed=5)
    g = torch.Generator().manual_seed(0)
    item = SimpleNamespace(ref_code=torch.randint(0, 4096, (100, 10), generator=g), ref_text="12 34 56 78 90")
    reqs = [dict(text=" ".join(str(int(x)) for x in torch.randint(0, 151643, (64,), generator=g)), item=item,
                 key="v0") for _ in range(n)]
    eng.admit(list(range(n)), reqs)
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    eng.admit(list(range(n, 2 * n)), reqs)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    err = a8.device_error()
    assert err[0] == 0, err
    print(json.dumps({"profile": "admit", "ok": True, "rows": int(eng.cpos[n])}), flush=True)


def profile_sample(rows=B_CFG2, V=4097, launches=4):
    """`launches` sampled draws (top-k 50, top-p 0.95, temperature 0.8) over rows x V logits rounded to bf16, as the
    semantic head gives them (capture the last with `ncu -s launches-1 -c 1`), then 20 timed with CUDA events."""
    import torch

    import __graft_entry__ as G
    G.build()
    a8 = G.load_package()
    L = a8._lib
    g = torch.Generator().manual_seed(0)
    lg = (torch.randn(rows, V + 3, generator=g) * 3).to(torch.bfloat16).float().cuda()
    out = torch.empty(rows, dtype=torch.int64, device="cuda")
    call = lambda: L.call("a8_sample", L.ptr(lg), V + 3, V, rows, 1, 50, 0.95, 0.8, 7, 16, None, L.ptr(out),
                          L.stream_handle())
    for _ in range(launches):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(20):
        call()
    e1.record()
    torch.cuda.synchronize()
    err = a8.device_error()
    assert err[0] == 0, err
    print(json.dumps({"profile": "sample", "rows": rows, "V": V, "us_per_launch": round(e0.elapsed_time(e1) * 50, 2)}),
          flush=True)


def profile_resample(b=B_CFG2, ticks=20):
    """The per-slot resampler (44.1 -> 16 kHz + PCM16) at the cfg2 bucket: `ticks` timed steps (CUDA events), then
    one step inside cudaProfilerStart/Stop. Prints one JSON line with the step time and its FMA rate."""
    import importlib

    import torch

    import __graft_entry__ as G
    G.build()
    a8 = G.load_package()
    RS = importlib.import_module(a8.__name__ + ".resample")
    dev = torch.device("cuda", torch.cuda.current_device())
    rs = RS.Resampler(b, 44100, 16000, 2048, dev)
    g = torch.Generator(device=dev).manual_seed(5)
    audio = (torch.rand(b, 2048, generator=g, device=dev) - 0.5).float()
    tok = torch.zeros(b, dtype=torch.int64, device=dev)
    rs.reset(list(range(b)), [1 << 30] * b, drop_first=False)
    for _ in range(3):
        rs.step(audio, tok, -1, b)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    outs = 0
    e0.record()
    for _ in range(ticks):
        _, cnt = rs.step(audio, tok, -1, b)
    e1.record()
    torch.cuda.synchronize()
    outs = int(cnt.sum())
    us = e0.elapsed_time(e1) * 1000 / ticks
    torch.cuda.profiler.start()
    rs.step(audio, tok, -1, b)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    err = a8.device_error()
    assert err[0] == 0, err
    fma = outs * rs.taps
    print(json.dumps({"profile": "resample", "ok": True, "rows": b, "us_per_step": round(us, 2),
                      "outputs_per_step": outs, "taps": rs.taps, "gfma_per_s": round(fma / us / 1e3, 1),
                      "bytes_per_step": b * (2048 * 4 + rs.out_max * 2 + 2 * rs.hist_len * 4)}), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="cfg2", choices=["cfg1", "cfg2", "cfg3", "streams"])
    ap.add_argument("--rate", type=float, default=40.0, help="cfg3/cfg4 arrivals a GPU (req/s)")
    ap.add_argument("--seconds", type=float, default=60.0, help="cfg3/cfg4/streams: trace length")
    ap.add_argument("--streams", type=int, default=512, help="streams: closed-loop users a GPU")
    ap.add_argument("--slots", type=int, default=1024, help="cfg3/streams: max_slots")
    ap.add_argument("--admit-every", type=int, default=2, help="admit every N ticks (serve/engine_worker.py default 2)")
    ap.add_argument("--admit-batch", type=int, default=8, help="or as soon as N wait (reference default 8)")
    ap.add_argument("--max-admit", type=int, default=64)
    ap.add_argument("--cpu-steps", type=int, default=None, help="CPU baseline sample: steps (cfg1 3, cfg2 6)")
    ap.add_argument("--cpu-rows", type=int, default=64, help="cfg2 CPU baseline sample: rows of the 192")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--profile", default=None, metavar="tick|conv:I|resample|admit|sample",
                    help="no timing: run one eager cfg2 tick (or decoder conv I alone at 192 rows, or the 44.1 -> "
                         "16 kHz resampler step at 192 rows, one admission of 8 config-0 prompts, or sampler draws over "
                         "192 x 4097 logits) between "
                         "cudaProfilerStart/Stop, for ncu "
                         "--profile-from-start off")
    ap.add_argument("--serve-streams", type=int, default=1408,
                    help="cfg2: closed-loop streams a GPU of the serving run reported under `serving`")
    ap.add_argument("--serve-seconds", type=float, default=30.0,
                    help="cfg2: length of that serving run (0: none)")
    ap.add_argument("--serve-slots", type=int, default=1536, help="cfg2: max_slots of that serving run")
    ap.add_argument("--out-sr", type=int, default=16000,
                    help="cfg3/streams: each stream converted to this rate + PCM16 on the GPU (the worker's "
                         "TTS_OUT_SR; 0 = read back fp32 frames at the codec rate)")
    args = ap.parse_args()
    if args.profile:
        return run_profile(args)
    args.warmup = max(3, args.warmup)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    args.gpus = world if world > 1 else args.gpus
    if args.cpu_steps is None:
        args.cpu_steps = 3 if args.workload == "cfg1" else 6        # ~10 s of CPU work either way
    if args.impl == "reference":
        if rank == 0:
            run_reference(args)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    run = {"cfg1": run_ours, "cfg2": run_ours_cfg2, "cfg3": run_serving, "streams": run_serving}[args.workload]
    line = run(args, rank, world, local)
    if args.workload == "cfg2" and args.serve_seconds > 0:
        # the headline metric's serving half: sustained streams at P95 RTF < 0.7 / P95 TTFA < 800 ms, measured by
        # the serving loop itself on every rank (one replica a GPU) after the tick timing above
        import gc

        import torch
        gc.collect()
        torch.cuda.empty_cache()
        sa = argparse.Namespace(**vars(args))
        sa.workload, sa.streams, sa.seconds, sa.slots = "streams", args.serve_streams, args.serve_seconds, \
            args.serve_slots
        srv = run_serving(sa, rank, world, local)
        if rank == 0 and line is not None and srv is not None:
            line["serving"] = {k: srv[k] for k in ("metric", "value", "unit", "meets_target", "rtf_p95", "rtf_p50",
                                                   "ttfa_ms_p95", "ttfa_ms_p50", "frames_per_s", "finished",
                                                   "mean_streams", "ms_per_step", "build_s", "clocks")}
            line["serving"]["streams_offered"] = args.serve_streams * world
            line["serving"]["config"] = srv["config"]["workload"] + f"; max_slots {args.serve_slots}; " + \
                srv["config"]["timing"]
    if rank == 0 and line is not None:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
