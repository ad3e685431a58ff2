#!/usr/bin/env python3
"""Benchmark of the NSRL integer transformer block on B200.

Workload (per GPU): one prenorm causal attention + gated-MLP block forward,
d_model 256, 4 heads x 64, MLP hidden 1024, seq 1024, batch 64 sequences
(65,536 tokens), Q15 Gaussian sigma 4096 activations, i8 uniform weights.
A step is one block forward over the batch; `value` is tokens/s over all
ranks (weak scaling: every rank runs its own 64 sequences, no collective on
the data path).  `e2e` is the same metric through the public C-ABI call with
the input copied from pinned host memory and the output copied back inside
the timed region.  The L2 is flushed (256 MiB memset) before every step.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

`--impl reference` times the CPU oracle (a C++ port of the reference's Rust
kernels) on all host threads over a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

D_MODEL, HEADS, HIDDEN, SEQ, BATCH = 256, 4, 1024, 1024, 64
HEAD_DIM = D_MODEL // HEADS
TOKENS = BATCH * SEQ
E2E_CHUNKS = (8, 16, 32)  # sequences per chunk of the host-buffer pipeline: each timed, the fastest reported
METRIC = "int attention-block tokens/s @1/2/4/8 B200, %INT8/HBM roofline, bit-exact"
WORKLOAD = "prenorm causal attention + gated-MLP block forward, d256 h4x64 ff1024 s1024 b64/gpu"
# dram__bytes_read.sum + dram__bytes_write.sum per launch, from the ncu captures
# summarised in profiles/ (attention: 342.1 MB read + 289.8 MB written; the gated
# linear: 35.9 MB + 81.6 MB; decode at batch 32: 544.6 MB + 3.8 MB).
NCU_TRAFFIC = {"attention_tc_hd64": 641520384, "linear_tc_gated": 117480704, "attention_decode": 548445696}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        j = json.load(open(p))
        return j["hbm_gbs"], j["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while running."""
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.FIELDS,
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[3:7]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def make_block_inputs(rank: int):
    """Block weights (shared seed) and this rank's input batch (rank-specific seed)."""
    from nsrl_b200 import synth as Y
    bw = Y.BlockWeights(seed=2024, d=D_MODEL, hidden=HIDDEN)
    chunks = []
    rows = BATCH * SEQ
    step = 1 << 12
    base = Y.tensor_seed(0xB200 + rank, 99)
    for r0 in range(0, rows, step):
        chunks.append(Y.q15_gaussian(Y.tensor_seed(base, r0), (min(step, rows - r0), D_MODEL)))
    return bw, np.concatenate(chunks)


def oracle_module():
    """The oracle, loaded as its -march=native build (every CPU leg times the same build)."""
    from oracle import oracle as O
    O.use_native()
    return O


def cpu_sample(bw, x, threads: int, sequences: int, heads: int = HEADS):
    """Times the oracle block (attention + MLP) over the first `sequences`
    sequences of x; returns (tokens/s, seconds, output)."""
    O = oracle_module()
    L = {nm: O.Linear(getattr(bw, nm), O.scales(1, bw.shift[nm], bw.out_dim(nm)))
         for nm in ("q", "k", "v", "o", "up", "gate", "down")}
    xs = x[:sequences * SEQ]
    t0 = time.perf_counter()
    y1, _ = O.prenorm_attention_block(xs, sequences, SEQ, D_MODEL, heads, bw.attn_gamma, 1,
                                      L["q"], L["k"], L["v"], L["o"], threads=threads)
    y2, _ = O.prenorm_mlp_block(y1, sequences * SEQ, D_MODEL, HIDDEN, bw.mlp_gamma, 1, L["up"], L["gate"], L["down"],
                                threads=threads)
    dt = time.perf_counter() - t0
    return sequences * SEQ / dt, dt, y2


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    oracle_module()
    threads = os.cpu_count() or 1
    bw, x = make_block_inputs(0)
    seqs = max(1, min(BATCH, threads))
    for _ in range(args.warmup):
        cpu_sample(bw, x, threads, seqs)
    rates = []
    t_total = 0.0
    for _ in range(args.steps):
        r, dt, _ = cpu_sample(bw, x, threads, seqs)
        rates.append(r)
        t_total += dt
    value = seqs * SEQ * args.steps / t_total
    sample = f"{seqs} sequences x {SEQ} tokens per step ({threads} threads, one sequence per thread)"
    out = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * t_total / args.steps,
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int16xint8->int32/int64",
           "data": "synthetic (seeded SplitMix64)",
           "config": {"workload": WORKLOAD, "d_model": D_MODEL, "heads": HEADS, "head_dim": HEAD_DIM,
                      "hidden_dim": HIDDEN, "seq_len": SEQ, "batch_per_step": seqs},
           "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
           "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)
    return 0


def kernel_table(core_lib):
    import ctypes as C
    n = core_lib.nsrl_profile_count()
    rows = {}
    name = C.c_char_p()
    ms, ops, byt = C.c_float(), C.c_double(), C.c_double()
    core_lib.nsrl_profile_entry.argtypes = [C.c_size_t, C.POINTER(C.c_char_p), C.POINTER(C.c_float),
                                            C.POINTER(C.c_double), C.POINTER(C.c_double)]
    for i in range(n):
        if core_lib.nsrl_profile_entry(i, C.byref(name), C.byref(ms), C.byref(ops), C.byref(byt)) != 0:
            raise RuntimeError("profile read failed")
        r = rows.setdefault(name.value.decode(), {"launches": 0, "ms": 0.0, "ops": 0.0, "bytes": 0.0})
        r["launches"] += 1
        r["ms"] += ms.value
        r["ops"] += ops.value
        r["bytes"] += byt.value
    return n, rows


TENSOR_KERNELS = ("linear_tc", "attention_prefill", "attention_tc", "accumulate_weight_grad",
                  "attention_grad_products", "attention_dlogit", "attention_bwd", "linear_simt")

# Config 5 (decode) and config 2 (linear sweep), measured after the headline.
DEC_LAYERS, DEC_D, DEC_H, DEC_F, DEC_B, DEC_PREFIX = 4, 512, 8, 2048, 256, 8192
SWEEP_M, SWEEP_KN = (4096, 16384, 65536), (256, 1024, 4096)


def run_decode(core, torch, steps, warmup, hbm, flush, batch=DEC_B):
    """4-layer KV-cache decode steps: per layer the prenorm attention decode block then the
    prenorm gated-MLP block over the batch's new tokens; the caches hold DEC_PREFIX + t rows."""
    DEC_B = batch
    from nsrl_b200 import synth as Y
    L = core.lib()
    gen = torch.Generator(device="cuda").manual_seed(5)
    lmax = DEC_PREFIX + warmup + 2 * steps + 1
    layers = []
    for li in range(DEC_LAYERS):
        bw = Y.BlockWeights(seed=77 + li, d=DEC_D, hidden=DEC_F)
        lin = {nm: core.Linear(torch.from_numpy(getattr(bw, nm)), core.make_scales(1, bw.shift[nm], bw.out_dim(nm)))
               for nm in ("q", "k", "v", "o", "up", "gate", "down")}
        caches = []
        for _ in range(2):  # K and V: Q15 Gaussian sigma 4096 (K narrower so that the softmax stays live)
            c = torch.empty((DEC_B, DEC_H, lmax, DEC_D // DEC_H), dtype=torch.int16, device="cuda")  # head-major
            c.copy_((torch.randn(c.shape, generator=gen, device="cuda") * 4096).clamp_(-32768, 32767).to(torch.int16))
            caches.append(c)
        caches[0] >>= 5
        layers.append((lin, caches, torch.from_numpy(bw.attn_gamma).cuda(), torch.from_numpy(bw.mlp_gamma).cuda()))
    x0 = (torch.randn((DEC_B, DEC_D), generator=gen, device="cuda") * 4096).clamp_(-32768, 32767).to(torch.int16)
    pos = torch.full((DEC_B,), DEC_PREFIX, dtype=torch.int32, device="cuda")
    ws = core.workspace(max(L.nsrl_decode_block_workspace_size(DEC_B, DEC_D, DEC_H),
                            L.nsrl_mlp_workspace_size(DEC_B, DEC_D, DEC_F)))
    st = core.Status()
    h = torch.empty_like(x0)
    y = torch.empty_like(x0)
    lp = {}

    def step(x):
        for lin, (kc, vc), ga, gm in layers:
            ps = [lin[n].c() for n in ("q", "k", "v", "o")]
            r = L.nsrl_prenorm_attention_decode_block(
                core._ptr(x), DEC_B, DEC_D, DEC_H, core._ptr(ga), 1, *[core.C.byref(p) for p in ps], core._ptr(kc),
                core._ptr(vc), core._ptr(pos), lmax, core._ptr(h), core._ptr(ws), ws.numel(), core._ptr(st.buf),
                core._stream())
            if r != 0:
                raise RuntimeError(L.nsrl_last_error())
            pm = [lin[n].c() for n in ("up", "gate", "down")]
            r = L.nsrl_prenorm_gated_mlp_residual_block(core._ptr(h), DEC_B, DEC_D, DEC_F, core._ptr(gm), 1,
                                                        *[core.C.byref(p) for p in pm], core._ptr(y), core._ptr(ws),
                                                        ws.numel(), core._ptr(st.buf), core._stream())
            if r != 0:
                raise RuntimeError(L.nsrl_last_error())
            x = y.clone()
        pos.add_(1)
        return x

    st.reset()
    x = x0
    for _ in range(warmup):
        x = step(x)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        x = step(x)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    # the same number of steps again with per-launch events, for the kernel table
    ctx_rows = DEC_PREFIX + warmup + steps  # keys attended at the first profiled step = this + 1
    L.nsrl_profile_reset()
    L.nsrl_profile_enable(1)
    for _ in range(steps):
        x = step(x)
    torch.cuda.synchronize()
    L.nsrl_profile_enable(0)
    code, hs = st.fetch()
    if code != 0:
        raise RuntimeError(f"decode rejected (flags {hs.flags:#x})")
    _, rows = kernel_table(L)
    dec = rows["attention_decode"]
    # algorithmic bytes of the profiled decode-attention launches: every cached K
    # and V row once (positions + 1 keys), plus q in and the context out
    keys = sum(DEC_B * (ctx_rows + t + 1) for t in range(steps)) * DEC_LAYERS
    dbytes = 2.0 * 2 * DEC_D * keys + 2.0 * 2 * DEC_D * DEC_B * steps * DEC_LAYERS
    ach = dbytes / (dec["ms"] / 1000.0) / 1e9
    return {"workload": f"{DEC_LAYERS}-layer decode step, d{DEC_D} h{DEC_H}x{DEC_D // DEC_H} ff{DEC_F}, "
                        f"batch {DEC_B}, KV prefix {DEC_PREFIX} (+t), i16 cache",
            "value": DEC_B * steps / (ms / 1000.0), "unit": "tokens/s", "steps": steps, "warmup": warmup,
            "ms_per_step": ms / steps,
            "roofline": {"kernel": "attention_decode", "bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s",
                         "frac": ach / hbm, "ms_per_launch": dec["ms"] / dec["launches"],
                         "algorithmic_bytes_per_launch": dbytes / dec["launches"]},
            "kernel_share": {k: round(v["ms"] / sum(r["ms"] for r in rows.values()), 4) for k, v in rows.items()}}


# Config 4 (training step): 4 layers, d256 h4x64 ff1024, seq 512, global batch
# 256 windows split over the ranks (strong scaling), byte vocabulary 256.
TR_LAYERS, TR_D, TR_H, TR_F, TR_S, TR_BATCH = 4, 256, 4, 1024, 512, 256
LINEARS = ("q", "k", "v", "o", "up", "gate", "down")


def make_train_model(core, torch):
    from nsrl_b200 import synth as Y
    from nsrl_b200 import train as TT
    tw = Y.TrainWeights(seed=4040, layers=TR_LAYERS, d=TR_D, hidden=TR_F, seq_len=TR_S)
    layers = []
    for bw in tw.blocks:
        e = {nm: core.Linear(torch.from_numpy(getattr(bw, nm)), core.make_scales(1, bw.shift[nm], bw.out_dim(nm)))
             for nm in LINEARS}
        e["attn_gamma"] = torch.from_numpy(bw.attn_gamma)
        e["mlp_gamma"] = torch.from_numpy(bw.mlp_gamma)
        layers.append(e)
    head = core.Linear(torch.from_numpy(tw.head), core.make_scales(1, tw.head_shift, 256))
    gm = TT.TrainModel(torch.from_numpy(tw.embeddings), torch.from_numpy(tw.positions), layers, head, TR_D, TR_H,
                       TR_F, TR_S)
    return tw, gm


def oracle_train_model(tw):
    """The oracle's copy of the synthetic training model (its own weight arrays)."""
    O = oracle_module()
    layers = []
    for bw in tw.blocks:
        e = {nm: O.Linear(getattr(bw, nm).copy(), O.scales(1, bw.shift[nm], bw.out_dim(nm))) for nm in LINEARS}
        e["attn_gamma"], e["mlp_gamma"] = bw.attn_gamma, bw.mlp_gamma
        layers.append(e)
    return O.TrainModel(tw.embeddings.copy(), tw.positions.copy(), layers,
                        O.Linear(tw.head.copy(), O.scales(1, tw.head_shift, 256)), TR_D, TR_H, TR_F, TR_S)


def train_cpu_sample(tw, ctx, tgt, threads):
    """The oracle's whole batch on `len(tgt)` windows with one worker per
    thread: forward + backward of every window, the merge in worker order and
    the requantising apply of every parameter."""
    O = oracle_module()
    m = oracle_train_model(tw)
    res = np.zeros(m.arena_layout()["total"], np.int64)
    t0 = time.perf_counter()
    r = O.train_step(m, res, ctx, tgt, workers=threads)
    dt = time.perf_counter() - t0
    if r is None:
        raise RuntimeError("oracle rejected the CPU sample")
    return len(tgt) * TR_S / dt, dt


def train_parity(core, torch, windows=4):
    """One step of the full training model on `windows` fresh windows, on the
    GPU and in the oracle from the same initial model: stats, every updated
    weight and embedding, and the carried residuals must be equal."""
    from nsrl_b200 import synth as Y
    from nsrl_b200 import train as TT
    O = oracle_module()
    tw, gm = make_train_model(core, torch)
    om = oracle_train_model(tw)
    ctx, tgt = Y.train_windows(0x9A41, windows, TR_S)
    cfg = TT.MiniTransformerTrainConfig()
    res = np.zeros(om.arena_layout()["total"], np.int64)
    ref = O.train_step(om, res, ctx, tgt, cfg={f: getattr(cfg, f) for f in O.DEFAULT_TRAIN_CONFIG}, workers=windows)
    state = TT.TrainState(gm)
    got = TT.mini_transformer_train_step(gm, state, torch.from_numpy(ctx).cuda(), torch.from_numpy(tgt).cuda(), cfg,
                                         TT.TrainStepBuffers(gm, windows))
    eq = ref is not None and got == ref
    eq = eq and np.array_equal(gm.head.weights.cpu().numpy(), om.head.weights)
    for gl, ol in zip(gm.layers, om.layers):
        for nm in LINEARS:
            eq = eq and np.array_equal(gl[nm].weights.cpu().numpy(), ol[nm].weights)
    eq = eq and np.array_equal(gm.embeddings.cpu().numpy(), om.embeddings)
    eq = eq and np.array_equal(gm.positions.cpu().numpy(), om.positions)
    eq = eq and np.array_equal(state.residuals.cpu().numpy(), res)
    return {"windows": windows, "compared": "stats, i8 weights, i16 embeddings and positions, residuals",
            "equal": bool(eq)}


def run_train(core, torch, dist, world, rank, steps, warmup, flush, hbm, tfl, src, cpu_baseline, batch=TR_BATCH):
    """Config 4: the data-parallel training step (windows forward + backward,
    exact int64 all-reduce, requantising apply) over `batch` windows per step
    (TR_BATCH for the measurement; smaller for profiling captures)."""
    from nsrl_b200 import synth as Y
    from nsrl_b200 import train as TT
    L = core.lib()
    TR_BATCH = batch
    if TR_BATCH % world:
        raise ValueError("the global batch must split evenly over the ranks")
    W = TR_BATCH // world
    tw, gm = make_train_model(core, torch)
    state = TT.TrainState(gm)
    buf = TT.TrainStepBuffers(gm, W)
    cfg = TT.MiniTransformerTrainConfig()
    e2e_steps = max(1, min(steps, 3))
    prof_steps = 1
    nsteps = warmup + steps + prof_steps + e2e_steps
    ctx_all, tgt_all = Y.train_windows(0x7EA1, nsteps * TR_BATCH, TR_S)
    lo, hi = rank * W, (rank + 1) * W
    win = lambda i, a: a[i * TR_BATCH + lo:i * TR_BATCH + hi]
    # device-resident windows of the warm-up, timed and profiled steps (the `value` leg)
    ndev = warmup + steps + prof_steps
    dctx = [torch.from_numpy(win(i, ctx_all)).cuda() for i in range(ndev)]
    dtgt = [torch.from_numpy(win(i, tgt_all)).cuda() for i in range(ndev)]
    stream = torch.cuda.current_stream()

    def one(i):
        r = TT.mini_transformer_train_step(gm, state, dctx[i], dtgt[i], cfg, buf)
        if r is None:
            raise RuntimeError(f"training batch {i} rejected")
        return r

    for i in range(warmup):
        one(i)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev = []
    last = None
    for i in range(warmup, warmup + steps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        last = one(i)
        b.record(stream)
        ev.append((a, b))
    torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in ev)
    t = torch.tensor([ms], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    # one more step with per-launch events, for the kernel table
    L.nsrl_profile_reset()
    L.nsrl_profile_enable(1)
    for i in range(warmup + steps, ndev):
        flush.zero_()
        one(i)
    torch.cuda.synchronize()
    L.nsrl_profile_enable(0)
    n_launches, rows = kernel_table(L)
    # end to end: each step's own windows copied from pinned host memory, the stats read back
    e2e_ms = 0.0
    for i in range(ndev, nsteps):
        hctx = torch.from_numpy(win(i, ctx_all)).pin_memory()
        htgt = torch.from_numpy(win(i, tgt_all)).pin_memory()
        flush.zero_()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        dc = hctx.cuda(non_blocking=True)
        dt_ = htgt.cuda(non_blocking=True)
        r = TT.mini_transformer_train_step(gm, state, dc, dt_, cfg, buf)
        b.record(stream)
        torch.cuda.synchronize()
        if r is None:
            raise RuntimeError("training batch rejected in the end-to-end loop")
        e2e_ms += a.elapsed_time(b)
    t = torch.tensor([e2e_ms], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item())
    if rank != 0:
        return None
    tokens = TR_BATCH * TR_S
    total = sum(r["ms"] for r in rows.values())
    out = {"workload": f"data-parallel training step, {TR_LAYERS} layers d{TR_D} h{TR_H}x{TR_D // TR_H} ff{TR_F} "
                       f"seq {TR_S}, global batch {TR_BATCH} windows over {world} GPU(s), byte vocabulary 256",
           "metric": "training tokens/s (windows x seq_len per step, whole job)",
           "value": tokens * steps / (ms / 1000.0), "unit": "tokens/s", "steps": steps, "warmup": warmup,
           "ms_per_step": ms / steps, "scaling": "strong", "n_gpus": world,
           "e2e": {"value": tokens * e2e_steps / (e2e_ms / 1000.0), "unit": "tokens/s",
                   "h2d_bytes_per_step": int(W * (TR_S + 1)), "d2h_bytes_per_step": 3 * 8 + 8 * 4 + 8 * 8,
                   "steps": e2e_steps},
           "gpu_launches_per_step": n_launches / prof_steps,
           "last_step": last,
           "roofline": roofline(rows, hbm, tfl, src),
           "kernel_table": f"{prof_steps} further step with per-launch events (the timed steps run without them)",
           "kernels": {k: {"launches": v["launches"], "ms": round(v["ms"], 3), "share": round(v["ms"] / total, 4)}
                       for k, v in sorted(rows.items(), key=lambda kv: -kv[1]["ms"])[:12]}}
    ap = rows.get("dp_apply")
    if ap:  # the requantising apply: algorithmic bytes (gradient, residual or Adam state, weight) over its time
        per = ap["ms"] / ap["launches"]
        gbs = ap["bytes"] / ap["launches"] / (per / 1000.0) / 1e9
        out["apply"] = {"ms_per_launch": round(per, 4), "algorithmic_bytes_per_launch": ap["bytes"] / ap["launches"],
                        "achieved_gbs": round(gbs, 1), "frac_of_hbm": round(gbs / hbm, 4)}
    if world == 1:
        out["parity"] = train_parity(core, torch)
        if not out["parity"]["equal"]:
            raise RuntimeError("training step differs from the oracle")
    if cpu_baseline and world == 1:
        threads = os.cpu_count() or 1
        n = max(1, min(3 * threads, 64))  # about 10 s of CPU work
        rate, dt = train_cpu_sample(tw, ctx_all[:n], tgt_all[:n], threads)
        out["cpu_baseline"] = {"value": rate, "unit": "tokens/s", "cores": threads, "kind": "port",
                               "sample": f"{n} windows x {TR_S} tokens: forward + backward, the merge and the apply "
                                         f"({dt:.1f} s, one worker per thread)"}
    return out


def run_sweep(core, torch, hbm, tflops, flush, reps=5):
    """Config 2: the i16 x i8 linear over M x K (K = N) through nsrl_linear_i16_i8_i16."""
    from nsrl_b200 import synth as Y
    L = core.lib()
    out = []
    for K in SWEEP_KN:
        N = K
        w = torch.from_numpy(Y.i8_uniform(K, (N, K)))
        lin = core.Linear(w, core.make_scales(1, Y.shift_for(K), N))
        for M in SWEEP_M:
            x = Y.q15_gaussian_torch(Y.tensor_seed(0x5EE9, M * 8192 + K), (M, K), "cuda")
            y = torch.empty((M, N), dtype=torch.int16, device="cuda")
            ws = core.workspace(L.nsrl_linear_workspace_size(M, K, N))
            st = core.Status()
            p = lin.c()

            def call():
                r = L.nsrl_linear_i16_i8_i16(core._ptr(x), M, core.C.byref(p), core._ptr(y), core._ptr(ws),
                                             ws.numel(), core._ptr(st.buf), core._stream())
                if r != 0:
                    raise RuntimeError(L.nsrl_last_error())

            for _ in range(3):
                call()
            tot = 0.0
            for _ in range(reps):
                flush.zero_()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                call()
                b.record()
                torch.cuda.synchronize()
                tot += a.elapsed_time(b)
            # the same calls again with per-launch events, for the GEMM's own time
            L.nsrl_profile_reset()
            L.nsrl_profile_enable(1)
            for _ in range(reps):
                flush.zero_()
                call()
            torch.cuda.synchronize()
            L.nsrl_profile_enable(0)
            _, rows = kernel_table(L)
            code, _ = st.fetch()
            if code != 0:
                raise RuntimeError("linear rejected in the sweep")
            gk = [v for k, v in rows.items() if k.startswith("linear_tc")][0]
            ops = 2.0 * M * N * K
            byts = 2.0 * M * K + N * K + 2.0 * M * N
            t_gemm = gk["ms"] / gk["launches"] / 1000.0
            t_call = tot / reps / 1000.0
            roof_s = max(ops / (tflops * 1e12), byts / (hbm * 1e9))
            out.append({"M": M, "K": K, "N": N, "bound": "tensor" if ops / (tflops * 1e12) > byts / (hbm * 1e9)
                        else "hbm", "ms_call": round(t_call * 1e3, 4), "ms_gemm": round(t_gemm * 1e3, 4),
                        "tops_call": ops / t_call / 1e12, "frac_call": roof_s / t_call, "frac_gemm": roof_s / t_gemm})
            del x, y
    return out


def roofline(rows, hbm_gbs, tflops, src):
    name = max(rows, key=lambda k: rows[k]["ms"])
    r = rows[name]
    per_launch_s = r["ms"] / 1000.0 / r["launches"]
    if name.startswith(TENSOR_KERNELS):
        ach = r["ops"] / r["launches"] / per_launch_s / 1e12
        out = {"kernel": name, "bound": "tensor", "achieved": ach, "peak": tflops, "unit": "TFLOP/s",
               "frac": ach / tflops,
               "peak_note": f"{src} dense bf16 burst = nominal int8 dense / 2 = ceiling of an i16xi8 MAC split "
                            "into two int8 MMAs; achieved counts algorithmic integer ops (2 per MAC)"}
    else:
        ach = r["bytes"] / r["launches"] / per_launch_s / 1e9
        out = {"kernel": name, "bound": "hbm", "achieved": ach, "peak": hbm_gbs, "unit": "GB/s",
               "frac": ach / hbm_gbs, "peak_note": f"{src} HBM copy bandwidth"}
    out["traffic"] = NCU_TRAFFIC.get(name)
    out["algorithmic_bytes_per_launch"] = r["bytes"] / r["launches"]
    out["algorithmic_ops_per_launch"] = r["ops"] / r["launches"]
    out["ms_per_launch"] = r["ms"] / r["launches"]
    return out


def run_config1(core, torch, flush, reps=50):
    """The reference's CPU-runnable case: one causal attention layer forward
    (Q, K, V, O linears and the exact softmax), batch 4, seq 128, d_model 128,
    2 heads x 64 (head_dim 32 is rejected by the reference).  A latency line:
    each call timed alone (L2 flushed before it), parity on the whole output."""
    from nsrl_b200 import synth as Y
    O = oracle_module()
    import ctypes as C
    B, S, d, H = 4, 128, 128, 2
    L = core.lib()
    bw = Y.BlockWeights(seed=101, d=d, hidden=4 * d)
    lin = {nm: core.Linear(torch.from_numpy(getattr(bw, nm)), core.make_scales(1, bw.shift[nm], d)) for nm in "qkvo"}
    olin = {nm: O.Linear(getattr(bw, nm), O.scales(1, bw.shift[nm], d)) for nm in "qkvo"}
    x_np = Y.q15_gaussian(Y.tensor_seed(0xC0F1, 1), (B * S, d))
    x = torch.from_numpy(x_np).cuda()
    y = torch.empty_like(x)
    ws = core.workspace(L.nsrl_attention_workspace_size(B, S, d, H))
    st = core.Status()
    ps = [lin[n].c() for n in "qkvo"]

    def call():
        r = L.nsrl_self_attention(core._ptr(x), B, S, d, H, 1, *[C.byref(p) for p in ps], core._ptr(y), core._ptr(ws),
                                  ws.numel(), core._ptr(st.buf), core._stream())
        if r != 0:
            raise RuntimeError(L.nsrl_last_error())

    st.reset()
    for _ in range(5):
        call()
    times = []
    for _ in range(reps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        call()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    code, _ = st.fetch()
    if code != 0:
        raise RuntimeError("config-1 attention rejected")
    ref = O.self_attention(x_np, B, S, d, H, *[olin[n] for n in "qkvo"], causal=True)
    eq = ref is not None and bool(np.array_equal(y.cpu().numpy(), ref))
    if not eq:
        raise RuntimeError("config-1 attention differs from the oracle")
    med = statistics.median(times)
    return {"workload": f"causal attention layer forward (q, k, v, o linears + exact softmax), batch {B}, seq {S}, "
                        f"d{d} h{H}x{d // H}",
            "latency_ms_median": med, "latency_ms_min": min(times), "value": B * S / (med / 1000.0),
            "unit": "tokens/s", "calls": reps, "parity": {"sequences": B, "of": B, "equal": eq}}


def run_block_hd16(core, torch, bw, x_np, flush, hbm, tfl, src, steps=5):
    """The headline block with 16 heads x 16 (the other legal head_dim at
    d_model 256): tokens/s, the kernel table of a profiled pass, parity on two
    sequences."""
    H = 16
    L = core.lib()
    lin = {nm: core.Linear(torch.from_numpy(getattr(bw, nm)), core.make_scales(1, bw.shift[nm], bw.out_dim(nm)))
           for nm in ("q", "k", "v", "o", "up", "gate", "down")}
    blk = core.TransformerBlock(D_MODEL, H, HIDDEN, *[lin[n] for n in ("q", "k", "v", "o", "up", "gate", "down")],
                                torch.from_numpy(bw.attn_gamma), torch.from_numpy(bw.mlp_gamma), 1)
    x = torch.from_numpy(x_np).cuda()
    y = torch.empty_like(x)
    ws = core.workspace(blk.workspace_bytes(BATCH, SEQ))
    st = core.Status()

    def step():
        if blk.launch(x, y, BATCH, SEQ, ws, st) != 0:
            raise RuntimeError(L.nsrl_last_error())

    st.reset()
    for _ in range(3):
        step()
    ms = 0.0
    for _ in range(steps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        step()
        b.record()
        torch.cuda.synchronize()
        ms += a.elapsed_time(b)
    L.nsrl_profile_reset()
    L.nsrl_profile_enable(1)
    for _ in range(steps):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    L.nsrl_profile_enable(0)
    _, rows = kernel_table(L)
    code, _ = st.fetch()
    if code != 0:
        raise RuntimeError("head_dim-16 block rejected")
    _, _, ref = cpu_sample(bw, x_np, 2, 2, heads=H)
    eq = bool(np.array_equal(y[:2 * SEQ].cpu().numpy(), ref))
    if not eq:
        raise RuntimeError("head_dim-16 block differs from the oracle")
    total = sum(r["ms"] for r in rows.values())
    return {"workload": f"the headline block with {H} heads x {D_MODEL // H}", "value": TOKENS * steps / (ms / 1000.0),
            "unit": "tokens/s", "ms_per_step": ms / steps, "steps": steps, "roofline": roofline(rows, hbm, tfl, src),
            "kernels": {k: {"launches": v["launches"], "ms": round(v["ms"], 4), "share": round(v["ms"] / total, 4)}
                        for k, v in sorted(rows.items(), key=lambda kv: -kv[1]["ms"])[:6]},
            "parity": {"sequences": 2, "of": BATCH, "equal": eq}}


def run_generate(core, torch, batch=64, steps=16, prompt_len=256, warmup=1):
    """Byte generation with the training workload's model (4 layers, d256,
    4 x 64 heads, seq 512): `batch` prompts of `prompt_len` bytes, `steps`
    sampled bytes each (top-k 40), every step the full forward of each
    512-byte window as the reference computes it.  Tokens/s = batch * steps
    / time; parity: sequence 0's first 4 bytes against the oracle."""
    from nsrl_b200 import generate as G
    from nsrl_b200 import synth as Y
    O = oracle_module()
    tw = Y.TrainWeights(seed=4040, layers=TR_LAYERS, d=TR_D, hidden=TR_F, seq_len=TR_S)
    head_shift = 15  # a live byte softmax at this model's feature scale
    layers = []
    olayers = []
    for bw in tw.blocks:
        e = {nm: core.Linear(torch.from_numpy(getattr(bw, nm)), core.make_scales(1, bw.shift[nm], bw.out_dim(nm)))
             for nm in LINEARS}
        e["attn_gamma"], e["mlp_gamma"] = torch.from_numpy(bw.attn_gamma), torch.from_numpy(bw.mlp_gamma)
        layers.append(e)
        o = {nm: O.Linear(getattr(bw, nm), O.scales(1, bw.shift[nm], bw.out_dim(nm))) for nm in LINEARS}
        o["attn_gamma"], o["mlp_gamma"] = bw.attn_gamma, bw.mlp_gamma
        olayers.append(o)
    from nsrl_b200 import train as TT
    gm = TT.TrainModel(torch.from_numpy(tw.embeddings), torch.from_numpy(tw.positions), layers,
                       core.Linear(torch.from_numpy(tw.head), core.make_scales(1, head_shift, 256)), TR_D, TR_H, TR_F,
                       TR_S)
    draws = Y.splitmix(0x6E4E, batch * prompt_len) >> np.uint64(57)
    prompts = [bytes((draws[b * prompt_len:(b + 1) * prompt_len] + 32).astype(np.uint8)) for b in range(batch)]
    gen = G.Generator(gm, batch, prompt_len, steps)
    host = torch.from_numpy(np.frombuffer(b"".join(prompts), np.uint8).reshape(batch, prompt_len).copy())
    for _ in range(warmup):
        gen(prompts, "sample", 40, 7)
    gen.contexts[:, :prompt_len].copy_(host)
    gen.status.reset()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    r = gen.launch([prompt_len] * batch, "sample", 40, 7)
    b.record()
    torch.cuda.synchronize()
    if r != 0 or gen.status.fetch()[0] != 0:
        raise RuntimeError("generation rejected")
    ms = a.elapsed_time(b)
    toks = gen.tokens.cpu().numpy()
    om = O.TrainModel(tw.embeddings, tw.positions, olayers, O.Linear(tw.head, O.scales(1, head_shift, 256)), TR_D,
                      TR_H, TR_F, TR_S)
    t0 = time.perf_counter()
    ref = O.generate(om, prompts[0], 4, "sample", 40, 7)
    cpu_s = time.perf_counter() - t0
    eq = ref is not None and bool(np.array_equal(toks[0, :4], ref[0]))
    if not eq:
        raise RuntimeError("generated bytes differ from the oracle")
    return {"workload": f"byte generation, {TR_LAYERS}-layer d{TR_D} h{TR_H}x{TR_D // TR_H} ff{TR_F} window {TR_S}, "
                        f"batch {batch}, prompts of {prompt_len} bytes, {steps} sampled bytes (top-k 40), full "
                        f"window forward per step",
            "value": batch * steps / (ms / 1000.0), "unit": "generated tokens/s", "ms_per_step": ms / steps,
            "steps": steps, "batch": batch,
            "cpu_oracle": {"value": 4 / cpu_s, "unit": "generated tokens/s", "cores": 1,
                           "sample": "4 bytes of one sequence"},
            "parity": {"sequences": 1, "bytes": 4, "equal": eq}}


def run_sharded(args):
    """The config-3 block with heads and batch sharded: ranks form batch groups
    of G ranks (G = --shard-heads, default min(N, heads)); each group runs its
    share of the global batch with positions split G ways for the token-wise
    work and heads split G ways for attention (nsrl_sharded_transformer_block:
    q|k|v and context rows cross NVLink as peer stores from the kernels'
    epilogues).  Total work is fixed as N grows (strong scaling)."""
    import datetime
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", str(29500 + os.getpid() % 1000))
        dist.init_process_group("gloo", rank=0, world_size=1)
    from nsrl_b200 import build, core, shard
    from nsrl_b200 import synth as Y
    build.build()
    L = core.lib()
    G = args.shard_heads or min(world, HEADS)
    Bg_total = args.shard_batch
    if world % G or HEADS % G or SEQ % G or Bg_total % (world // G):
        raise SystemExit(f"--shard-heads {G} does not split {world} ranks / {HEADS} heads / batch {Bg_total}")
    ngroups = world // G
    grp_id, grank = rank // G, rank % G
    groups = [dist.new_group(list(range(g * G, (g + 1) * G))) for g in range(ngroups)] if world > 1 else [None]
    pg = groups[grp_id]
    Bg = Bg_total // ngroups
    bw = Y.BlockWeights(seed=2024, d=D_MODEL, hidden=HIDDEN)
    lin = {nm: core.Linear(torch.from_numpy(getattr(bw, nm)), core.make_scales(1, bw.shift[nm], bw.out_dim(nm)))
           for nm in ("q", "k", "v", "o", "up", "gate", "down")}
    blk = core.TransformerBlock(D_MODEL, HEADS, HIDDEN, *[lin[n] for n in ("q", "k", "v", "o", "up", "gate", "down")],
                                torch.from_numpy(bw.attn_gamma), torch.from_numpy(bw.mlp_gamma), 1)
    # the group's sequences (seeded by sequence index), this rank's positions of each
    seqs = [Y.q15_gaussian(Y.tensor_seed(0x5A4D, grp_id * Bg + b), (SEQ, D_MODEL)) for b in range(Bg)]
    a, b_ = shard.positions(SEQ, G, grank)
    x_np = np.ascontiguousarray(np.stack([q[a:b_] for q in seqs]).reshape(-1, D_MODEL))
    x = torch.from_numpy(x_np).cuda()
    y = torch.empty_like(x)
    g = shard.ShardGroup(Bg, SEQ, D_MODEL, HEADS, group=pg, timeout_ms=20000)
    ws = core.workspace(g.workspace_bytes(HIDDEN))
    st = core.Status()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()

    def step(xin, yout):
        r = g.block(blk, xin, yout, ws, st)
        if r != 0:
            raise RuntimeError(f"sharded block failed: {r} {L.nsrl_last_error()}")
        core._check(g.allreduce_status(st))

    for _ in range(args.warmup):
        st.reset()
        flush.zero_()
        step(x, y)
    code, hs = st.fetch()
    if code != 0:
        raise RuntimeError(f"sharded block rejected during warm-up (flags {hs.flags:#x})")
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    dist.barrier()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        flush.zero_()
        starts[i].record(stream)
        st.buf.zero_()
        step(x, y)
        ends[i].record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    clk = clocks.stop()
    ms = torch.tensor([sum(s_.elapsed_time(e_) for s_, e_ in zip(starts, ends))], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    elapsed_ms = float(ms.item())
    code, hs = st.fetch()
    if code != 0:
        raise RuntimeError(f"sharded block rejected in the timed region (flags {hs.flags:#x})")
    L.nsrl_profile_reset()
    L.nsrl_profile_enable(1)
    for _ in range(3):
        flush.zero_()
        st.buf.zero_()
        step(x, y)
    torch.cuda.synchronize()
    L.nsrl_profile_enable(0)
    n_launches, rows = kernel_table(L)
    launches_per_step = n_launches // 3
    # end to end: this rank's rows from pinned host memory, the block, the rows and the status back
    xh = torch.from_numpy(x_np).pin_memory()
    yh = torch.empty_like(xh).pin_memory()
    sh = torch.empty(8, dtype=torch.int64).pin_memory()
    xd, yd = torch.empty_like(x), torch.empty_like(y)
    e2e_steps = max(3, min(args.steps, 20))
    e_s = [torch.cuda.Event(enable_timing=True) for _ in range(e2e_steps)]
    e_e = [torch.cuda.Event(enable_timing=True) for _ in range(e2e_steps)]
    dist.barrier()
    torch.cuda.synchronize()
    for i in range(e2e_steps):
        flush.zero_()
        e_s[i].record(stream)
        xd.copy_(xh, non_blocking=True)
        st.buf.zero_()
        step(xd, yd)
        yh.copy_(yd, non_blocking=True)
        sh.copy_(st.buf, non_blocking=True)
        e_e[i].record(stream)
    torch.cuda.synchronize()
    if int(sh[0]) != 0 or not torch.equal(yh, y.cpu()):
        raise RuntimeError("end-to-end sharded output differs from the device run")
    t = torch.tensor([sum(a_.elapsed_time(b2) for a_, b2 in zip(e_s, e_e))], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item())
    # parity: every rank checks its rows of its group's first sequence against the oracle
    O = oracle_module()
    ol = {nm: O.Linear(getattr(bw, nm), O.scales(1, bw.shift[nm], bw.out_dim(nm)))
          for nm in ("q", "k", "v", "o", "up", "gate", "down")}
    threads = max(1, (os.cpu_count() or 1) // max(1, min(world, 8)))
    y1, _ = O.prenorm_attention_block(seqs[0], 1, SEQ, D_MODEL, HEADS, bw.attn_gamma, 1, ol["q"], ol["k"], ol["v"],
                                      ol["o"], threads=threads)
    ref, _ = O.prenorm_mlp_block(y1, SEQ, D_MODEL, HIDDEN, bw.mlp_gamma, 1, ol["up"], ol["gate"], ol["down"],
                                 threads=threads)
    eq = torch.tensor([int(np.array_equal(y.cpu().numpy()[:b_ - a], ref[a:b_]))], device="cuda")
    if world > 1:
        dist.all_reduce(eq, op=dist.ReduceOp.MIN)
    g.close()
    if rank == 0:
        hbm, tfl, src = peaks()
        tokens = Bg_total * SEQ
        total_ms = sum(r["ms"] for r in rows.values())
        kernels = {k: {"launches": v["launches"] // 3, "ms": round(v["ms"] / 3, 4), "share": round(v["ms"] / total_ms, 4)}
                   for k, v in sorted(rows.items(), key=lambda kv: -kv[1]["ms"])}
        out = {"metric": METRIC, "value": tokens * args.steps / (elapsed_ms / 1000.0), "unit": "tokens/s",
               "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps,
               "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
               "dtype": "int16xint8->int32/int64",
               "data": "synthetic (seeded SplitMix64: Irwin-Hall Q15 sigma 4096, uniform i8 weights)",
               "config": {"workload": f"prenorm causal attention + gated-MLP block forward, d{D_MODEL} "
                                      f"h{HEADS}x{HEAD_DIM} ff{HIDDEN} s{SEQ}, global batch {Bg_total}",
                          "global_batch": Bg_total, "seq_len": SEQ,
                          "parallelism": f"heads/positions x{G}, batch x{ngroups}",
                          "l2": "flushed before every step (256 MiB memset, outside the timed events)"},
               "e2e": {"value": tokens * e2e_steps / (e2e_ms / 1000.0), "unit": "tokens/s",
                       "h2d_bytes_per_step": int(x.numel() * 2) * world,
                       "d2h_bytes_per_step": int(y.numel() * 2 + 64) * world, "steps": e2e_steps},
               "gpu_launches": launches_per_step * args.steps,
               "roofline": roofline(rows, hbm, tfl, src),
               "kernels": kernels, "clocks": clk,
               "parity": {"compared": "each rank's rows of its group's first sequence, last timed step",
                          "equal": bool(int(eq.item()))}}
        print(json.dumps(out), flush=True)
        if not int(eq.item()):
            raise RuntimeError("the sharded block output differs from the oracle")
    dist.barrier()
    dist.destroy_process_group()
    return 0


def run_secondary(args):
    """One secondary measurement alone on cuda:0 (its JSON object on one line)."""
    import torch
    from nsrl_b200 import build, core
    build.build()
    hbm, tfl, _ = peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    if args.case == "decode":
        out = run_decode(core, torch, steps=args.steps, warmup=args.warmup, hbm=hbm, flush=flush,
                         batch=args.decode_batch)
    elif args.case == "generate":
        out = run_generate(core, torch)
    elif args.case == "train":
        out = run_train(core, torch, None, 1, 0, steps=args.steps, warmup=args.warmup, flush=flush, hbm=hbm, tfl=tfl,
                        src=peaks()[2], cpu_baseline=not args.no_cpu_baseline, batch=args.train_windows)
    else:
        out = run_sweep(core, torch, hbm, tfl, flush)
    print(json.dumps(out), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the decode and linear-sweep measurements")
    ap.add_argument("--case", default="block", choices=["block", "decode", "sweep", "train", "generate", "sharded"],
                    help="decode / sweep / train / generate: run only that secondary measurement on one GPU; "
                         "sharded: the block with heads and batch sharded over the ranks")
    ap.add_argument("--shard-heads", type=int, default=0, help="--case sharded: ranks per head group (default "
                                                                 "min(N, heads))")
    ap.add_argument("--shard-batch", type=int, default=BATCH, help="--case sharded: global batch (sequences)")
    ap.add_argument("--decode-batch", type=int, default=DEC_B)
    ap.add_argument("--train-steps", type=int, default=10, help="timed steps of the training-step measurement")
    ap.add_argument("--train-windows", type=int, default=TR_BATCH,
                    help="--case train: windows per step (the measurement uses the global batch of 256)")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.case == "sharded":
        return run_sharded(args)
    if args.case != "block":
        return run_secondary(args)

    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))

    from nsrl_b200 import build, core
    build.build()
    L = core.lib()
    bw, x_np = make_block_inputs(rank)
    lin = {nm: core.Linear(torch.from_numpy(getattr(bw, nm)),
                           core.make_scales(1, bw.shift[nm], bw.out_dim(nm)))
           for nm in ("q", "k", "v", "o", "up", "gate", "down")}
    blk = core.TransformerBlock(D_MODEL, HEADS, HIDDEN, *[lin[n] for n in ("q", "k", "v", "o", "up", "gate", "down")],
                                torch.from_numpy(bw.attn_gamma), torch.from_numpy(bw.mlp_gamma), 1)
    x = torch.from_numpy(x_np).cuda()
    y = torch.empty_like(x)
    ws = core.workspace(blk.workspace_bytes(BATCH, SEQ))
    st = core.Status()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()

    def step():
        r = blk.launch(x, y, BATCH, SEQ, ws, st)
        if r != 0:
            raise RuntimeError(f"block launch failed: {r} {L.nsrl_last_error()}")

    st.reset()
    for _ in range(args.warmup):
        flush.zero_()
        step()
    code, hs = st.fetch()
    if code != 0:
        raise RuntimeError(f"block rejected during warm-up (flags {hs.flags:#x})")

    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        flush.zero_()
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clk = clocks.stop()
    elapsed_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    t = torch.tensor([elapsed_ms], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms = float(t.item())
    code, hs = st.fetch()
    if code != 0:
        raise RuntimeError(f"block rejected in the timed region (flags {hs.flags:#x})")
    y_timed = y.cpu().numpy()
    # the same steps again with per-launch events (the in-library profiler) for the
    # kernel table and the roofline; the timed steps above ran without them
    L.nsrl_profile_reset()
    L.nsrl_profile_enable(1)
    for i in range(args.steps):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    L.nsrl_profile_enable(0)
    n_launches, rows = kernel_table(L)

    # ---- end to end through the public host-buffer call: pinned host in, host out,
    # the batch in chunks of sequences with copies overlapping compute ----
    e2e_steps = max(3, min(args.steps, 20))
    xh = torch.from_numpy(x_np).pin_memory()
    yh = torch.empty_like(xh).pin_memory()
    sh = torch.empty(8, dtype=torch.int64).pin_memory()
    hws = core.workspace(max(blk.host_workspace_bytes(c, SEQ) for c in E2E_CHUNKS))

    def e2e_run(chunk, nsteps):
        e_s = [torch.cuda.Event(enable_timing=True) for _ in range(nsteps)]
        e_e = [torch.cuda.Event(enable_timing=True) for _ in range(nsteps)]
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        for i in range(nsteps):
            flush.zero_()
            e_s[i].record(stream)
            st.buf.zero_()
            r = blk.launch_host(xh, yh, BATCH, SEQ, chunk, hws, st)
            if r != 0:
                raise RuntimeError(f"host block launch failed: {r} {L.nsrl_last_error()}")
            sh.copy_(st.buf, non_blocking=True)
            e_e[i].record(stream)
            torch.cuda.synchronize()
            if int(sh[0]) != 0:
                raise RuntimeError("block rejected in the end-to-end loop")
        if not np.array_equal(yh.numpy(), y.cpu().numpy()):
            raise RuntimeError("host-buffer block output differs from the device call")
        ms = sum(a.elapsed_time(b) for a, b in zip(e_s, e_e))
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        if dist:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dist.barrier()
        return float(t.item())

    # every rank takes the same steps: one untimed call per chunk size (the
    # pipeline's streams and events are created on the first call), a short
    # run of each, then the timed run with the fastest (the max over ranks
    # decides on every rank)
    for c in E2E_CHUNKS:
        e2e_run(c, 1)
    chunk_ms = {c: e2e_run(c, 3) / 3.0 for c in E2E_CHUNKS}
    e2e_chunk = min(E2E_CHUNKS, key=lambda c: chunk_ms[c])
    e2e_ms = e2e_run(e2e_chunk, e2e_steps)

    # config 4 on every rank (its exchange is a collective)
    train_out = None
    if not args.no_extras:
        hbm, tfl, src = peaks()
        train_out = run_train(core, torch, dist, world, rank, steps=args.train_steps, warmup=3, flush=flush, hbm=hbm,
                              tfl=tfl, src=src, cpu_baseline=not args.no_cpu_baseline)
    if rank == 0:
        hbm, tfl, src = peaks()
        value = world * TOKENS * args.steps / (elapsed_ms / 1000.0)
        e2e_value = world * TOKENS * e2e_steps / (e2e_ms / 1000.0)
        total_ms = sum(r["ms"] for r in rows.values())
        kernels = {k: {"launches": v["launches"], "ms": round(v["ms"], 4), "share": round(v["ms"] / total_ms, 4)}
                   for k, v in sorted(rows.items(), key=lambda kv: -kv[1]["ms"])}
        out = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
               "scaling": "weak", "vs_baseline": None, "dtype": "int16xint8->int32/int64",
               "data": "synthetic (seeded SplitMix64: Irwin-Hall Q15 sigma 4096, uniform i8 weights)",
               "config": {"workload": WORKLOAD, "d_model": D_MODEL, "heads": HEADS, "head_dim": HEAD_DIM,
                          "hidden_dim": HIDDEN, "seq_len": SEQ, "batch_per_gpu": BATCH,
                          "global_batch": BATCH * world, "parallelism": f"dp{world} (batch-sharded replicas)",
                          "l2": "flushed before every step (256 MiB memset, outside the timed events)"},
               "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": int(x.numel() * 2),
                       "d2h_bytes_per_step": int(y.numel() * 2 + 64), "steps": e2e_steps,
                       "chunk_sequences": e2e_chunk,
                       "ms_per_step_by_chunk": {str(c): round(v, 4) for c, v in chunk_ms.items()}},
               "gpu_launches": n_launches,
               "roofline": roofline(rows, hbm, tfl, src),
               "kernels": kernels,
               "clocks": clk}
        # parity: the timed output against the oracle on the first sequences of the
        # batch (the same sequences the CPU baseline computes)
        threads = os.cpu_count() or 1
        seqs = max(1, min(BATCH, threads, 16))
        _, dt, ref = cpu_sample(bw, x_np, threads, seqs)
        eq = bool(np.array_equal(y_timed[:seqs * SEQ], ref))
        out["parity"] = {"sequences": seqs, "of": BATCH, "compared": "block output of the last timed step",
                         "equal": eq}
        if not eq:
            print(json.dumps(out), flush=True)
            raise RuntimeError("the timed block output differs from the oracle")
        if not args.no_extras and world == 1:
            out["config1_latency"] = run_config1(core, torch, flush)
            out["block_hd16"] = run_block_hd16(core, torch, bw, x_np, flush, hbm, tfl, src)
            out["decode"] = run_decode(core, torch, steps=8, warmup=2, hbm=hbm, flush=flush)
            out["generate"] = run_generate(core, torch)
            out["linear_sweep"] = run_sweep(core, torch, hbm, tfl, flush)
        if train_out is not None:
            out["train"] = train_out
        if world == 1 and not args.no_cpu_baseline:
            passes, dt = 1, dt
            while dt < 10.0 and passes < 64:  # about 10 s of CPU work
                dt += cpu_sample(bw, x_np, threads, seqs)[1]
                passes += 1
            out["cpu_baseline"] = {"value": passes * seqs * SEQ / dt, "unit": "tokens/s", "cores": threads,
                                   "kind": "port",
                                   "sample": f"{passes} passes of {seqs} sequences x {SEQ} tokens of the same block "
                                             f"({dt:.1f} s, one sequence per thread)"}
        print(json.dumps(out), flush=True)
    if dist:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
