"""Benchmark of the chain-of-edits (multi-segment RoPE) attention fwd+bwd.

Headline workload (the default): Qwen3-8B-shaped attention
layer, bf16, B=4, T=4096, Hq=32, Hkv=8, head_dim=128, rope_theta=1e6, two
head-dim RoPE sections (slots [0,32) follow arange, slots [32,64) an
edit-cursor stream), every batch row packs documents with lengths
~ U[256, 2048] (causal inside each document, one position block per
document).  Synthetic seeded inputs.  A step = forward + backward of the
attention over the batch.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config 1|E|4|2a|3] [--compare-triton]

Other workloads (``--config``), one JSON line each:

* ``E``: the reference's own workload, a CPT edit chain built by its sampler
  (``tests/golden/chain_e.npz``: T=3072, 71 blocks, abs keys, keys at
  block-dependent positions), B=1, Hq=32, Hkv=8, one RoPE section;
* ``4``: 64 sequences of U[64, 2048] tokens packed into one 65,536-token row,
  two sections;
* ``2a``: the attention layer of config 2 (one causal sequence of 8,192
  tokens, micro-batch 1), two sections;
* ``3``: one causal sequence of 32,768 tokens, three sections (24/24/16
  frequency slots).  Under torchrun its heads are split by KV head over the
  ranks and O, dQ, dK, dV are all-gathered (NCCL), strong scaling.

Under torchrun (N > 1) configs 1, E, 4 and 2a run one batch per rank (weak
scaling, no collective on the data path); the step time is the max over
ranks.  ``--impl reference`` times the reference's own eager attention (fp32,
all host cores) on a bounded sample of the workload.  ``--compare-triton``
times the reference's Triton backend against this library on the same GPU
and inputs (configs 1 and E).
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from dataclasses import dataclass
from typing import Any, List

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

B, T, HQ, HKV, D = 4, 4096, 32, 8, 128
THETA = 1e6
SECTIONS = [(0, 32), (32, 64)]
SECTIONS3 = [(0, 24), (24, 48), (48, 64)]
WORKLOAD = ("cfg1: bf16 B=4 T=4096 Hq=32 Hkv=8 D=128 theta=1e6, docs U[256,2048] packed per row, "
            "2 RoPE sections (32+32 freq slots: arange, cursor stream)")
METRIC = "multi-seg RoPE attn fwd+bwd TFLOP/s (causal-adjusted, 14*D*pairs*Hq)"
DOM_KERNEL_NAMES = {"fwd": "fwd_pers_kernel (forward)", "dq": "dq_pers_kernel (dQ)", "dkdv": "dkdv_ws_kernel (dK/dV)",
                    "simt": "simt fp32 kernels (forward + backward)"}
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of the
# dominant kernel on the config-1 workload, from one `ncu --set full` capture
# of it on the current build (the summary sits with the other profiles).
TRAFFIC_BYTES = {"dkdv": 408681728}
REF_PATH = os.path.join(ROOT, "baseline", "_ref")


def make_rows(seed: int):
    """The seeded document layout of one rank: per batch row, documents of
    U[256, 2048] tokens packed to T; the second RoPE section's cursor stream."""
    import autoindexer_b200 as ab
    from autoindexer_b200.positions import split_documents

    rng = np.random.default_rng(seed)
    streams = [np.arange(T), ab.cursor_stream(T, rng)]
    rows = ab.RowLayouts()
    for _ in range(B):
        lens = split_documents(T, 256, 2048, rng)
        rows.append(ab.document_blocks(lens, position_ids=np.arange(T)))
    return rows, streams


def _inputs(seed, b, hq, hkv, t, dtype=None):
    import torch

    dtype = dtype or torch.bfloat16
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, hq, t, D, generator=g).to(dtype)
    k = torch.randn(b, hkv, t, D, generator=g).to(dtype)
    v = torch.randn(b, hkv, t, D, generator=g).to(dtype)
    dout = torch.randn(b, t, hq, D, generator=g).to(dtype)
    return q, k, v, dout


def make_workload(seed: int, device):
    """Config-1 inputs: the document layout is the same on every rank (seed 0:
    fixed per-GPU work for weak scaling), q/k/v/dO values are seeded by `seed`."""
    import torch

    import autoindexer_b200 as ab

    rows, streams = make_rows(0)
    rope = ab.SectionedRope(D, THETA, [torch.as_tensor(s) for s in streams], SECTIONS, device=device)
    return rows, rope, streams, _inputs(seed, B, HQ, HKV, T)


@dataclass
class Workload:
    cfg: str
    desc: str
    batch: int
    seq_len: int
    rows: Any          # the layout handed to the attention (RowLayouts or a shared list)
    rope: Any          # RotaryEmbeddingFunc (torch module)
    streams: List[np.ndarray]
    sections: List[tuple]
    host: tuple        # q, k, v, dout (CPU tensors of the workload's dtype)
    full_cpu: bool = False  # the CPU baseline runs the whole workload (else one row x KV group slice)

    def row_lists(self):
        """One position-block list per batch row."""
        from autoindexer_b200.meta import layout_rows

        return layout_rows(self.rows, self.batch)


CONFIG_DESC = {
    "0": ("cfg0: fp32 B=2 T=1024 Hq=32 Hkv=8 D=128 theta=1e6, one causal sequence per row, 2 RoPE sections "
          "(32+32 freq slots: arange, cursor stream); the fp32 kernels"),
    "1": WORKLOAD,
    "E": ("cfgE: bf16 B=1 T=3072 Hq=32 Hkv=8 D=128 theta=1e6, CPT edit chain from the reference's sampler "
          "(autoindexer_8B.yaml perturbation: 71 blocks, sum E=145958, 12798 abs keys), 1 RoPE section"),
    "4": ("cfg4: bf16 B=1 T=65536 Hq=32 Hkv=8 D=128 theta=1e6, 64 sequences U[64,2048] rescaled to 65536 tokens, "
          "2 RoPE sections"),
    "2a": ("cfg2 attention layer: bf16 B=1 T=8192 Hq=32 Hkv=8 D=128 theta=1e6, one causal sequence, "
           "2 RoPE sections"),
    "3": ("cfg3: bf16 B=1 T=32768 Hq=32 Hkv=8 D=128 theta=1e6, one causal sequence, 3 RoPE sections "
          "(24/24/16 freq slots: arange, two cursor streams)"),
}


def build_workload(cfg: str, seed: int, device) -> Workload:
    """The seeded workload of a configuration: the layout is fixed per
    configuration; q/k/v/dO are seeded by ``seed``."""
    import torch

    import autoindexer_b200 as ab

    if cfg == "1":
        rows, rope, streams, host = make_workload(seed, device)
        return Workload(cfg, CONFIG_DESC[cfg], B, T, rows, rope, streams, SECTIONS, host)
    if cfg == "E":
        with np.load(os.path.join(ROOT, "tests", "golden", "chain_e.npz")) as z:
            g = {k: z[k] for k in z.files}
        lay = ab.blocks_from_concat(g["boundary_indices"], g["query_pos_ids"], g["concat_key_pos_ids"],
                                    g["concat_attn_masks"], g["concat_abs_pos_masks"])
        t = int(g["T_model"])
        pmax = int(max(g["query_pos_ids"].max(), g["concat_key_pos_ids"].max())) + 1
        streams = [np.arange(pmax)]
        rope = ab.SectionedRope(D, THETA, [torch.as_tensor(streams[0])], [(0, D // 2)], device=device)
        return Workload(cfg, CONFIG_DESC[cfg], 1, t, lay, rope, streams, [(0, D // 2)], _inputs(seed, 1, HQ, HKV, t))
    if cfg == "0":
        t = 1024
        rng = np.random.default_rng(0)
        streams = [np.arange(t), ab.cursor_stream(t, rng)]
        rows = ab.RowLayouts([ab.document_blocks([t], position_ids=np.arange(t)) for _ in range(2)])
        rope = ab.SectionedRope(D, THETA, [torch.as_tensor(s) for s in streams], SECTIONS, device=device)
        return Workload(cfg, CONFIG_DESC[cfg], 2, t, rows, rope, streams, SECTIONS,
                        _inputs(seed, 2, HQ, HKV, t, torch.float32), full_cpu=True)
    if cfg == "4":
        t = 65536
        rng = np.random.default_rng(4)
        raw = rng.integers(64, 2049, 64).astype(np.float64)
        lens = np.maximum(np.round(raw / raw.sum() * t).astype(int), 1)
        lens[-1] += t - lens.sum()
        streams = [np.arange(t), ab.cursor_stream(t, rng)]
        rows = ab.RowLayouts([ab.document_blocks([int(x) for x in lens], position_ids=np.arange(t))])
        sections = SECTIONS
    elif cfg == "2a":
        t = 8192
        rng = np.random.default_rng(2)
        streams = [np.arange(t), ab.cursor_stream(t, rng)]
        rows = ab.RowLayouts([ab.document_blocks([t], position_ids=np.arange(t))])
        sections = SECTIONS
    elif cfg == "3":
        t = 32768
        rng = np.random.default_rng(3)
        streams = [np.arange(t), ab.cursor_stream(t, rng), ab.cursor_stream(t, rng)]
        rows = ab.RowLayouts([ab.document_blocks([t], position_ids=np.arange(t))])
        sections = SECTIONS3
    else:
        raise ValueError(f"unknown config {cfg}")
    rope = ab.SectionedRope(D, THETA, [torch.as_tensor(s) for s in streams], sections, device=device)
    return Workload(cfg, CONFIG_DESC[cfg], 1, t, rows, rope, streams, sections, _inputs(seed, 1, HQ, HKV, t))


class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons while running."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for n, p in zip(names, parts[3:7]):
                if p.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p["bf16_tflops_sustained"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, 1400.0, "fallback"


def max_over_ranks(t: float, world: int, device) -> float:
    """The largest of the ranks' values (every rank calls it; world 1: t)."""
    if world <= 1:
        return t
    import torch
    import torch.distributed as dist

    tt = torch.tensor([t], device=device, dtype=torch.float64)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    return float(tt.item())


def sum_over_ranks(x: float, world: int, device) -> float:
    """Sum of the ranks' values (every rank calls it; world 1: x)."""
    if world <= 1:
        return x
    import torch
    import torch.distributed as dist

    tt = torch.tensor([x], device=device, dtype=torch.float64)
    dist.all_reduce(tt, op=dist.ReduceOp.SUM)
    return float(tt.item())


def workload_config(wl, world: int, sharded: bool) -> dict:
    """The ``config`` of a bench line for workload ``wl`` at ``world`` ranks:
    this library's arm and the reference arm report the same dict (the
    reference arm's bounded CPU sample is described in its ``cpu_baseline``)."""
    return {"workload": wl.desc, "global_batch": wl.batch * (1 if sharded else world), "seq_len": wl.seq_len,
            "parallelism": (f"kv-head shards over {world} ranks + NCCL all-gather" if sharded
                            else f"dp{world} (independent rows)"),
            "l2": "flushed between timed steps (256 MB write, untimed)"}


def job_tflops(job_flops_per_step: float, steps: int, t_max: float) -> float:
    """Whole-job throughput: job FLOPs per step (summed over ranks for weak
    scaling, the one problem's FLOPs for strong scaling) over the slowest
    rank's time."""
    return job_flops_per_step * steps / t_max / 1e12


def _e2e(args, dev, host, apply, out_shapes, world, dtype):
    """End to end through a public function: every step copies its inputs in
    from pinned host memory (copy-in stream, two device buffer sets), runs
    ``apply(q, k, v) -> out`` and its autograd backward (compute stream), and
    copies (out, dq, dk, dv) back to pinned host memory (copy-out stream);
    the three streams overlap consecutive steps the way a training loop
    feeding host data runs them.  Returns (seconds for ``args.steps`` steps,
    max over ranks; bytes in; bytes out) per step."""
    import torch
    import torch.distributed as dist

    pinned = [x.pin_memory() for x in host]
    outs_host = [torch.empty(s, dtype=dtype).pin_memory() for s in out_shapes]
    h2d = sum(x.numel() * x.element_size() for x in pinned)
    d2h = sum(x.numel() * x.element_size() for x in outs_host)
    s_in, s_comp, s_out = (torch.cuda.Stream(dev) for _ in range(3))
    dev_in = [[torch.empty(x.shape, dtype=x.dtype, device=dev) for x in pinned] for _ in range(2)]

    def run(nsteps, ev_start=None, ev_end=None):
        comp_done = []
        if ev_start is not None:
            ev_start.record(s_in)
        for i in range(nsteps):
            buf = dev_in[i % 2]
            if i >= 2:
                s_in.wait_event(comp_done[i - 2])  # buffer set free again
            with torch.cuda.stream(s_in):
                for d_, h_ in zip(buf, pinned):
                    d_.copy_(h_, non_blocking=True)
                in_done = torch.cuda.Event()
                in_done.record(s_in)
            s_comp.wait_event(in_done)
            with torch.cuda.stream(s_comp):
                xq, xk, xv = (b.detach().requires_grad_(True) for b in buf[:3])
                o = apply(xq, xk, xv)
                o.backward(buf[3])
                res = (o.detach(), xq.grad, xk.grad, xv.grad)
                ev = torch.cuda.Event()
                ev.record(s_comp)
                comp_done.append(ev)
            s_out.wait_event(ev)
            with torch.cuda.stream(s_out):
                for dst, src in zip(outs_host, res):
                    src.record_stream(s_out)
                    dst.copy_(src, non_blocking=True)
        if ev_end is not None:
            ev_end.record(s_out)

    run(max(1, args.warmup))
    torch.cuda.synchronize(dev)
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    run(args.steps, e_start, e_end)
    torch.cuda.synchronize(dev)
    t_e2e = max_over_ranks(e_start.elapsed_time(e_end) / 1e3, world, dev)
    return t_e2e, h2d, d2h


def run_ours(args):
    import torch
    import torch.distributed as dist

    from autoindexer_b200.attention import KernelTimes, attn_bwd, attn_fwd, fused_chain_of_edits_attn_b200, read_status
    from autoindexer_b200.meta import compile_layout
    from autoindexer_b200 import sharding

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        os.environ.setdefault("NCCL_DEBUG", "WARN")  # keep stdout to the one JSON line
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    sharded = args.config == "3" and world > 1
    # Weak scaling: every rank its own seeded values on the same layout.
    # Strong scaling (sharded config 3): one problem, the same inputs everywhere.
    wl = build_workload(args.config, seed=0 if sharded else rank, device=dev)
    Bw, Tw = wl.batch, wl.seq_len
    q, k, v, dout = (x.to(dev) for x in wl.host)
    scale = D ** -0.5
    wdtype = wl.host[0].dtype
    layout = compile_layout(wl.rows, Bw, Tw, D, wdtype, wl.rope, dev)
    flops = 14.0 * D * HQ * layout.pairs_per_head
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    G = HQ // HKV
    if sharded:
        k0, k1 = sharding.head_range(HKV, rank, world)
        ql, kl, vl = q[:, k0 * G:k1 * G], k[:, k0:k1], v[:, k0:k1]
        dol = dout[:, :, k0 * G:k1 * G].contiguous()
        bufs = sharding.GatherBuffers(q, k)
    gather_ev = []

    def step(timed=None):
        """One forward + backward; ``timed``: (e0, e1, e2) events recorded
        around the forward and the backward."""
        if timed:
            timed[0].record(stream)
        if not sharded:
            out, lse, ws = attn_fwd(q, k, v, layout, scale, keep_workspace=True)
            if timed:
                timed[1].record(stream)
            grads = attn_bwd(q, k, v, out, lse, dout, layout, scale, fwd_workspace=ws)
            if timed:
                timed[2].record(stream)
            return
        out = sharding.sharded_forward(ql, kl, vl, layout, scale, bufs)
        if timed:
            timed[1].record(stream)
        sharding.sharded_backward(dol, bufs)
        if timed:
            timed[2].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    assert read_status(dev) == 0

    # Device-timed steps: events around each step, L2 flushed (untimed) between steps.
    ev = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(3)) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    if sharded:
        bufs.gather_ms()  # forget the warm-up's gathers
    with ClockSampler(local) as clocks:
        for i in range(args.steps):
            flush.fill_(float(i))
            step(ev[i])
        torch.cuda.synchronize(dev)
    gather_ms = bufs.gather_ms() if sharded else None
    if world > 1:
        dist.barrier()
    t_fwd = sum(a.elapsed_time(b) for a, b, _ in ev) / 1e3
    t_bwd = sum(b.elapsed_time(c) for _, b, c in ev) / 1e3
    t_step = t_fwd + t_bwd
    t_max = max_over_ranks(t_step, world, dev)
    job_flops = flops if sharded else sum_over_ranks(flops, world, dev)
    value = job_tflops(job_flops, args.steps, t_max)
    ms_per_step = t_max / args.steps * 1e3

    # Per-kernel device times: the same steps again with the library's launch
    # events on (ai_attn_profile_*); they give the dominant kernel's duration
    # for the roofline and the count of our launches.
    torch.cuda.synchronize(dev)
    with KernelTimes() as kt:
        for i in range(args.steps):
            flush.fill_(float(i))
            step()
        torch.cuda.synchronize(dev)

    # End to end through the public API.
    if sharded:
        def apply(xq, xk, xv):
            return sharding.kv_sharded_attention(xq, xk, xv, layout, scale)
    else:
        def apply(xq, xk, xv):
            return fused_chain_of_edits_attn_b200(wl.rope, xq, xk, xv, wl.rows)[0]
    out_shapes = [(Bw, Tw, HQ, D), (Bw, HQ, Tw, D), (Bw, HKV, Tw, D), (Bw, HKV, Tw, D)]
    t_e2e, h2d, d2h = _e2e(args, dev, wl.host, apply, out_shapes, world, wdtype)
    e2e_value = job_tflops(job_flops, args.steps, t_e2e)
    assert read_status(dev) == 0

    # Layout compile per new position-block list (a training step builds one):
    # fresh list objects (no cache), native tables, one copy to the device,
    # the rotary table from the module on the device; median of three.
    t_layouts = []
    for _ in range(3):
        fresh = build_workload(args.config, seed=0, device=dev).rows
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        compile_layout(fresh, Bw, Tw, D, wdtype, wl.rope, dev)
        torch.cuda.synchronize(dev)
        t_layouts.append((time.perf_counter() - t0) * 1e3)
    layout_ms = float(np.median(t_layouts))

    peak, peak_sus, peak_kind = peaks()
    # Dominant kernel: algorithmic FLOPs per launch (per query head and finite
    # (query, key) pair: forward 4·D, dQ 6·D — S, dP, dQ — and dK/dV 8·D — S,
    # dP, dV, dK) over its event-timed duration.
    hq_local = (HQ // world) if sharded else HQ
    kflops = {kk: c * D * hq_local * layout.pairs_per_head for kk, c in (("fwd", 4.0), ("dq", 6.0), ("dkdv", 8.0))}
    if wdtype == torch.float32:  # one fp32 (SIMT) kernel family does forward and backward
        kflops = {"simt": 14.0 * D * hq_local * layout.pairs_per_head}
    dom = max(kflops, key=lambda kk: kt.ms[kk])
    dom_ms = kt.ms[dom] / max(1, kt.launches[dom])  # per launch
    achieved = kflops[dom] * args.steps / (kt.ms[dom] * 1e-3) / 1e12
    launches_per_step = sum(kt.launches.values()) / args.steps
    tokens = (1 if sharded else world) * Bw * Tw * args.steps / t_max
    n_ranks_work = 1 if sharded else world
    line = {
        "metric": METRIC,
        "value": round(value, 3),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True,
        "scaling": "strong" if sharded else "weak",
        "vs_baseline": None,
        "dtype": "f32" if wdtype == torch.float32 else "bf16",
        "data": "synthetic (seeded randn q/k/v/dO; seeded layouts and cursor streams)",
        "config": workload_config(wl, world, sharded),
        "fwd_ms": round(max_over_ranks(t_fwd, world, dev) / args.steps * 1e3, 4),
        "bwd_ms": round(max_over_ranks(t_bwd, world, dev) / args.steps * 1e3, 4),
        "tokens_per_s": round(tokens, 1),
        "pairs_per_head": layout.pairs_per_head,
        "pct_bf16_peak": round(100 * value / n_ranks_work / peak, 2) if not sharded else
        round(100 * value / world / peak, 2),
        "pct_bf16_spec_2250": round(100 * value / (world if sharded else n_ranks_work) / 2250.0, 2),
        "roofline": {"bound": "tensor" if dom != "simt" else "fp32 fma", "kernel": DOM_KERNEL_NAMES[dom],
                     "achieved": round(achieved, 3), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "peak_kind": f"{peak_kind} burst bf16",
                     "launch_ms": round(dom_ms, 4),
                     "traffic": TRAFFIC_BYTES.get(dom) if args.config == "1" else None},
        "kernel_ms_per_step": {kk: round(v_ / args.steps, 4) for kk, v_ in kt.ms.items() if v_ > 0},
        "e2e": {"value": round(e2e_value, 3), "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": int(round(launches_per_step * args.steps)),
        "layout_compile_ms": round(layout_ms, 3),
        "clocks": clocks.summary(),
    }
    if gather_ms is not None:
        line["allgather_ms_per_step"] = round(max_over_ranks(gather_ms / args.steps, world, dev), 4)
    if world == 1 and args.config in ("0", "1") and not args.no_cpu_baseline:  # the CPU baseline is an N=1 figure
        line["cpu_baseline"] = cpu_baseline(wl, seed=0, min_seconds=10.0)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def _reference_modules():
    """The reference's own attention code from its offline install under
    ``baseline/_ref`` (``pip install --no-deps --target baseline/_ref``), or
    None when it is not there."""
    if not os.path.isdir(REF_PATH):
        return None
    if REF_PATH not in sys.path:
        sys.path.insert(0, REF_PATH)
    try:
        from autoindexer.models.autoindexer.attention import reference as ref
        from autoindexer.models.autoindexer import perturb_labels as pl
        from autoindexer.models.autoindexer import type_utils as tu
    except Exception:  # noqa: BLE001 - any import failure means "not available"
        return None
    return ref, pl, tu


def cpu_baseline(wl: Workload, seed=0, reps=1, min_seconds=0.0):
    """The reference's eager attention (``chain_of_edits_attn_ref``,
    ``attention/reference.py:116-141``, from ``baseline/_ref``) forward +
    autograd backward in fp32 on all host cores, on one (batch row, KV group)
    slice of the workload: 4 query heads of batch row 0, K/V expanded as the
    reference's interface does.  Without the install, the oracle (numpy
    restatement of the same code) on the same slice.  The slice runs ``reps``
    times, and again until ``min_seconds`` have passed (at most 64 times);
    the figure is the mean per run."""
    import torch

    def timed(run_once):
        t0, n = time.perf_counter(), 0
        while True:
            run_once()
            n += 1
            el = time.perf_counter() - t0
            if n >= reps and (el >= min_seconds or n >= 64):
                return el / n, n

    q, k, v, dout = wl.host
    G = HQ // HKV
    lay = wl.row_lists()[0]
    Tw = wl.seq_len
    pairs = sum(int(np.cumsum(np.asarray(lay.concat_attn_masks[ks:ke], dtype=np.int64))[s:e].sum())
                for s, e, ks, ke in lay.boundary_indices)
    flops = 14.0 * D * G * pairs
    if wl.full_cpu:  # the whole workload: every row (same list here) and every head
        flops *= wl.batch * (HQ // G)
    mods = _reference_modules()
    from threadpoolctl import threadpool_limits

    cores = os.cpu_count()
    if mods is not None:
        ref, pl, tu = mods
        import autoindexer_b200 as ab

        rlay = ab.blocks_from_concat(lay.boundary_indices, lay.query_pos_ids, lay.concat_key_pos_ids,
                                     lay.concat_attn_masks, lay.concat_abs_pos_masks,
                                     block_cls=tu.PositionBlock, list_cls=pl.PositionBlockList)
        rope = ab.SectionedRope(D, THETA, [torch.as_tensor(s) for s in wl.streams], wl.sections)
        prev = torch.get_num_threads()
        torch.set_num_threads(cores)
        def run_once():
            rlay._query_rotary_pos_emb = rlay._keys_rotary_pos_emb = None
            if wl.full_cpu:
                from transformers.models.llama.modeling_llama import repeat_kv

                qs, ks, vs = (x.float().requires_grad_(True) for x in (q, k, v))
                out, _ = ref.chain_of_edits_attn_ref(rope, qs, repeat_kv(ks, G), repeat_kv(vs, G), rlay)
                out.backward(dout.float())
                return
            qs = q[:1, :G].float().requires_grad_(True)
            ks = k[:1, :1].float().requires_grad_(True)
            vs = v[:1, :1].float().requires_grad_(True)
            out, _ = ref.chain_of_edits_attn_ref(rope, qs, ks.expand(1, G, Tw, D), vs.expand(1, G, Tw, D), rlay)
            out.backward(dout[:1, :, :G].float())

        try:
            dt, n_runs = timed(run_once)
        finally:
            torch.set_num_threads(prev)
        kind, what = "reference", "reference eager chain_of_edits_attn_ref + autograd, torch fp32"
    else:
        from oracle import attn_oracle as O

        rope = O.make_sectioned_rope(wl.rope.inv_freq.cpu().numpy(), wl.streams, wl.sections)
        if wl.full_cpu:
            lay = wl.row_lists()
            qs, ks, vs, dos = (x.float().numpy() for x in (q, k, v, dout))
        else:
            qs, ks, vs = (x[:1, :n].float().numpy() for x, n in ((q, G), (k, 1), (v, 1)))
            dos = dout[:1, :, :G].float().numpy()
        def run_once():
            O.attn_forward(qs, ks, vs, lay, rope, dtype=np.float32)
            O.attn_backward(qs, ks, vs, dos, lay, rope, dtype=np.float32)

        with threadpool_limits(limits=cores):
            dt, n_runs = timed(run_once)
        kind, what = "port", "oracle (numpy restatement of the reference's eager path), fp32"
    sample = (f"the whole workload (B={wl.batch}, {HQ} query heads), T={Tw}" if wl.full_cpu
              else f"batch row 0, kv group 0 ({G} query heads), T={Tw}")
    return {"value": round(flops / dt / 1e12, 6), "unit": "TFLOP/s", "cores": cores, "kind": kind,
            "sample": f"{sample}: fwd+bwd, {what}, {dt:.2f} s a run, "
                      f"{n_runs} run{'s' if n_runs != 1 else ''} ({dt * n_runs:.1f} s)"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    wl = build_workload(args.config, seed=0, device="cpu")
    for _ in range(args.warmup):
        cpu_baseline(wl)
    vals = [cpu_baseline(wl) for _ in range(args.steps)]
    value = float(np.median([x["value"] for x in vals]))
    cb = dict(vals[0])
    cb["value"] = round(value, 6)
    line = {
        "metric": METRIC, "value": round(value, 6), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (same generator as the GPU arm)", "impl": "reference",
        "config": workload_config(wl, world, args.config == "3" and world > 1),
        "cpu_baseline": cb,
        "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_compare_triton(args):
    """This library against the reference's Triton backend
    (``fused_chain_of_edits_attn_triton``, ``attention/triton_wrapper.py:57-101``,
    from ``baseline/_ref``) on the same GPU and the same inputs: forward +
    autograd backward through each public function, L2 flushed between
    steps.  The reference's kernel takes one position-block list shared by
    the batch and expanded K/V (its interface calls ``repeat_kv``,
    ``attention/__init__.py:36-37``), so it runs one call per batch row with
    K/V expanded; the expansion is part of its step, as in the reference."""
    import torch

    import autoindexer_b200 as ab
    from autoindexer_b200.attention import fused_chain_of_edits_attn_b200

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    wl = build_workload(args.config, seed=0, device=dev)
    q, k, v, dout = (x.to(dev) for x in wl.host)
    Bw, Tw = wl.batch, wl.seq_len
    G = HQ // HKV
    flush = torch.empty(64 * 1024 * 1024, device=dev)
    line = {"metric": "fwd+bwd ms per step, this library vs the reference's Triton backend (same GPU, inputs)",
            "config": {"workload": wl.desc, "l2": "flushed between timed steps"}, "steps": args.steps,
            "warmup": args.warmup, "dtype": "bf16", "higher_is_better": False}

    def timed(fn):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize(dev)
        tot = 0.0
        for i in range(args.steps):
            flush.fill_(float(i))
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize(dev)
            tot += e0.elapsed_time(e1)
        return tot / args.steps

    def ours():
        xq, xk, xv = (x.detach().requires_grad_(True) for x in (q, k, v))
        o, _ = fused_chain_of_edits_attn_b200(wl.rope, xq, xk, xv, wl.rows)
        o.backward(dout)
        return o.detach(), xq.grad, xk.grad, xv.grad

    from autoindexer_b200.meta import compile_layout

    pairs = compile_layout(wl.rows, Bw, Tw, D, torch.bfloat16, wl.rope, dev).pairs_per_head
    flops = 14.0 * D * HQ * pairs
    with ClockSampler(0) as clocks:
        t_ours = timed(ours)
    line["ours_ms"] = round(t_ours, 4)
    line["ours_tflops"] = round(flops / t_ours / 1e9, 3)
    mods = _reference_modules()
    try:
        if mods is None:
            raise RuntimeError("baseline/_ref (the reference's offline install) is missing")
        ref, pl, tu = mods
        from autoindexer.models.autoindexer.attention.triton_wrapper import _HAS_TRITON, fused_chain_of_edits_attn_triton

        if not _HAS_TRITON:
            raise RuntimeError("the reference's Triton kernels did not import")
        rls = [ab.blocks_from_concat(r.boundary_indices, r.query_pos_ids, r.concat_key_pos_ids, r.concat_attn_masks,
                                     r.concat_abs_pos_masks, block_cls=tu.PositionBlock,
                                     list_cls=pl.PositionBlockList, device=dev) for r in wl.row_lists()]

        def triton_step():
            res = []
            for b in range(Bw):
                xq = q[b:b + 1].detach().requires_grad_(True)
                xk = k[b:b + 1].detach().requires_grad_(True)
                xv = v[b:b + 1].detach().requires_grad_(True)
                ke = xk.repeat_interleave(G, dim=1)
                ve = xv.repeat_interleave(G, dim=1)
                o, _ = fused_chain_of_edits_attn_triton(wl.rope, xq, ke, ve, rls[b])
                o.backward(dout[b:b + 1])
                res.append((o.detach(), xq.grad, xk.grad, xv.grad))
            return [torch.cat(x, dim=0) for x in zip(*res)]

        with ClockSampler(0) as clocks_t:
            t_tri = timed(triton_step)
        a, b_ = ours(), triton_step()
        # Rows past a row's last block (diagonal-only in the reference's eager
        # function, reference.py:42-43: out = v, dV += dO) are left out: the
        # reference's Triton kernel does not write them.
        covs = [int(r.boundary_indices[-1][1]) for r in wl.row_lists()]
        par = {}
        for name, x, y in zip(("out", "dq", "dk", "dv"), a, b_):
            tdim = 1 if name == "out" else 2
            keep = torch.zeros(x.shape[0], x.shape[tdim], dtype=torch.bool, device=x.device)
            for bi, c in enumerate(covs):
                keep[bi, :c] = True
            shape = [x.shape[0]] + [1] * (x.dim() - 1)
            shape[tdim] = x.shape[tdim]
            m = keep.view(shape)
            x, y = (x.float() * m), (y.float() * m)
            par[name] = {"max_abs": round(float((x - y).abs().max()), 5),
                         "rel_l2": round(float((x - y).norm() / y.norm().clamp_min(1e-30)), 6)}
        par["rows_compared"] = "rows below each row's last block end (all rows of config 1; 3062 of 3072 for E)"
        line.update({"triton_ms": round(t_tri, 4), "triton_tflops": round(flops / t_tri / 1e9, 3),
                     "speedup_vs_triton": round(t_tri / t_ours, 2), "parity_ours_vs_triton": par,
                     "clocks_triton": clocks_t.summary()})
    except Exception as e:  # noqa: BLE001 - report why the comparison arm could not run
        line["triton"] = f"unavailable: {type(e).__name__}: {e}"
    line["clocks"] = clocks.summary()
    line["cutedsl"] = ("unavailable: the reference's CuTeDSL backend needs flash-attn-4==4.0.0b29 "
                       "(flash_attn.cute), which is not installed in this image and cannot be installed offline")
    print(json.dumps(line), flush=True)


PREFILL_B = 8
PREFILL_WORKLOAD = ("prefill: bf16 B=8 T=4096 Hq=32 Hkv=8 D=128 theta=1e6, left padding U[0, T/2) per row "
                    "(seed 0), RoPE positions arange(T)")


def run_prefill(args):
    """Prefill attention (``plain_causal_attn_b200``) against the reference's
    own prefill path on the same GPU: RoPE by ``apply_cos_sin``, K/V expanded
    for GQA (``repeat_kv``), ``scaled_dot_product_attention`` under the causal
    & key-padding mask (``prefill_sdpa.py:55-70``, ``attention/__init__.py:
    36-37``).  Forward only (prefill is inference), L2 flushed between steps;
    one JSON line, not the headline metric."""
    import torch
    import torch.nn.functional as F

    import autoindexer_b200 as ab

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    Bp = PREFILL_B
    rng = np.random.default_rng(0)
    pads = rng.integers(0, T // 2, size=Bp)
    keep = np.arange(T)[None, :] >= pads[:, None]
    mask = torch.as_tensor(keep)[:, None, None, :].to(dev)
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(Bp, h, T, D, generator=g).to(torch.bfloat16).to(dev) for h in (HQ, HKV, HKV))
    rope = ab.SectionedRope(D, THETA, [torch.arange(T)], [(0, D // 2)], device=dev)
    # valid (query, key) pairs: row b, query i >= pad_b sees keys [pad_b, i]
    pairs_all = int(sum(((T - p) * (T - p + 1)) // 2 for p in pads))
    flops = 4.0 * D * HQ * pairs_all
    flush = torch.empty(64 * 1024 * 1024, device=dev)

    def ours():
        return ab.plain_causal_attn_b200(rope, q, k, v, attention_mask=mask)[0]

    pos = torch.arange(T, device=dev).unsqueeze(0)
    causal = torch.tril(torch.ones((T, T), dtype=torch.bool, device=dev))

    def reference():
        cos, sin = rope(q, pos)
        cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)

        def rot(x):
            h = x.shape[-1] // 2
            return x * cos + torch.cat((-x[..., h:], x[..., :h]), dim=-1) * sin

        ke = k.repeat_interleave(HQ // HKV, dim=1)
        ve = v.repeat_interleave(HQ // HKV, dim=1)
        o = F.scaled_dot_product_attention(rot(q), rot(ke), ve, attn_mask=causal & mask, is_causal=False)
        return o.transpose(1, 2).contiguous()

    def timed(fn):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize(dev)
        tot = 0.0
        for i in range(args.steps):
            flush.fill_(float(i))
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize(dev)
            tot += e0.elapsed_time(e1) / 1e3
        return tot / args.steps

    t_ours = timed(ours)
    t_ref = timed(reference)
    a, b = ours(), reference()
    valid = torch.as_tensor(keep).to(dev)[:, :, None, None]  # rows that attend a key
    diff = float(((a.float() - b.float()).abs() * valid).max())
    print(json.dumps({
        "metric": "prefill attention fwd TFLOP/s (4*D*valid pairs*Hq)", "value": round(flops / t_ours / 1e12, 3),
        "unit": "TFLOP/s", "ms_per_step": round(t_ours * 1e3, 4), "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "dtype": "bf16", "data": "synthetic (seeded randn q/k/v, seeded pads)",
        "config": {"workload": PREFILL_WORKLOAD, "l2": "flushed between timed steps"},
        "reference_sdpa": {"value": round(flops / t_ref / 1e12, 3), "ms_per_step": round(t_ref * 1e3, 4),
                           "what": "rotate + repeat_kv + torch scaled_dot_product_attention, same GPU"},
        "max_abs_diff_valid_rows": round(diff, 5),
    }), flush=True)


DECODE_WORKLOAD = ("decode: bf16 B=8 Hq=32 Hkv=8 D=128 theta=1e6, one query token against an unrotated "
                   "cache of L=32768 keys, relative key positions, every key attended")


def run_decode(args):
    """One decode step (``decode_attention``) against the reference's eager
    decode branch on the same GPU (``repeat_kv``, the whole cache rotated,
    ``q . k_rot``, mask, scale, fp32 softmax, ``P . V``:
    ``attention/__init__.py:36-51``, ``attn_layers.py:15-27``).  HBM-bound:
    the metric is the cache bytes one step must read (K and V once) over its
    time, against the measured copy bandwidth.  One JSON line, not the
    headline metric."""
    import torch

    import autoindexer_b200 as ab

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    Bd, L = 8, 32768
    g = torch.Generator().manual_seed(0)
    q = torch.randn(Bd, HQ, 1, D, generator=g).to(torch.bfloat16).to(dev)
    k, v = (torch.randn(Bd, HKV, L, D, generator=g).to(torch.bfloat16).to(dev) for _ in range(2))
    rope = ab.SectionedRope(D, THETA, [torch.arange(L)], [(0, D // 2)], device=dev)

    class Pos:  # the IterPositions fields attention reads (type_utils.py:48-67)
        key_pos_ids = torch.arange(L, device=dev) - (L - 1)
        attn_mask = torch.ones(L, dtype=torch.bool, device=dev)

        def get_rotary_pos_emb(self, rotary_emb, x):
            return rotary_emb(x, (self.key_pos_ids + (L - 1)).unsqueeze(0))

    pp = Pos()
    flush = torch.empty(64 * 1024 * 1024, device=dev)

    def ours():
        return ab.decode_attention(q, k, v, pp, rope)

    def reference():
        G = HQ // HKV
        ke, ve = k.repeat_interleave(G, dim=1), v.repeat_interleave(G, dim=1)
        cos, sin = pp.get_rotary_pos_emb(rope, ke)
        cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
        h = D // 2
        kr = ke * cos + torch.cat((-ke[..., h:], ke[..., :h]), dim=-1) * sin
        w = q @ kr.transpose(-1, -2)
        w.masked_fill_(~pp.attn_mask.view(-1, 1, 1, L), float("-inf"))
        w = torch.softmax(w * D ** -0.5, dim=-1, dtype=torch.float32).to(q.dtype)
        return w @ ve

    def timed(fn):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize(dev)
        tot = 0.0
        for i in range(args.steps):
            flush.fill_(float(i))
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize(dev)
            tot += e0.elapsed_time(e1) / 1e3
        return tot / args.steps

    t_ours, t_ref = timed(ours), timed(reference)
    from autoindexer_b200.attention import KernelTimes

    with KernelTimes() as kt:  # the two decode launches alone, CUDA events on their stream
        for i in range(args.steps):
            flush.fill_(float(i))
            ours()
        torch.cuda.synchronize(dev)
    t_kern = kt.ms["decode"] / max(1, kt.launches["decode"]) / 1e3
    diff = float((ours().float() - reference().float()).abs().max())
    nbytes = 2 * Bd * HKV * L * D * 2  # K and V read once
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            hbm = float(json.load(f).get("hbm_gbs"))
    except (OSError, ValueError, TypeError):
        hbm = 6650.0
    gbs = nbytes / t_ours / 1e9
    print(json.dumps({
        "metric": "decode step cache read GB/s (K and V bytes / step time)", "value": round(gbs, 1), "unit": "GB/s",
        "ms_per_step": round(t_ours * 1e3, 4), "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "dtype": "bf16", "data": "synthetic (seeded randn q/k/v)",
        "config": {"workload": DECODE_WORKLOAD, "l2": "flushed between timed steps (cache 1.07 GB > L2)"},
        "kernel_ms": round(t_kern * 1e3, 4),
        "roofline": {"bound": "hbm", "achieved": round(nbytes / t_kern / 1e9, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(nbytes / t_kern / 1e9 / hbm, 4), "traffic": None},
        "reference_eager": {"value": round(nbytes / t_ref / 1e9, 1), "ms_per_step": round(t_ref * 1e3, 4),
                            "what": "repeat_kv + rotate the cache + matmul + fp32 softmax + matmul, same GPU"},
        "max_abs_diff": round(diff, 5),
    }), flush=True)




INDEX_B = 4
INDEX_WORKLOAD = ("index head: bf16 B=4, 2 heads (start / end cursor), D=128, theta=1e6, the +E edit chain "
                  "(46 edits, T=3072), cursor targets drawn among each row's attendable keys")


def run_index(args):
    """Index-head cursor losses (``compute_index_losses_b200``) against the
    reference's ``compute_index_losses`` (``attn_layers.py:40-110``, from
    ``baseline/_ref``) on the same GPU and inputs: losses of every edit
    forward, backward of ``start + 2 * end``, L2 flushed between steps.  The
    per-call host work (the rows of every edit, the rotary table) is inside
    both steps, as it is in training.  One JSON line, not the headline
    metric."""
    import torch

    import autoindexer_b200 as ab
    from autoindexer_b200.index_head import index_rows

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    with np.load(os.path.join(ROOT, "tests", "golden", "ops_cases.npz")) as z:
        ops = z["chain_e"]
    lay = ab.positions_from_operations(ops)
    rng = np.random.default_rng(7)
    cursor = {}
    for blk, (s_, e_, _, _) in zip(lay, lay.boundary_indices):
        if int(blk.block_type) == 1:
            cursor[int(e_) - 1] = (0, 0)
    probe = index_rows(lay, cursor)
    for r in range(0, probe.rows.shape[0], 2):
        picks = []
        for rr in (r, r + 1):
            _, _, n, off = probe.rows[rr]
            cand = np.flatnonzero(probe.ok[off:off + n])
            picks.append(int(rng.choice(cand)) if cand.size else 0)
        cursor[int(probe.edits[r])] = tuple(picks)
    T = int(lay.boundary_indices[-1][1])
    inv = 1.0 / (THETA ** (np.arange(0, D, 2, dtype=np.float64) / D))

    class PlainRope(torch.nn.Module):  # transformers' default rotary: cos/sin of pos * inv_freq, in x.dtype
        def __init__(self):
            super().__init__()
            self.register_buffer("inv_freq", torch.as_tensor(inv, dtype=torch.float32), persistent=False)

        @torch.no_grad()
        def forward(self, x, position_ids):
            f = position_ids.to(self.inv_freq.device).float()[..., None] * self.inv_freq
            emb = torch.cat((f, f), dim=-1)
            return emb.cos().to(x.dtype), emb.sin().to(x.dtype)

    rope = PlainRope().to(dev)
    g = torch.Generator().manual_seed(11)
    q0 = torch.randn(INDEX_B, 2, T, D, generator=g).to(torch.bfloat16).to(dev)
    k0 = torch.randn(INDEX_B, 2, T, D, generator=g).to(torch.bfloat16).to(dev)
    q, k = q0.clone().requires_grad_(True), k0.clone().requires_grad_(True)
    flush = torch.empty(64 * 1024 * 1024, device=dev)
    mods = _reference_modules()
    ref_lay = None
    if mods is not None:
        from autoindexer.models.autoindexer import attn_layers as ref_al

        _, pl, tu = mods
        ref_lay = ab.positions_from_operations(ops, device=dev, block_cls=tu.PositionBlock,
                                               list_cls=pl.PositionBlockList)

    def ours():
        q.grad = k.grad = None
        (sl, el), _ = ab.compute_index_losses_b200(rope, q, k, lay, cursor)
        (sl + 2 * el).backward()
        return sl, el

    def reference():
        q.grad = k.grad = None
        (sl, el), _ = ref_al.compute_index_losses(rope, q, k, ref_lay, cursor)
        (sl + 2 * el).backward()
        return sl, el

    def timed(fn):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize(dev)
        tot = 0.0
        for i in range(args.steps):
            flush.fill_(float(i))
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize(dev)
            tot += e0.elapsed_time(e1) / 1e3
        return tot / args.steps

    t_ours = timed(ours)
    sl, el = ours()
    got = (float(sl), float(el), q.grad.float().clone(), k.grad.float().clone())
    n_rows = probe.rows.shape[0]
    # algorithmic bytes: every (row, key) reads the key's K row once forward and once per backward pass
    key_bytes = int(probe.rows[:, 2].astype(np.int64).sum()) * D * 2 * INDEX_B
    line = {
        "metric": "index-head cursor losses fwd+bwd ms per step", "value": round(t_ours * 1e3, 4), "unit": "ms",
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": False, "dtype": "bf16",
        "data": "synthetic (seeded randn q/k, seeded cursor targets)",
        "config": {"workload": INDEX_WORKLOAD, "edits": n_rows // 2, "l2": "flushed between timed steps"},
        "key_bytes_per_pass": key_bytes,
    }
    if mods is not None:
        t_ref = timed(reference)
        rl, re_ = reference()
        line["reference"] = {"ms_per_step": round(t_ref * 1e3, 4),
                             "what": "reference compute_index_losses + autograd (Python loop over edits), same GPU"}
        line["speedup_vs_reference"] = round(t_ref / t_ours, 2)
        line["diff_vs_reference"] = {
            "start_loss": round(abs(got[0] - float(rl)), 5), "end_loss": round(abs(got[1] - float(re_)), 5),
            "dq_rel_l2": round(float((got[2] - q.grad.float()).norm() / q.grad.float().norm()), 5),
            "dk_rel_l2": round(float((got[3] - k.grad.float()).norm() / k.grad.float().norm()), 5)}
    else:
        line["reference"] = "unavailable: the reference is not installed under baseline/_ref"
    print(json.dumps(line), flush=True)



TRAIN_T = 8192
TRAIN_WORKLOAD = ("cfg2: Qwen3-8B-architecture decoder (36 layers, hidden 4096, Hq=32, Hkv=8, D=128, SwiGLU 12288, "
                  "RMSNorm, vocab 151936), random-init bf16 weights, T=8192, micro-batch 1 per GPU, tokens U[vocab] "
                  "with 5% from 4 marker ids, 2 RoPE sections, gradient checkpointing, AdamW (fused), DDP over ranks")


def run_train(args):
    """Config 2: full training steps of a Qwen3-8B-architecture model whose
    attention is this library (``attn_implementation="autoindexer_b200"``),
    driven the way the reference's model drives its backbone
    (``AutoIndexerModelBase.decode``, ``autoindexer.py:474-509``): the
    backbone's rotary module swapped for an identity rotation
    (``models/utils/model_utils.py:4-20``) so q/k reach the attention
    unrotated, and ``parsed_positions`` / ``rotary_emb`` passed through as
    keyword arguments.  A step = forward (loss) + backward + optimizer step.
    Tokens/s as the reference's ``ThroughputCallback`` counts them
    (``training_monitors.py:74-105``: input tokens summed over ranks over
    the elapsed time); DDP (``configs/accelerate/ddp.yaml``) across ranks,
    gradient all-reduce by NCCL."""
    import torch
    import torch.distributed as dist
    from torch import nn
    from transformers import Qwen3Config, Qwen3ForCausalLM

    import autoindexer_b200 as ab
    from autoindexer_b200.attention import KernelTimes, read_status
    from autoindexer_b200.meta import compile_layout

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        os.environ.setdefault("NCCL_DEBUG", "WARN")
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    class Identity(nn.Module):
        def __init__(self, head_dim):
            super().__init__()
            self.head_dim = head_dim

        def forward(self, x, position_ids):
            shape = (*position_ids.shape, self.head_dim)
            return x.new_ones(shape), x.new_zeros(shape)

    ab.register_autoindexer_b200_attention()
    cfg = Qwen3Config(vocab_size=151936, hidden_size=4096, intermediate_size=12288, num_hidden_layers=36,
                      num_attention_heads=HQ, num_key_value_heads=HKV, head_dim=D, rope_theta=THETA,
                      max_position_embeddings=40960, tie_word_embeddings=False, rms_norm_eps=1e-6,
                      attn_implementation="autoindexer_b200", use_cache=False)
    torch.manual_seed(0)
    prev_dtype = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    with torch.device(dev):
        model = Qwen3ForCausalLM(cfg)
    torch.set_default_dtype(prev_dtype)
    model.model.rotary_emb = Identity(D)
    model.gradient_checkpointing_enable(gradient_checkpointing_kwargs={"use_reentrant": False})
    model.train()
    n_params = sum(p.numel() for p in model.parameters())
    n_embed = model.model.embed_tokens.weight.numel() + model.lm_head.weight.numel()

    class LossStep(nn.Module):
        """The loss of one sequence; the position-block list and the rotary
        function are held here and passed to the backbone inside forward (as
        AutoIndexerModelBase.decode passes the lists it builds), so that DDP's
        input handling never sees them."""

        def __init__(self, m):
            super().__init__()
            self.m = m
            self.layout = None
            object.__setattr__(self, "rope", None)  # not a submodule: its tables are not DDP buffers

        def forward(self, ids):
            return self.m(input_ids=ids, labels=ids, parsed_positions=self.layout, rotary_emb=self.rope).loss

    step_mod = LossStep(model)
    net = step_mod
    if world > 1:
        net = nn.parallel.DistributedDataParallel(step_mod, device_ids=[local], gradient_as_bucket_view=True,
                                                  bucket_cap_mb=256, broadcast_buffers=False)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4, weight_decay=0.0, fused=True)

    rng = np.random.default_rng(100 + rank)
    ids = rng.integers(0, cfg.vocab_size - 4, size=(1, TRAIN_T))
    marks = rng.random(TRAIN_T) < 0.05
    ids[0, marks] = cfg.vocab_size - 4 + rng.integers(0, 4, size=int(marks.sum()))
    ids_host = torch.as_tensor(ids, dtype=torch.long).pin_memory()
    ids_dev = torch.empty_like(ids_host, device=dev)
    srng = np.random.default_rng(2)
    streams = [np.arange(TRAIN_T), ab.cursor_stream(TRAIN_T, srng)]
    rope = ab.SectionedRope(D, THETA, [torch.as_tensor(s) for s in streams], SECTIONS, device=dev)
    layout = ab.RowLayouts([ab.document_blocks([TRAIN_T], position_ids=np.arange(TRAIN_T))])
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()
    stream = torch.cuda.current_stream(dev)
    step_mod.layout = layout
    object.__setattr__(step_mod, "rope", rope)

    def step():
        ids_dev.copy_(ids_host, non_blocking=True)
        loss = net(ids_dev)
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        loss_host.copy_(loss.detach().float(), non_blocking=True)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    assert read_status(dev) == 0
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clocks:
        for i in range(args.steps):
            ev[i][0].record(stream)
            step()
            ev[i][1].record(stream)
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    t_step = max_over_ranks(sum(a.elapsed_time(b) for a, b in ev) / 1e3, world, dev)
    tokens_per_s = world * TRAIN_T * args.steps / t_step
    # The attention launches of one step (36 layers forward, their
    # recomputation under gradient checkpointing, 36 backward), by CUDA events.
    with KernelTimes() as kt:
        step()
        torch.cuda.synchronize(dev)
    pairs = compile_layout(layout, 1, TRAIN_T, D, torch.bfloat16, rope, dev).pairs_per_head
    attn_flops = cfg.num_hidden_layers * 14.0 * D * HQ * pairs  # credited: forward + backward, no recompute
    attn_ms = sum(kt.ms.values())
    dense_flops = 6.0 * (n_params - n_embed) * TRAIN_T + 6.0 * model.lm_head.weight.numel() * TRAIN_T
    peak, _, peak_kind = peaks()
    ms = t_step / args.steps * 1e3
    line = {
        "metric": "train tokens/s (Qwen3-8B architecture, T=8192, micro-batch 1 per GPU)",
        "value": round(tokens_per_s, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 2), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded uniform token ids with 5% marker ids)",
        "config": {"workload": TRAIN_WORKLOAD, "global_batch": world, "seq_len": TRAIN_T,
                   "parallelism": f"ddp{world}", "params": n_params},
        "tokens_per_s_per_gpu": round(tokens_per_s / world, 1),
        "model_tflops_per_gpu": round((dense_flops + attn_flops) / (ms / 1e3) / 1e12, 1),
        "attention": {"ms_per_step": round(attn_ms, 3), "share_of_step": round(attn_ms / ms, 4),
                      "credited_tflops": round(attn_flops / (attn_ms / 1e3) / 1e12, 1),
                      "launches": int(sum(kt.launches.values())),
                      "note": "credited fwd+bwd FLOPs of the 36 layers over the time of all attention launches "
                              "of a step (forward, checkpoint recompute, backward)"},
        "peak": {"bf16_tflops": peak, "kind": peak_kind},
        "e2e": {"value": round(tokens_per_s, 1), "unit": "tokens/s", "h2d_bytes_per_step": TRAIN_T * 8,
                "d2h_bytes_per_step": 4},
        "gpu_launches": int(sum(kt.launches.values())),
        "loss": round(float(loss_host), 4),
        "clocks": clocks.summary(),
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="1", choices=sorted(CONFIG_DESC) + ["2"],
                    help="workload (default: config 1; 2 = full-model training steps)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--compare-triton", action="store_true",
                    help="time the reference's Triton backend against this library (one extra JSON line)")
    ap.add_argument("--prefill", action="store_true", help="time the prefill path instead (one extra JSON line)")
    ap.add_argument("--decode", action="store_true", help="time one decode step instead (one extra JSON line)")
    ap.add_argument("--index", action="store_true",
                    help="time the index-head cursor losses instead (one extra JSON line)")
    args = ap.parse_args()
    if args.index:
        run_index(args)
    elif args.prefill:
        run_prefill(args)
    elif args.decode:
        run_decode(args)
    elif args.compare_triton:
        run_compare_triton(args)
    elif args.config == "2" and args.impl == "ours":
        run_train(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
