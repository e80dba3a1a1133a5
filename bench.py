"""Benchmark of the chain-of-edits (multi-segment RoPE) attention fwd+bwd.

Workload: Qwen3-8B-shaped attention layer, bf16,
B=4, T=4096, Hq=32, Hkv=8, head_dim=128, rope_theta=1e6, two head-dim RoPE
sections (slots [0,32) follow arange, slots [32,64) an edit-cursor stream),
every batch row packs documents with lengths ~ U[256, 2048] (causal inside
each document, one position-block per document).  Synthetic seeded inputs.

A step = forward + backward of the attention over the batch.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Under torchrun (N > 1) every rank runs its own batch (weak scaling, no
collective on the data path); the step time is the max over ranks.
``--impl reference`` times the CPU oracle (numpy restatement of the
reference's eager path) on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

B, T, HQ, HKV, D = 4, 4096, 32, 8, 128
THETA = 1e6
SECTIONS = [(0, 32), (32, 64)]
WORKLOAD = ("cfg1: bf16 B=4 T=4096 Hq=32 Hkv=8 D=128 theta=1e6, docs U[256,2048] packed per row, "
            "2 RoPE sections (32+32 freq slots: arange, cursor stream)")
METRIC = "multi-seg RoPE attn fwd+bwd TFLOP/s (causal-adjusted, 14*D*pairs*Hq)"
DOM_KERNEL_NAMES = {"fwd": "fwd_pers_kernel (forward)", "dq": "dq_pers_kernel (dQ)", "dkdv": "dkdv_ws_kernel (dK/dV)"}
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch on this
# workload, from one ncu capture of the three kernels (profiles/).
TRAFFIC_BYTES = {"fwd": 368016640, "dq": 549332224, "dkdv": 401622016}


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


def make_workload(seed: int, device):
    """Config-1 inputs: the document layout is the same on every rank (seed 0:
    fixed per-GPU work for weak scaling), q/k/v/dO values are seeded by `seed`."""
    import torch

    import autoindexer_b200 as ab

    rows, streams = make_rows(0)
    rope = ab.SectionedRope(D, THETA, [torch.as_tensor(s) for s in streams], SECTIONS, device=device)
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, HQ, T, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, HKV, T, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, HKV, T, D, generator=g).to(torch.bfloat16)
    dout = torch.randn(B, T, HQ, D, generator=g).to(torch.bfloat16)
    return rows, rope, streams, (q, k, v, dout)


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


def job_tflops(job_flops_per_step: float, steps: int, t_max: float) -> float:
    """Whole-job throughput: every rank processes its own seeded batch (weak
    scaling), so the job's FLOPs per step are the sum over ranks; the job
    takes as long as its slowest rank."""
    return job_flops_per_step * steps / t_max / 1e12


def run_ours(args):
    import torch
    import torch.distributed as dist

    from autoindexer_b200 import _lib
    from autoindexer_b200.attention import KernelTimes, attn_bwd, attn_fwd, fused_chain_of_edits_attn_b200, read_status
    from autoindexer_b200.meta import compile_layout

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        os.environ.setdefault("NCCL_DEBUG", "WARN")  # keep stdout to the one JSON line
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    rows, rope, _, host = make_workload(seed=rank, device=dev)
    q, k, v, dout = (x.to(dev) for x in host)
    scale = D ** -0.5
    layout = compile_layout(rows, B, T, D, torch.bfloat16, rope, dev)
    flops = 14.0 * D * HQ * layout.pairs_per_head
    flops_fwd = 4.0 * D * HQ * layout.pairs_per_head
    flops_bwd = 10.0 * D * HQ * layout.pairs_per_head
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        out, lse, ws = attn_fwd(q, k, v, layout, scale, keep_workspace=True)
        return attn_bwd(q, k, v, out, lse, dout, layout, scale, fwd_workspace=ws)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    assert read_status(dev) == 0

    # Device-timed steps: events around each step, L2 flushed (untimed) between steps.
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clocks:
        for i in range(args.steps):
            flush.fill_(float(i))
            e0, e1, e2 = ev[i]
            e0.record(stream)
            out, lse, ws = attn_fwd(q, k, v, layout, scale, keep_workspace=True)
            e1.record(stream)
            grads = attn_bwd(q, k, v, out, lse, dout, layout, scale, fwd_workspace=ws)
            e2.record(stream)
            # Release this step's tensors as the warm-up does, so that every
            # step reuses the same allocator blocks.
            del out, lse, ws, grads
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    t_fwd = sum(a.elapsed_time(b) for a, b, _ in ev) / 1e3
    t_bwd = sum(b.elapsed_time(c) for _, b, c in ev) / 1e3
    t_step = t_fwd + t_bwd
    t_max = max_over_ranks(t_step, world, dev)
    job_flops = sum_over_ranks(flops, world, dev)
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

    # End to end through the public API: pinned host inputs -> device, forward +
    # backward via autograd, results (out, dq, dk, dv) back to pinned host memory.
    pinned = [x.pin_memory() for x in host]
    outs_host = [torch.empty(B, T, HQ, D, dtype=torch.bfloat16).pin_memory(),
                 torch.empty(B, HQ, T, D, dtype=torch.bfloat16).pin_memory(),
                 torch.empty(B, HKV, T, D, dtype=torch.bfloat16).pin_memory(),
                 torch.empty(B, HKV, T, D, dtype=torch.bfloat16).pin_memory()]
    h2d = sum(x.numel() * x.element_size() for x in pinned)
    d2h = sum(x.numel() * x.element_size() for x in outs_host)

    # The steps are pipelined over three streams: step i's inputs are copied in
    # (copy-in stream, two device buffer sets) while step i - 1 computes and
    # step i - 2's results are copied out (copy-out stream), the way a training
    # loop feeding host data would run them; every step copies its own inputs
    # in and its own results out inside the timed span.
    s_in, s_comp, s_out = (torch.cuda.Stream(dev) for _ in range(3))
    dev_in = [[torch.empty(x.shape, dtype=x.dtype, device=dev) for x in pinned] for _ in range(2)]

    def e2e_run(nsteps, ev_start=None, ev_end=None):
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
                o, _ = fused_chain_of_edits_attn_b200(rope, xq, xk, xv, rows)
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

    e2e_run(max(1, args.warmup))
    torch.cuda.synchronize(dev)
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    e2e_run(args.steps, e_start, e_end)
    torch.cuda.synchronize(dev)
    t_e2e = max_over_ranks(e_start.elapsed_time(e_end) / 1e3, world, dev)
    e2e_value = job_tflops(job_flops, args.steps, t_e2e)
    assert read_status(dev) == 0

    peak, peak_sus, peak_kind = peaks()
    # Dominant kernel: algorithmic FLOPs per launch (per query head and finite
    # (query, key) pair: forward 4·D, dQ 6·D — S, dP, dQ — and dK/dV 8·D — S,
    # dP, dV, dK) over its event-timed duration.
    kflops = {"fwd": 4.0 * D * HQ * layout.pairs_per_head, "dq": 6.0 * D * HQ * layout.pairs_per_head,
              "dkdv": 8.0 * D * HQ * layout.pairs_per_head}
    dom = max(kflops, key=lambda kk: kt.ms[kk])
    dom_ms = kt.ms[dom] / max(1, kt.launches[dom])  # per launch
    achieved = kflops[dom] * args.steps / (kt.ms[dom] * 1e-3) / 1e12
    launches_per_step = sum(kt.launches.values()) / args.steps
    tokens = world * B * T * args.steps / t_max

    line = {
        "metric": METRIC,
        "value": round(value, 3),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded randn q/k/v/dO; seeded document lengths and cursor streams)",
        "config": {"workload": WORKLOAD, "global_batch": B * world, "seq_len": T, "parallelism": f"dp{world} (independent rows)",
                   "l2": "flushed between timed steps (256 MB write, untimed)"},
        "fwd_ms": round(t_fwd / args.steps * 1e3, 4),
        "bwd_ms": round(t_bwd / args.steps * 1e3, 4),
        "tokens_per_s": round(tokens, 1),
        "pairs_per_head": layout.pairs_per_head,
        "pct_bf16_peak": round(100 * value / world / peak, 2),
        "pct_bf16_spec_2250": round(100 * value / world / 2250.0, 2),
        "roofline": {"bound": "tensor", "kernel": DOM_KERNEL_NAMES[dom],
                     "achieved": round(achieved, 3), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "peak_kind": f"{peak_kind} burst bf16",
                     "launch_ms": round(dom_ms, 4), "traffic": TRAFFIC_BYTES.get(dom)},
        "kernel_ms_per_step": {kk: round(v / args.steps, 4) for kk, v in kt.ms.items() if v > 0},
        "e2e": {"value": round(e2e_value, 3), "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": int(round(launches_per_step * args.steps)),
        "clocks": clocks.summary(),
    }
    if world == 1 and not args.no_cpu_baseline:  # the CPU baseline is an N=1 figure
        line["cpu_baseline"] = cpu_baseline(rows, host, seed=0)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def cpu_baseline(rows, host, seed=0, reps=1):
    """Oracle (numpy port of the reference's eager path, fp32, all host
    threads) on one (row, kv-group) slice: 4 query heads of batch row 0."""
    import torch

    import autoindexer_b200 as ab
    from oracle import attn_oracle as O

    q, k, v, dout = host
    G = HQ // HKV
    rng = np.random.default_rng(seed)
    streams = [np.arange(T), ab.cursor_stream(T, rng)]
    rope_mod = ab.SectionedRope(D, THETA, [torch.as_tensor(s) for s in streams], SECTIONS)
    rope = O.make_sectioned_rope(rope_mod.inv_freq.numpy(), streams, SECTIONS)
    lay = rows[0]
    qs = q[:1, :G].float().numpy()
    ks = k[:1, :1].float().numpy()
    vs = v[:1, :1].float().numpy()
    dos = dout[:1, :, :G].float().numpy()
    pairs = O.count_pairs(lay, T)
    # All host threads for the BLAS calls, also under torchrun (which sets
    # OMP_NUM_THREADS=1 for its workers).
    from threadpoolctl import threadpool_limits

    with threadpool_limits(limits=os.cpu_count()):
        t0 = time.perf_counter()
        for _ in range(reps):
            O.attn_forward(qs, ks, vs, lay, rope, dtype=np.float32)
            O.attn_backward(qs, ks, vs, dos, lay, rope, dtype=np.float32)
        dt = (time.perf_counter() - t0) / reps
    flops = 14.0 * D * G * pairs
    return {"value": round(flops / dt / 1e12, 6), "unit": "TFLOP/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"batch row 0, kv group 0 ({G} query heads), T={T}: fwd+bwd, numpy fp32, {dt:.2f} s"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    import torch

    rows, _, _, host = make_workload(seed=0, device="cpu")
    for _ in range(args.warmup):
        cpu_baseline(rows, host)
    vals = [cpu_baseline(rows, host) for _ in range(args.steps)]
    value = float(np.median([x["value"] for x in vals]))
    cb = dict(vals[0])
    cb["value"] = round(value, 6)
    line = {
        "metric": METRIC, "value": round(value, 6), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (same generator as the GPU arm)", "impl": "reference",
        "config": {"workload": WORKLOAD, "global_batch": B, "seq_len": T, "parallelism": "cpu"},
        "cpu_baseline": cb,
        "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--prefill", action="store_true", help="time the prefill path instead (one extra JSON line)")
    ap.add_argument("--decode", action="store_true", help="time one decode step instead (one extra JSON line)")
    args = ap.parse_args()
    if args.prefill:
        run_prefill(args)
    elif args.decode:
        run_decode(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
