"""KV-head sharding of the attention over the GPUs of one node.

For long sequences (the T = 32,768 configuration of the path) one GPU's work
is split by GQA group: every rank holds the same q, k, v, rank r computes
the query heads of KV heads [r·Hkv/n, (r+1)·Hkv/n) — a group's heads see
only their own K/V, so the ranks need nothing from each other while they
compute — and the results are all-gathered along the head dimension over the
process group (NCCL over NVLink for CUDA tensors): O after the forward,
dQ, dK and dV after the backward.  The gathered tensors are the same on
every rank, as replicated inputs require.

The gathers need no copy: the full results live in head-major buffers
(``(B, H, T, D)``), every rank's kernels write their heads straight into
their own slice, and ``all_gather_into_tensor`` fills the other slices in
place (with one batch row a rank's heads are one contiguous run; with more
rows the slice is gathered through a staging buffer).  O is returned as the
``(B, T, Hq, D)`` view of its head-major buffer.

The reference has no multi-GPU attention path; its training runs one
replica per GPU (DDP), which the batch-row split of ``bench.py --gpus N``
mirrors.  This module is the head split the long-context configuration
needs.
"""

from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist
from torch import Tensor

from .meta import CompiledLayout

# local_fwd(q, k, v, layout, scale, out_bhtd) -> (out (B, T, h, D), state); out_bhtd, when not None, is
#   the (B, h, T, D) view the result must be written into
# local_bwd(state, dout (B, T, h, D), grads, after_dq=None) -> (dq, dk, dv); grads, when not None, are the
#   views to fill; after_dq, when not None, is called once dQ is complete in stream order (before dK / dV
#   are: a local backward that computes all three at once calls it at the end)
LocalFwd = Callable[..., Tuple[Tensor, object]]
LocalBwd = Callable[..., Tuple[Tensor, Tensor, Tensor]]


def kernel_fwd(q: Tensor, k: Tensor, v: Tensor, layout: CompiledLayout, scale: float,
               out_bhtd: Optional[Tensor] = None):
    """The library's forward for one rank's heads (``ai_attn_fwd``); keeps
    what the backward needs, the once-rotated Q/K copies included."""
    from .attention import _dense_d, attn_fwd

    q, k, v = _dense_d(q), _dense_d(k), _dense_d(v)
    out, lse, ws = attn_fwd(q, k, v, layout, scale, keep_workspace=True, out_bhtd=out_bhtd)
    return out, (q, k, v, out, lse, ws, layout, scale)


def kernel_bwd(state, dout: Tensor, grads=None, after_dq=None):
    """The library's backward for one rank's heads (``ai_attn_bwd``; with
    ``after_dq`` as two calls, dQ then dK / dV)."""
    from .attention import attn_bwd

    q, k, v, out, lse, ws, layout, scale = state
    return attn_bwd(q, k, v, out, lse, dout.contiguous(), layout, scale, fwd_workspace=ws, grads=grads,
                    after_dq=after_dq)


def head_range(num_heads: int, rank: int, world: int) -> Tuple[int, int]:
    """Heads [h0, h1) of ``rank`` when ``num_heads`` are split evenly."""
    if num_heads % world:
        raise ValueError(f"{num_heads} heads do not split over {world} ranks")
    n = num_heads // world
    return rank * n, (rank + 1) * n


def _world(group) -> Tuple[int, int]:
    if group is None and not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def gather_heads_inplace(full: Tensor, group: Optional[dist.ProcessGroup], async_op: bool = False):
    """All-gather along dim 1 of the head-major buffer ``full`` ``(B, H, T,
    D)``, whose own head slice this rank has written: afterwards every slice
    holds its rank's heads.  With ``B == 1`` the slices are contiguous and
    NCCL gathers in place (with ``async_op`` the work handle is returned and
    the caller waits on it); otherwise through a staging buffer, at once."""
    world, rank = _world(group)
    if world == 1:
        return None
    Bf, H = full.shape[0], full.shape[1]
    h0, h1 = head_range(H, rank, world)
    if Bf == 1 and full.is_contiguous():
        flat = full.view(-1)
        n = flat.numel() // world
        return dist.all_gather_into_tensor(flat, flat[rank * n:(rank + 1) * n], group=group, async_op=async_op)
    stage = torch.empty((world,) + tuple(full[:, h0:h1].shape), dtype=full.dtype, device=full.device)
    dist.all_gather_into_tensor(stage, full[:, h0:h1].contiguous(), group=group)
    full.copy_(stage.permute(1, 0, 2, 3, 4).reshape(full.shape))
    return None


def gather_heads(x: Tensor, axis: int, group: Optional[dist.ProcessGroup]) -> Tensor:
    """All-gather of each rank's head slice ``x`` along ``axis``, in rank
    order (a new tensor; for callers that hold only their own slice)."""
    world, _ = _world(group)
    if world == 1:
        return x
    x = x.contiguous()
    stage = torch.empty((world,) + tuple(x.shape), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(stage, x, group=group)
    return torch.movedim(stage, 0, axis).flatten(axis, axis + 1)


class GatherBuffers:
    """The head-major result buffers of one sharded attention shape, kept
    across steps: O ``(B, Hq, T, D)``, dQ like q, dK and dV like k.  Event
    pairs around every gather give the time spent in them
    (``gather_ms``)."""

    def __init__(self, q: Tensor, k: Tensor, group: Optional[dist.ProcessGroup] = None, timing: bool = True):
        self.group = group
        self.world, self.rank = _world(group)
        Hq, Hkv = q.shape[1], k.shape[1]
        self.kv_heads = head_range(Hkv, self.rank, self.world)
        G = Hq // Hkv
        self.q_heads = (self.kv_heads[0] * G, self.kv_heads[1] * G)
        self.out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
        self.dq = torch.empty(q.shape, dtype=q.dtype, device=q.device)
        self.dk = torch.empty(k.shape, dtype=k.dtype, device=k.device)
        self.dv = torch.empty(k.shape, dtype=k.dtype, device=k.device)
        self.timing = timing
        self.events = []
        self.state = None

    def gather(self, *fulls: Tensor) -> None:
        if self.world == 1:
            return
        stream = torch.cuda.current_stream(fulls[0].device) if fulls[0].is_cuda else None
        if self.timing and stream is not None:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        for f in fulls:
            gather_heads_inplace(f, self.group)
        if self.timing and stream is not None:
            e1.record(stream)
            self.events.append((e0, e1))

    def gather_async(self, full: Tensor):
        """Starts the gather of ``full`` (returns what ``finish`` takes): in
        place on NCCL's stream when the layout allows it, at once otherwise."""
        work = gather_heads_inplace(full, self.group, async_op=True)
        if work is None:
            return None
        return work

    def finish(self, work) -> None:
        """Makes the current stream wait for a gather started by
        ``gather_async``; the time it waits counts as gather time."""
        if work is None:
            return
        stream = torch.cuda.current_stream() if torch.cuda.is_available() and self.out.is_cuda else None
        if self.timing and stream is not None:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            work.wait()
            e1.record(stream)
            self.events.append((e0, e1))
        else:
            work.wait()

    def gather_ms(self) -> float:
        """Milliseconds spent in the gathers recorded so far (synchronises),
        then forgets them."""
        ms = sum(a.elapsed_time(b) for a, b in self.events)
        self.events = []
        return ms


def sharded_forward(q_l: Tensor, k_l: Tensor, v_l: Tensor, layout: CompiledLayout, scale: float,
                    bufs: GatherBuffers, local_fwd: LocalFwd = kernel_fwd) -> Tensor:
    """This rank's heads (``q_l``, ``k_l``, ``v_l``) written into its slice of
    ``bufs.out``, then gathered: returns the full ``(B, T, Hq, D)`` output on
    every rank."""
    q0, q1 = bufs.q_heads
    _, bufs.state = local_fwd(q_l, k_l, v_l, layout, scale, bufs.out[:, q0:q1])
    bufs.gather(bufs.out)
    return bufs.out.permute(0, 2, 1, 3)


def sharded_backward(dout_l: Tensor, bufs: GatherBuffers, local_bwd: LocalBwd = kernel_bwd, overlap: bool = False):
    """This rank's dQ, dK, dV written into its slices of the buffers, then
    gathered: returns the full ``(dq, dk, dv)`` on every rank.  With
    ``overlap`` the backward runs in two parts and the dQ gather is issued
    as soon as dQ is complete (``after_dq``), on NCCL's stream while the
    dK / dV kernels run; the caller's stream waits for it before returning.
    (Off by default: on two B200s the NCCL kernels then share the SMs with
    dK / dV and the dK / dV launch no longer starts under the tail of the dQ
    kernel, which cost more than the 0.4 ms of dQ gather it hid.)"""
    q0, q1 = bufs.q_heads
    k0, k1 = bufs.kv_heads
    grads = (bufs.dq[:, q0:q1], bufs.dk[:, k0:k1], bufs.dv[:, k0:k1])
    if not overlap:
        local_bwd(bufs.state, dout_l, grads)
        bufs.state = None
        bufs.gather(bufs.dq, bufs.dk, bufs.dv)
        return bufs.dq, bufs.dk, bufs.dv
    pending = []

    def after_dq():
        if bufs.world > 1:
            pending.append(bufs.gather_async(bufs.dq))

    local_bwd(bufs.state, dout_l, grads, after_dq=after_dq)
    bufs.state = None
    bufs.gather(bufs.dk, bufs.dv)
    for w in pending:
        bufs.finish(w)
    return bufs.dq, bufs.dk, bufs.dv


class KVShardedAttention(torch.autograd.Function):
    """Attention with its heads split over the ranks of ``group`` by KV head;
    q ``(B, Hq, T, D)``, k and v ``(B, Hkv, T, D)`` replicated, out
    ``(B, T, Hq, D)`` and the gradients gathered on every rank."""

    @staticmethod
    def forward(ctx, q, k, v, layout: CompiledLayout, scale: float, group, local_fwd: LocalFwd,
                local_bwd: LocalBwd, overlap: bool = False):
        Hq, Hkv = q.shape[1], k.shape[1]
        if Hq % Hkv:
            raise ValueError(f"num_q_heads {Hq} is not a multiple of num_kv_heads {Hkv}")
        bufs = GatherBuffers(q, k, group, timing=False)
        k0, k1 = bufs.kv_heads
        q0, q1 = bufs.q_heads
        out = sharded_forward(q[:, q0:q1], k[:, k0:k1], v[:, k0:k1], layout, scale, bufs, local_fwd)
        ctx.bufs, ctx.local_bwd, ctx.overlap = bufs, local_bwd, overlap
        return out

    @staticmethod
    def backward(ctx, dout):
        bufs = ctx.bufs
        q0, q1 = bufs.q_heads
        dq, dk, dv = sharded_backward(dout[:, :, q0:q1], bufs, ctx.local_bwd, ctx.overlap)
        ctx.bufs = None
        return dq, dk, dv, None, None, None, None, None, None


def kv_sharded_attention(q: Tensor, k: Tensor, v: Tensor, layout: CompiledLayout, scale: float,
                         group: Optional[dist.ProcessGroup] = None, local_fwd: LocalFwd = kernel_fwd,
                         local_bwd: LocalBwd = kernel_bwd, overlap: bool = False) -> Tensor:
    """Differentiable KV-head-sharded attention (see the module docstring);
    with one rank, or no process group, it is the single-GPU attention.
    ``overlap``: start the dQ all-gather while dK / dV are computed (see
    ``sharded_backward``)."""
    return KVShardedAttention.apply(q, k, v, layout, scale, group, local_fwd, local_bwd, overlap)
