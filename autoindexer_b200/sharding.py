"""KV-head sharding of the attention over the GPUs of one node.

For long sequences (the T = 32,768 configuration of the path) one GPU's work
is split by GQA group: every rank holds the same q, k, v, rank r computes
the query heads of KV heads [r·Hkv/n, (r+1)·Hkv/n) — a group's heads see
only their own K/V, so the ranks need nothing from each other while they
compute — and the results are all-gathered along the head dimension over the
process group (NCCL over NVLink for CUDA tensors): O after the forward,
dQ, dK and dV after the backward.  The gathered tensors are the same on
every rank, as replicated inputs require.

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

# local_fwd(q, k, v, layout, scale) -> (out (B, T, h, D), state)
# local_bwd(state, dout (B, T, h, D)) -> (dq, dk, dv)
LocalFwd = Callable[[Tensor, Tensor, Tensor, CompiledLayout, float], Tuple[Tensor, object]]
LocalBwd = Callable[[object, Tensor], Tuple[Tensor, Tensor, Tensor]]


def kernel_fwd(q: Tensor, k: Tensor, v: Tensor, layout: CompiledLayout, scale: float):
    """The library's forward for one rank's heads (``ai_attn_fwd``); keeps
    what the backward needs, the once-rotated Q/K copies included."""
    from .attention import _dense_d, attn_fwd

    q, k, v = _dense_d(q), _dense_d(k), _dense_d(v)
    out, lse, ws = attn_fwd(q, k, v, layout, scale, keep_workspace=True)
    return out, (q, k, v, out, lse, ws, layout, scale)


def kernel_bwd(state, dout: Tensor):
    """The library's backward for one rank's heads (``ai_attn_bwd``)."""
    from .attention import attn_bwd

    q, k, v, out, lse, ws, layout, scale = state
    return attn_bwd(q, k, v, out, lse, dout.contiguous(), layout, scale, fwd_workspace=ws)


def head_range(num_heads: int, rank: int, world: int) -> Tuple[int, int]:
    """Heads [h0, h1) of ``rank`` when ``num_heads`` are split evenly."""
    if num_heads % world:
        raise ValueError(f"{num_heads} heads do not split over {world} ranks")
    n = num_heads // world
    return rank * n, (rank + 1) * n


def gather_heads(x: Tensor, axis: int, group: Optional[dist.ProcessGroup]) -> Tensor:
    """All-gather of each rank's head slice ``x`` along ``axis``, in rank order."""
    world = dist.get_world_size(group) if group is not None or dist.is_initialized() else 1
    if world == 1:
        return x
    x = x.contiguous()
    parts = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(parts, x, group=group)
    return torch.cat(parts, dim=axis)


class KVShardedAttention(torch.autograd.Function):
    """Attention with its heads split over the ranks of ``group`` by KV head;
    q ``(B, Hq, T, D)``, k and v ``(B, Hkv, T, D)`` replicated, out
    ``(B, T, Hq, D)`` and the gradients gathered on every rank."""

    @staticmethod
    def forward(ctx, q, k, v, layout: CompiledLayout, scale: float, group, local_fwd: LocalFwd,
                local_bwd: LocalBwd):
        world = dist.get_world_size(group) if group is not None or dist.is_initialized() else 1
        rank = dist.get_rank(group) if world > 1 else 0
        Hq, Hkv = q.shape[1], k.shape[1]
        if Hq % Hkv:
            raise ValueError(f"num_q_heads {Hq} is not a multiple of num_kv_heads {Hkv}")
        k0, k1 = head_range(Hkv, rank, world)
        G = Hq // Hkv
        q0, q1 = k0 * G, k1 * G
        out_l, state = local_fwd(q[:, q0:q1], k[:, k0:k1], v[:, k0:k1], layout, scale)
        ctx.state, ctx.group, ctx.local_bwd, ctx.q_heads = state, group, local_bwd, (q0, q1)
        return gather_heads(out_l, 2, group)

    @staticmethod
    def backward(ctx, dout):
        q0, q1 = ctx.q_heads
        dq_l, dk_l, dv_l = ctx.local_bwd(ctx.state, dout[:, :, q0:q1])
        ctx.state = None
        g = ctx.group
        return gather_heads(dq_l, 1, g), gather_heads(dk_l, 1, g), gather_heads(dv_l, 1, g), None, None, None, None, None


def kv_sharded_attention(q: Tensor, k: Tensor, v: Tensor, layout: CompiledLayout, scale: float,
                         group: Optional[dist.ProcessGroup] = None, local_fwd: LocalFwd = kernel_fwd,
                         local_bwd: LocalBwd = kernel_bwd) -> Tensor:
    """Differentiable KV-head-sharded attention (see the module docstring);
    with one rank, or no process group, it is the single-GPU attention."""
    return KVShardedAttention.apply(q, k, v, layout, scale, group, local_fwd, local_bwd)
