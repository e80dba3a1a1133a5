"""Rotary-embedding plugins and the position-indexed cos/sin table.

The reference hands every backend a ``RotaryEmbeddingFunc``
(``type_utils.py:57``: ``(x, position_ids) -> (cos, sin)``, shapes
``(1, L, D)``) and applies it rotate-half style (``attention/utils.py:5-6``).
Because the function depends on the position id alone, the kernels consume it
as a table: one fp32 row of ``D/2`` cos and ``D/2`` sin values per position id
in ``[p_min, p_max]``, obtained by calling the module itself on
``arange(p_min, p_max + 1)`` with an fp32 probe tensor.  The table is built
once per layout and shared by every layer.

``SectionedRope`` expresses head-dim "RoPE segments" through the same plugin
type: the position id is a token index, and frequency slot ``k`` of section
``s`` rotates by ``streams[s][token]``.  With rotate-half pairing (dims ``k`` and
``k + D/2`` share slot ``k``) a section owns whole slots: slots ``[a, b)`` are
the dims ``[a, b)`` and ``[D/2 + a, D/2 + b)``.  With one section it is the
standard RoPE of the reference.
"""

from __future__ import annotations

from typing import Sequence, Tuple

import torch
from torch import Tensor, nn

__all__ = ["default_inv_freq", "SectionedRope", "rope_table"]


def default_inv_freq(head_dim: int, theta: float, device=None) -> Tensor:
    """``theta ** (-2k / D)`` in fp32, computed as transformers' default RoPE
    initialisation does."""
    exps = torch.arange(0, head_dim, 2, dtype=torch.int64, device=device).float() / head_dim
    return 1.0 / (theta ** exps)


class SectionedRope(nn.Module):
    """``RotaryEmbeddingFunc`` with per-section position streams.

    ``streams``: ``S`` integer tensors indexed by token; ``slot_sections``:
    ``S`` half-open slot ranges ``(a, b)`` covering ``[0, D/2)``."""

    def __init__(self, head_dim: int, theta: float, streams: Sequence[Tensor],
                 slot_sections: Sequence[Tuple[int, int]], device=None):
        super().__init__()
        half = head_dim // 2
        assert len(streams) == len(slot_sections) and len(streams) >= 1
        owner = torch.empty(half, dtype=torch.long)
        covered = torch.zeros(half, dtype=torch.bool)
        for si, (a, b) in enumerate(slot_sections):
            owner[a:b] = si
            covered[a:b] = True
        assert bool(covered.all()), "sections must cover every frequency slot"
        self.head_dim = head_dim
        self.rope_theta = float(theta)
        self.slot_sections = [tuple(s) for s in slot_sections]
        self.register_buffer("inv_freq", default_inv_freq(head_dim, theta, device), persistent=False)
        self.register_buffer("owner", owner.to(device), persistent=False)
        self.register_buffer("streams", torch.stack([torch.as_tensor(s, dtype=torch.long) for s in streams]).to(device),
                             persistent=False)

    @torch.no_grad()
    def forward(self, x: Tensor, position_ids: Tensor) -> Tuple[Tensor, Tensor]:
        idx = position_ids.long().clamp_min(0).to(self.streams.device)
        # (S, *idx.shape) gathered positions, then per-slot choice of section.
        pos = self.streams[:, idx.reshape(-1)].T.float()  # (L, S)
        pos = pos[:, self.owner]  # (L, D/2)
        freqs = (pos * self.inv_freq[None, :].float()).reshape(*idx.shape, -1)
        emb = torch.cat((freqs, freqs), dim=-1)
        return emb.cos().to(x.dtype), emb.sin().to(x.dtype)


def rope_table(rotary_emb, p_min: int, p_max: int, head_dim: int, device) -> Tuple[Tensor, Tensor]:
    """fp32 ``(n_pos, D/2)`` cos and sin tables of ``rotary_emb`` for the
    position ids ``p_min .. p_max``.  Raises if the module's two halves differ
    (the kernels implement rotate-half RoPE only)."""
    ids = torch.arange(p_min, p_max + 1, dtype=torch.long, device=device)
    probe = torch.zeros(1, dtype=torch.float32, device=device)
    with torch.no_grad():
        cos, sin = rotary_emb(probe, ids[None])
    cos = cos.reshape(-1, cos.shape[-1]).float()
    sin = sin.reshape(-1, sin.shape[-1]).float()
    if cos.shape != (ids.numel(), head_dim):
        raise ValueError(f"rotary_emb returned cos of shape {tuple(cos.shape)}, expected ({ids.numel()}, {head_dim})")
    h = head_dim // 2
    if not (torch.equal(cos[:, :h], cos[:, h:]) and torch.equal(sin[:, :h], sin[:, h:])):
        raise NotImplementedError("rotary_emb halves differ: only rotate-half RoPE (cat(freqs, freqs)) is supported")
    return cos[:, :h].contiguous(), sin[:, :h].contiguous()
