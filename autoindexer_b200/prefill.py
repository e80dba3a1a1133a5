"""Prefill attention on the B200 kernels: ``plain_causal_attn_b200``.

The counterpart of the reference's ``plain_causal_attn_sdpa``
(``src/autoindexer/models/autoindexer/attention/prefill_sdpa.py:11-71``),
registered there as ``"autoindexer_prefill_sdpa"``
(``attention/__init__.py:81``) and selected by ``_prefill_prompt``
(``autoindexer.py:584``): a from-scratch forward of left-padded prompts,
rotary positions ``arange(T)`` shared by every row, causal attention, and an
optional per-row key-validity mask ``(B, 1, 1, T)`` (nonzero = real token).

Here that is one COMPLETE position block per row — query rows ``[0, T)``,
keys ``[0, T)`` at their own positions, key ``j`` attended iff the row's mask
holds it — run by the same kernels as the chain-of-edits path: a
left-padding mask becomes the block's first attended key (``kv_lo``), any
other mask the per-key flags.  Query rows with no attended key at or before
them (the padding rows of a left-padded prompt) return zeros; the reference
leaves them to SDPA, whose math backend returns NaN there, and its callers
ignore them.
"""

from __future__ import annotations

from collections import OrderedDict
from typing import Optional, Tuple

import torch
from torch import Tensor

from .attention import AttentionFn
from .meta import RowLayouts, compile_layout
from .positions import BlockType, PositionBlock, PositionBlockList

# Position-block lists by (T, row mask bytes) and row layouts by the whole
# mask: a repeated prompt shape reuses the same objects, so compile_layout's
# per-object cache finds its device tables.
_ROWS: "OrderedDict[tuple, PositionBlockList]" = OrderedDict()
_LAYOUTS: "OrderedDict[tuple, RowLayouts]" = OrderedDict()  # by (B, T, mask bytes)
_MAX_ROWS = 64


def _row_blocks(seq_len: int, keep: Optional[Tensor]) -> PositionBlockList:
    """One block over the whole row; ``keep`` (bool, ``(T,)``) marks the
    attended keys (all when ``None``)."""
    key = (seq_len, None if keep is None else keep.numpy().tobytes())
    hit = _ROWS.get(key)
    if hit is not None:
        _ROWS.move_to_end(key)
        return hit
    pos = torch.arange(seq_len)
    am = torch.ones(seq_len, dtype=torch.bool) if keep is None else keep.clone()
    blocks = PositionBlockList([PositionBlock(key_pos_ids=pos, query_pos_ids=pos.clone(), attn_mask=am,
                                              start_idx=0, end_idx=seq_len,
                                              block_type=BlockType.COMPLETE)]).concat()
    _ROWS[key] = blocks
    if len(_ROWS) > _MAX_ROWS:
        _ROWS.popitem(last=False)
    return blocks


def prefill_layout(attention_mask: Optional[Tensor], batch: int, seq_len: int):
    """The position-block layout of a prefill forward: one shared block list
    without a mask, else one per row (rows with equal masks share theirs)."""
    if attention_mask is None:
        return _row_blocks(seq_len, None)
    m = attention_mask
    if m.dim() != 4 or m.shape[0] != batch or m.shape[1] != 1 or m.shape[2] != 1 or m.shape[3] != seq_len:
        raise ValueError(f"attention_mask must be (batch, 1, 1, kv_len) = ({batch}, 1, 1, {seq_len}), "
                         f"got {tuple(m.shape)}")
    keep = m.reshape(batch, seq_len).to(torch.bool).cpu()
    key = (batch, seq_len, keep.numpy().tobytes())
    rows = _LAYOUTS.get(key)
    if rows is None:
        rows = RowLayouts()
        for b in range(batch):
            rows.append(_row_blocks(seq_len, keep[b]))
        _LAYOUTS[key] = rows
        if len(_LAYOUTS) > _MAX_ROWS:
            _LAYOUTS.popitem(last=False)
    else:
        _LAYOUTS.move_to_end(key)
    return rows


def plain_causal_attn_b200(
    rotary_emb,
    query: Tensor,
    keys: Tensor,
    values: Tensor,
    attention_mask: Optional[Tensor] = None,
    dropout_p: float = 0.0,
    scaling: Optional[float] = None,
    **kwargs,
) -> Tuple[Tensor, None]:
    """Plain causal prefill attention (same contract as the reference's
    ``plain_causal_attn_sdpa``): ``query`` ``(B, Hq, T, D)``, ``keys`` and
    ``values`` ``(B, Hkv, T, D)`` unrotated; returns ``(out (B, T, Hq, D),
    None)``.  Differentiable (the chain-of-edits backward)."""
    B, Hq, q_len, D = query.shape
    kv_len = keys.shape[2]
    assert q_len == kv_len, "plain_causal_attn_b200 assumes a from-scratch forward (no KV cache yet)"
    if keys.shape[1] == 0 or Hq % keys.shape[1] != 0:
        raise ValueError(f"num_q_heads {Hq} is not a multiple of num_kv_heads {keys.shape[1]}")
    if dropout_p:
        raise NotImplementedError("autoindexer_b200 attention has no dropout")
    if not query.is_cuda:
        raise RuntimeError("autoindexer_b200 attention runs on CUDA tensors only")
    scale = float(scaling) if scaling is not None else D ** -0.5
    layout = compile_layout(prefill_layout(attention_mask, B, q_len), B, q_len, D, query.dtype, rotary_emb,
                            query.device)
    return AttentionFn.apply(query, keys, values, layout, scale), None


def prefill_attention_interface(module, query: Tensor, key: Tensor, value: Tensor,
                                attention_mask: Optional[Tensor], dropout: float = 0.0,
                                scaling: Optional[float] = None, rotary_emb=None, **kwargs):
    """transformers attention function (``ALL_ATTENTION_FUNCTIONS`` signature)
    for the prefill forward: the reference registers its SDPA prefill under
    ``"autoindexer_prefill_sdpa"`` behind a wrapper that expands K/V for GQA
    (``attention/__init__.py:36-37,78-84``); the kernels read GQA K/V as they
    are, so none is expanded here."""
    return plain_causal_attn_b200(rotary_emb, query, key, value, attention_mask=attention_mask,
                                  dropout_p=dropout, scaling=scaling)
