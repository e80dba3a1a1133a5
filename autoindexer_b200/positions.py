"""Position-block formats of the chain-of-edits attention.

``PositionBlock`` / ``PositionBlockList`` carry the same fields, with the same
meaning, as the reference's types (``type_utils.py:32-40`` and
``perturb_labels.py:278-357`` of AutodeskAILab/autoindexer's
``src/autoindexer/models/autoindexer``), so that a list built by the reference's
own edit-chain code and a list built here are interchangeable inputs of
``autoindexer_b200``'s attention function:

* block ``b`` owns query rows ``[start, end)`` of the sequence; its keys are the
  prefix ``[0, end)``;
* ``key_pos_ids[j]`` is the rotary position id of key ``j`` *inside this block*
  (the same physical key gets a different position in different blocks);
* ``attn_mask[j]`` false masks key ``j`` out of the block;
* ``abs_pos_mask[j]`` true makes the logit against key ``j`` use the unrotated
  query (``None`` = all false);
* ``query_pos_ids`` are the positions of the block's own query rows.

``concat()`` builds the flattened view every backend reads: concatenated
per-block key arrays and ``boundary_indices = (start, end, key_start, key_end)``.

The builders below generate the synthetic layouts the benchmarks use: packed
documents (one COMPLETE block per document, keys before the document masked)
and cursor-style position streams for head-dim sections.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import IntEnum
from typing import List, Optional, Sequence

import numpy as np
import torch
from torch import Tensor

__all__ = [
    "BlockType",
    "PositionBlock",
    "PositionBlockList",
    "document_blocks",
    "blocks_from_concat",
    "positions_from_operations",
    "cursor_stream",
]


class BlockType(IntEnum):
    EXTEND = 1
    EDIT = 2
    COMPLETE = 3


@dataclass
class PositionBlock:
    key_pos_ids: Tensor
    query_pos_ids: Optional[Tensor] = None
    abs_pos_mask: Optional[Tensor] = None
    attn_mask: Optional[Tensor] = None
    start_idx: Optional[int] = None
    end_idx: Optional[int] = None
    block_type: Optional[BlockType] = None


class PositionBlockList(list):
    """List of ``PositionBlock``; ``concat()`` fills the flattened arrays."""

    def __init__(self, *args):
        super().__init__(*args)
        self.query_pos_ids: Optional[Tensor] = None
        self.concat_key_pos_ids: Optional[Tensor] = None
        self.concat_abs_pos_masks: Optional[Tensor] = None
        self.concat_attn_masks: Optional[Tensor] = None
        self.boundary_indices = []

    def concat(self) -> "PositionBlockList":
        self.query_pos_ids = torch.cat([blk.query_pos_ids for blk in self], dim=0)
        self.concat_key_pos_ids = torch.cat([blk.key_pos_ids for blk in self], dim=0)
        masks = []
        for blk in self:
            am = blk.attn_mask
            if am is None:
                am = torch.ones(len(blk.key_pos_ids), dtype=torch.bool, device=blk.key_pos_ids.device)
            masks.append(am)
        self.concat_attn_masks = torch.cat(masks, dim=0)
        self.concat_abs_pos_masks = torch.zeros_like(self.concat_attn_masks)
        self.boundary_indices = []
        offset = 0
        for blk in self:
            n_keys = len(blk.key_pos_ids)
            first_row = n_keys - len(blk.query_pos_ids)
            self.boundary_indices.append((first_row, n_keys, offset, offset + n_keys))
            if blk.abs_pos_mask is not None:
                self.concat_abs_pos_masks[offset:offset + n_keys] = blk.abs_pos_mask
            offset += n_keys
        return self

    def get_rotary_pos_emb(self, rotary_emb, x: Tensor, seq_len: int):
        """``(cos, sin)`` of the zero-padded query positions and of the
        concatenated key positions, as the reference's eager backend expects
        (``perturb_labels.py:333-339``); memoised per (module, dtype, device,
        seq_len)."""
        key = (id(rotary_emb), x.dtype, str(x.device), seq_len)
        cache = self.__dict__.setdefault("_rotary_cache", {})
        if key not in cache:
            q = self.query_pos_ids
            padded = torch.nn.functional.pad(q, (0, seq_len - len(q))).to(x.device)
            cache[key] = (rotary_emb(x, padded.unsqueeze(0)),
                          rotary_emb(x, self.concat_key_pos_ids.to(x.device).unsqueeze(0)))
        return cache[key]

    @property
    def device(self):
        return self[0].key_pos_ids.device if len(self) else None


def document_blocks(doc_lens: Sequence[int], position_ids: Optional[Sequence[int]] = None,
                    device=None) -> PositionBlockList:
    """One COMPLETE block per packed document: rows ``[s, e)``, keys ``[0, e)``
    with ``attn_mask = (j >= s)`` so attention stays inside the document.

    ``position_ids`` (length ``sum(doc_lens)``) gives the rotary position id of
    every token; by default positions restart at 0 in each document.  With a
    ``SectionedRope`` the position ids are token indices (``arange``) and the
    per-section positions live in the rope's streams."""
    total = int(sum(doc_lens))
    if position_ids is None:
        pos = np.concatenate([np.arange(n, dtype=np.int64) for n in doc_lens]) if total else np.zeros(0, np.int64)
    else:
        pos = np.asarray(position_ids, dtype=np.int64)
        assert pos.shape[0] == total
    pos_t = torch.as_tensor(pos, device=device)
    blocks = PositionBlockList()
    s = 0
    for n in doc_lens:
        e = s + int(n)
        am = torch.zeros(e, dtype=torch.bool, device=device)
        am[s:e] = True
        blocks.append(PositionBlock(
            key_pos_ids=pos_t[:e].clone(),
            query_pos_ids=pos_t[s:e].clone(),
            abs_pos_mask=None,
            attn_mask=am,
            start_idx=s,
            end_idx=e,
            block_type=BlockType.COMPLETE,
        ))
        s = e
    return blocks.concat()


def blocks_from_concat(boundary_indices, query_pos_ids, concat_key_pos_ids, concat_attn_masks,
                       concat_abs_pos_masks, block_cls=None, list_cls=None, device=None):
    """The position-block list whose ``concat()`` gives these flattened arrays
    (the inverse of ``concat()``, ``perturb_labels.py:341-357``): block ``b``
    with ``boundary_indices[b] = (s, e, ks, ke)`` gets query positions
    ``query_pos_ids[s:e]`` and the key arrays ``[ks, ke)``.  ``block_cls`` /
    ``list_cls`` choose the block and list types (default: this module's; the
    reference's own types have the same fields)."""
    block_cls = block_cls or PositionBlock
    list_cls = list_cls or PositionBlockList

    def t(x, dtype):
        return torch.as_tensor(np.asarray(x.detach().cpu() if hasattr(x, "detach") else x), dtype=dtype,
                               device=device)

    qp = t(query_pos_ids, torch.long)
    kp = t(concat_key_pos_ids, torch.long)
    am = t(concat_attn_masks, torch.bool)
    ab = t(concat_abs_pos_masks, torch.bool)
    out = list_cls()
    for s, e, ks, ke in np.asarray(boundary_indices, dtype=np.int64).reshape(-1, 4):
        s, e, ks, ke = int(s), int(e), int(ks), int(ke)
        a = ab[ks:ke]
        out.append(block_cls(key_pos_ids=kp[ks:ke].clone(), query_pos_ids=qp[s:e].clone(),
                             abs_pos_mask=a.clone() if bool(a.any()) else None, attn_mask=am[ks:ke].clone(),
                             start_idx=s, end_idx=e, block_type=None))
    out.concat()
    return out


def positions_from_operations(operations, device=None, block_cls=None, list_cls=None) -> PositionBlockList:
    """The position-block list of an edit chain, built natively
    (``ai_attn_positions_from_ops``): the same list the reference's
    ``perturb_labels_per_sequence`` + ``get_parsed_positions_from_perturbations``
    (``perturb_labels.py:236-275, 395-467``) build from these operations, in
    one pass over host arrays instead of per-operation device ops with a host
    sync each.  ``operations``: the ``Operation`` objects
    ``sample_cursor_operations`` returns, or rows of (num_insert, num_delete,
    start_rel_pos, end_rel_pos, num_extend).  Returns the concat()-ed list."""
    import ctypes

    from . import _lib

    rows = [(o.num_insert, o.num_delete, o.start_rel_pos, o.end_rel_pos, o.num_extend) if hasattr(o, "num_insert")
            else tuple(o) for o in operations]
    ops = np.ascontiguousarray(np.asarray(rows, dtype=np.int64).reshape(-1, 5))
    lib = _lib.lib()
    nb, nq, nk = ctypes.c_int32(0), ctypes.c_int64(0), ctypes.c_int64(0)
    _lib.check(lib.ai_attn_positions_from_ops_sizes(ops.ctypes.data, ops.shape[0], ctypes.byref(nb), ctypes.byref(nq),
                                                    ctypes.byref(nk)), "ai_attn_positions_from_ops")
    bounds = np.empty((nb.value, 4), dtype=np.int64)
    qpos = np.empty(nq.value, dtype=np.int64)
    kpos = np.empty(nk.value, dtype=np.int64)
    attn = np.empty(nk.value, dtype=np.uint8)
    absm = np.empty(nk.value, dtype=np.uint8)
    types = np.empty(nb.value, dtype=np.int32)
    _lib.check(lib.ai_attn_positions_from_ops(ops.ctypes.data, ops.shape[0], bounds.ctypes.data, qpos.ctypes.data,
                                              kpos.ctypes.data, attn.ctypes.data, absm.ctypes.data,
                                              types.ctypes.data), "ai_attn_positions_from_ops")
    lay = blocks_from_concat(bounds, qpos, kpos, attn.astype(bool), absm.astype(bool), block_cls=block_cls,
                             list_cls=list_cls, device=device)
    for blk, t in zip(lay, types):
        blk.block_type = BlockType(int(t))
    return lay


def cursor_stream(n: int, rng: np.random.Generator, p_step: float = 0.8) -> np.ndarray:
    """Edit-chain cursor positions: start at 0; with probability ``p_step`` step
    by +1, otherwise jump back to a uniform position in ``[0, current]``."""
    out = np.zeros(n, dtype=np.int64)
    cur = 0
    u = rng.random(n)
    for t in range(1, n):
        if u[t] < p_step:
            cur += 1
        else:
            cur = int(rng.integers(0, cur + 1))
        out[t] = cur
    return out


def split_documents(total: int, lo: int, hi: int, rng: np.random.Generator) -> List[int]:
    """Document lengths ~ U[lo, hi] packed into ``total`` tokens; the last
    document is truncated to fit."""
    lens = []
    acc = 0
    while acc < total:
        n = int(rng.integers(lo, hi + 1))
        n = min(n, total - acc)
        lens.append(n)
        acc += n
    return lens
