"""Compiles a position-block layout into the device tables the kernels read.

Input: the flattened arrays of a ``PositionBlockList`` after ``concat()``
(``perturb_labels.py:341-357`` of the reference): ``boundary_indices`` (per
block ``(s, e, key_start, key_end)``), ``query_pos_ids``,
``concat_key_pos_ids``, ``concat_attn_masks``, ``concat_abs_pos_masks``.  The
reference shares one list across the batch (``cutedsl/meta.py:20-22``); a
``RowLayouts`` list with one ``PositionBlockList`` per batch row gives every
row its own layout (packed documents of different lengths per row).

Output (``CompiledLayout``), all int32 / fp32 device tensors:

* ``blocks [n, 8]``: row, s, e, key_off, kv_lo, flags, abs_lo, abs_hi (see
  ``AI_BLOCK_*``); ``kv_lo`` is the first key the block attends to, so packed
  documents skip the masked prefix; flags mark blocks with masked keys inside
  ``[kv_lo, e)`` and blocks with abs keys, whose abs keys lie in
  ``[abs_lo, abs_hi)``;
* ``key_info [sum E]``: per concatenated key, the rotary table row (bits
  0..29), attn mask (bit 30), abs mask (bit 31);
* ``q_pos [B, T]``: table row of every query row (rows past the covered
  length use position 0, as ``perturb_labels.py:335`` pads); ``k_own [B, T]``
  the table row of key j in the block whose query rows hold j (a block
  flagged OWNPOS attends every key at that row, e.g. packed documents);
* ``rope_cos / rope_sin [n_pos, D/2]``: fp32 table of the rotary module, and
  ``rope_cs16 [n_pos, D/2, 2]`` the same angles as fp16 (cos, sin) pairs for
  the bf16 tensor-core kernels;
* ``fwd_items [m, 4]``: (block, q0, q1) query tiles: those of blocks with
  abs keys, then those with at most half a tile of rows, then the rest, each
  group longest first;
* ``kv_items [k, 4]``: (row, j0, j1) key tiles of the dK/dV pass: those that
  hold an abs key of some block first, then the rest, longest first.

The tables are built by the native builder ``ai_attn_prep``
(``csrc/ai_prep.cpp``) into one host buffer (pinned for a GPU target) and
copied to the device in one transfer; the rotary table comes from the
caller's rotary module evaluated on the device.  They are built once per
layout object and cached on it (the reference caches its own per-backend
metadata the same way, ``perturb_labels.py:298-331``), so all layers of a
forward share them.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np
import torch

from . import _lib
from .rope import rope_table

__all__ = ["RowLayouts", "CompiledLayout", "compile_layout", "layout_rows", "dtype_code"]

BLOCKF_MASKED, BLOCKF_ABS, BLOCKF_OWNPOS = 1, 2, 4


class RowLayouts(list):
    """One position-block list per batch row."""


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return _lib.DTYPE_BF16
    if dtype == torch.float16:
        return _lib.DTYPE_F16
    if dtype == torch.float32:
        return _lib.DTYPE_F32
    raise TypeError(f"unsupported dtype {dtype}")


def _np(x):
    if hasattr(x, "detach"):
        return x.detach().cpu().numpy()
    return np.asarray(x)


def layout_rows(parsed_positions, batch: int) -> list:
    """Per-row layouts: a ``RowLayouts`` (or a list whose items carry
    ``boundary_indices``) as is, anything else shared by every row."""
    if isinstance(parsed_positions, RowLayouts) or (
            isinstance(parsed_positions, (list, tuple)) and len(parsed_positions) > 0
            and hasattr(parsed_positions[0], "boundary_indices")):
        rows = list(parsed_positions)
        if len(rows) != batch:
            raise ValueError(f"{len(rows)} row layouts for a batch of {batch}")
        return rows
    return [parsed_positions] * batch


@dataclass
class CompiledLayout:
    batch: int
    seq_len: int
    head_dim: int
    dtype: int
    n_pos: int
    p_min: int
    fwd_tile: int
    kv_tile: int
    blocks: torch.Tensor
    row_blocks: torch.Tensor
    row_cov: torch.Tensor
    key_info: torch.Tensor
    q_pos: torch.Tensor
    k_own: torch.Tensor
    rope_cos: torch.Tensor
    rope_sin: torch.Tensor
    rope_cs16: torch.Tensor
    fwd_items: torch.Tensor
    kv_items: torch.Tensor
    n_fwd_abs_items: int         # leading fwd_items whose block has abs keys
    n_kv_abs_items: int          # leading kv_items that a block with abs keys sees
    n_fwd_short_items: int       # fwd_items after the abs ones with at most fwd_tile / 2 rows
    n_fwd_abs_short_items: int   # the first abs items, with at most fwd_tile / 2 rows
    kv_chunks: torch.Tensor      # [c, 4]: kv item, first / end query tile, partial slot (-1: whole item)
    kv_reduce: torch.Tensor      # [r, 4]: kv item, first slot, slots (items split into chunks)
    n_kv_partials: int           # partial slots of the split items
    kv_cost_max: int             # cost of the costliest key tile (query tiles + 2 per block)
    kv_cost_total: int           # cost of all key tiles
    blk_cls: torch.Tensor        # [n_blocks]: first rotation-class entry of the block in chunk_cls, -1: none
    chunk_cls: torch.Tensor      # [n]: rotation class of each 64-key chunk of the blocks that have classes
    rot_classes: torch.Tensor    # [c, 2]: block and first key whose chunk defines the class
    pairs_per_head: int          # finite (query, key) logits of one head summed over the batch
    all_rows_owned: bool = False  # every row of every batch row belongs to a block (no fill launches)
    host_blocks: np.ndarray = field(repr=False, default=None)
    _host_buffer: Optional[torch.Tensor] = field(repr=False, default=None)  # pinned source of the tables' copy

    def c_struct(self) -> "_lib.AiAttnLayout":
        L = _lib.AiAttnLayout()
        L.n_blocks = int(self.blocks.shape[0])
        L.blocks = self.blocks.data_ptr()
        L.row_blocks = self.row_blocks.data_ptr()
        L.row_cov = self.row_cov.data_ptr()
        L.key_info = self.key_info.data_ptr()
        L.n_keys = int(self.key_info.numel())
        L.q_pos = self.q_pos.data_ptr()
        L.k_own = self.k_own.data_ptr()
        L.rope_cos = self.rope_cos.data_ptr()
        L.rope_sin = self.rope_sin.data_ptr()
        L.rope_cs16 = self.rope_cs16.data_ptr()
        L.n_pos = int(self.n_pos)
        L.fwd_tile = int(self.fwd_tile)
        L.fwd_items = self.fwd_items.data_ptr() if self.fwd_items.numel() else None
        L.n_fwd_items = int(self.fwd_items.shape[0])
        L.n_fwd_abs_items = int(self.n_fwd_abs_items)
        L.kv_tile = int(self.kv_tile)
        L.kv_items = self.kv_items.data_ptr() if self.kv_items.numel() else None
        L.n_kv_items = int(self.kv_items.shape[0])
        L.n_kv_abs_items = int(self.n_kv_abs_items)
        L.all_rows_owned = int(self.all_rows_owned)
        L.n_fwd_short_items = int(self.n_fwd_short_items)
        L.kv_chunks = self.kv_chunks.data_ptr() if self.kv_chunks.numel() else None
        L.n_kv_chunks = int(self.kv_chunks.shape[0])
        L.n_kv_partials = int(self.n_kv_partials)
        L.kv_reduce = self.kv_reduce.data_ptr() if self.kv_reduce.numel() else None
        L.n_kv_reduce = int(self.kv_reduce.shape[0])
        L.kv_cost_max = int(self.kv_cost_max)
        L.kv_cost_total = int(self.kv_cost_total)
        L.blk_cls = self.blk_cls.data_ptr() if self.blk_cls.numel() else None
        L.chunk_cls = self.chunk_cls.data_ptr() if self.chunk_cls.numel() else None
        L.n_chunk_cls = int(self.chunk_cls.shape[0])
        L.rot_classes = self.rot_classes.data_ptr() if self.rot_classes.numel() else None
        L.n_rot_classes = int(self.rot_classes.shape[0])
        L.n_fwd_abs_short_items = int(self.n_fwd_abs_short_items)
        return L


def compile_layout(parsed_positions, batch: int, seq_len: int, head_dim: int, dtype: torch.dtype,
                   rotary_emb, device) -> CompiledLayout:
    """Builds (or fetches from the layout's cache) the device tables."""
    device = torch.device(device)
    code = dtype_code(dtype)
    cache_owner = parsed_positions if not isinstance(parsed_positions, tuple) else None
    key = None
    if cache_owner is not None:
        rows_probe = layout_rows(parsed_positions, batch)
        key = (batch, seq_len, head_dim, code, id(rotary_emb), str(device),
               tuple(id(getattr(r, "concat_key_pos_ids", None)) for r in rows_probe[:1]))
        cache = getattr(cache_owner, "_b200_layout_cache", None)
        if cache is not None and key in cache:
            return cache[key]
    compiled = _compile(parsed_positions, batch, seq_len, head_dim, code, rotary_emb, device)
    if cache_owner is not None:
        try:
            cache = getattr(cache_owner, "_b200_layout_cache", None)
            if cache is None:
                cache = {}
                setattr(cache_owner, "_b200_layout_cache", cache)
            cache[key] = compiled
        except AttributeError:
            pass  # plain list: no attribute storage, no caching
    return compiled


def _prep_list(lay, seq_len: int):
    """The AiPrepList of one concat()-ed list, with the numpy arrays it
    points into (kept alive by the caller)."""
    if getattr(lay, "concat_key_pos_ids", None) is None:
        raise ValueError("position-block list has not been concat()-ed")
    bounds = np.ascontiguousarray(np.asarray([tuple(int(v) for v in b) for b in lay.boundary_indices],
                                             dtype=np.int64).reshape(-1, 4))
    if bounds.shape[0] == 0:
        raise ValueError("position-block list has no blocks")
    qpos = np.ascontiguousarray(_np(lay.query_pos_ids).astype(np.int64).reshape(-1))
    kpos = np.ascontiguousarray(_np(lay.concat_key_pos_ids).astype(np.int64).reshape(-1))
    attn = np.ascontiguousarray(_np(lay.concat_attn_masks).astype(np.uint8).reshape(-1))
    ab = np.ascontiguousarray(_np(lay.concat_abs_pos_masks).astype(np.uint8).reshape(-1))
    if attn.shape[0] != kpos.shape[0] or ab.shape[0] != kpos.shape[0]:
        raise ValueError("concatenated key arrays do not match boundary_indices")
    pl = _lib.AiPrepList()
    pl.n_blocks = bounds.shape[0]
    pl.boundary = bounds.ctypes.data
    pl.n_query = qpos.shape[0]
    pl.query_pos = qpos.ctypes.data
    pl.n_keys = kpos.shape[0]
    pl.key_pos = kpos.ctypes.data
    pl.attn_mask = attn.ctypes.data
    pl.abs_mask = ab.ctypes.data
    return pl, (bounds, qpos, kpos, attn, ab)


def _compile(parsed_positions, batch, seq_len, head_dim, code, rotary_emb, device) -> CompiledLayout:
    """The tables of ``AiAttnLayout`` from the native builder (``ai_attn_prep``):
    one host buffer (pinned when the target is a GPU), one copy to the
    device, the rotary table from the caller's module."""
    rows = layout_rows(parsed_positions, batch)
    uniq: List = []
    index_of = {}
    for r in rows:
        if id(r) not in index_of:
            index_of[id(r)] = len(uniq)
            uniq.append(r)
    preps = [_prep_list(r, seq_len) for r in uniq]
    lists = (_lib.AiPrepList * len(preps))(*[p for p, _ in preps])
    list_of_row = np.asarray([index_of[id(r)] for r in rows], dtype=np.int32)
    lib = _lib.lib()
    fwd_tile = lib.ai_attn_fwd_tile_rows(code, head_dim)
    kv_tile = lib.ai_attn_kv_tile_rows(code, head_dim)
    sz = _lib.AiPrepSizes()
    rc = lib.ai_attn_prep_sizes(lists, len(preps), list_of_row.ctypes.data, batch, seq_len, fwd_tile, kv_tile,
                                ctypes.byref(sz))
    if rc != 0:
        raise ValueError(f"position-block layout rejected: {_lib.strerror(rc)}")
    # One int32 buffer holds every table (sections 16-byte aligned).
    parts = [("blocks", sz.n_blocks * 8), ("row_blocks", batch + 1), ("row_cov", batch), ("key_info", sz.n_keys),
             ("q_pos", batch * seq_len), ("k_own", batch * seq_len), ("fwd_items", sz.n_fwd_items * 4),
             ("kv_items", sz.n_kv_items * 4), ("kv_chunks", sz.n_kv_chunks * 4), ("kv_reduce", sz.n_kv_reduce * 4),
             ("blk_cls", sz.n_blocks), ("chunk_cls", sz.n_chunk_cls), ("rot_classes", sz.n_rot_classes * 2)]
    offs, total = {}, 0
    for name, n in parts:
        offs[name] = (total, int(n))
        total += (int(n) + 3) // 4 * 4
    pin = torch.device(device).type == "cuda"
    host = torch.empty(max(total, 4), dtype=torch.int32, pin_memory=pin)
    base = host.data_ptr()
    t = _lib.AiPrepTables()
    for name, _ in parts:
        setattr(t, name, base + 4 * offs[name][0])
    rc = lib.ai_attn_prep(lists, len(preps), list_of_row.ctypes.data, batch, seq_len, fwd_tile, kv_tile,
                          ctypes.byref(t))
    if rc != 0:
        raise ValueError(f"position-block layout rejected: {_lib.strerror(rc)}")
    dev_all = host.to(device, non_blocking=pin)

    def view(name, shape):
        o, n = offs[name]
        return dev_all[o:o + n].view(*shape)

    lo, hi = int(sz.p_min), int(sz.p_max)
    cos, sin = rope_table(rotary_emb, lo, hi, head_dim, device)
    blocks_host = host[offs["blocks"][0]:offs["blocks"][0] + offs["blocks"][1]].view(-1, 8).numpy().copy()
    return CompiledLayout(
        batch=batch, seq_len=seq_len, head_dim=head_dim, dtype=code, n_pos=hi - lo + 1, p_min=lo,
        fwd_tile=fwd_tile, kv_tile=kv_tile,
        blocks=view("blocks", (-1, 8)), row_blocks=view("row_blocks", (-1,)), row_cov=view("row_cov", (-1,)),
        key_info=view("key_info", (-1,)), q_pos=view("q_pos", (batch, seq_len)), k_own=view("k_own", (batch, seq_len)),
        rope_cos=cos, rope_sin=sin, rope_cs16=torch.stack([cos, sin], dim=-1).to(torch.float16).contiguous(),
        fwd_items=view("fwd_items", (-1, 4)), kv_items=view("kv_items", (-1, 4)),
        kv_chunks=view("kv_chunks", (-1, 4)), kv_reduce=view("kv_reduce", (-1, 4)), n_kv_partials=int(t.n_kv_partials),
        blk_cls=view("blk_cls", (-1,)), chunk_cls=view("chunk_cls", (-1,)), rot_classes=view("rot_classes", (-1, 2)),
        kv_cost_max=int(t.kv_cost_max), kv_cost_total=int(t.kv_cost_total),
        n_fwd_abs_items=int(t.n_fwd_abs_items), n_kv_abs_items=int(t.n_kv_abs_items),
        n_fwd_short_items=int(t.n_fwd_short_items), n_fwd_abs_short_items=int(t.n_fwd_abs_short_items),
        pairs_per_head=int(t.pairs_per_head),
        all_rows_owned=bool(t.all_rows_owned), host_blocks=blocks_host, _host_buffer=host,
    )
