"""Numpy restatement of the layout tables ``ai_attn_prep`` builds.

TEST INFRASTRUCTURE ONLY: the checker the native builder
(``autoindexer_b200/csrc/ai_prep.cpp``, called by
``autoindexer_b200.meta.compile_layout``) is compared against in
``tests/test_layout.py``.  It derives the same tables from a concat()-ed
position-block list (``perturb_labels.py:341-357``) with numpy array
operations: key words, own-block rows, block records, query rows, work
lists and counts.
"""

from dataclasses import dataclass
from typing import List

import numpy as np

_KEY_ATTN = np.uint32(1 << 30)
_KEY_ABS = np.uint32(1 << 31)
_ROW_MASK = (1 << 30) - 1
BLOCKF_MASKED, BLOCKF_ABS, BLOCKF_OWNPOS = 1, 2, 4


def _np(x):
    if hasattr(x, "detach"):
        return x.detach().cpu().numpy()
    return np.asarray(x)


def layout_rows(parsed_positions, batch):
    if isinstance(parsed_positions, (list, tuple)) and len(parsed_positions) > 0 and hasattr(
            parsed_positions[0], "boundary_indices"):
        return list(parsed_positions)
    return [parsed_positions] * batch


@dataclass
class _HostLayout:
    bounds: np.ndarray   # [n, 4] int64
    qpos: np.ndarray     # [T_cov]
    kpos: np.ndarray     # [sum E]
    attn: np.ndarray     # [sum E] bool
    abs_: np.ndarray     # [sum E] bool


def _host_layout(lay, seq_len: int) -> _HostLayout:
    if getattr(lay, "concat_key_pos_ids", None) is None:
        raise ValueError("position-block list has not been concat()-ed")
    bounds = np.asarray([tuple(int(v) for v in b) for b in lay.boundary_indices], dtype=np.int64).reshape(-1, 4)
    qpos = _np(lay.query_pos_ids).astype(np.int64).reshape(-1)
    kpos = _np(lay.concat_key_pos_ids).astype(np.int64).reshape(-1)
    attn = _np(lay.concat_attn_masks).astype(bool).reshape(-1)
    ab = _np(lay.concat_abs_pos_masks).astype(bool).reshape(-1)
    if bounds.shape[0] == 0:
        raise ValueError("position-block list has no blocks")
    expect_s = 0
    for s, e, ks, ke in bounds:
        if s != expect_s or e <= s or ke - ks != e or e > seq_len:
            raise ValueError(f"blocks must partition [0, T_cov) in order with key range [0, e): got {(s, e, ks, ke)}")
        expect_s = e
    if qpos.shape[0] != expect_s:
        raise ValueError(f"query_pos_ids has {qpos.shape[0]} entries, blocks cover {expect_s} rows")
    if kpos.shape[0] != bounds[-1, 3] or attn.shape[0] != kpos.shape[0] or ab.shape[0] != kpos.shape[0]:
        raise ValueError("concatenated key arrays do not match boundary_indices")
    return _HostLayout(bounds, qpos, kpos, attn, ab)


def _pairs(h: _HostLayout) -> int:
    n = 0
    for s, e, ks, ke in h.bounds:
        c = np.cumsum(h.attn[ks:ke].astype(np.int64))
        n += int(c[s:e].sum())
    return n


def _tiles(fwd_tile: int, kv_tile: int, blocks: np.ndarray, row_cov: np.ndarray):
    fwd = []
    for bi, (row, s, e, koff, kv_lo, flags, _, _) in enumerate(blocks):
        for q0 in range(s, e, fwd_tile):
            q1 = min(q0 + fwd_tile, e)
            cost = (q1 - q0) * max(0, min(e, q1) - kv_lo)
            fwd.append((cost, bi, q0, q1))
    # Items of blocks with abs keys first (short ones, then the others), then
    # the other short items (at most half a tile of rows: the tensor-core
    # kernels pack several heads of such an item into one tile), then the
    # rest; longest first within each group.
    def group(t):
        short = t[3] - t[2] <= fwd_tile // 2
        if int(blocks[t[1], 5]) & BLOCKF_ABS:
            return 0 if short else 1
        return 2 if short else 3
    fwd.sort(key=lambda t: (group(t), -t[0]))
    n_abs = sum(1 for t in fwd if group(t) <= 1)
    n_abs_short = sum(1 for t in fwd if group(t) == 0)
    n_short = sum(1 for t in fwd if group(t) == 2)
    # Key tiles: cost = query rows that see them; tiles that hold an abs key
    # of some block first (the abs pass adds those blocks' part), then
    # longest first.
    kv = []
    for row, cov in enumerate(row_cov):
        rb = blocks[blocks[:, 0] == row]
        for j0 in range(0, int(cov), kv_tile):
            j1 = min(j0 + kv_tile, int(cov))
            seen = (rb[:, 2] > j0) & (rb[:, 4] < j1)
            cost = int(np.maximum(rb[seen, 2] - np.maximum(rb[seen, 1], j0), 0).sum())
            # an abs key of a block among these keys (its range [abs_lo, abs_hi) meets [j0, j1))
            has_abs = bool(((rb[seen, 5] & BLOCKF_ABS) != 0)[(rb[seen, 6] < j1) & (rb[seen, 7] > j0)].any())
            kv.append((has_abs, cost, row, j0, j1))
    kv.sort(key=lambda t: (-int(t[0]), -t[1]))
    n_kv_abs = sum(1 for t in kv if t[0])
    fwd_arr = np.asarray([(bi, q0, q1, 0) for _, bi, q0, q1 in fwd], dtype=np.int32).reshape(-1, 4)
    kv_arr = np.asarray([(row, j0, j1, 0) for _, _, row, j0, j1 in kv], dtype=np.int32).reshape(-1, 4)
    return fwd_arr, kv_arr, n_abs, n_kv_abs, n_short, n_abs_short


def host_tables(parsed_positions, batch, seq_len, fwd_tile, kv_tile):
    """The layout tables as numpy arrays (see the module docstring)."""
    rows = layout_rows(parsed_positions, batch)
    uniq: List = []
    index_of = {}
    for r in rows:
        if id(r) not in index_of:
            index_of[id(r)] = len(uniq)
            uniq.append(r)
    hosts = [_host_layout(r, seq_len) for r in uniq]

    # Table range: every owned query position, every attended key position, and 0 (padding).
    lo, hi = 0, 0
    for h in hosts:
        if h.qpos.size:
            lo, hi = min(lo, int(h.qpos.min())), max(hi, int(h.qpos.max()))
        if h.attn.any():
            kp = h.kpos[h.attn]
            lo, hi = min(lo, int(kp.min())), max(hi, int(kp.max()))
    n_pos = hi - lo + 1
    if n_pos > _ROW_MASK:
        raise ValueError("position range too large for the kernel tables")

    key_info_parts, key_base, own_rows, own_flags = [], [], [], []
    base = 0
    for h in hosts:
        rowidx = np.clip(h.kpos - lo, 0, n_pos - 1).astype(np.uint32)
        info = rowidx | (h.attn.astype(np.uint32) * _KEY_ATTN) | ((h.abs_ & h.attn).astype(np.uint32) * _KEY_ABS)
        key_info_parts.append(info)
        key_base.append(base)
        base += info.shape[0]
        # Key j's table row in the block whose query rows hold j; a block whose
        # attended keys all use that row can read a once-rotated copy of K.
        own = np.zeros(seq_len, dtype=np.int64)
        for s, e, ks, ke in h.bounds:
            own[s:e] = rowidx[ks + s:ks + e]
        own_rows.append(own)
        own_flags.append([bool(np.all(rowidx[ks:ke][h.attn[ks:ke]] == own[:e][h.attn[ks:ke]]))
                          for s, e, ks, ke in h.bounds])
    key_info = np.concatenate(key_info_parts).view(np.int32)

    blocks, row_blocks, row_cov = [], [0], []
    q_pos = np.zeros((batch, seq_len), dtype=np.int32)
    k_own = np.zeros((batch, seq_len), dtype=np.int32)
    pairs = 0
    host_pairs = [_pairs(h) for h in hosts]
    for b, r in enumerate(rows):
        u = index_of[id(r)]
        h = hosts[u]
        k_own[b] = own_rows[u]
        for bi, (s, e, ks, ke) in enumerate(h.bounds):
            am = h.attn[ks:ke]
            nz = np.flatnonzero(am)
            kv_lo = int(nz[0]) if nz.size else int(e)
            flags = 0
            if nz.size and not am[kv_lo:].all():
                flags |= BLOCKF_MASKED
            if (h.abs_[ks:ke] & am).any():
                flags |= BLOCKF_ABS
            if own_flags[u][bi]:
                flags |= BLOCKF_OWNPOS
            abs_lo = abs_hi = 0
            if flags & BLOCKF_ABS:
                na = np.flatnonzero(h.abs_[ks:ke] & am)
                abs_lo, abs_hi = int(na[0]), int(na[-1]) + 1
            blocks.append((b, int(s), int(e), key_base[u] + int(ks), kv_lo, flags, abs_lo, abs_hi))
        row_blocks.append(len(blocks))
        cov = int(h.bounds[-1, 1])
        row_cov.append(cov)
        qp = np.zeros(seq_len, dtype=np.int64)
        qp[:cov] = h.qpos
        q_pos[b] = np.clip(qp - lo, 0, n_pos - 1)
        pairs += host_pairs[u]

    blocks_np = np.asarray(blocks, dtype=np.int32).reshape(-1, 8)
    row_cov_np = np.asarray(row_cov, dtype=np.int32)
    fwd_items, kv_items, n_abs, n_kv_abs, n_short, n_abs_short = _tiles(fwd_tile, kv_tile, blocks_np, row_cov_np)

    return dict(blocks=blocks_np, row_blocks=np.asarray(row_blocks, dtype=np.int32), row_cov=row_cov_np,
                key_info=key_info, q_pos=q_pos, k_own=k_own, fwd_items=fwd_items, kv_items=kv_items,
                n_fwd_abs_items=n_abs, n_kv_abs_items=n_kv_abs, n_fwd_short_items=n_short,
                n_fwd_abs_short_items=n_abs_short, pairs_per_head=pairs,
                all_rows_owned=bool(np.all(row_cov_np >= seq_len)), p_min=lo, n_pos=n_pos)
