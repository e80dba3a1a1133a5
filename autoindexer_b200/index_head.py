"""Index-head cursor losses on the B200 kernels.

``compute_index_losses_b200`` has the signature and results of the
reference's ``compute_index_losses`` (``attn_layers.py:40-110`` of
AutodeskAILab/autoindexer's ``src/autoindexer/models/autoindexer``): for every
edit of the position-block list (an EXTEND block, its last row the edit
marker) the start-cursor head (head 0, the query just before the marker) and
the end-cursor head (head 1, the marker) attend over the key prefix with keys
rotated by their position relative to the query, masked keys excluded (the
end head also excludes keys at relative positions <= 0), and the losses are
``-log_softmax`` at the cursor keys, averaged over the batch and the edits.

The reference loops over the edits in Python, a dozen small torch ops each;
here the rows of all edits are built once on the host (``index_rows``) and
run by one forward launch and two backward launches of ``ai_index_fwd`` /
``ai_index_bwd`` (``csrc/ai_index.cu``), differentiable through autograd.
"""

from __future__ import annotations

import ctypes
from typing import Dict, Optional, Tuple

import numpy as np
import torch
from torch import Tensor

from . import _lib
from .positions import BlockType
from .rope import rope_table

__all__ = ["IndexRows", "index_rows", "compute_index_losses_b200"]


def _np(x):
    if hasattr(x, "detach"):
        return x.detach().cpu().numpy()
    return np.asarray(x)


class IndexRows:
    """The host-built rows of one (list, cursors, editable_start): per row
    (head, query row, key count, key offset), its cursor target, and per key
    its position relative to the query and whether it may be attended."""

    def __init__(self, rows, targets, rel, ok, edits):
        self.rows = rows          # [n_rows, 4] int32
        self.targets = targets    # [n_rows] int32
        self.rel = rel            # [n_keys] int64
        self.ok = ok              # [n_keys] uint8
        self.edits = edits        # [n_rows] edit marker index of the row


def index_rows(parsed_positions, cursor_indices, editable_start: int = 0) -> IndexRows:
    """Rows of ``compute_index_losses`` for a concat()-ed position-block
    list whose blocks carry ``block_type`` (``cursor_indices``: edit marker
    index -> (start cursor, end cursor), as ``batch_perturb_labels`` returns
    them with ``return_indices_as_dict``)."""
    rows, targets, rels, oks, edits = [], [], [], [], []
    off = 0
    kpos_all = _np(parsed_positions.concat_key_pos_ids).astype(np.int64)
    attn_all = _np(parsed_positions.concat_attn_masks).astype(bool)
    qpos_all = _np(parsed_positions.query_pos_ids).astype(np.int64)
    for blk, (s, e, ks, ke) in zip(parsed_positions, parsed_positions.boundary_indices):
        if int(blk.block_type or 0) != int(BlockType.EXTEND):
            continue
        s, e, ks, ke = int(s), int(e), int(ks), int(ke)
        ed = e - 1
        kp, att, qp = kpos_all[ks:ke], attn_all[ks:ke], qpos_all[s:e]
        tgt_s, tgt_e = (int(x) for x in cursor_indices[ed])
        for head, qi, rel, ok, tgt in (
                (0, ed - 1, kp[:-1] - qp[-2], att[:-1] & (kp[:-1] >= editable_start), tgt_s),
                (1, ed, kp - qp[-1], att & (kp >= editable_start), tgt_e)):
            if head == 1:
                ok = ok & (rel > 0)  # compute_end_index_mask, attn_layers.py:30-37
            n = rel.shape[0]
            rows.append((head, qi, n, off))
            targets.append(tgt)
            rels.append(rel)
            oks.append(ok.astype(np.uint8))
            edits.append(ed)
            off += n
    return IndexRows(np.asarray(rows, dtype=np.int32).reshape(-1, 4), np.asarray(targets, dtype=np.int32),
                     np.concatenate(rels) if rels else np.zeros(0, np.int64),
                     np.concatenate(oks) if oks else np.zeros(0, np.uint8), np.asarray(edits, dtype=np.int64))


def _t4(x: Tensor) -> "_lib.AiTensor4":
    t = _lib.AiTensor4()
    t.ptr = x.data_ptr()
    t.stride_b, t.stride_h, t.stride_t = x.stride(0), x.stride(1), x.stride(2)
    return t


class _Prepared:
    """Device copies of the rows and the rotary table for one call: the
    row table, targets, key table rows and key flags go over in one copy
    from one pinned host buffer (filled by the native builder,
    ``ai_index_rows``, in ``native``)."""

    @classmethod
    def native(cls, parsed_positions, cursor_indices, editable_start: int, rotary_emb, head_dim: int, device):
        """The rows of every edit built by ``ai_index_rows`` straight into the
        pinned buffer; ``None`` when the list has no edit."""
        from .meta import _prep_list

        pl, keep = _prep_list(parsed_positions, 0)
        types = np.ascontiguousarray(np.asarray([int(b.block_type or 0) for b in parsed_positions], dtype=np.int32))
        if types.shape[0] != pl.n_blocks:
            raise ValueError("block_type count does not match boundary_indices")
        lib = _lib.lib()
        n_rows, n_keys = ctypes.c_int32(0), ctypes.c_int64(0)
        edits = np.zeros(max(1, pl.n_blocks), dtype=np.int64)
        _lib.check(lib.ai_index_rows_sizes(ctypes.byref(pl), types.ctypes.data, ctypes.byref(n_rows),
                                           ctypes.byref(n_keys), edits.ctypes.data), "ai_index_rows_sizes")
        self = cls.__new__(cls)
        self.n_rows, self.n_keys = int(n_rows.value), int(n_keys.value)
        if self.n_rows == 0:
            return None
        self.edits = np.repeat(edits[:self.n_rows // 2], 2)
        tg = np.asarray([cursor_indices[int(e)] for e in edits[:self.n_rows // 2]], dtype=np.int32).reshape(-1)
        self._fill(tg, device, lambda rows, key_rows, key_ok: cls._native_fill(pl, types, editable_start, rows,
                                                                                key_rows, key_ok))
        self.cos, self.sin = rope_table(rotary_emb, self.lo, self.hi, head_dim, device)
        self.n_pos = self.hi - self.lo + 1
        del keep
        return self

    @staticmethod
    def _native_fill(pl, types, editable_start, rows, key_rows, key_ok):
        out = _lib.AiIndexRowsOut()
        out.rows, out.key_rows, out.key_ok = rows.ctypes.data, key_rows.ctypes.data, key_ok.ctypes.data
        _lib.check(_lib.lib().ai_index_rows(ctypes.byref(pl), types.ctypes.data, int(editable_start),
                                            ctypes.byref(out)), "ai_index_rows")
        return int(out.rel_lo), int(out.rel_hi)

    def _fill(self, targets, device, writer):
        # int32 sections (16-byte aligned): rows [n_rows][4], targets, key rows; then the uint8 key flags
        n_rows4, n_keys4 = 4 * self.n_rows, (self.n_keys + 3) // 4 * 4
        o_tg = n_rows4
        o_kr = o_tg + (self.n_rows + 3) // 4 * 4
        o_ok = o_kr + n_keys4
        host = torch.empty(4 * o_ok + n_keys4, dtype=torch.uint8, pin_memory=True)
        h32 = host[:4 * o_ok].view(torch.int32).numpy()
        h32[o_tg:o_tg + self.n_rows] = targets
        rows = h32[:n_rows4].reshape(-1, 4)
        self.lo, self.hi = writer(rows, h32[o_kr:o_kr + self.n_keys], host[4 * o_ok:4 * o_ok + self.n_keys].numpy())
        self.host_rows = rows
        dev = host.to(device, non_blocking=True)
        d32 = dev[:4 * o_ok].view(torch.int32)
        self.rows = d32[:n_rows4]
        self.targets = d32[o_tg:o_tg + self.n_rows]
        self.key_rows = d32[o_kr:o_kr + self.n_keys]
        self.key_ok = dev[4 * o_ok:4 * o_ok + self.n_keys]
        self._host = host  # the copy reads it asynchronously


def _args(q, k, prep: _Prepared, scale, logits, lse, loss):
    from .attention import status_word

    a = _lib.AiIndexArgs()
    a.batch, _, a.seq_len, a.head_dim = q.shape
    a.dtype = _lib.DTYPE_BF16 if q.dtype == torch.bfloat16 else _lib.DTYPE_F32
    a.scale = float(scale)
    a.q, a.k = _t4(q), _t4(k)
    a.n_rows = prep.n_rows
    a.rows = prep.rows.data_ptr()
    a.targets = prep.targets.data_ptr()
    a.n_keys = prep.n_keys
    a.key_rows = prep.key_rows.data_ptr()
    a.key_ok = prep.key_ok.data_ptr()
    a.rope_cos, a.rope_sin, a.n_pos = prep.cos.data_ptr(), prep.sin.data_ptr(), prep.n_pos
    a.logits, a.lse, a.loss = logits.data_ptr(), lse.data_ptr(), loss.data_ptr()
    a.status = status_word(q.device).data_ptr()
    return a


class IndexLossFn(torch.autograd.Function):
    """Per-(batch row, index row) losses ``(B, n_rows)`` fp32 and the logits
    ``(B, n_keys)``; backward through ``ai_index_bwd``."""

    @staticmethod
    def forward(ctx, q, k, prep: _Prepared, scale: float):
        B = q.shape[0]
        logits = torch.empty((B, prep.n_keys), dtype=torch.float32, device=q.device)
        lse = torch.empty((B, prep.n_rows), dtype=torch.float32, device=q.device)
        loss = torch.empty((B, prep.n_rows), dtype=torch.float32, device=q.device)
        a = _args(q, k, prep, scale, logits, lse, loss)
        stream = torch.cuda.current_stream(q.device).cuda_stream
        _lib.check(_lib.lib().ai_index_fwd(ctypes.byref(a), ctypes.c_void_p(stream)), "ai_index_fwd")
        ctx.save_for_backward(q, k, logits, lse)
        ctx.prep, ctx.scale = prep, scale
        ctx.mark_non_differentiable(logits)
        return loss, logits

    @staticmethod
    def backward(ctx, dloss, _dlogits):
        q, k, logits, lse = ctx.saved_tensors
        prep = ctx.prep
        dq = torch.zeros_like(q)
        dk = torch.empty_like(k)
        dl = dloss.float().contiguous() if dloss is not None else torch.zeros_like(lse)
        loss_dummy = torch.empty_like(lse)
        b = _lib.AiIndexBwdArgs()
        b.fwd = _args(q, k, prep, ctx.scale, logits, lse, loss_dummy)
        b.dloss = dl.data_ptr()
        b.dq, b.dk = _t4(dq), _t4(dk)
        stream = torch.cuda.current_stream(q.device).cuda_stream
        _lib.check(_lib.lib().ai_index_bwd(ctypes.byref(b), ctypes.c_void_p(stream)), "ai_index_bwd")
        return dq, dk, None, None


def compute_index_losses_b200(
        rotary_emb,
        query: Tensor,
        keys: Tensor,
        parsed_positions,
        cursor_indices,
        scaling: Optional[float] = None,
        return_weights: bool = False,
        editable_start: int = 0,
) -> Tuple[Tuple[Tensor, Tensor], Dict[int, Tuple[Tensor, Tensor]]]:
    """Same contract as the reference's ``compute_index_losses``: ``query``
    and ``keys`` ``(B, 2, T, D)`` (head 0 start cursor, head 1 end cursor,
    unrotated), a concat()-ed position-block list shared by the batch,
    ``cursor_indices`` {edit marker index: (start, end)}; returns
    ``((start_loss, end_loss), weights)`` with ``weights[edit] = (start
    logits (B, 1, 1, ed), end logits (B, 1, 1, ed + 1))`` when
    ``return_weights``.  CUDA tensors (bf16 or fp32, head_dim 32 / 64 / 128)."""
    B, H, T, D = query.shape
    if H != 2:
        raise ValueError("the index head has two heads (start and end cursor)")
    if keys.shape[2] != T:
        raise AssertionError("q_len must equal kv_len")
    if not query.is_cuda:
        raise RuntimeError("autoindexer_b200 index losses run on CUDA tensors only")
    if query.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError(f"unsupported dtype {query.dtype}")
    scale = float(scaling) if scaling is not None else D ** -0.5
    prep = _Prepared.native(parsed_positions, cursor_indices, editable_start, rotary_emb, D, query.device)
    if prep is None:
        # as the reference: keep q/k in the graph with a zero contribution
        zero = (query.sum() + keys.sum()) * 0.0
        return (zero.to(query.dtype), zero.to(query.dtype)), {}
    n_edits = prep.n_rows // 2
    q = query if query.stride(-1) == 1 else query.contiguous()
    k = keys if keys.stride(-1) == 1 else keys.contiguous()
    loss, logits = IndexLossFn.apply(q, k, prep, scale)
    # rows come in (start, end) pairs per edit; mean over the batch as .mean() in the reference
    per_edit = loss.mean(dim=0).view(n_edits, 2).sum(dim=0) / n_edits
    start_loss, end_loss = per_edit[0], per_edit[1]
    weights = {}
    if return_weights:
        for r in range(prep.n_rows):
            h, _, n, off = (int(x) for x in prep.host_rows[r])
            w = logits[:, off:off + n].to(query.dtype).view(B, 1, 1, n)
            ed = int(prep.edits[r])
            s_w, e_w = weights.get(ed, (None, None))
            weights[ed] = (w, e_w) if h == 0 else (s_w, w)
    return (start_loss.to(query.dtype), end_loss.to(query.dtype)), weights
