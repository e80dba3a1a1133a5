"""CPU oracle for the chain-of-edits (multi-segment RoPE) causal attention.

TEST INFRASTRUCTURE ONLY.  This module is the checker that the CUDA path of
``autoindexer_b200`` is compared against.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The product path never imports, calls or
falls back to it.

It is a numpy restatement of the reference's eager path (AutodeskAILab/
autoindexer, package ``src/autoindexer/models/autoindexer``):

* ``attention/utils.py:5-6``            ``apply_cos_sin``  (rotate-half RoPE)
* ``attention/reference.py:11-64``      ``compute_attn_weights_over_segments_ref``
* ``attention/reference.py:96-113``     ``compute_attn_weights_ref``  (causal + scale)
* ``attention/reference.py:116-141``    ``chain_of_edits_attn_ref``   (softmax, P.V)
* ``attention/__init__.py:36-37``       GQA expansion (``repeat_kv``) in the wrapper
* ``perturb_labels.py:333-339``         query positions zero-padded to ``T``
* ``attention/prefill_sdpa.py:11-71``   ``plain_causal_attn_sdpa`` (prefill)
* ``attention/__init__.py:36-51``, ``attn_layers.py:15-27``  decode step (``IterPositions``)

The reference obtains gradients through autograd; ``attn_backward`` writes the
same gradients out by hand (softmax backward, then the per-block split of the
logit gradient into the rotated-query part and the ``abs`` part, then the
transpose of the rotation).

Pinning: ``tests/test_oracle_golden.py`` checks this module against golden
vectors produced by running the reference itself (``tests/golden/make_golden.py``)
and against the reference's own known-answer position matrix
(``src/autoindexer/models/autoindexer/tests/labels/position_matrix.json``).

Layouts follow the reference: ``q`` is ``(B, Hq, T, D)``, ``k``/``v`` are
``(B, Hkv, T, D)`` (un-expanded, ``Hq = G * Hkv``), the output is
``(B, T, Hq, D)`` and ``lse`` is ``(B, Hq, T)``.

A ``layout`` is any object with the attributes the reference's
``PositionBlockList`` carries after ``concat()`` (``perturb_labels.py:341-357``):
``boundary_indices`` (list of ``(start, end, key_start, key_end)``),
``query_pos_ids``, ``concat_key_pos_ids``, ``concat_attn_masks`` and
``concat_abs_pos_masks`` (numpy arrays or torch CPU tensors).  ``layout`` may
also be a list with one such object per batch row.

``rope`` is a callable ``rope(position_ids) -> (cos, sin)`` returning arrays
of shape ``(L, D)``, the role ``RotaryEmbeddingFunc`` plays in the reference
(``type_utils.py:57``).
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "default_inv_freq",
    "make_rope",
    "make_sectioned_rope",
    "apply_cos_sin",
    "segment_logits",
    "attn_logits",
    "attn_forward",
    "attn_backward",
    "count_pairs",
    "attn_chunked",
    "index_rows",
    "index_losses",
]


def _np(x):
    if hasattr(x, "detach"):
        x = x.detach().cpu().numpy()
    return np.asarray(x)


# ---------------------------------------------------------------------------
# Rotary tables
# ---------------------------------------------------------------------------

def default_inv_freq(head_dim: int, theta: float) -> np.ndarray:
    """``inv_freq[k] = theta ** (-2k / D)`` in float32 (HF default RoPE init,
    transformers ``_compute_default_rope_parameters``).  Bit equality with
    torch's ``pow`` is not guaranteed; tests that need exact agreement take
    ``inv_freq`` from the rotary module itself."""
    exps = np.arange(0, head_dim, 2, dtype=np.int64).astype(np.float32) / np.float32(head_dim)
    return (np.float32(1.0) / (np.float32(theta) ** exps)).astype(np.float32)


def make_rope(inv_freq: np.ndarray):
    """Standard RoPE as HF computes it: the angle is the float32 product
    ``float32(pos) * inv_freq`` and ``cos``/``sin`` are taken of that float32
    angle; the half-table is repeated (``cat(freqs, freqs)``)."""
    inv_freq = np.asarray(inv_freq, dtype=np.float32)

    def rope(position_ids):
        pos = _np(position_ids).astype(np.float32).reshape(-1)
        ang = (pos[:, None] * inv_freq[None, :]).astype(np.float32).astype(np.float64)
        c, s = np.cos(ang), np.sin(ang)
        return np.concatenate([c, c], axis=-1), np.concatenate([s, s], axis=-1)

    return rope


def make_sectioned_rope(inv_freq: np.ndarray, streams, slot_sections):
    """Head-dim sections expressed through the reference's plugin type: the
    position id handed to the rotary function is a token index ``t``; frequency
    slot ``k`` that belongs to section ``s`` rotates by ``streams[s][t]``.
    ``slot_sections`` lists ``(slot_begin, slot_end)`` per section (rotate-half
    pairs dims ``k`` and ``k + D/2``, so a section owns whole slots)."""
    inv_freq = np.asarray(inv_freq, dtype=np.float32)
    streams = [np.asarray(_np(s), dtype=np.int64) for s in streams]
    half = inv_freq.shape[0]
    owner = np.empty(half, dtype=np.int64)
    for si, (a, b) in enumerate(slot_sections):
        owner[a:b] = si

    def rope(position_ids):
        idx = _np(position_ids).astype(np.int64).reshape(-1)
        idx = np.clip(idx, 0, None)
        pos = np.stack([streams[owner[k]][idx] for k in range(half)], axis=-1).astype(np.float32)
        ang = (pos * inv_freq[None, :]).astype(np.float32).astype(np.float64)
        c, s = np.cos(ang), np.sin(ang)
        return np.concatenate([c, c], axis=-1), np.concatenate([s, s], axis=-1)

    return rope


def _rotate_half(x):
    h = x.shape[-1] // 2
    return np.concatenate([-x[..., h:], x[..., :h]], axis=-1)


def apply_cos_sin(x, cos, sin):
    """``x * cos + rotate_half(x) * sin`` (``attention/utils.py:5-6``); ``cos`` and
    ``sin`` are ``(L, D)`` and broadcast over the leading dims of ``x``."""
    return x * cos + _rotate_half(x) * sin


def _rotate_half_T(g):
    """Transpose of ``rotate_half``: ``rotate_half(x) = [-x2, x1]`` so the
    adjoint maps ``[g1, g2]`` to ``[g2, -g1]``."""
    h = g.shape[-1] // 2
    return np.concatenate([g[..., h:], -g[..., :h]], axis=-1)


def apply_cos_sin_T(g, cos, sin):
    """Adjoint of ``apply_cos_sin`` with respect to ``x``."""
    return g * cos + _rotate_half_T(g * sin)


# ---------------------------------------------------------------------------
# Layout helpers
# ---------------------------------------------------------------------------

def _layout_arrays(layout):
    return (
        [tuple(int(v) for v in b) for b in layout.boundary_indices],
        _np(layout.query_pos_ids).astype(np.int64),
        _np(layout.concat_key_pos_ids).astype(np.int64),
        _np(layout.concat_attn_masks).astype(bool),
        _np(layout.concat_abs_pos_masks).astype(bool),
    )


def _per_row(layout, batch):
    if isinstance(layout, (list, tuple)) and len(layout) > 0 and hasattr(layout[0], "boundary_indices"):
        assert len(layout) == batch, "one layout per batch row expected"
        return list(layout)
    return [layout] * batch


def count_pairs(layout, seq_len: int) -> int:
    """Number of finite logits of one head of one batch row for ``layout``
    (owned rows only; the diagonal-only unowned rows are not counted)."""
    bounds, _, _, am, _ = _layout_arrays(layout)
    n = 0
    for s, e, ks, ke in bounds:
        m = am[ks:ke]
        c = np.cumsum(m.astype(np.int64))
        # row i in [s, e) sees keys j <= i with attn mask set
        n += int(c[s:e].sum())
    return n


# ---------------------------------------------------------------------------
# Forward
# ---------------------------------------------------------------------------

def segment_logits(q, q_rot, k, key_cos, key_sin, abs_mask, attn_mask, bounds):
    """Restates ``compute_attn_weights_over_segments_ref`` (reference.py:11-64)
    for one batch row: ``q``, ``q_rot``, ``k`` are ``(H, T, D)``; returns the
    ``(H, T, T)`` logits with ``-inf`` outside blocks and a zero diagonal on
    rows no block owns."""
    H, T, D = q.shape
    w = np.full((H, T, T), -np.inf, dtype=q.dtype)
    idx = np.arange(T)
    w[:, idx, idx] = 0
    for s, e, ks, ke in bounds:
        k_rot = apply_cos_sin(k[:, :e, :], key_cos[ks:ke], key_sin[ks:ke])  # (H, e, D)
        kt = np.swapaxes(k_rot, -1, -2)
        blk = q_rot[:, s:e, :] @ kt
        blk = blk + ((q[:, s:e, :] - q_rot[:, s:e, :]) @ kt) * abs_mask[ks:ke]
        blk = np.where(attn_mask[ks:ke], blk, -np.inf)
        w[:, s:e, :e] = blk
    return w


def _row_rope(rope, qpos, kpos, T):
    qp = np.zeros(T, dtype=np.int64)
    qp[: qpos.shape[0]] = qpos  # perturb_labels.py:335 pads with zeros
    qc, qs = rope(qp)
    kc, ks = rope(kpos)
    return qc, qs, kc, ks


def attn_logits(q_row, k_row, layout_row, rope, scale):
    """Restates ``compute_attn_weights_ref`` (reference.py:96-113) for one row:
    segment logits, global causal mask, then ``* scale``."""
    H, T, D = q_row.shape
    bounds, qpos, kpos, am, ab = _layout_arrays(layout_row)
    qc, qs, kc, ks = _row_rope(rope, qpos, kpos, T)
    q_rot = apply_cos_sin(q_row, qc, qs)
    w = segment_logits(q_row, q_rot, k_row, kc, ks, ab, am, bounds)
    causal = np.tril(np.ones((T, T), dtype=bool))
    w = np.where(causal, w, -np.inf)
    return w * scale


def _softmax(w):
    m = np.max(w, axis=-1, keepdims=True)
    e = np.exp(w - m)
    ssum = e.sum(axis=-1, keepdims=True)
    return e / ssum, (m + np.log(ssum))[..., 0]


def _expand(x, groups):
    return np.repeat(x, groups, axis=1) if groups > 1 else x


def attn_forward(q, k, v, layout, rope, scale=None, dtype=np.float64):
    """Restates ``chain_of_edits_attn_ref`` (reference.py:116-141) with the
    wrapper's GQA expansion (``attention/__init__.py:36-37``).

    Returns ``(out (B, T, Hq, D), lse (B, Hq, T))``; ``lse`` is the
    log-sum-exp of the scaled logits of each row (the quantity the fused
    kernels save for the backward pass)."""
    q, k, v = (_np(t).astype(dtype) for t in (q, k, v))
    B, Hq, T, D = q.shape
    G = Hq // k.shape[1]
    if scale is None:
        scale = D ** -0.5
    out = np.empty((B, T, Hq, D), dtype=dtype)
    lse = np.empty((B, Hq, T), dtype=dtype)
    for b, lay in enumerate(_per_row(layout, B)):
        w = attn_logits(q[b], _expand(k[b:b + 1], G)[0], lay, rope, scale)
        p, l = _softmax(w)
        out[b] = np.swapaxes(p @ _expand(v[b:b + 1], G)[0], 0, 1)
        lse[b] = l
    return out, lse


# ---------------------------------------------------------------------------
# Backward
# ---------------------------------------------------------------------------

def attn_backward(q, k, v, dout, layout, rope, scale=None, dtype=np.float64):
    """Gradients of ``attn_forward`` with respect to ``q``, ``k``, ``v`` for the
    upstream gradient ``dout (B, T, Hq, D)``; the same quantities the reference
    obtains through autograd on ``chain_of_edits_attn_ref``.

    Returns ``(dq (B, Hq, T, D), dk (B, Hkv, T, D), dv (B, Hkv, T, D))``."""
    q, k, v, dout = (_np(t).astype(dtype) for t in (q, k, v, dout))
    B, Hq, T, D = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    if scale is None:
        scale = D ** -0.5
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    for b, lay in enumerate(_per_row(layout, B)):
        bounds, qpos, kpos, am, ab = _layout_arrays(lay)
        qc, qs, kc, ks = _row_rope(rope, qpos, kpos, T)
        qb = q[b]
        kb = _expand(k[b:b + 1], G)[0]
        vb = _expand(v[b:b + 1], G)[0]
        q_rot = apply_cos_sin(qb, qc, qs)
        w = segment_logits(qb, q_rot, kb, kc, ks, ab, am, bounds)
        causal = np.tril(np.ones((T, T), dtype=bool))
        w = np.where(causal, w, -np.inf) * scale
        p, _ = _softmax(w)
        do = np.swapaxes(dout[b], 0, 1)  # (Hq, T, D)
        dvb = np.swapaxes(p, -1, -2) @ do
        dp = do @ np.swapaxes(vb, -1, -2)
        ds = p * (dp - np.sum(dp * p, axis=-1, keepdims=True))
        dl = np.where(np.isfinite(w), ds * scale, 0.0)  # gradient of the unscaled logits
        dq_rot = np.zeros_like(qb)
        dq_raw = np.zeros_like(qb)
        dkb = np.zeros_like(kb)
        for s, e, kst, ke in bounds:
            cos_b, sin_b = kc[kst:ke], ks[kst:ke]
            k_rot = apply_cos_sin(kb[:, :e, :], cos_b, sin_b)
            g = dl[:, s:e, :e]
            absm = ab[kst:ke].astype(dtype)
            g_rot = g * (1.0 - absm)
            g_abs = g * absm
            dq_rot[:, s:e, :] += g_rot @ k_rot
            dq_raw[:, s:e, :] += g_abs @ k_rot
            dk_rot = np.swapaxes(g_rot, -1, -2) @ q_rot[:, s:e, :] + np.swapaxes(g_abs, -1, -2) @ qb[:, s:e, :]
            dkb[:, :e, :] += apply_cos_sin_T(dk_rot, cos_b, sin_b)
        dq[b] = apply_cos_sin_T(dq_rot, qc, qs) + dq_raw
        dk[b] = dkb.reshape(Hkv, G, T, D).sum(axis=1)
        dv[b] = dvb.reshape(Hkv, G, T, D).sum(axis=1)
    return dq, dk, dv


# ---------------------------------------------------------------------------
# Query-chunked forward + backward (long sequences)
# ---------------------------------------------------------------------------

def attn_chunked(q, k, v, dout, layout, rope, scale=None, dtype=np.float64, chunk=512, backward=True):
    """The same function as ``attn_forward`` / ``attn_backward``, evaluated one
    block and one chunk of its query rows at a time, so that no ``(H, T, T)``
    array is ever held (the reference's eager path needs one; at T = 8192 and
    beyond it does not fit).  Per block ``[s, e)`` (``reference.py:46-62``) a
    chunk of rows ``[r0, r1)`` sees keys ``[kv_lo, r1)``: the causal limit of
    its last row, from the block's first attended key on (every key before
    it is masked, so its logit is ``-inf`` and its weight 0).  Softmax is
    per row, so chunking rows changes nothing; dK / dV are summed over the
    chunks and blocks that see a key.  Rows no block owns follow
    ``reference.py:42-43`` (only their own key, logit 0).

    Returns ``(out, lse, dq, dk, dv)`` (the gradients are ``None`` when
    ``backward`` is false); shapes as in ``attn_forward`` / ``attn_backward``."""
    q, k, v = (_np(t).astype(dtype) for t in (q, k, v))
    B, Hq, T, D = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    if scale is None:
        scale = D ** -0.5
    out = np.empty((B, T, Hq, D), dtype=dtype)
    lse = np.empty((B, Hq, T), dtype=dtype)
    if backward:
        dout = _np(dout).astype(dtype)
        dq = np.zeros_like(q)
        dk = np.zeros_like(k)
        dv = np.zeros_like(v)
    for b, lay in enumerate(_per_row(layout, B)):
        bounds, qpos, kpos, am, ab = _layout_arrays(lay)
        qc, qs, kc, ks = _row_rope(rope, qpos, kpos, T)
        qb = q[b]
        kb = _expand(k[b:b + 1], G)[0]
        vb = _expand(v[b:b + 1], G)[0]
        q_rot = apply_cos_sin(qb, qc, qs)
        if backward:
            do_b = np.swapaxes(dout[b], 0, 1)  # (Hq, T, D)
            dq_rot = np.zeros_like(qb)
            dq_raw = np.zeros_like(qb)
            dkb = np.zeros_like(kb)
            dvb = np.zeros_like(vb)
        cov = bounds[-1][1] if bounds else 0
        # rows no block owns: p = 1 on the own key, so out = v, lse = 0, dV += dO
        out[b, cov:] = np.swapaxes(vb[:, cov:], 0, 1)
        lse[b, :, cov:] = 0
        if backward:
            dvb[:, cov:] += do_b[:, cov:]
        for s, e, kst, ke in bounds:
            attm = am[kst:ke]
            absm = ab[kst:ke]
            nz = np.flatnonzero(attm)
            lo = int(nz[0]) if nz.size else e
            if lo >= e:
                out[b, s:e] = np.nan  # softmax over no key (the reference gives NaN as well)
                lse[b, :, s:e] = -np.inf
                continue
            k_rot = apply_cos_sin(kb[:, lo:e, :], kc[kst + lo:ke], ks[kst + lo:ke])  # keys [lo, e)
            has_abs = bool(absm[lo:e].any())
            if backward:
                dk_rot = np.zeros_like(k_rot)
            for r0 in range(s, e, chunk):
                r1 = min(r0 + chunk, e)
                n = r1 - lo
                kr = k_rot[:, :n]
                krt = np.swapaxes(kr, -1, -2)
                w = q_rot[:, r0:r1] @ krt
                if has_abs:
                    w = w + ((qb[:, r0:r1] - q_rot[:, r0:r1]) @ krt) * absm[lo:r1]
                rows = np.arange(r0, r1)[:, None]
                cols = np.arange(lo, r1)[None, :]
                ok = attm[lo:r1][None, :] & (cols <= rows)
                w = np.where(ok, w, -np.inf) * scale
                p, l = _softmax(w)
                out[b, r0:r1] = np.swapaxes(p @ vb[:, lo:r1], 0, 1)
                lse[b, :, r0:r1] = l
                if not backward:
                    continue
                do = do_b[:, r0:r1]
                dvb[:, lo:r1] += np.swapaxes(p, -1, -2) @ do
                dp = do @ np.swapaxes(vb[:, lo:r1], -1, -2)
                ds = p * (dp - np.sum(dp * p, axis=-1, keepdims=True))
                dl = np.where(ok, ds * scale, 0.0)
                if has_abs:
                    a_ = absm[lo:r1].astype(dtype)
                    g_rot, g_abs = dl * (1.0 - a_), dl * a_
                    dq_raw[:, r0:r1] += g_abs @ kr
                    dk_rot[:, :n] += np.swapaxes(g_abs, -1, -2) @ qb[:, r0:r1]
                else:
                    g_rot = dl
                dq_rot[:, r0:r1] += g_rot @ kr
                dk_rot[:, :n] += np.swapaxes(g_rot, -1, -2) @ q_rot[:, r0:r1]
            if backward:
                dkb[:, lo:e] += apply_cos_sin_T(dk_rot, kc[kst + lo:ke], ks[kst + lo:ke])
        if backward:
            dq[b] = apply_cos_sin_T(dq_rot, qc, qs) + dq_raw
            dk[b] = dkb.reshape(Hkv, G, T, D).sum(axis=1)
            dv[b] = dvb.reshape(Hkv, G, T, D).sum(axis=1)
    if not backward:
        return out, lse, None, None, None
    return out, lse, dq, dk, dv


# ---------------------------------------------------------------------------
# Index head: edit-cursor losses
# ---------------------------------------------------------------------------

BLOCK_EXTEND = 1


def index_rows(layout, block_type, edits, editable_start=0):
    """The rows of ``compute_index_losses`` (``attn_layers.py:40-110``): for
    every EXTEND block (an edit; its last row is the edit marker ``ed``) a
    start row (head 0, query ``ed - 1``, keys ``[0, ed)`` at positions
    ``key_pos[:-1] - query_pos[-2]``, attended where ``attn_mask[:-1] &
    key_pos >= editable_start``) and an end row (head 1, query ``ed``, keys
    ``[0, ed]`` at ``key_pos - query_pos[-1]``, attended where ``attn_mask &
    key_pos >= editable_start`` and the relative position is > 0,
    ``compute_end_index_mask`` ``:30-37``).  ``edits``: rows of (edit marker
    index, start cursor, end cursor).  Returns a list of
    ``(head, query_row, rel_pos, ok, target, edit)``."""
    bounds, qpos, kpos, am, _ = _layout_arrays(layout)
    cursor = {int(e): (int(s), int(t)) for e, s, t in np.asarray(edits).reshape(-1, 3)}
    rows = []
    for bi, (s, e, ks, ke) in enumerate(bounds):
        if int(block_type[bi]) != BLOCK_EXTEND:
            continue
        ed = e - 1
        kp, att, qp = kpos[ks:ke], am[ks:ke], qpos[s:e]
        tgt_s, tgt_e = cursor[ed]
        rel = kp[:-1] - qp[-2]
        rows.append((0, ed - 1, rel, att[:-1] & (kp[:-1] >= editable_start), tgt_s, ed))
        rel = kp - qp[-1]
        rows.append((1, ed, rel, att & (kp >= editable_start) & (rel > 0), tgt_e, ed))
    return rows


def index_losses(q, k, layout, block_type, edits, rope, scale=None, editable_start=0, w_start=1.0, w_end=1.0,
                 dtype=np.float64):
    """Restates ``compute_index_losses`` (``attn_layers.py:40-110``) with
    ``compute_attn_weights_iter`` (``:15-27``: the query unrotated, every key
    rotated by its relative position, masked keys ``-inf``, times ``scale``):
    ``start_loss`` / ``end_loss`` are the means over the batch of
    ``-log_softmax`` at the cursor key, averaged over the edits.  Also
    returns the gradients of ``w_start * start_loss + w_end * end_loss`` with
    respect to ``q`` and ``k`` (``(B, 2, T, D)``), written out by hand:
    ``dlogit_j = w * (softmax_j - [j == target]) / (B * n_edits)``,
    ``dq = scale sum_j dlogit_j R(rel_j) k_j``,
    ``dk_j = scale dlogit_j R(rel_j)^T q``."""
    q, k = (_np(t).astype(dtype) for t in (q, k))
    B, H, T, D = q.shape
    assert H == 2
    if scale is None:
        scale = D ** -0.5
    rows = index_rows(layout, block_type, edits, editable_start)
    n_edits = len(rows) // 2
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    totals = [0.0, 0.0]
    for h, qi, rel, ok, tgt, _ in rows:
        n = rel.shape[0]
        cos, sin = rope(rel)
        kr = apply_cos_sin(k[:, h, :n, :], cos, sin)  # (B, n, D)
        w = np.einsum("bd,bnd->bn", q[:, h, qi, :], kr) * scale
        w = np.where(ok[None, :], w, -np.inf)
        p, lse = _softmax(w)
        totals[h] += float(np.mean(lse - w[:, tgt]))
        weight = (w_start if h == 0 else w_end) / (B * max(n_edits, 1))
        g = p.copy()
        g[:, tgt] -= 1.0
        g = np.where(ok[None, :], g * weight, 0.0)  # masked logits are constants (masked_fill)
        dq[:, h, qi, :] += scale * np.einsum("bn,bnd->bd", g, kr)
        dk[:, h, :n, :] += scale * apply_cos_sin_T(g[:, :, None] * q[:, h, qi, None, :], cos, sin)
    if n_edits > 0:
        totals = [t / n_edits for t in totals]
    return totals[0], totals[1], dq, dk


# ---------------------------------------------------------------------------
# Prefill (plain causal attention of left-padded prompts)
# ---------------------------------------------------------------------------

def plain_causal_forward(q, k, v, keep, rope, scale=None, dtype=np.float64):
    """Restates ``plain_causal_attn_sdpa`` (``attention/prefill_sdpa.py:11-71``)
    after the registry wrapper's GQA expansion (``attention/__init__.py:36-37``):
    ``q`` and ``k`` rotated by ``rope(arange(T))`` (one position table for
    every row, ``prefill_sdpa.py:55-58``), then softmax attention under
    ``tril(T, T) & keep[b]`` (``prefill_sdpa.py:60-68``; ``keep`` ``(B, T)``
    bool or ``None`` for plain causal).  A query row that attends no key has
    no defined result in the reference (SDPA); here it is zero, with lse
    ``-inf``.  Returns ``(out (B, T, Hq, D), lse (B, Hq, T))``."""
    q, k, v = (_np(t).astype(dtype) for t in (q, k, v))
    B, Hq, T, D = q.shape
    G = Hq // k.shape[1]
    if scale is None:
        scale = D ** -0.5
    cos, sin = rope(np.arange(T))
    qr = apply_cos_sin(q, cos, sin)
    kr = apply_cos_sin(_expand(k, G), cos, sin)
    ve = _expand(v, G)
    causal = np.tril(np.ones((T, T), dtype=bool))
    out = np.zeros((B, T, Hq, D), dtype=dtype)
    lse = np.full((B, Hq, T), -np.inf, dtype=dtype)
    for b in range(B):
        allowed = causal if keep is None else causal & np.asarray(keep[b], dtype=bool)[None, :]
        rows = allowed.any(axis=1)
        w = np.einsum("htd,hsd->hts", qr[b], kr[b]) * scale
        w = np.where(allowed[None], w, -np.inf)
        p, l = _softmax(w[:, rows])
        out[b][rows] = np.swapaxes(p @ ve[b], 0, 1)
        lse[b][:, rows] = l
    return out, lse


# ---------------------------------------------------------------------------
# Decode step (IterPositions)
# ---------------------------------------------------------------------------

def decode_forward(q, k, v, key_pos, attn_mask, rope, scale=None, attention_mask=None, dtype=np.float64):
    """Restates the IterPositions branch of the registered interface
    (``attention/__init__.py:36-51``): K/V expanded for GQA (``repeat_kv``),
    ``compute_attn_weights_iter`` (``attn_layers.py:15-27``: keys rotated by
    ``rope(key_pos)``, the query unrotated, ``q . k_rot``, ``attn_mask``
    positions set to -inf, times ``scale``), a boolean ``attention_mask``
    applied as a fill and a float one added, softmax, ``P . V``.

    ``q`` ``(B, Hq, 1, D)``; ``k``, ``v`` ``(B, Hkv, L, D)``; ``key_pos``
    ``(L,)`` or ``(B, L)``; ``attn_mask`` the same shape (bool) or ``None``.
    Returns ``(B, Hq, 1, D)``."""
    q, k, v = (_np(t).astype(dtype) for t in (q, k, v))
    B, Hq, _, D = q.shape
    L = k.shape[2]
    G = Hq // k.shape[1]
    if scale is None:
        scale = D ** -0.5
    kp = np.asarray(_np(key_pos)).reshape(-1, L)
    cos, sin = rope(kp.reshape(-1))
    cos, sin = cos.reshape(kp.shape[0], 1, L, D), sin.reshape(kp.shape[0], 1, L, D)
    kr = apply_cos_sin(_expand(k, G), cos, sin)
    w = np.einsum("bhqd,bhkd->bhqk", q, kr)
    if attn_mask is not None:
        am = np.asarray(_np(attn_mask), dtype=bool).reshape(-1, 1, 1, L)
        w = np.where(am, w, -np.inf)
    w = w * scale
    if attention_mask is not None:
        m = _np(attention_mask)
        w = np.where(m, w, -np.inf) if m.dtype == bool else w + m.astype(dtype)
    p, _ = _softmax(w)
    return p @ _expand(v, G)
