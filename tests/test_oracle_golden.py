"""Pins the CPU oracle (``oracle/attn_oracle.py``) against the reference.

* every golden case under ``tests/golden`` was produced by running the
  reference's own eager attention and autograd (``make_golden.py``); the
  oracle must reproduce output, log-sum-exp and dQ/dK/dV;
* the reference's known-answer test (``tests/test_generalized_rope.py`` with
  ``labels/position_matrix.json``): recovering integer relative positions
  from ``acos`` of the logits with ``head_dim = 2`` and ``inv_freq / 100``.
"""

import numpy as np
import pytest

from conftest import ArrayLayout, golden_inputs, golden_names, golden_rope, load_golden
from oracle import attn_oracle as O


@pytest.mark.parametrize("name", golden_names())
def test_oracle_matches_reference(name):
    g = load_golden(name)
    lay = ArrayLayout.from_golden(g)
    _, rope = golden_rope(g)
    q, k, v, dout = golden_inputs(g)
    out, lse = O.attn_forward(q, k, v, lay, rope)
    dq, dk, dv = O.attn_backward(q, k, v, dout, lay, rope)
    for label, got, want in (("out", out, g["out"]), ("lse", lse, g["lse"]), ("dq", dq, g["dq"]),
                             ("dk", dk, g["dk"]), ("dv", dv, g["dv"])):
        np.testing.assert_allclose(got, want, rtol=2e-5, atol=2e-5, err_msg=f"{name}:{label}")


def test_oracle_known_answer_position_matrix():
    """Restates the reference's KAT (test_generalized_rope.py:20-64) through
    the oracle's logits."""
    import os
    from conftest import GOLDEN

    with np.load(os.path.join(GOLDEN, "kat_position_matrix.npz")) as z:
        g = {k: z[k] for k in z.files}
    lay = ArrayLayout.from_golden(g)
    T = g["position_matrix"].shape[0]
    inv = np.asarray([1.0 / 100.0], dtype=np.float32)  # head_dim 2, theta 1e4 -> inv_freq 1.0, divided by 100
    rope = O.make_rope(inv)
    q = np.zeros((1, 1, T, 2))
    q[..., 0] = 1
    k = q.copy()
    k_sign = np.ones((1, 1, T, 2))
    k_sign[..., 0] = 0
    w = O.attn_logits(q[0], k[0], lay, rope, 1.0)[0]
    ws = O.attn_logits(q[0], k_sign[0], lay, rope, 1.0)[0]
    mask = w != -np.inf
    sign = -np.sign(np.where(np.isfinite(ws), ws, 0) * 100)
    rec = np.round(sign * np.arccos(np.clip(np.where(mask, w, 0), -1, 1)) / inv[0]).astype(np.int64)
    rec = np.where(mask, rec, 0)
    np.testing.assert_array_equal(mask.astype(np.int64), g["attention_mask"].astype(np.int64))
    np.testing.assert_array_equal(rec, g["position_matrix"].astype(np.int64))


def test_oracle_unowned_rows_are_diagonal_only():
    """Rows past the blocks' coverage see only their own key with logit 0
    (reference.py:42-43): out = v of the row, lse = 0."""
    g = load_golden("op7_d32")
    lay = ArrayLayout.from_golden(g)
    _, rope = golden_rope(g)
    q, k, v, dout = golden_inputs(g)
    T = q.shape[2]
    pad = 7
    qp, kp, vp = (np.concatenate([x, np.random.default_rng(0).standard_normal(x.shape[:2] + (pad, x.shape[3]))], axis=2)
                  for x in (q, k, v))
    out, lse = O.attn_forward(qp, kp, vp, lay, rope)
    np.testing.assert_allclose(out[0, T:, :, :], np.repeat(vp[0, :, T:, :], 2, axis=0).transpose(1, 0, 2), atol=1e-12)
    np.testing.assert_allclose(lse[0, :, T:], 0.0, atol=1e-12)
    np.testing.assert_allclose(out[0, :T], g["out"][0], rtol=2e-5, atol=2e-5)


def test_count_pairs_matches_logits():
    g = load_golden("op0_d32")
    lay = ArrayLayout.from_golden(g)
    _, rope = golden_rope(g)
    q, k, _, _ = golden_inputs(g)
    w = O.attn_logits(q[0], np.repeat(k[0], 2, axis=0), lay, rope, 1.0)
    assert int(np.isfinite(w[0]).sum()) == O.count_pairs(lay, q.shape[2])


@pytest.mark.parametrize("name", ["op0_d32", "op5_d32", "op9_d32", "sec3", "chain_e"])
def test_chunked_oracle_matches_dense_oracle(name):
    """The query-chunked restatement (used at sizes where the dense one's
    (H, T, T) arrays do not fit) gives the dense oracle's results; chunks of
    a few rows put chunk edges inside every block."""
    g = load_golden(name)
    lay = ArrayLayout.from_golden(g)
    _, rope = golden_rope(g)
    q, k, v, dout = golden_inputs(g)
    want = O.attn_forward(q, k, v, lay, rope) + O.attn_backward(q, k, v, dout, lay, rope)
    got = O.attn_chunked(q, k, v, dout, lay, rope, chunk=37 if name == "chain_e" else 5)
    for label, a, b in zip(("out", "lse", "dq", "dk", "dv"), got, want):
        np.testing.assert_allclose(a, b, rtol=1e-10, atol=1e-10, err_msg=f"{name}:{label}")
    np.testing.assert_allclose(got[0], g["out"], rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("case", range(10))
@pytest.mark.parametrize("es", [0, 3])
def test_index_loss_oracle_matches_reference(case, es):
    """The index-head oracle reproduces the reference's compute_index_losses
    (attn_layers.py:40-110) and its autograd gradients on the reference's own
    operation cases (tests/golden/make_index_golden.py), editable_start 0 and 3."""
    g = load_golden(f"index_op{case}")
    lay = ArrayLayout.from_golden(g)
    rope = O.make_rope(g["inv_freq"])
    from golden_inputs import make_inputs

    q, k, _, _ = make_inputs(int(g["seed"]), int(g["B"]), 2, 2, int(g["T"]), int(g["D"]))
    sl, el, dq, dk = O.index_losses(q, k, lay, g["block_type"], g["cursor_edits"], rope, editable_start=es,
                                    w_start=1.0, w_end=2.0)
    np.testing.assert_allclose(sl, g[f"start_loss_es{es}"], rtol=1e-6)
    np.testing.assert_allclose(el, g[f"end_loss_es{es}"], rtol=1e-6)
    np.testing.assert_allclose(dq, g[f"dq_es{es}"], rtol=2e-5, atol=2e-6)
    np.testing.assert_allclose(dk, g[f"dk_es{es}"], rtol=2e-5, atol=2e-6)
