"""Index-head cursor losses (``autoindexer_b200.compute_index_losses_b200``,
kernels ``ai_index_fwd`` / ``ai_index_bwd``) against the reference's
``compute_index_losses`` (``attn_layers.py:40-110``).

* CPU: the host-built rows equal the oracle's restatement of the reference's
  per-edit rows;
* GPU, fp32: the losses and the gradients of ``start + 2 * end`` match the
  vectors the reference produced on its own operation cases
  (``tests/golden/index_op*.npz``), 1e-4;
* GPU, bf16, the +E training chain (T = 3072, 46 edits, head_dim 128): the
  losses within 1e-2 relative and the gradients within relative L2 1e-2 of
  the oracle, and the returned weights equal the logits the oracle builds.
"""

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, ArrayLayout, HFRope, load_golden, rel_l2
from oracle import attn_oracle as O


def _golden_case(i):
    g = load_golden(f"index_op{i}")
    lay = ArrayLayout.from_golden(g)
    blocks = _typed_list(lay, g["block_type"])
    cursor = {int(e): (int(s), int(t)) for e, s, t in g["cursor_edits"]}
    from golden_inputs import make_inputs

    q, k, _, _ = make_inputs(int(g["seed"]), int(g["B"]), 2, 2, int(g["T"]), int(g["D"]))
    return g, blocks, cursor, q, k


def _typed_list(lay, block_type):
    """The concat()-ed list as blocks carrying their types (what the
    reference's PositionBlockList holds)."""
    from autoindexer_b200.positions import BlockType, blocks_from_concat

    out = blocks_from_concat(lay.boundary_indices, lay.query_pos_ids, lay.concat_key_pos_ids, lay.concat_attn_masks,
                             lay.concat_abs_pos_masks)
    for blk, t in zip(out, block_type):
        blk.block_type = BlockType(int(t))
    return out


@pytest.mark.parametrize("case", [0, 3, 9])
@pytest.mark.parametrize("es", [0, 3])
def test_index_rows_match_oracle(case, es):
    from autoindexer_b200.index_head import index_rows

    g, blocks, cursor, _, _ = _golden_case(case)
    ir = index_rows(blocks, cursor, editable_start=es)
    want = O.index_rows(blocks, g["block_type"], g["cursor_edits"], editable_start=es)
    assert ir.rows.shape[0] == len(want)
    off = 0
    for r, (h, qi, rel, ok, tgt, ed) in enumerate(want):
        assert tuple(ir.rows[r]) == (h, qi, rel.shape[0], off)
        assert ir.targets[r] == tgt and ir.edits[r] == ed
        assert np.array_equal(ir.rel[off:off + rel.shape[0]], rel)
        assert np.array_equal(ir.ok[off:off + rel.shape[0]].astype(bool), ok)
        off += rel.shape[0]


@pytest.mark.gpu
@pytest.mark.parametrize("case", range(10))
@pytest.mark.parametrize("es", [0, 3])
def test_fp32_index_losses_match_reference(case, es, cuda_device):
    from autoindexer_b200 import compute_index_losses_b200

    g, blocks, cursor, q, k = _golden_case(case)
    rope = HFRope(g["inv_freq"]).to(cuda_device)
    tq, tk = (torch.as_tensor(x).to(cuda_device).requires_grad_(True) for x in (q, k))
    (sl, el), _ = compute_index_losses_b200(rope, tq, tk, blocks, cursor, editable_start=es)
    (sl + 2 * el).backward()
    np.testing.assert_allclose(sl.item(), g[f"start_loss_es{es}"], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(el.item(), g[f"end_loss_es{es}"], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(tq.grad.cpu().numpy(), g[f"dq_es{es}"], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(tk.grad.cpu().numpy(), g[f"dk_es{es}"], rtol=1e-4, atol=1e-4)


@pytest.mark.gpu
def test_bf16_index_losses_on_the_training_chain(cuda_device):
    """The +E chain (built by the reference's sampler), batch 2, head_dim
    128, theta 1e6; cursor targets drawn among each row's attended keys."""
    from autoindexer_b200 import compute_index_losses_b200, positions_from_operations
    from autoindexer_b200.index_head import index_rows

    with np.load(os.path.join(GOLDEN, "ops_cases.npz")) as z:
        ops = z["chain_e"]
    lay = positions_from_operations(ops)
    types = np.asarray([int(b.block_type) for b in lay])
    rng = np.random.default_rng(7)
    cursor = {}
    for blk, (s, e, ks, ke) in zip(lay, lay.boundary_indices):
        if int(blk.block_type) != 1:
            continue
        cursor[int(e) - 1] = (0, 0)
    probe = index_rows(lay, cursor)
    for r in range(0, probe.rows.shape[0], 2):
        picks = []
        for rr in (r, r + 1):
            _, _, n, off = probe.rows[rr]
            cand = np.flatnonzero(probe.ok[off:off + n])
            picks.append(int(rng.choice(cand)) if cand.size else 0)
        cursor[int(probe.edits[r])] = tuple(picks)
    B, T, D = 2, int(lay.boundary_indices[-1][1]), 128
    inv = O.default_inv_freq(D, 1e6)
    g = torch.Generator().manual_seed(5)
    q = torch.randn(B, 2, T, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, 2, T, D, generator=g).to(torch.bfloat16)
    tq, tk = (x.to(cuda_device).requires_grad_(True) for x in (q, k))
    (sl, el), w = compute_index_losses_b200(HFRope(inv).to(cuda_device), tq, tk, lay, cursor, return_weights=True)
    (sl + 2 * el).backward()
    edits = np.asarray([(e, s, t) for e, (s, t) in sorted(cursor.items())])
    osl, oel, odq, odk = O.index_losses(q.double().numpy(), k.double().numpy(), lay, types, edits,
                                        O.make_rope(inv), w_start=1.0, w_end=2.0)
    assert abs(sl.item() - osl) <= 1e-2 * abs(osl) + 1e-2
    assert abs(el.item() - oel) <= 1e-2 * abs(oel) + 1e-2
    assert rel_l2(tq.grad.double().cpu().numpy(), odq) <= 1e-2
    assert rel_l2(tk.grad.double().cpu().numpy(), odk) <= 1e-2
    # returned weights: the masked, scaled logits of the first edit's rows
    ed = min(cursor)
    ws, we = w[ed]
    assert ws.shape == (B, 1, 1, ed) and we.shape == (B, 1, 1, ed + 1)
    rows = O.index_rows(lay, types, edits)
    h, qi, rel, ok, _, _ = rows[0]
    cos, sin = O.make_rope(inv)(rel)
    kr = O.apply_cos_sin(k[:, 0, :rel.shape[0]].double().numpy(), cos, sin)
    want = np.einsum("bd,bnd->bn", q[:, 0, qi].double().numpy(), kr) * D ** -0.5
    got = ws.float().cpu().numpy()[:, 0, 0]
    fin = ok[None, :].repeat(B, 0)
    assert np.all(np.isneginf(got[~fin]))
    assert np.max(np.abs(got[fin] - want[fin])) <= 0.1


@pytest.mark.parametrize("case", [0, 3, 9, "chain_e"])
@pytest.mark.parametrize("es", [0, 3])
def test_native_index_rows_match_python_rows(case, es):
    """ai_index_rows (the rows compute_index_losses_b200 uploads) equals
    index_rows, the Python statement of the reference's per-edit loop: row
    table, edit markers, key flags and the keys' table rows (relative
    position minus the lowest attended one)."""
    import ctypes

    from autoindexer_b200 import _lib
    from autoindexer_b200.index_head import _Prepared, index_rows
    from autoindexer_b200.meta import _prep_list

    if case == "chain_e":
        from autoindexer_b200 import positions_from_operations

        with np.load(os.path.join(GOLDEN, "ops_cases.npz")) as z:
            blocks = positions_from_operations(z["chain_e"])
    else:
        _, blocks, _, _, _ = _golden_case(case)
    types = np.asarray([int(b.block_type or 0) for b in blocks], dtype=np.int32)
    pl, keep = _prep_list(blocks, 0)
    n_rows, n_keys = ctypes.c_int32(0), ctypes.c_int64(0)
    edits = np.zeros(len(types), dtype=np.int64)
    lib = _lib.lib()
    assert lib.ai_index_rows_sizes(ctypes.byref(pl), types.ctypes.data, ctypes.byref(n_rows), ctypes.byref(n_keys),
                                   edits.ctypes.data) == 0
    cursor = {int(e): (0, 1) for e in edits[:n_rows.value // 2]}
    want = index_rows(blocks, cursor, editable_start=es)
    assert n_rows.value == want.rows.shape[0] and n_keys.value == want.rel.shape[0]
    rows = np.zeros((n_rows.value, 4), dtype=np.int32)
    key_rows = np.zeros(n_keys.value, dtype=np.int32)
    key_ok = np.zeros(n_keys.value, dtype=np.uint8)
    lo, hi = _Prepared._native_fill(pl, types, es, rows, key_rows, key_ok)
    assert np.array_equal(rows, want.rows)
    assert np.array_equal(np.repeat(edits[:n_rows.value // 2], 2), want.edits)
    assert np.array_equal(key_ok, want.ok)
    ok = want.ok.astype(bool)
    assert lo == min(0, int(want.rel[ok].min())) and hi == max(0, int(want.rel[ok].max()))
    assert np.array_equal(key_rows[ok], (want.rel[ok] - lo).astype(np.int32))
