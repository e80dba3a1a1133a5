"""Layout compiler (``autoindexer_b200.meta``): the device tables the kernels
read, built on the CPU from reference-format position-block lists."""

import os

import numpy as np
import pytest
import torch

from conftest import ArrayLayout, golden_names, golden_rope, load_golden
from autoindexer_b200 import RowLayouts, document_blocks
from autoindexer_b200.meta import compile_layout
from oracle import attn_oracle as O

KEY_ATTN, KEY_ABS = 1 << 30, 1 << 31


def _compile(lay, B, T, D, dtype, rope_mod):
    return compile_layout(lay, B, T, D, dtype, rope_mod, "cpu")


@pytest.mark.parametrize("name", golden_names())
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_tables_match_layout(name, dtype):
    g = load_golden(name)
    lay = ArrayLayout.from_golden(g)
    mod, rope = golden_rope(g)
    T, D = int(g["T"]), int(g["D"])
    c = _compile(lay, 2, T + 5, D, dtype, mod)
    blocks = c.blocks.numpy()
    info = c.key_info.numpy().view(np.uint32)
    bounds = np.asarray(lay.boundary_indices)
    assert blocks.shape[0] == 2 * bounds.shape[0]
    am = lay.concat_attn_masks.numpy()
    ab = lay.concat_abs_pos_masks.numpy()
    kp = lay.concat_key_pos_ids.numpy()
    for bi, (row, s, e, koff, kv_lo, flags, _, _) in enumerate(blocks):
        S, E, KS, KE = bounds[bi % bounds.shape[0]]
        assert (row, s, e, koff) == (bi // bounds.shape[0], S, E, KS)
        m = am[KS:KE]
        assert kv_lo == (np.flatnonzero(m)[0] if m.any() else E)
        assert bool(flags & 2) == bool((ab[KS:KE] & m).any())
        assert bool(flags & 1) == bool(m.any() and not m[kv_lo:].all())
        word = info[KS:KE]
        assert np.array_equal((word & KEY_ATTN) != 0, m)
        assert np.array_equal((word & KEY_ABS) != 0, ab[KS:KE] & m)
        rows = (word & ((1 << 30) - 1)).astype(np.int64)
        assert np.array_equal(rows[m] + c.p_min, kp[KS:KE][m])
    # the table reproduces the rotary module at every used position
    cos_ref, sin_ref = rope(np.arange(c.p_min, c.p_min + c.n_pos))
    np.testing.assert_allclose(c.rope_cos.numpy(), cos_ref[:, : D // 2], atol=1e-6)
    np.testing.assert_allclose(c.rope_sin.numpy(), sin_ref[:, : D // 2], atol=1e-6)
    # query rows: owned rows carry their position, the padding carries position 0
    qp = c.q_pos.numpy()[0] + c.p_min
    assert np.array_equal(qp[:T], lay.query_pos_ids.numpy())
    assert np.all(qp[T:] == 0)
    assert c.pairs_per_head == 2 * O.count_pairs(lay, T)
    # abs items lead the forward work list, then the short items (at most
    # half a tile of rows), then the rest
    items = c.fwd_items.numpy()
    is_abs = (blocks[items[:, 0], 5] & 2) != 0
    assert is_abs.sum() == c.n_fwd_abs_items and is_abs[:c.n_fwd_abs_items].all()
    rest = items[c.n_fwd_abs_items:]
    short = (rest[:, 2] - rest[:, 1]) <= c.fwd_tile // 2
    assert short.sum() == c.n_fwd_short_items and short[:c.n_fwd_short_items].all()
    # abs-key ranges: [abs_lo, abs_hi) is the span of the block's abs keys
    for (s_, e_, KS, KE), blk in zip(lay.boundary_indices, blocks):
        a_ = ab[KS:KE] & am[KS:KE]
        if a_.any():
            nz = np.flatnonzero(a_)
            assert (blk[6], blk[7]) == (nz[0], nz[-1] + 1)
        else:
            assert (blk[6], blk[7]) == (0, 0)
    # key tiles holding an abs key of some block lead the dK/dV work list
    kv = c.kv_items.numpy()
    hold = [any(b_[5] & 2 and b_[6] < j1 and b_[7] > j0 and b_[2] > j0 for b_ in blocks) for _, j0, j1, _ in kv]
    assert sum(hold) == c.n_kv_abs_items and all(hold[:c.n_kv_abs_items])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_work_items_cover_rows_and_keys_once(dtype):
    rng = np.random.default_rng(0)
    lens_a, lens_b = [300, 77, 190], [128, 128, 311]
    rows = RowLayouts([document_blocks(lens_a), document_blocks(lens_b)])
    T = 600
    mod, _ = golden_rope(load_golden("op0_d32"))
    D = 32
    c = _compile(rows, 2, T, D, dtype, mod)
    blocks = c.blocks.numpy()
    seen = np.zeros((2, T), dtype=np.int64)
    for bi, q0, q1, _ in c.fwd_items.numpy():
        row, s, e = blocks[bi, :3]
        assert s <= q0 < q1 <= e and q1 - q0 <= c.fwd_tile
        seen[row, q0:q1] += 1
    assert np.all(seen[0, :sum(lens_a)] == 1) and np.all(seen[0, sum(lens_a):] == 0)
    assert np.all(seen[1, :sum(lens_b)] == 1) and np.all(seen[1, sum(lens_b):] == 0)
    keys = np.zeros((2, T), dtype=np.int64)
    for row, j0, j1, _ in c.kv_items.numpy():
        assert j1 - j0 <= c.kv_tile
        keys[row, j0:j1] += 1
    assert np.all(keys[0, :sum(lens_a)] == 1) and np.all(keys[1, :sum(lens_b)] == 1)
    assert list(c.row_cov.numpy()) == [sum(lens_a), sum(lens_b)]
    # documents: each block attends from its own first row on
    for row, s, e, koff, kv_lo, flags, _, _ in blocks:
        # no masked keys, no abs keys, every key at its own-block position
        assert kv_lo == s and flags == 4
    own = c.k_own.numpy()
    assert np.array_equal(own[0, :sum(lens_a)] + c.p_min,
                          np.concatenate([np.arange(n) for n in lens_a]))


def test_layout_rejects_malformed_lists():
    g = load_golden("op1_d32")
    mod, _ = golden_rope(g)
    lay = ArrayLayout.from_golden(g)
    bad = ArrayLayout(np.asarray(lay.boundary_indices)[1:], lay.query_pos_ids, lay.concat_key_pos_ids,
                      lay.concat_attn_masks, lay.concat_abs_pos_masks)
    with pytest.raises(ValueError):
        _compile(bad, 1, int(g["T"]), 32, torch.float32, mod)
    with pytest.raises(ValueError):
        _compile(lay, 1, int(g["T"]) - 1, 32, torch.float32, mod)


def test_layout_cache_is_reused():
    g = load_golden("op2_d32")
    mod, _ = golden_rope(g)
    lay = ArrayLayout.from_golden(g)
    a = _compile(lay, 1, int(g["T"]), 32, torch.float32, mod)
    b = _compile(lay, 1, int(g["T"]), 32, torch.float32, mod)
    assert a is b


def test_all_rows_owned_flag():
    """The layout tells the library when no row is diagonal-only, so the fill
    launches are skipped; rows past the blocks' coverage keep them."""
    g = load_golden("op2_d32")
    mod, _ = golden_rope(g)
    T = int(g["T"])
    padded = _compile(ArrayLayout.from_golden(g), 1, T + 5, 32, torch.float32, mod)
    assert not padded.all_rows_owned and padded.c_struct().all_rows_owned == 0
    rows = RowLayouts()
    rows.append(document_blocks([T // 2, T - T // 2], position_ids=np.arange(T)))
    docs = _compile(rows, 1, T, 32, torch.float32, mod)
    assert docs.all_rows_owned and docs.c_struct().all_rows_owned == 1


def test_external_mask_check():
    """An external 4-D mask is accepted when it removes nothing inside the
    causal triangle (bool or additive), rejected otherwise, and rechecked
    after an in-place change."""
    from autoindexer_b200.attention import _check_mask_is_causal

    T = 260
    tri = torch.tril(torch.ones(T, T, dtype=torch.bool))
    m = tri[None, None].expand(2, 1, T, T)
    _check_mask_is_causal(m, T)
    _check_mask_is_causal(m, T)  # cached for this tensor and version
    f = torch.zeros(2, 1, T, T).masked_fill_(~tri, float("-inf"))
    _check_mask_is_causal(f, T)
    f[1, 0, 200, 150] = float("-inf")  # in place: a new version, checked again
    with pytest.raises(NotImplementedError):
        _check_mask_is_causal(f, T)
    b = tri[None, None].repeat(1, 1, 1, 1)
    b[0, 0, 7, 3] = False
    with pytest.raises(NotImplementedError):
        _check_mask_is_causal(b, T)
    with pytest.raises(NotImplementedError):
        _check_mask_is_causal(torch.ones(1, 1, T, T + 1, dtype=torch.bool), T)


def test_blocks_from_concat_inverts_concat():
    """Rebuilding a list from the concat()-ed arrays of the +E chain (built by
    the reference's own sampler) gives the same arrays back."""
    from autoindexer_b200 import blocks_from_concat

    g = load_golden("chain_e")
    lay = blocks_from_concat(g["boundary_indices"], g["query_pos_ids"], g["concat_key_pos_ids"],
                             g["concat_attn_masks"], g["concat_abs_pos_masks"])
    assert np.array_equal(np.asarray(lay.boundary_indices), g["boundary_indices"])
    assert np.array_equal(lay.query_pos_ids.numpy(), g["query_pos_ids"])
    assert np.array_equal(lay.concat_key_pos_ids.numpy(), g["concat_key_pos_ids"])
    assert np.array_equal(lay.concat_attn_masks.numpy(), g["concat_attn_masks"])
    assert np.array_equal(lay.concat_abs_pos_masks.numpy(), g["concat_abs_pos_masks"])


@pytest.mark.parametrize("case", [f"op{i}" for i in range(10)] + ["chain_e"])
def test_positions_from_operations_match_reference(case):
    """The native edit-chain builder reproduces the layouts the reference's
    get_parsed_positions_from_perturbations built from the same operations
    (the ten operation_tuples.json cases and the +E chain)."""
    from conftest import GOLDEN
    from autoindexer_b200 import positions_from_operations

    with np.load(os.path.join(GOLDEN, "ops_cases.npz")) as z:
        ops = z[case]
    g = load_golden(case if case == "chain_e" else f"{case}_d32")
    lay = positions_from_operations(ops)
    assert np.array_equal(np.asarray(lay.boundary_indices), g["boundary_indices"])
    assert np.array_equal(lay.query_pos_ids.numpy(), g["query_pos_ids"])
    assert np.array_equal(lay.concat_key_pos_ids.numpy(), g["concat_key_pos_ids"])
    assert np.array_equal(lay.concat_attn_masks.numpy(), g["concat_attn_masks"])
    assert np.array_equal(lay.concat_abs_pos_masks.numpy(), g["concat_abs_pos_masks"])


def test_positions_from_operations_rejects_invalid_chains():
    from autoindexer_b200 import positions_from_operations

    with pytest.raises(RuntimeError):
        positions_from_operations([(3, 0, 0, 0, 5)])  # an edit cannot open the sequence
    with pytest.raises(RuntimeError):
        positions_from_operations([(0, 0, 0, 0, 5), (1, 1, 4, 9, 0)])  # cursor range past the text


@pytest.mark.parametrize("which", ["golden", "bench1", "benchE", "bench4"])
def test_native_tables_match_numpy_restatement(which):
    """ai_attn_prep (the native builder behind compile_layout) gives the
    tables of the numpy restatement in tests/layout_numpy.py, on every golden
    layout (shared by two rows) and on the benchmark layouts."""
    import layout_numpy as LN

    if which == "golden":
        cases = []
        for name in golden_names():
            g = load_golden(name)
            cases.append((ArrayLayout.from_golden(g), 2, int(g["T"]) + 5, golden_rope(g)[0], int(g["D"])))
    else:
        import bench

        wl = bench.build_workload(which[5:], 0, "cpu")
        cases = [(wl.rows, wl.batch, wl.seq_len, wl.rope, 128)]
    for lay, B, T, mod, D in cases:
        c = compile_layout(lay, B, T, D, torch.bfloat16, mod, "cpu")
        want = LN.host_tables(lay, B, T, c.fwd_tile, c.kv_tile)
        for name in ("blocks", "row_blocks", "row_cov", "key_info", "q_pos", "k_own", "fwd_items", "kv_items"):
            assert np.array_equal(getattr(c, name).numpy(), np.asarray(want[name]).reshape(getattr(c, name).shape)), name
        for name in ("n_fwd_abs_items", "n_kv_abs_items", "n_fwd_short_items", "n_fwd_abs_short_items",
                     "pairs_per_head", "all_rows_owned",
                     "p_min", "n_pos"):
            assert getattr(c, name) == want[name], name


@pytest.mark.parametrize("which", ["bench1", "benchE", "bench2a"])
def test_kv_chunks_partition_each_key_tile(which):
    """dK/dV chunks: the query tiles of every key tile (64-row tiles of the
    blocks that see it, blocks with an abs key among its keys left out) are
    covered once, in order; split tiles own consecutive partial slots listed
    in kv_reduce; the costs are query tiles plus two per block."""
    import bench

    wl = bench.build_workload(which[5:], 0, "cpu")
    c = compile_layout(wl.rows, wl.batch, wl.seq_len, 128, torch.bfloat16, wl.rope, "cpu")
    blocks, kv, ch, red = (x.numpy() for x in (c.blocks, c.kv_items, c.kv_chunks, c.kv_reduce))
    row_blocks = c.row_blocks.numpy()
    any_abs = c.n_kv_abs_items > 0
    cost_max = cost_total = 0
    by_item = {}
    for item, q0, q1, slot in ch:
        by_item.setdefault(int(item), []).append((int(q0), int(q1), int(slot)))
    assert sorted(by_item) == list(range(kv.shape[0]))
    reduce_of = {int(r[0]): (int(r[1]), int(r[2])) for r in red}
    for k, (row, j0, j1, _) in enumerate(kv):
        nq, cost = 0, 0
        for bi in range(row_blocks[row], row_blocks[row + 1]):
            _, s, e, _, kv_lo, flags, alo, ahi = blocks[bi]
            if not (e > j0 and kv_lo < j1 and max(s, j0) < e):
                continue
            if any_abs and flags & 2 and (ahi <= alo or (j0 < ahi and alo < j1)):
                continue
            n = (e - max(s, j0) + 63) // 64
            nq += n
            cost += n + 2
        cost_max, cost_total = max(cost_max, cost), cost_total + cost
        parts = sorted(by_item[k])
        assert parts[0][0] == 0 and parts[-1][1] == nq
        assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
        if len(parts) == 1:
            assert parts[0][2] == -1 and k not in reduce_of
        else:
            first, n = reduce_of[k]
            assert n == len(parts) and [p[2] for p in parts] == list(range(first, first + n))
    assert c.kv_cost_max == cost_max and c.kv_cost_total == cost_total
    assert c.n_kv_partials == sum(n for _, n in reduce_of.values())


def _class_cases():
    import bench

    out = []
    for which in ("E", "1"):
        wl = bench.build_workload(which, 0, "cpu")
        out.append((wl.rows, wl.batch, wl.seq_len, wl.rope, 128))
    # the golden edit chains shared by two batch rows: classes are per row
    for name in golden_names()[:4]:
        g = load_golden(name)
        out.append((ArrayLayout.from_golden(g), 2, int(g["T"]) + 5, golden_rope(g)[0], int(g["D"])))
    return out


@pytest.mark.parametrize("case", range(6))
def test_rotation_classes_describe_each_chunk(case):
    """Rotation classes: every 64-key chunk of a block without own positions
    (kv_lo on a chunk boundary) has a class whose defining chunk (same batch
    row, same first key) gives each key the same attended / past-the-end
    state and every attended key the same rotary table row; padding chunks of
    the last 128-key tile repeat the last real chunk's class; no two classes
    describe the same chunk; own-position blocks have none."""
    lay, B, T, rope, D = _class_cases()[case]
    c = compile_layout(lay, B, T, D, torch.bfloat16, rope, "cpu")
    blocks, info = c.blocks.numpy(), c.key_info.numpy().view(np.uint32)
    blk_cls, chunk_cls, rc = c.blk_cls.numpy(), c.chunk_cls.numpy(), c.rot_classes.numpy()
    assert blk_cls.shape == (blocks.shape[0],)

    def describe(bi, k0):
        row, s, e, off, kv_lo = (int(x) for x in blocks[bi][:5])
        d = [row, k0]
        for j in range(k0, k0 + 64):
            if j >= e:
                d.append(-1)
            elif info[off + j] & 0x40000000:
                d.append(int(info[off + j] & 0x3FFFFFFF))
            else:
                d.append(-2)
        return tuple(d)

    descs = [describe(int(bi), int(k0)) for bi, k0 in rc]
    assert len(set(descs)) == len(descs)
    for bi, (row, s, e, off, kv_lo, flags, _, _) in enumerate(blocks):
        if (flags & 4) or kv_lo >= e or kv_lo % 64:
            assert blk_cls[bi] == -1
            continue
        if blk_cls[bi] < 0:
            continue  # over the class cap (not reached here)
        n = 2 * ((e - kv_lo + 127) // 128)
        ent = chunk_cls[blk_cls[bi]:blk_cls[bi] + n]
        assert ent.shape[0] == n
        for i in range(n):
            k0 = kv_lo + 64 * i
            if k0 >= e:
                assert ent[i] == ent[i - 1]
                continue
            assert descs[ent[i]] == describe(bi, k0)
    if c.rot_classes.shape[0]:
        assert chunk_cls.max() == c.rot_classes.shape[0] - 1
