"""Parity of the CUDA kernels with the oracle at the sizes the benchmarks run.

Every case calls the kernels through the C ABI and compares with the
query-chunked oracle (``oracle.attn_chunked``, itself checked against the
dense oracle and the reference's golden vectors on the CPU):

* the +E edit chain: a CPT training step's layout built by the reference's
  own sampler (``tests/golden/chain_e.npz``, ``make_edit_chain_golden.py``):
  T = 3072, 71 blocks, abs keys, keys at block-dependent positions, keys
  seen by many blocks; bf16 at the specification's tolerances and fp32 at
  1e-4;
* one causal sequence of 8192 tokens with config 3's three RoPE sections
  (24 / 24 / 16 frequency slots: arange and two cursor streams): every row
  and every key, out, lse, dQ, dK and dV;
* fp32 at head_dim 128 on config 0's shape (B=2, T=1024, Hq=32, Hkv=8,
  two sections, causal), 1e-4;
* the exact layout ``bench.py`` times (``make_rows(0)``: config 1, B=4,
  T=4096, packed documents): every document of row 0 and the last document
  of rows 1-3, two KV groups.

Tolerances (specification): bf16 out / lse max-abs 2e-2 and relative L2
1e-2, dQ / dK / dV relative L2 1e-2; fp32 1e-4 absolute and relative.
"""

import os
import sys

import numpy as np
import pytest
import torch

from conftest import ROOT, ArrayLayout, HFRope, load_golden, rel_l2
from autoindexer_b200 import RowLayouts, SectionedRope, document_blocks
from autoindexer_b200.attention import attn_bwd, attn_fwd, read_status
from autoindexer_b200.meta import compile_layout
from autoindexer_b200.positions import cursor_stream
from oracle import attn_oracle as O

pytestmark = pytest.mark.gpu

BF16_ABS = 2e-2
BF16_REL = 1e-2
FP32_TOL = 1e-4


def _run(lay, q, k, v, dout, mod, dtype, device):
    """Forward + backward through the C ABI on host arrays; float64 results."""
    B, Hq, T, D = q.shape
    tq, tk, tv, tdo = (torch.as_tensor(x).to(device=device, dtype=dtype) for x in (q, k, v, dout))
    layout = compile_layout(lay, B, T, D, dtype, mod.to(device), device)
    out, lse = attn_fwd(tq, tk, tv, layout, D ** -0.5)
    dq, dk, dv = attn_bwd(tq, tk, tv, out, lse, tdo, layout, D ** -0.5)
    torch.cuda.synchronize(device)
    assert read_status(device) == 0
    return [t.double().cpu().numpy() for t in (out, lse, dq, dk, dv)]


def _bf16(*xs):
    return [torch.as_tensor(np.asarray(x)).to(torch.bfloat16).double().numpy() for x in xs]


def _check_bf16(got, want, label):
    names = ("out", "lse", "dq", "dk", "dv")
    for name, a, b in zip(names, got, want):
        fin = np.isfinite(b)
        assert np.array_equal(fin, np.isfinite(a)), f"{label} {name}: non-finite entries differ"
        a, b = a[fin], b[fin]
        if name in ("out", "lse"):
            assert np.max(np.abs(a - b)) <= BF16_ABS, f"{label} {name} max-abs {np.max(np.abs(a - b))}"
        if name != "lse":
            assert rel_l2(a, b) <= BF16_REL, f"{label} {name} rel-L2 {rel_l2(a, b)}"


def _check_fp32(got, want, label):
    for name, a, b in zip(("out", "lse", "dq", "dk", "dv"), got, want):
        np.testing.assert_allclose(a, b, rtol=FP32_TOL, atol=FP32_TOL, err_msg=f"{label}:{name}")


# ---------------------------------------------------------------- +E edit chain

def _chain_e(Hq, Hkv, D, seed):
    g = load_golden("chain_e")
    lay = ArrayLayout.from_golden(g)
    T = int(g["T_model"])
    rng = np.random.default_rng(seed)
    q, k, v = (rng.standard_normal(s) for s in ((1, Hq, T, D), (1, Hkv, T, D), (1, Hkv, T, D)))
    dout = rng.standard_normal((1, T, Hq, D))
    inv = O.default_inv_freq(D, float(g["theta"]))
    return lay, q, k, v, dout, HFRope(inv), O.make_rope(inv)


def test_bf16_edit_chain_e_matches_oracle(cuda_device):
    """T = 3072 CPT edit chain (abs keys, block-dependent key positions, the
    multi-block dK fold), one KV group of 4 query heads, head_dim 128."""
    lay, q, k, v, dout, mod, rope = _chain_e(4, 1, 128, 20)
    q, k, v, dout = _bf16(q, k, v, dout)
    got = _run(lay, q, k, v, dout, mod, torch.bfloat16, cuda_device)
    want = O.attn_chunked(q, k, v, dout, lay, rope, chunk=512)
    _check_bf16(got, want, "chain E bf16")


def test_fp32_edit_chain_e_matches_oracle(cuda_device):
    lay, q, k, v, dout, mod, rope = _chain_e(4, 1, 128, 21)
    q, k, v, dout = (x.astype(np.float32) for x in (q, k, v, dout))
    got = _run(lay, q, k, v, dout, mod, torch.float32, cuda_device)
    want = O.attn_chunked(q, k, v, dout, lay, rope, chunk=512)
    _check_fp32(got, want, "chain E fp32")


# ---------------------------------------------------------------- T = 8192, three sections

def test_bf16_causal_8192_three_sections_full(cuda_device):
    """Config 3's sections on one causal sequence of 8192 tokens: every row
    and every key of one KV group (4 query heads)."""
    T, Hq, Hkv, D = 8192, 4, 1, 128
    rng = np.random.default_rng(33)
    sections = [(0, 24), (24, 48), (48, 64)]
    streams = [np.arange(T), cursor_stream(T, rng), cursor_stream(T, rng)]
    mod = SectionedRope(D, 1e6, [torch.as_tensor(x) for x in streams], sections)
    rope = O.make_sectioned_rope(mod.inv_freq.numpy(), streams, sections)
    lay = document_blocks([T], position_ids=np.arange(T))
    q, k, v = (rng.standard_normal(s) for s in ((1, Hq, T, D), (1, Hkv, T, D), (1, Hkv, T, D)))
    dout = rng.standard_normal((1, T, Hq, D))
    q, k, v, dout = _bf16(q, k, v, dout)
    got = _run(lay, q, k, v, dout, mod, torch.bfloat16, cuda_device)
    want = O.attn_chunked(q, k, v, dout, lay, rope, chunk=1024)
    _check_bf16(got, want, "T=8192 3 sections")


# ---------------------------------------------------------------- fp32, head_dim 128, config 0

def test_fp32_config0_head_dim_128(cuda_device):
    """Config 0: B=2, T=1024, Hq=32, Hkv=8, head_dim 128, two sections of
    32 frequency slots (arange; a cursor stream), theta 1e6, causal; fp32
    kernels at 1e-4."""
    B, T, Hq, Hkv, D = 2, 1024, 32, 8, 128
    rng = np.random.default_rng(0)
    sections = [(0, 32), (32, 64)]
    streams = [np.arange(T), cursor_stream(T, rng)]
    mod = SectionedRope(D, 1e6, [torch.as_tensor(x) for x in streams], sections)
    rope = O.make_sectioned_rope(mod.inv_freq.numpy(), streams, sections)
    lay = document_blocks([T], position_ids=np.arange(T))
    q, k, v = (rng.standard_normal(s).astype(np.float32) for s in ((B, Hq, T, D), (B, Hkv, T, D), (B, Hkv, T, D)))
    dout = rng.standard_normal((B, T, Hq, D)).astype(np.float32)
    got = _run(lay, q, k, v, dout, mod, torch.float32, cuda_device)
    want = O.attn_chunked(q, k, v, dout, lay, rope, chunk=256)
    _check_fp32(got, want, "config 0 fp32")


# ---------------------------------------------------------------- the bench's own layout

def test_bf16_bench_layout_documents(cuda_device):
    """``bench.make_rows(0)`` and ``bench.make_workload``'s inputs, the whole
    config-1 batch on the kernels; checked: every document of row 0 and the
    last document of rows 1-3, KV groups 0 and 7 (query heads 0-3, 28-31).
    A document depends only on its own rows, so each is checked against the
    oracle run on that document alone."""
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    import bench

    rows, mod, streams, host = bench.make_workload(seed=0, device="cpu")
    q, k, v, dout = host
    B, Hq, T, D = q.shape
    got = _run(rows, q.float().numpy(), k.float().numpy(), v.float().numpy(), dout.float().numpy(), mod,
               torch.bfloat16, cuda_device)
    rope = O.make_sectioned_rope(mod.inv_freq.cpu().numpy(), streams, bench.SECTIONS)
    G = Hq // k.shape[1]
    checked = 0
    for b in range(B):
        bounds = rows[b].boundary_indices
        docs = range(len(bounds)) if b == 0 else [len(bounds) - 1]
        for di in docs:
            s, e = int(bounds[di][0]), int(bounds[di][1])
            for grp in (0, k.shape[1] - 1):
                hq = slice(grp * G, (grp + 1) * G)
                sub = document_blocks([e - s], position_ids=np.arange(s, e))
                qs = q[b:b + 1, hq, s:e].double().numpy()
                ks = k[b:b + 1, grp:grp + 1, s:e].double().numpy()
                vs = v[b:b + 1, grp:grp + 1, s:e].double().numpy()
                dos = dout[b:b + 1, s:e, hq].double().numpy()
                want = O.attn_chunked(qs, ks, vs, dos, sub, rope, chunk=512)
                sl = [got[0][b:b + 1, s:e, hq], got[1][b:b + 1, hq, s:e], got[2][b:b + 1, hq, s:e],
                      got[3][b:b + 1, grp:grp + 1, s:e], got[4][b:b + 1, grp:grp + 1, s:e]]
                _check_bf16(sl, want, f"bench row {b} doc {di} group {grp}")
                checked += 1
    assert checked >= 2 * (len(rows[0].boundary_indices) + 3)


def _dq_scratch_bytes(layout, Hq, D=128):
    """Backward workspace bytes of the abs split's dQ partials (they follow
    the split key tiles' partials)."""
    return (layout.n_fwd_abs_items * Hq * 128 * D * 4 + 255) // 256 * 256 if layout.n_fwd_abs_items else 0


def test_bf16_split_key_tiles_match_whole_key_tiles(cuda_device):
    """The +E chain's long key tiles are split into chunks of query tiles
    whose fp32 partial sums a second launch adds up (when the workspace holds
    them); without room for the partials every key tile runs whole.  Both
    give the same gradients up to the order of the fp32 sums."""
    import ctypes

    from autoindexer_b200 import _lib
    from autoindexer_b200.attention import _fwd_args, _t4

    lay, q, k, v, dout, mod, _ = _chain_e(8, 2, 128, 22)
    tq, tk, tv, tdo = (torch.as_tensor(x).to(cuda_device, torch.bfloat16) for x in (q, k, v, dout))
    B, Hq, T, D = tq.shape
    layout = compile_layout(lay, B, T, D, torch.bfloat16, mod.to(cuda_device), cuda_device)
    assert layout.n_kv_partials > 0
    out, lse, fws = attn_fwd(tq, tk, tv, layout, D ** -0.5, keep_workspace=True)
    lib = _lib.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    res = []
    for split in (True, False):
        grads = [torch.empty_like(x) for x in (tq, tk, tv)]
        a = _lib.AiAttnBwdArgs()
        a.fwd = _fwd_args(tq, tk, tv, out.permute(0, 2, 1, 3), lse, layout, D ** -0.5)
        a.dout = _t4(tdo.permute(0, 2, 1, 3))
        a.dq, a.dk, a.dv = (_t4(x) for x in grads)
        a.fwd.workspace, a.fwd.workspace_bytes, a.fwd_rotated = fws.data_ptr(), fws.numel(), 1
        nbytes = ctypes.c_size_t(0)
        assert lib.ai_attn_bwd_workspace(ctypes.byref(a), ctypes.byref(nbytes)) == 0
        delta_only = (B * Hq * T * 4 + 255) // 256 * 256
        # the abs splits' partials come after the split key tiles' ones: left out of both runs
        dq_part = _dq_scratch_bytes(layout, Hq, D)
        assert nbytes.value > delta_only + dq_part  # the dK/dV partials are asked for
        ws = torch.empty(nbytes.value - dq_part if split else delta_only, dtype=torch.uint8, device=cuda_device)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
        assert lib.ai_attn_bwd(ctypes.byref(a), stream) == 0
        torch.cuda.synchronize(cuda_device)
        assert read_status(cuda_device) == 0
        res.append([x.double().cpu().numpy() for x in grads])
    for name, a_, b_ in zip(("dq", "dk", "dv"), *res):
        assert rel_l2(a_, b_) <= 2e-3, (name, rel_l2(a_, b_))
    assert np.array_equal(res[0][0], res[1][0])  # dQ does not take part in the split


def test_bf16_rotation_classes_match_shared_memory_rotation(cuda_device):
    """The +E chain's blocks read their keys from the rotation-class copies
    (each distinct 64-key chunk rotated once); with the classes removed from
    the layout the same kernels rotate every K tile in shared memory.  The
    rotation arithmetic is the same, so out, lse, dQ and dV are equal bit for
    bit; dK differs by the order of its fp32 sums (with classes, consecutive
    blocks that rotate a key tile alike accumulate in TMEM and are folded
    once)."""
    import dataclasses

    lay, q, k, v, dout, mod, _ = _chain_e(8, 2, 128, 23)
    tq, tk, tv, tdo = (torch.as_tensor(x).to(cuda_device, torch.bfloat16) for x in (q, k, v, dout))
    B, Hq, T, D = tq.shape
    layout = compile_layout(lay, B, T, D, torch.bfloat16, mod.to(cuda_device), cuda_device)
    assert layout.rot_classes.shape[0] > 0
    none = dataclasses.replace(layout, chunk_cls=layout.chunk_cls[:0], rot_classes=layout.rot_classes[:0])
    res = []
    for lo in (layout, none):
        out, lse, fws = attn_fwd(tq, tk, tv, lo, D ** -0.5, keep_workspace=True)
        dq, dk, dv = attn_bwd(tq, tk, tv, out, lse, tdo, lo, D ** -0.5, fwd_workspace=fws)
        torch.cuda.synchronize(cuda_device)
        assert read_status(cuda_device) == 0
        res.append((out, lse, dq, dk, dv))
    for name, a_, b_ in zip(("out", "lse", "dq", "dv"), *(r[:3] + r[4:] for r in res)):
        assert torch.equal(a_, b_), name
    assert rel_l2(res[0][3].double().cpu().numpy(), res[1][3].double().cpu().numpy()) <= 2e-3


def test_bf16_abs_split_matches_whole_abs_items(cuda_device):
    """The abs split: the persistent kernels run the abs blocks' key tiles
    without abs keys and leave partial rows (forward: O / l and the log-sum;
    dQ: the rotated accumulator) that the one-head kernels finish with the
    tiles holding abs keys.  Without room for the partials in the
    workspaces the one-head kernels run those items whole.  Both agree to
    the rounding of the merge; the split one is also checked against the
    oracle by the +E parity tests."""
    import ctypes

    from autoindexer_b200 import _lib
    from autoindexer_b200.attention import _fwd_args, _t4

    lay, q, k, v, dout, mod, _ = _chain_e(8, 2, 128, 24)
    tq, tk, tv, tdo = (torch.as_tensor(x).to(cuda_device, torch.bfloat16) for x in (q, k, v, dout))
    B, Hq, T, D = tq.shape
    layout = compile_layout(lay, B, T, D, torch.bfloat16, mod.to(cuda_device), cuda_device)
    n_abs = layout.n_fwd_abs_items
    assert n_abs > 0
    fwd_part = (n_abs * Hq * 128 * (D + 1) * 4 + 255) // 256 * 256
    dq_part = _dq_scratch_bytes(layout, Hq, D)
    lib = _lib.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    res = []
    for split in (True, False):
        out = torch.empty((B, T, Hq, D), dtype=torch.bfloat16, device=cuda_device)
        lse = torch.empty((B, Hq, T), dtype=torch.float32, device=cuda_device)
        a = _fwd_args(tq, tk, tv, out.permute(0, 2, 1, 3), lse, layout, D ** -0.5)
        nbytes = ctypes.c_size_t(0)
        assert lib.ai_attn_fwd_workspace(ctypes.byref(a), ctypes.byref(nbytes)) == 0
        fws = torch.empty(nbytes.value, dtype=torch.uint8, device=cuda_device)
        a.workspace, a.workspace_bytes = fws.data_ptr(), nbytes.value - (0 if split else fwd_part)
        assert lib.ai_attn_fwd(ctypes.byref(a), stream) == 0
        grads = [torch.empty_like(x) for x in (tq, tk, tv)]
        b = _lib.AiAttnBwdArgs()
        b.fwd = a
        b.fwd_rotated = 1
        b.dout = _t4(tdo.permute(0, 2, 1, 3))
        b.dq, b.dk, b.dv = (_t4(x) for x in grads)
        assert lib.ai_attn_bwd_workspace(ctypes.byref(b), ctypes.byref(nbytes)) == 0
        ws = torch.empty(nbytes.value, dtype=torch.uint8, device=cuda_device)
        b.workspace, b.workspace_bytes = ws.data_ptr(), nbytes.value - (0 if split else dq_part)
        assert lib.ai_attn_bwd(ctypes.byref(b), stream) == 0
        torch.cuda.synchronize(cuda_device)
        assert read_status(cuda_device) == 0
        res.append([x.double().cpu().numpy() for x in (out, lse, *grads)])
    for name, a_, b_ in zip(("out", "lse", "dq", "dk", "dv"), *res):
        fin = np.isfinite(a_) & np.isfinite(b_)
        assert np.array_equal(np.isfinite(a_), np.isfinite(b_)), name
        assert rel_l2(a_[fin], b_[fin]) <= 5e-3, (name, rel_l2(a_[fin], b_[fin]))


def test_bf16_backward_in_two_parts_equals_one_call(cuda_device):
    """ai_attn_bwd with parts = dQ, then parts = dK/dV on the same
    arguments and workspace (what the sharded backward does to start the dQ
    all-gather early) gives the one-call gradients bit for bit, on the +E
    chain (abs split, split key tiles, rotation classes)."""
    lay, q, k, v, dout, mod, _ = _chain_e(8, 2, 128, 25)
    tq, tk, tv, tdo = (torch.as_tensor(x).to(cuda_device, torch.bfloat16) for x in (q, k, v, dout))
    B, Hq, T, D = tq.shape
    layout = compile_layout(lay, B, T, D, torch.bfloat16, mod.to(cuda_device), cuda_device)
    out, lse, fws = attn_fwd(tq, tk, tv, layout, D ** -0.5, keep_workspace=True)
    one = attn_bwd(tq, tk, tv, out, lse, tdo, layout, D ** -0.5, fwd_workspace=fws)
    seen = []
    two = attn_bwd(tq, tk, tv, out, lse, tdo, layout, D ** -0.5, fwd_workspace=fws, after_dq=lambda: seen.append(1))
    torch.cuda.synchronize(cuda_device)
    assert seen == [1] and read_status(cuda_device) == 0
    for name, a_, b_ in zip(("dq", "dk", "dv"), one, two):
        assert torch.equal(a_, b_), name
