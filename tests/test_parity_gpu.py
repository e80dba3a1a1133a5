"""Parity of the CUDA kernels (called through the C ABI) with the reference.

* fp32: against the golden fixtures the reference itself produced
  (``tests/golden``), tolerance 1e-4 (absolute and relative);
* bf16 (tcgen05 forward, head_dim 128): against the float64 oracle evaluated
  on the same bf16-rounded inputs, tolerances of the specification: output and
  lse max-abs 2e-2 and relative L2 1e-2, dQ/dK/dV relative L2 1e-2;
* full-size layouts: a causal prefix closed at a document boundary is
  independent of everything after it, so the kernels' results on that prefix
  of a full-size batch must match the oracle run on the prefix alone;
* determinism (no atomics anywhere: bitwise-equal reruns) and a clean device
  status word.
"""

import numpy as np
import pytest
import torch

from conftest import (ArrayLayout, HFRope, golden_inputs, golden_names, golden_rope, load_golden, max_rel, rel_l2)
from autoindexer_b200 import RowLayouts, SectionedRope, document_blocks
from autoindexer_b200.attention import attn_bwd, attn_fwd, read_status
from autoindexer_b200.meta import compile_layout
from autoindexer_b200.positions import cursor_stream, split_documents
from oracle import attn_oracle as O

pytestmark = pytest.mark.gpu

BF16_OUT_ABS = 2e-2
BF16_REL = 1e-2
FP32_TOL = 1e-4


def run_kernels(lay, q, k, v, dout, rope_mod, dtype, device, scale=None):
    """Forward + backward through the C ABI; numpy float64 results."""
    B, Hq, T, D = q.shape
    scale = D ** -0.5 if scale is None else scale
    tq, tk, tv = (torch.as_tensor(x).to(device=device, dtype=dtype) for x in (q, k, v))
    tdo = torch.as_tensor(dout).to(device=device, dtype=dtype)
    layout = compile_layout(lay, B, T, D, dtype, rope_mod.to(device), device)
    out, lse = attn_fwd(tq, tk, tv, layout, scale)
    dq, dk, dv = attn_bwd(tq, tk, tv, out, lse, tdo, layout, scale)
    torch.cuda.synchronize(device)
    assert read_status(device) == 0
    return [t.double().cpu().numpy() for t in (out, lse, dq, dk, dv)]


def bf16_round(*xs):
    return [torch.as_tensor(x).to(torch.bfloat16).double().numpy() for x in xs]


def check_bf16(got, want, label):
    out, lse, dq, dk, dv = got
    wo, wl, wdq, wdk, wdv = want
    assert np.max(np.abs(out - wo)) <= BF16_OUT_ABS, f"{label} out max-abs {np.max(np.abs(out - wo))}"
    assert rel_l2(out, wo) <= BF16_REL, f"{label} out rel-L2 {rel_l2(out, wo)}"
    assert np.max(np.abs(lse - wl)) <= BF16_OUT_ABS, f"{label} lse max-abs {np.max(np.abs(lse - wl))}"
    for name, a, b in (("dq", dq, wdq), ("dk", dk, wdk), ("dv", dv, wdv)):
        assert rel_l2(a, b) <= BF16_REL, f"{label} {name} rel-L2 {rel_l2(a, b)}"


# ---------------------------------------------------------------- fp32 vs golden

@pytest.mark.parametrize("name", golden_names())
def test_fp32_matches_reference_golden(name, cuda_device):
    g = load_golden(name)
    lay = ArrayLayout.from_golden(g)
    mod, _ = golden_rope(g, device=cuda_device)
    q, k, v, dout = golden_inputs(g)
    out, lse, dq, dk, dv = run_kernels(lay, q, k, v, dout, mod, torch.float32, cuda_device)
    for label, got, want in (("out", out, g["out"]), ("lse", lse, g["lse"]), ("dq", dq, g["dq"]),
                             ("dk", dk, g["dk"]), ("dv", dv, g["dv"])):
        np.testing.assert_allclose(got, want, rtol=FP32_TOL, atol=FP32_TOL, err_msg=f"{name}:{label}")


# ---------------------------------------------------------------- bf16 vs oracle

def _edit_chain_case(name, B, Hq, Hkv, D, seed):
    g = load_golden(name)
    lay = ArrayLayout.from_golden(g)
    T = int(g["T"])
    rng = np.random.default_rng(seed)
    q, k, v = (rng.standard_normal(s) for s in ((B, Hq, T, D), (B, Hkv, T, D), (B, Hkv, T, D)))
    dout = rng.standard_normal((B, T, Hq, D))
    inv = O.default_inv_freq(D, 1e4)
    return lay, q, k, v, dout, HFRope(inv), O.make_rope(inv)


@pytest.mark.parametrize("name,hq,hkv", [("op0_d32", 4, 2), ("op5_d32", 4, 2), ("op9_d32", 4, 2), ("op5_d32", 8, 2),
                                         ("op9_d32", 4, 1)])
def test_bf16_edit_chains_match_oracle(name, hq, hkv, cuda_device):
    """GQA groups of 1 query-head pair and of 2 pairs (one CTA per pair)."""
    lay, q, k, v, dout, mod, rope = _edit_chain_case(name, 2, hq, hkv, 128, 11)
    q, k, v, dout = bf16_round(q, k, v, dout)
    got = run_kernels(lay, q, k, v, dout, mod, torch.bfloat16, cuda_device)
    out, lse = O.attn_forward(q, k, v, lay, rope)
    want = [out, lse, *O.attn_backward(q, k, v, dout, lay, rope)]
    check_bf16(got, want, name)


def _sectioned_docs(B, T, D, n_sections, seed, lo=64, hi=300):
    rng = np.random.default_rng(seed)
    half = D // 2
    cuts = np.linspace(0, half, n_sections + 1).astype(int)
    sections = [(int(cuts[i]), int(cuts[i + 1])) for i in range(n_sections)]
    streams = [np.arange(T)] + [cursor_stream(T, rng) for _ in range(n_sections - 1)]
    rows = RowLayouts()
    for _ in range(B):
        lens = split_documents(T - int(rng.integers(0, 40)), lo, hi, rng)
        rows.append(document_blocks(lens, position_ids=np.arange(sum(lens))))
    mod = SectionedRope(D, 1e6, [torch.as_tensor(s) for s in streams], sections)
    rope = O.make_sectioned_rope(mod.inv_freq.numpy(), streams, sections)
    return rows, mod, rope


@pytest.mark.parametrize("n_sections", [1, 2, 3])
def test_bf16_sectioned_documents_match_oracle(n_sections, cuda_device):
    B, T, Hq, Hkv, D = 2, 520, 4, 1, 128
    rows, mod, rope = _sectioned_docs(B, T, D, n_sections, seed=n_sections)
    rng = np.random.default_rng(5)
    q, k, v = (rng.standard_normal(s) for s in ((B, Hq, T, D), (B, Hkv, T, D), (B, Hkv, T, D)))
    dout = rng.standard_normal((B, T, Hq, D))
    q, k, v, dout = bf16_round(q, k, v, dout)
    got = run_kernels(rows, q, k, v, dout, mod, torch.bfloat16, cuda_device)
    out, lse = O.attn_forward(q, k, v, list(rows), rope)
    want = [out, lse, *O.attn_backward(q, k, v, dout, list(rows), rope)]
    check_bf16(got, want, f"sections{n_sections}")


def test_fp32_sectioned_documents_match_oracle(cuda_device):
    B, T, Hq, Hkv, D = 2, 300, 4, 2, 64
    rows, mod, rope = _sectioned_docs(B, T, D, 2, seed=9, lo=40, hi=120)
    rng = np.random.default_rng(6)
    q, k, v = (rng.standard_normal(s).astype(np.float32) for s in ((B, Hq, T, D), (B, Hkv, T, D), (B, Hkv, T, D)))
    dout = rng.standard_normal((B, T, Hq, D)).astype(np.float32)
    got = run_kernels(rows, q, k, v, dout, mod, torch.float32, cuda_device)
    out, lse = O.attn_forward(q, k, v, list(rows), rope)
    want = [out, lse, *O.attn_backward(q, k, v, dout, list(rows), rope)]
    for label, a, b in zip(("out", "lse", "dq", "dk", "dv"), got, want):
        np.testing.assert_allclose(a, b, rtol=FP32_TOL, atol=FP32_TOL, err_msg=label)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_unowned_tail_rows(dtype, cuda_device):
    """Rows past the blocks' coverage: out = v, lse = 0, dV = sum of the
    group's dO, dQ = dK = 0 (reference.py:42-43 diagonal-only rows)."""
    lay, q, k, v, dout, mod, rope = _edit_chain_case("op3_d32", 1, 4, 2, 128 if dtype == torch.bfloat16 else 64, 3)
    T0 = q.shape[2]
    pad = 37
    rng = np.random.default_rng(8)
    q, k, v = (np.concatenate([x, rng.standard_normal(x.shape[:2] + (pad, x.shape[3]))], axis=2) for x in (q, k, v))
    dout = np.concatenate([dout, rng.standard_normal((1, pad) + dout.shape[2:])], axis=1)
    if dtype == torch.bfloat16:
        q, k, v, dout = bf16_round(q, k, v, dout)
    got = run_kernels(lay, q, k, v, dout, mod, dtype, cuda_device)
    out, lse = O.attn_forward(q, k, v, lay, rope)
    want = [out, lse, *O.attn_backward(q, k, v, dout, lay, rope)]
    tol = 1e-2 if dtype == torch.bfloat16 else FP32_TOL
    np.testing.assert_allclose(got[0][:, T0:], want[0][:, T0:], atol=tol, rtol=tol)
    np.testing.assert_allclose(got[1][:, :, T0:], 0.0, atol=1e-6)
    np.testing.assert_allclose(got[3][:, :, T0:], 0.0, atol=0)
    np.testing.assert_allclose(got[2][:, :, T0:], 0.0, atol=0)
    np.testing.assert_allclose(got[4][:, :, T0:], want[4][:, :, T0:], atol=tol, rtol=tol)


# ---------------------------------------------------------------- full size

def test_bf16_full_size_prefix_matches_oracle(cuda_device):
    """Config-1 shape (B=4, T=4096, Hq=32, Hkv=8, D=128, packed documents,
    2 sections): run the whole batch, then check the rows and keys of the
    documents inside the first ~1.2k tokens of row 0 against the oracle."""
    B, T, Hq, Hkv, D = 4, 4096, 32, 8, 128
    rows, mod, rope = _sectioned_docs(B, T, D, 2, seed=21, lo=256, hi=2048)
    rows[0] = document_blocks([700, 500] + split_documents(T - 1200, 256, 2048, np.random.default_rng(3)),
                              position_ids=np.arange(T))
    g = torch.Generator().manual_seed(0)
    q = torch.randn(B, Hq, T, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, T, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, T, D, generator=g).to(torch.bfloat16)
    dout = torch.randn(B, T, Hq, D, generator=g).to(torch.bfloat16)
    got = run_kernels(rows, q, k, v, dout, mod, torch.bfloat16, cuda_device)
    P = 1200
    qs, ks, vs = (x[:1, :, :P].double().numpy() for x in (q[:, :8], k[:, :2], v[:, :2]))
    dos = dout[:1, :P, :8].double().numpy()
    prefix = document_blocks([700, 500], position_ids=np.arange(P))
    out, lse = O.attn_forward(qs, ks, vs, prefix, rope)
    want = [out, lse, *O.attn_backward(qs, ks, vs, dos, prefix, rope)]
    sl = [got[0][:1, :P, :8], got[1][:1, :8, :P], got[2][:1, :8, :P], got[3][:1, :2, :P], got[4][:1, :2, :P]]
    check_bf16(sl, want, "full-size prefix")


def _full_size_run(rows, mod, B, T, Hq, Hkv, D, device, seed):
    """Seeded bf16 inputs on the device, forward + backward through the C ABI;
    returns the inputs and the outputs, all on the device."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, T, D, generator=g).to(torch.bfloat16).to(device)
    k = torch.randn(B, Hkv, T, D, generator=g).to(torch.bfloat16).to(device)
    v = torch.randn(B, Hkv, T, D, generator=g).to(torch.bfloat16).to(device)
    dout = torch.randn(B, T, Hq, D, generator=g).to(torch.bfloat16).to(device)
    layout = compile_layout(rows, B, T, D, torch.bfloat16, mod.to(device), device)
    out, lse = attn_fwd(q, k, v, layout, D ** -0.5)
    dq, dk, dv = attn_bwd(q, k, v, out, lse, dout, layout, D ** -0.5)
    torch.cuda.synchronize(device)
    assert read_status(device) == 0
    return (q, k, v, dout), (out, lse, dq, dk, dv)


def test_bf16_config4_varlen_prefix_matches_oracle(cuda_device):
    """Config-4 shape: 64 sequences of U[64, 2048] tokens rescaled to sum to
    65,536, packed in one row (Hq=32, Hkv=8, D=128, 2 RoPE sections).  A
    sequence depends on nothing outside itself, so the first two (made 500
    and 400 tokens long) are checked in full — out, lse, dQ, dK, dV — against
    the oracle."""
    T, Hq, Hkv, D, P = 65536, 32, 8, 128, 900
    rng = np.random.default_rng(4)
    raw = rng.integers(64, 2049, 62).astype(np.float64)
    lens = np.maximum(np.round(raw / raw.sum() * (T - P)).astype(int), 1)
    lens[-1] += (T - P) - lens.sum()
    lens = [500, 400] + [int(x) for x in lens]
    assert len(lens) == 64 and sum(lens) == T
    sections = [(0, 32), (32, 64)]
    streams = [np.arange(T), cursor_stream(T, rng)]
    mod = SectionedRope(D, 1e6, [torch.as_tensor(x) for x in streams], sections)
    rope = O.make_sectioned_rope(mod.inv_freq.numpy(), streams, sections)
    rows = RowLayouts()
    rows.append(document_blocks(lens, position_ids=np.arange(T)))
    (q, k, v, dout), got = _full_size_run(rows, mod, 1, T, Hq, Hkv, D, cuda_device, seed=4)
    qs, ks, vs = (x[:, :h, :P].double().cpu().numpy() for x, h in ((q, 8), (k, 2), (v, 2)))
    dos = dout[:, :P, :8].double().cpu().numpy()
    prefix = document_blocks([500, 400], position_ids=np.arange(P))
    out, lse = O.attn_forward(qs, ks, vs, prefix, rope)
    want = [out, lse, *O.attn_backward(qs, ks, vs, dos, prefix, rope)]
    o, l, dq, dk, dv = got
    sl = [t.double().cpu().numpy() for t in (o[:, :P, :8], l[:, :8, :P], dq[:, :8, :P], dk[:, :2, :P], dv[:, :2, :P])]
    check_bf16(sl, want, "config-4 prefix")


def test_bf16_config3_long_causal_prefix_matches_oracle(cuda_device):
    """Config-3 shape: one causal sequence of 32,768 tokens (Hq=32, Hkv=8,
    D=128) with three RoPE sections of 24 / 24 / 16 frequency slots (arange
    and two cursor streams).  Rows below 1,024 depend only on keys below
    1,024, so their output, lse and dQ are checked against the oracle on that
    prefix (dK / dV of those keys also take every later row)."""
    T, Hq, Hkv, D, P = 32768, 32, 8, 128, 1024
    rng = np.random.default_rng(3)
    sections = [(0, 24), (24, 48), (48, 64)]
    streams = [np.arange(T), cursor_stream(T, rng), cursor_stream(T, rng)]
    mod = SectionedRope(D, 1e6, [torch.as_tensor(x) for x in streams], sections)
    rope = O.make_sectioned_rope(mod.inv_freq.numpy(), streams, sections)
    rows = RowLayouts()
    rows.append(document_blocks([T], position_ids=np.arange(T)))
    (q, k, v, dout), got = _full_size_run(rows, mod, 1, T, Hq, Hkv, D, cuda_device, seed=3)
    qs, ks, vs = (x[:, :h, :P].double().cpu().numpy() for x, h in ((q, 8), (k, 2), (v, 2)))
    dos = dout[:, :P, :8].double().cpu().numpy()
    prefix = document_blocks([P], position_ids=np.arange(P))
    wo, wl = O.attn_forward(qs, ks, vs, prefix, rope)
    wdq, _, _ = O.attn_backward(qs, ks, vs, dos, prefix, rope)
    o, l, dq = (t.double().cpu().numpy() for t in (got[0][:, :P, :8], got[1][:, :8, :P], got[2][:, :8, :P]))
    assert np.max(np.abs(o - wo)) <= BF16_OUT_ABS, f"config-3 out max-abs {np.max(np.abs(o - wo))}"
    assert rel_l2(o, wo) <= BF16_REL
    assert np.max(np.abs(l - wl)) <= BF16_OUT_ABS, f"config-3 lse max-abs {np.max(np.abs(l - wl))}"
    assert rel_l2(dq, wdq) <= BF16_REL, f"config-3 dq rel-L2 {rel_l2(dq, wdq)}"


@pytest.mark.parametrize("layout_kind", ["documents", "edit_chain", "edit_chain_g4"])
def test_bf16_rotated_copies_match_in_kernel_rotation(layout_kind, cuda_device):
    """The fast path (Q and K rotated once into scratch, read by TMA) and the
    small-workspace path (every tile rotated in shared memory) agree."""
    if layout_kind == "documents":
        B, T, Hq, Hkv, D = 2, 700, 8, 2, 128
        rows, mod, _ = _sectioned_docs(B, T, D, 2, seed=31)
        lay = rows
        rng = np.random.default_rng(2)
        q, k, v = (rng.standard_normal(s) for s in ((B, Hq, T, D), (B, Hkv, T, D), (B, Hkv, T, D)))
        dout = rng.standard_normal((B, T, Hq, D))
    else:
        hq = 8 if layout_kind == "edit_chain_g4" else 4
        lay, q, k, v, dout, mod, _ = _edit_chain_case("op2_d32", 2, hq, 2, 128, 13)
        B, Hq, T, D = q.shape
    tq, tk, tv, tdo = (torch.as_tensor(x).to(cuda_device, torch.bfloat16) for x in (q, k, v, dout))
    layout = compile_layout(lay, B, T, D, torch.bfloat16, mod.to(cuda_device), cuda_device)
    res = []
    for copies in (True, False):
        out, lse = attn_fwd(tq, tk, tv, layout, D ** -0.5, rotated_copies=copies)
        grads = attn_bwd(tq, tk, tv, out, lse, tdo, layout, D ** -0.5, rotated_copies=copies)
        res.append([t.double().cpu().numpy() for t in (out, lse, *grads)])
    torch.cuda.synchronize(cuda_device)
    assert read_status(cuda_device) == 0
    for name, a_, b_ in zip(("out", "lse", "dq", "dk", "dv"), *res):
        assert rel_l2(a_, b_) <= 1e-3, (name, rel_l2(a_, b_))


@pytest.mark.parametrize("layout_kind", ["documents", "edit_chain"])
def test_bf16_backward_reuses_forward_rotation(layout_kind, cuda_device):
    """ai_attn_bwd with fwd_rotated = 1 (reading the rotated Q/K copies the
    forward left in its workspace) gives bit-identical gradients to a backward
    that rotates Q and K itself."""
    if layout_kind == "documents":
        B, T, Hq, Hkv, D = 2, 640, 8, 2, 128
        rows, mod, _ = _sectioned_docs(B, T, D, 2, seed=41)
        lay = rows
        rng = np.random.default_rng(3)
        q, k, v = (rng.standard_normal(s) for s in ((B, Hq, T, D), (B, Hkv, T, D), (B, Hkv, T, D)))
        dout = rng.standard_normal((B, T, Hq, D))
    else:
        lay, q, k, v, dout, mod, _ = _edit_chain_case("op7_d32", 2, 4, 2, 128, 17)
        B, Hq, T, D = q.shape
    tq, tk, tv, tdo = (torch.as_tensor(x).to(cuda_device, torch.bfloat16) for x in (q, k, v, dout))
    layout = compile_layout(lay, B, T, D, torch.bfloat16, mod.to(cuda_device), cuda_device)
    out, lse, ws = attn_fwd(tq, tk, tv, layout, D ** -0.5, keep_workspace=True)
    assert ws is not None
    reuse = attn_bwd(tq, tk, tv, out, lse, tdo, layout, D ** -0.5, fwd_workspace=ws)
    own = attn_bwd(tq, tk, tv, out, lse, tdo, layout, D ** -0.5)
    torch.cuda.synchronize(cuda_device)
    assert read_status(cuda_device) == 0
    for name, a_, b_ in zip(("dq", "dk", "dv"), reuse, own):
        assert torch.equal(a_, b_), name


def test_kernel_times_count_launches(cuda_device):
    """ai_attn_profile_*: one forward + backward on a documents layout records
    the rotation, forward, delta, dQ and dK/dV launches with positive times."""
    from autoindexer_b200.attention import KernelTimes

    B, T, Hq, Hkv, D = 2, 640, 8, 2, 128
    rows, mod, _ = _sectioned_docs(B, T, D, 2, seed=43)
    rng = np.random.default_rng(4)
    tq, tk, tv = (torch.as_tensor(rng.standard_normal(s)).to(cuda_device, torch.bfloat16)
                  for s in ((B, Hq, T, D), (B, Hkv, T, D), (B, Hkv, T, D)))
    tdo = torch.as_tensor(rng.standard_normal((B, T, Hq, D))).to(cuda_device, torch.bfloat16)
    layout = compile_layout(rows, B, T, D, torch.bfloat16, mod.to(cuda_device), cuda_device)
    with KernelTimes() as kt:
        out, lse, ws = attn_fwd(tq, tk, tv, layout, D ** -0.5, keep_workspace=True)
        attn_bwd(tq, tk, tv, out, lse, tdo, layout, D ** -0.5, fwd_workspace=ws)
    assert kt.launches["prerot"] == 1  # the backward reuses the forward's copies
    for kind in ("fwd", "delta", "dq", "dkdv"):
        assert kt.launches[kind] >= 1 and kt.ms[kind] > 0.0, kind
    # the fill launches run exactly when some row is diagonal-only
    fills = 0 if layout.all_rows_owned else 1
    assert kt.launches["fwd_fill"] == fills and kt.launches["bwd_fill"] == fills
    assert kt.launches["simt"] == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_deterministic_reruns(dtype, cuda_device):
    D = 128 if dtype == torch.bfloat16 else 64
    lay, q, k, v, dout, mod, _ = _edit_chain_case("op0_d32", 2, 4, 2, D, 4)
    a = run_kernels(lay, q, k, v, dout, mod, dtype, cuda_device)
    b = run_kernels(lay, q, k, v, dout, mod, dtype, cuda_device)
    for x, y in zip(a, b):
        assert np.array_equal(x, y)


def test_autograd_and_registry(cuda_device):
    """The registered transformers attention function (un-expanded GQA K/V)
    and the autograd path give the kernels' results."""
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    import autoindexer_b200 as ab

    ab.register_autoindexer_b200_attention()
    fn = ALL_ATTENTION_FUNCTIONS["autoindexer_b200"]
    lay, q, k, v, dout, mod, rope = _edit_chain_case("op1_d32", 2, 4, 2, 128, 12)
    tq, tk, tv = (torch.as_tensor(x).to(cuda_device, torch.bfloat16).requires_grad_(True) for x in (q, k, v))

    class M(torch.nn.Module):
        num_key_value_groups = 2

    out, w = fn(M(), tq, tk, tv, None, dropout=0.0, scaling=None, rotary_emb=mod.to(cuda_device), parsed_positions=lay)
    assert w is None and out.shape == (2, q.shape[2], 4, 128)
    out.backward(torch.as_tensor(dout).to(cuda_device, torch.bfloat16))
    ref = run_kernels(lay, *(x.detach().float().cpu().numpy() for x in (tq, tk, tv)), dout, mod, torch.bfloat16,
                      cuda_device)
    assert np.array_equal(out.detach().double().cpu().numpy(), ref[0])
    assert np.array_equal(tq.grad.double().cpu().numpy(), ref[2])
    with pytest.raises(NotImplementedError):
        fn(M(), tq, tk, tv, None, dropout=0.1, rotary_emb=mod, parsed_positions=lay)
