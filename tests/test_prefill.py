"""Prefill attention (``plain_causal_attn_b200``, the counterpart of the
reference's ``plain_causal_attn_sdpa``, ``attention/prefill_sdpa.py:11-71``).

CPU: the prefill layout (one block per row; a left-padding mask becomes the
block's first attended key, any other mask per-key flags) and, through the
chain-of-edits oracle run on that layout, the same results as the direct
restatement of the reference's SDPA prefill (``oracle.plain_causal_forward``)
on every row that attends a key.  GPU: the kernels through the public
function against that restatement (bf16 tolerances of the path), zeros on
padding rows, gradients against the oracle's, GQA, and the transformers
interface.
"""

import sys

import numpy as np
import pytest
import torch

from conftest import ROOT, HFRope, rel_l2

sys.path.insert(0, ROOT)

from autoindexer_b200 import compile_layout, prefill_layout  # noqa: E402
from autoindexer_b200.meta import BLOCKF_MASKED, BLOCKF_OWNPOS  # noqa: E402
from oracle import attn_oracle as O  # noqa: E402

D = 128


def _masks(B, T, kind):
    keep = np.ones((B, T), dtype=bool)
    if kind == "left":
        pads = [0, 37, T // 2][:B]
        for b, p in enumerate(pads):
            keep[b, :p] = False
    elif kind == "right":
        lens = [T, T - 29, T // 3][:B]
        for b, n in enumerate(lens):
            keep[b, n:] = False
    elif kind == "holes":
        rng = np.random.default_rng(5)
        keep = rng.random((B, T)) > 0.2
        keep[:, 0] = True
    return keep


def _mask_tensor(keep):
    return None if keep is None else torch.as_tensor(keep)[:, None, None, :]


def test_prefill_layout_blocks():
    B, T = 3, 200
    rope = HFRope(O.default_inv_freq(D, 1e6))
    left = _masks(B, T, "left")
    lay = compile_layout(prefill_layout(_mask_tensor(left), B, T), B, T, D, torch.bfloat16, rope, "cpu")
    blk = lay.host_blocks
    assert [tuple(r[:3]) for r in blk] == [(b, 0, T) for b in range(B)]
    assert list(blk[:, 4]) == [0, 37, T // 2]          # kv_lo = first real key
    assert all(int(f) & BLOCKF_OWNPOS and not int(f) & BLOCKF_MASKED for f in blk[:, 5])
    right = _masks(B, T, "right")
    lay = compile_layout(prefill_layout(_mask_tensor(right), B, T), B, T, D, torch.bfloat16, rope, "cpu")
    assert [bool(int(f) & BLOCKF_MASKED) for f in lay.host_blocks[:, 5]] == [False, True, True]
    # rows with the same mask share one block list; no mask: one list for all rows
    same = np.ones((2, T), dtype=bool)
    rows = prefill_layout(_mask_tensor(same), 2, T)
    assert rows[0] is rows[1]
    assert not isinstance(prefill_layout(None, 2, T), type(rows))
    with pytest.raises(ValueError):
        prefill_layout(torch.ones(2, T, dtype=torch.bool), 2, T)


@pytest.mark.parametrize("kind", ["none", "left", "right", "holes"])
def test_oracle_on_prefill_layout_equals_sdpa_restatement(kind):
    B, Hq, Hkv, T, Dh = 3, 4, 2, 48, 16
    rng = np.random.default_rng(11)
    q, k, v = (rng.standard_normal(s) for s in ((B, Hq, T, Dh), (B, Hkv, T, Dh), (B, Hkv, T, Dh)))
    keep = None if kind == "none" else _masks(B, T, kind)
    rope = O.make_rope(O.default_inv_freq(Dh, 1e4))
    want, want_lse = O.plain_causal_forward(q, k, v, keep, rope)
    rows = prefill_layout(_mask_tensor(keep), B, T)
    with np.errstate(invalid="ignore"):  # rows that attend nothing: NaN in the chain oracle, not compared
        got, got_lse = O.attn_forward(q, k, v, rows, rope)
    valid = np.ones((B, T), dtype=bool) if keep is None else np.cumsum(keep, axis=1) > 0
    for b in range(B):
        np.testing.assert_allclose(got[b][valid[b]], want[b][valid[b]], rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(got_lse[b][:, valid[b]], want_lse[b][:, valid[b]], rtol=1e-12, atol=1e-12)


# ---------------------------------------------------------------- GPU

def _gpu_case(B, Hq, Hkv, T, kind, seed, device):
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(B, h, T, D, generator=g).to(torch.bfloat16) for h in (Hq, Hkv, Hkv))
    keep = None if kind == "none" else _masks(B, T, kind)
    inv = O.default_inv_freq(D, 1e6)
    return q, k, v, keep, HFRope(inv).to(device), O.make_rope(inv)


@pytest.mark.gpu
@pytest.mark.parametrize("kind,hq,hkv", [("none", 4, 4), ("left", 4, 4), ("left", 8, 2), ("right", 4, 2),
                                         ("holes", 4, 4)])
def test_prefill_forward_matches_sdpa_restatement(kind, hq, hkv, cuda_device):
    from autoindexer_b200 import plain_causal_attn_b200, read_status

    B, T = 3, 333
    q, k, v, keep, mod, rope = _gpu_case(B, hq, hkv, T, kind, 3, cuda_device)
    out, none = plain_causal_attn_b200(mod, q.to(cuda_device), k.to(cuda_device), v.to(cuda_device),
                                       attention_mask=None if keep is None else _mask_tensor(keep).to(cuda_device))
    torch.cuda.synchronize(cuda_device)
    assert none is None and read_status(cuda_device) == 0
    assert out.shape == (B, T, hq, D)
    got = out.double().cpu().numpy()
    want, _ = O.plain_causal_forward(q.double().numpy(), k.double().numpy(), v.double().numpy(), keep, rope)
    valid = np.ones((B, T), dtype=bool) if keep is None else np.cumsum(keep, axis=1) > 0
    for b in range(B):
        assert np.max(np.abs(got[b][valid[b]] - want[b][valid[b]])) <= 2e-2, f"row {b}"
        assert rel_l2(got[b][valid[b]], want[b][valid[b]]) <= 1e-2, f"row {b}"
        assert np.all(got[b][~valid[b]] == 0.0)  # padding rows: zeros


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["none", "right"])
def test_prefill_gradients_match_oracle(kind, cuda_device):
    from autoindexer_b200 import plain_causal_attn_b200

    B, Hq, Hkv, T = 2, 4, 2, 260
    q, k, v, keep, mod, rope = _gpu_case(B, Hq, Hkv, T, kind, 4, cuda_device)
    dout = torch.randn(B, T, Hq, D, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16)
    xs = [x.to(cuda_device).requires_grad_(True) for x in (q, k, v)]
    out, _ = plain_causal_attn_b200(mod, *xs, attention_mask=None if keep is None else
                                    _mask_tensor(keep).to(cuda_device))
    out.backward(dout.to(cuda_device))
    rows = prefill_layout(_mask_tensor(keep), B, T)
    want = O.attn_backward(q.double().numpy(), k.double().numpy(), v.double().numpy(), dout.double().numpy(),
                           rows, rope)
    for name, x, w in zip(("dq", "dk", "dv"), xs, want):
        assert rel_l2(x.grad.double().cpu().numpy(), w) <= 1e-2, name


@pytest.mark.gpu
def test_prefill_transformers_interface(cuda_device):
    from autoindexer_b200 import plain_causal_attn_b200, prefill_attention_interface

    B, T = 2, 130
    q, k, v, keep, mod, _ = _gpu_case(B, 4, 2, T, "left", 6, cuda_device)
    args = [x.to(cuda_device) for x in (q, k, v)]
    m = _mask_tensor(keep).to(cuda_device)
    a, _ = prefill_attention_interface(None, *args, m, rotary_emb=mod)
    b, _ = plain_causal_attn_b200(mod, *args, attention_mask=m)
    assert torch.equal(a, b)
    with pytest.raises(NotImplementedError):
        prefill_attention_interface(None, *args, m, dropout=0.1, rotary_emb=mod)
