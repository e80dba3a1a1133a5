"""Decode step (``autoindexer_b200.decode``, C ABI ``ai_attn_decode``): the
IterPositions branch of the reference's interface (``attention/__init__.py:
36-51``, ``attn_layers.py:15-27``).

CPU: the oracle restatement (``oracle.decode_forward``) against the golden
vectors the reference's own decode branch wrote (``tests/golden/
decode_iter.npz``, ``make_decode_golden.py``).  GPU: the kernels against the
oracle (bf16 tolerances of the path) for shared and per-row key positions,
masks, GQA groups of 1-8, caches split over many CTAs; all-masked rows give
zeros; the transformers interface routes a decode step to the kernels.
"""

import os
import sys
from dataclasses import dataclass
from typing import Optional

import numpy as np
import pytest
import torch

from conftest import ROOT, HFRope, rel_l2

sys.path.insert(0, ROOT)

from oracle import attn_oracle as O  # noqa: E402

GOLDEN = os.path.join(ROOT, "tests", "golden", "decode_iter.npz")


def test_oracle_matches_reference_decode_golden():
    g = np.load(GOLDEN)
    rope = O.make_rope(g["inv_freq"])
    out = O.decode_forward(g["q"], g["k"], g["v"], g["key_pos"], g["attn_mask"], rope)
    np.testing.assert_allclose(out, g["out"], rtol=1e-10, atol=1e-10)


@dataclass
class Iter:
    """The fields of the reference's ``IterPositions`` that attention reads."""
    key_pos_ids: torch.Tensor
    attn_mask: Optional[torch.Tensor] = None

    def get_rotary_pos_emb(self, rotary_emb, x):
        kp = self.key_pos_ids.unsqueeze(0) if self.key_pos_ids.ndim == 1 else self.key_pos_ids
        return rotary_emb(x, kp)


def _case(B, Hq, Hkv, L, per_row, masked, seed, device):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, 1, 128, generator=g).to(torch.bfloat16)
    k, v = (torch.randn(B, Hkv, L, 128, generator=g).to(torch.bfloat16) for _ in range(2))
    rng = np.random.default_rng(seed)
    kp = (np.stack([np.arange(L) - (L - 1) - 3 * b for b in range(B)]) if per_row else np.arange(L) - (L - 1))
    am = None
    if masked:
        am = rng.random((B, L) if per_row else (L,)) > 0.3
        am[..., -1] = True
    inv = O.default_inv_freq(128, 1e6)
    pp = Iter(torch.as_tensor(kp).to(device), None if am is None else torch.as_tensor(am).to(device))
    return q, k, v, kp, am, pp, HFRope(inv).to(device), O.make_rope(inv)


@pytest.mark.gpu
@pytest.mark.parametrize("B,Hq,Hkv,L,per_row,masked", [
    (2, 4, 4, 300, False, False), (3, 8, 2, 1000, True, True), (1, 8, 1, 5000, False, True),
    (4, 32, 8, 2049, True, False), (2, 16, 2, 257, False, True)])
def test_decode_matches_oracle(B, Hq, Hkv, L, per_row, masked, cuda_device):
    from autoindexer_b200 import decode_attention, read_status

    q, k, v, kp, am, pp, mod, rope = _case(B, Hq, Hkv, L, per_row, masked, 7, cuda_device)
    out = decode_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), pp, mod)
    torch.cuda.synchronize(cuda_device)
    assert read_status(cuda_device) == 0
    got = out.double().cpu().numpy()
    want = O.decode_forward(q.double().numpy(), k.double().numpy(), v.double().numpy(), kp, am, rope)
    assert np.max(np.abs(got - want)) <= 2e-2
    assert rel_l2(got, want) <= 1e-2


@pytest.mark.gpu
def test_decode_unaligned_cache_matches_oracle(cuda_device):
    """A V cache that is 8- but not 16-byte aligned cannot be read by TMA:
    the register-streaming split kernel runs it; both kernels match the
    oracle (the aligned case takes the TMA kernel)."""
    from autoindexer_b200 import decode_attention, read_status

    B, Hq, Hkv, L = 2, 8, 2, 777
    q, k, v, kp, am, pp, mod, rope = _case(B, Hq, Hkv, L, True, True, 11, cuda_device)
    want = O.decode_forward(q.double().numpy(), k.double().numpy(), v.double().numpy(), kp, am, rope)
    wide = torch.zeros(B, Hkv, L, 136, dtype=torch.bfloat16)
    wide[..., 4:132] = v
    v_odd = wide.to(cuda_device)[..., 4:132]  # base 8 bytes past a 16-byte boundary
    assert v_odd.data_ptr() % 16 == 8
    outs = [decode_attention(q.to(cuda_device), k.to(cuda_device), vv, pp, mod) for vv in (v.to(cuda_device), v_odd)]
    torch.cuda.synchronize(cuda_device)
    assert read_status(cuda_device) == 0
    for out in outs:
        got = out.double().cpu().numpy()
        assert np.max(np.abs(got - want)) <= 2e-2
        assert rel_l2(got, want) <= 1e-2


@pytest.mark.gpu
def test_decode_all_masked_row_is_zero(cuda_device):
    from autoindexer_b200 import decode_attention

    B, L = 2, 600
    q, k, v, kp, _, _, mod, rope = _case(B, 4, 2, L, True, False, 3, cuda_device)
    am = np.ones((B, L), dtype=bool)
    am[1] = False
    pp = Iter(torch.as_tensor(kp).to(cuda_device), torch.as_tensor(am).to(cuda_device))
    out = decode_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), pp, mod).double().cpu()
    assert torch.all(out[1] == 0)
    want = O.decode_forward(q[:1].double().numpy(), k[:1].double().numpy(), v[:1].double().numpy(), kp[:1],
                            am[:1], rope)
    assert rel_l2(out[:1].numpy(), want) <= 1e-2


@pytest.mark.gpu
def test_interface_routes_decode_to_kernels(cuda_device):
    from autoindexer_b200 import attention_interface

    B, Hq, Hkv, L = 2, 8, 2, 700
    q, k, v, kp, am, pp, mod, rope = _case(B, Hq, Hkv, L, False, True, 5, cuda_device)
    hf_mask = torch.ones(B, 1, 1, L, dtype=torch.bool)
    hf_mask[0, ..., :100] = False
    out, w = attention_interface(None, q.to(cuda_device), k.to(cuda_device), v.to(cuda_device),
                                 hf_mask.to(cuda_device), scaling=0.1, rotary_emb=mod, parsed_positions=pp)
    assert w is None and out.shape == (B, Hq, 1, 128)
    want = O.decode_forward(q.double().numpy(), k.double().numpy(), v.double().numpy(), kp, am, rope, scale=0.1,
                            attention_mask=hf_mask.numpy())
    assert rel_l2(out.double().cpu().numpy(), want) <= 1e-2
