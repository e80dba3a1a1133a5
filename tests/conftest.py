"""Shared test helpers.

``-m "not gpu"`` runs the oracle-vs-golden checks, the layout compiler and
the C-ABI surface on the CPU; ``-m gpu`` runs the CUDA kernels through the C
ABI against the oracle and the golden fixtures.
"""

import os
import sys

import numpy as np
import pytest
import torch
from torch import nn

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, GOLDEN):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100) device")


def golden_names():
    """The chain-of-edits golden cases (not the known-answer tables or the
    decode-step vectors)."""
    return sorted(f[:-4] for f in os.listdir(GOLDEN)
                  if f.endswith(".npz") and not f.startswith(("kat_", "decode_", "ops_", "index_")))


def load_golden(name):
    with np.load(os.path.join(GOLDEN, name + ".npz")) as z:
        return {k: z[k] for k in z.files}


class ArrayLayout(list):
    """A concat()-ed position-block layout given directly by its flattened
    arrays (what a reference ``PositionBlockList`` exposes after concat())."""

    def __init__(self, boundary_indices, query_pos_ids, concat_key_pos_ids, concat_attn_masks, concat_abs_pos_masks):
        super().__init__()
        self.boundary_indices = [tuple(int(v) for v in b) for b in np.asarray(boundary_indices).reshape(-1, 4)]
        self.query_pos_ids = torch.as_tensor(np.asarray(query_pos_ids, dtype=np.int64))
        self.concat_key_pos_ids = torch.as_tensor(np.asarray(concat_key_pos_ids, dtype=np.int64))
        self.concat_attn_masks = torch.as_tensor(np.asarray(concat_attn_masks, dtype=bool))
        self.concat_abs_pos_masks = torch.as_tensor(np.asarray(concat_abs_pos_masks, dtype=bool))

    @classmethod
    def from_golden(cls, g):
        return cls(g["boundary_indices"], g["query_pos_ids"], g["concat_key_pos_ids"], g["concat_attn_masks"],
                   g["concat_abs_pos_masks"])


class HFRope(nn.Module):
    """Standard rotate-half RoPE computed as transformers' rotary modules do
    (fp32 angle = float(pos) * inv_freq, cos/sin in fp32, cast to x.dtype)."""

    def __init__(self, inv_freq):
        super().__init__()
        self.register_buffer("inv_freq", torch.as_tensor(np.asarray(inv_freq, dtype=np.float32)), persistent=False)

    @torch.no_grad()
    def forward(self, x, position_ids):
        f = position_ids.to(self.inv_freq.device).float()[..., None] * self.inv_freq.float()
        emb = torch.cat((f, f), dim=-1)
        return emb.cos().to(x.dtype).to(x.device), emb.sin().to(x.dtype).to(x.device)


def golden_rope(g, device="cpu"):
    """(torch module, oracle rope function) for a golden case."""
    from oracle import attn_oracle as O
    from autoindexer_b200.rope import SectionedRope

    if "streams" in g:
        sections = [tuple(int(v) for v in s) for s in g["sections"]]
        D = int(g["D"])
        mod = SectionedRope(D, float(g["theta"]), [torch.as_tensor(s) for s in g["streams"]], sections, device=device)
        fn = O.make_sectioned_rope(mod.inv_freq.cpu().numpy(), list(g["streams"]), sections)
        return mod, fn
    return HFRope(g["inv_freq"]).to(device), O.make_rope(g["inv_freq"])


def golden_inputs(g):
    from golden_inputs import make_inputs

    return make_inputs(int(g["seed"]), 1, int(g["Hq"]), int(g["Hkv"]), int(g["T"]), int(g["D"]))


def max_rel(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.max(np.abs(a - b)) / max(1e-30, float(np.max(np.abs(b)))))


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(1e-30, float(np.linalg.norm(b))))


@pytest.fixture(scope="session")
def cuda_device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
