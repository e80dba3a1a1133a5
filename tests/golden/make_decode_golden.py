"""Writes tests/golden/decode_iter.npz: the reference's own decode branch
(the IterPositions path of ``attention/__init__.py:36-51``, with
``attn_layers.py:15-27`` ``compute_attn_weights_iter`` and
``type_utils.py:48-67`` ``IterPositions``) run in float64 on seeded inputs.

Run once in a checkout that has the reference importable:
    python tests/golden/make_decode_golden.py /path/to/reference/src
"""

import os
import sys

import numpy as np
import torch


def main(ref_src):
    sys.path.insert(0, ref_src)
    from autoindexer.models.autoindexer.attn_layers import compute_attn_weights_iter
    from autoindexer.models.autoindexer.type_utils import IterPositions

    B, Hq, Hkv, L, D = 2, 4, 2, 37, 16
    rng = np.random.default_rng(21)
    q = rng.standard_normal((B, Hq, 1, D))
    k = rng.standard_normal((B, Hkv, L, D))
    v = rng.standard_normal((B, Hkv, L, D))
    key_pos = np.stack([np.arange(L) - (L - 1), rng.integers(-50, 1, size=L)])  # relative positions, per row
    attn_mask = rng.random((B, L)) > 0.25
    attn_mask[:, -1] = True
    theta, half = 1e4, D // 2
    inv_freq = (1.0 / theta ** (np.arange(0, D, 2, dtype=np.float64) / D)).astype(np.float32)

    def rotary_emb(x, position_ids):  # HF-style: fp32 angle, cat(freqs, freqs)
        ang = position_ids.to(torch.float32)[..., None] * torch.as_tensor(inv_freq)
        emb = torch.cat((ang, ang), dim=-1).double()
        return emb.cos().to(x.dtype), emb.sin().to(x.dtype)

    tq, tk, tv = (torch.as_tensor(x) for x in (q, k, v))
    pp = IterPositions(key_pos_ids=torch.as_tensor(key_pos), attn_mask=torch.as_tensor(attn_mask))
    G = Hq // Hkv
    tk_e, tv_e = tk.repeat_interleave(G, dim=1), tv.repeat_interleave(G, dim=1)  # repeat_kv
    w = compute_attn_weights_iter(rotary_emb, tq, tk_e, pp, scaling=None)
    p = torch.softmax(w, dim=-1)
    out = torch.matmul(p, tv_e)
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "decode_iter.npz")
    np.savez(path, q=q, k=k, v=v, key_pos=key_pos, attn_mask=attn_mask, inv_freq=inv_freq, out=out.numpy())
    print("wrote", path)


if __name__ == "__main__":
    main(sys.argv[1])
