"""Deterministic inputs shared by the golden-fixture generator and the tests.

Q/K/V/dO are drawn from numpy's PCG64 generator (bit-stable across platforms)
as standard normals rounded to float32, so the fp32 CUDA path sees exactly the
values the reference was run on.
"""

import numpy as np


def make_inputs(seed: int, batch: int, num_q_heads: int, num_kv_heads: int, seq_len: int, head_dim: int):
    rng = np.random.Generator(np.random.PCG64(seed))

    def draw(*shape):
        return rng.standard_normal(shape).astype(np.float32)

    q = draw(batch, num_q_heads, seq_len, head_dim)
    k = draw(batch, num_kv_heads, seq_len, head_dim)
    v = draw(batch, num_kv_heads, seq_len, head_dim)
    dout = draw(batch, seq_len, num_q_heads, head_dim)
    return q, k, v, dout
