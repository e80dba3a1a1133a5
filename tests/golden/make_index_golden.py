"""Generates ``tests/golden/index_op{i}.npz``: the reference's index-head
cursor losses and their gradients on its own edit-chain test cases.

Run in a container that holds the reference checkout (read-only is fine):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_index_golden.py /path/to/autoindexer

Per case of the reference's ``tests/cases/operation_tuples.json``
(``generate_sequences.OPERATION_CASES``), as its own
``test_index_loss_parity.py`` sets it up (``build_synthetic_sequence``, the
parsed positions truncated to the decoder input length): query and key
states ``(B=2, 2, T, D=32)`` from ``golden_inputs.make_inputs`` (float64),
``compute_index_losses`` (``attn_layers.py:40-110``) with a Llama rotary
embedding and ``editable_start`` 0 and 3, then autograd on
``start_loss + 2 * end_loss``.  Stored: the truncated layout (with block
types), the cursor targets per edit, the losses and dQ / dK.
"""

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

from golden_inputs import make_inputs  # noqa: E402


def main(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "src"))
    import torch
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding

    from autoindexer.models.autoindexer.attn_layers import compute_index_losses
    from autoindexer.models.autoindexer.config import AutoIndexerConfig
    from autoindexer.models.autoindexer.perturb_labels import get_parsed_positions_from_perturbations
    from autoindexer.models.autoindexer.tests.generate_sequences import (DEFAULT_MARKER_MAP, OPERATION_CASES,
                                                                          build_synthetic_sequence)
    from autoindexer.models.autoindexer.tests.test_index_loss_parity import _truncate_parsed_positions

    B, D = 2, 32
    for i, oc in enumerate(OPERATION_CASES):
        tokens, _, cursor, perts = build_synthetic_sequence(oc, DEFAULT_MARKER_MAP, B, torch.device("cpu"))
        T = tokens.shape[1] - 1
        pp = _truncate_parsed_positions(get_parsed_positions_from_perturbations(perts), T)
        rot = LlamaRotaryEmbedding(AutoIndexerConfig(hidden_size=D, head_dim=D, max_position_embeddings=1000))
        q, k, _, _ = make_inputs(4000 + i, B, 2, 2, T, D)
        res = {}
        for es in (0, 3):
            qt = torch.tensor(q, dtype=torch.float64, requires_grad=True)
            kt = torch.tensor(k, dtype=torch.float64, requires_grad=True)
            (sl, el), _ = compute_index_losses(rot, qt, kt, pp, cursor, editable_start=es)
            (sl + 2 * el).backward()
            res[f"start_loss_es{es}"] = np.float64(sl.item())
            res[f"end_loss_es{es}"] = np.float64(el.item())
            res[f"dq_es{es}"] = qt.grad.numpy().astype(np.float32)
            res[f"dk_es{es}"] = kt.grad.numpy().astype(np.float32)
        edits = np.asarray([(e, s, t) for e, (s, t) in sorted(cursor.items())], dtype=np.int64).reshape(-1, 3)
        np.savez_compressed(
            os.path.join(HERE, f"index_op{i}.npz"), **res,
            boundary_indices=np.asarray(pp.boundary_indices, dtype=np.int64).reshape(-1, 4),
            query_pos_ids=pp.query_pos_ids.numpy().astype(np.int64),
            concat_key_pos_ids=pp.concat_key_pos_ids.numpy().astype(np.int64),
            concat_attn_masks=pp.concat_attn_masks.numpy().astype(bool),
            concat_abs_pos_masks=pp.concat_abs_pos_masks.numpy().astype(bool),
            block_type=np.asarray([int(b.block_type) for b in pp], dtype=np.int32),
            cursor_edits=edits, seed=np.int64(4000 + i), B=np.int64(B), T=np.int64(T), D=np.int64(D),
            inv_freq=rot.inv_freq.numpy().astype(np.float32))
        print(f"index_op{i}", T, edits.shape[0])


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_index_golden.py <reference checkout>")
    main(sys.argv[1])
