"""Generates ``tests/golden/ops_cases.npz``: the edit-operation lists whose
position-block layouts the other golden files hold, so that the native
builder ``ai_attn_positions_from_ops`` can be checked against the layouts
the reference built from the same operations.

Run in a container that holds the reference checkout (read-only is fine):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_ops_golden.py /path/to/autoindexer

Stored (int64, rows of (num_insert, num_delete, start_rel_pos, end_rel_pos,
num_extend)):

* ``op{i}``: the operations of the reference's ``tests/cases/operation_tuples.json``
  case ``i`` (``generate_sequences.OPERATION_CASES``), whose layouts
  ``op{i}_d32.npz`` holds (``make_golden.py``);
* ``chain_e``: the operations ``make_edit_chain_golden.py`` draws from the
  reference's sampler (same seed and parameters), whose layout
  ``chain_e.npz`` holds.
"""

import os
import random
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)


def main(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "src"))
    from autoindexer.models.autoindexer.config import AutoIndexerConfig
    from autoindexer.models.autoindexer.perturb_labels import sample_cursor_operations
    from autoindexer.models.autoindexer.tests.generate_sequences import OPERATION_CASES

    from make_edit_chain_golden import LABEL_LEN, MAX_LENGTH, PERTURB

    out = {}
    for i, oc in enumerate(OPERATION_CASES):
        out[f"op{i}"] = np.asarray(oc.operations, dtype=np.int64).reshape(-1, 5)
    random.seed(0)
    np.random.seed(0)
    cfg = AutoIndexerConfig(num_heads=2, head_dim=32, edit_type_ratio=[1, 1, 1], **PERTURB)
    perturb = dict(cfg.perturb)
    perturb.pop("append_eos", None)
    while True:
        ops, token_count = sample_cursor_operations(LABEL_LEN, **perturb)
        if token_count + 1 <= MAX_LENGTH:
            break
    out["chain_e"] = np.asarray([(o.num_insert, o.num_delete, o.start_rel_pos, o.end_rel_pos, o.num_extend)
                                 for o in ops], dtype=np.int64)
    np.savez_compressed(os.path.join(HERE, "ops_cases.npz"), **out)
    print({k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_ops_golden.py <reference checkout>")
    main(sys.argv[1])
