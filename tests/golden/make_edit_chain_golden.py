"""Generates ``tests/golden/chain_e.npz``: a training-scale edit chain built by
the reference's own edit-chain machinery, with the reference's eager
attention outputs on it.

Run in a container that holds the reference checkout (read-only is fine):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_edit_chain_golden.py /path/to/autoindexer

The chain is what one CPT training step of the reference feeds its attention
(``AutoIndexerModelBase.forward``, ``src/autoindexer/models/autoindexer/
autoindexer.py:282-306``):

* ``sample_cursor_operations`` (``perturb_labels.py:135-233``) with the
  perturbation parameters of ``configs/cpt_datamix/autoindexer_8B.yaml:17-29``
  (mean_num_edits 50, mean_insert 5, mean_delete 5, mean_extend 40,
  edit_type_ratio [1, 1, 1], edit_lag_prob 0.5, mean_edit_lag 5), resampled
  until it fits ``max_seq_length`` = 3072 as ``batch_perturb_labels`` does
  (``perturb_labels.py:505-510``), from ``random`` / ``numpy.random`` seeded
  with 0 and a label length of 2800 tokens;
* ``perturb_labels_per_sequence`` (``:236-275``) and
  ``get_parsed_positions_from_perturbations`` (``:395-467``), whose
  ``concat()``-ed arrays are stored as they are.

Stored: the layout arrays, ``T_model`` = 3072 (the attention's sequence
length; rows past the covered length belong to no block), and the reference's
float64 eager forward / autograd results (``attention/reference.py:116-141``)
on ``golden_inputs.make_inputs(seed, 1, Hq=2, Hkv=1, T_cov, D=32)`` with a
Llama rotary embedding at theta 1e6, as float32 (the same recipe as
``make_golden.py``).
"""

import os
import random
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, HERE)

MAX_LENGTH = 3072
LABEL_LEN = 2800
PERTURB = dict(mean_num_edits=50, mean_insert=5, mean_delete=5, mean_extend=40, inplace_edits=False,
               sort_edits=False, edit_lag_prob=0.5, mean_edit_lag=5)


def main(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "src"))
    import torch
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding

    from autoindexer.models.autoindexer.attention import reference as ref
    from autoindexer.models.autoindexer.config import AutoIndexerConfig
    from autoindexer.models.autoindexer.perturb_labels import (get_parsed_positions_from_perturbations,
                                                                perturb_labels_per_sequence,
                                                                sample_cursor_operations)
    from make_golden import _layout_dict, run_reference

    torch.set_num_threads(os.cpu_count())
    random.seed(0)
    np.random.seed(0)
    cfg = AutoIndexerConfig(num_heads=2, head_dim=32, edit_type_ratio=[1, 1, 1], **PERTURB)
    perturb = dict(cfg.perturb)
    perturb.pop("append_eos", None)  # batch_perturb_labels' own argument, not the sampler's
    while True:
        ops, token_count = sample_cursor_operations(LABEL_LEN, **perturb)
        if token_count + 1 <= MAX_LENGTH:
            break
    perts = perturb_labels_per_sequence(ops)
    pp = get_parsed_positions_from_perturbations(perts, None)
    lay = _layout_dict(pp)
    print("blocks", lay["boundary_indices"].shape[0], "T_cov", lay["query_pos_ids"].shape[0], "sum E",
          lay["concat_key_pos_ids"].shape[0], "abs keys", int(lay["concat_abs_pos_masks"].sum()))
    rcfg = AutoIndexerConfig(num_heads=2, head_dim=32, rope_theta=1e6)
    rot = LlamaRotaryEmbedding(rcfg)
    res = run_reference(ref, rot, pp, seed=3000, Hq=2, Hkv=1, D=32)
    np.savez_compressed(os.path.join(HERE, "chain_e.npz"), **res, **lay, T_model=np.int64(MAX_LENGTH),
                        theta=np.float64(1e6))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_edit_chain_golden.py <reference checkout>")
    main(sys.argv[1])
