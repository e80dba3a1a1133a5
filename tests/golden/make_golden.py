"""Generates the golden fixtures under tests/golden/ by running the reference.

Run in a container that holds the reference checkout (read-only is fine):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py /path/to/autoindexer

It imports the reference's own eager attention
(``src/autoindexer/models/autoindexer/attention/reference.py``,
``chain_of_edits_attn_ref`` / ``compute_attn_weights_ref``) and its own
edit-chain machinery (``perturb_labels.py``,
``tests/generate_sequences.py``), runs them in float64 on the inputs of
``golden_inputs.make_inputs`` and stores, per case, the concat()-ed position
layout, the rotary ``inv_freq``, and the reference's forward output, row
log-sum-exp and the autograd gradients dQ/dK/dV (float32).

Cases:
* ``kat_position_matrix``: the layout of the reference's known-answer test
  (``tests/test_generalized_rope.py``) and its expected 82x82 position / mask
  matrices (``tests/labels/position_matrix.json``);
* ``op{i}``: the ten edit chains of ``tests/cases/operation_tuples.json``
  (B=1, Hq=2, Hkv=1, D=32; cases 3 and 7 also at D=64);
* ``sec2``, ``sec3``: packed documents with 2 and 3 head-dim RoPE sections
  (``autoindexer_b200.SectionedRope``), D=64.
"""

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, HERE)

from golden_inputs import make_inputs  # noqa: E402


def _layout_dict(pp):
    return dict(
        boundary_indices=np.asarray(pp.boundary_indices, dtype=np.int64).reshape(-1, 4),
        query_pos_ids=pp.query_pos_ids.cpu().numpy().astype(np.int64),
        concat_key_pos_ids=pp.concat_key_pos_ids.cpu().numpy().astype(np.int64),
        concat_attn_masks=pp.concat_attn_masks.cpu().numpy().astype(bool),
        concat_abs_pos_masks=pp.concat_abs_pos_masks.cpu().numpy().astype(bool),
    )


def run_reference(ref, rotary_emb, pp, seed, Hq, Hkv, D):
    import torch
    from transformers.models.llama.modeling_llama import repeat_kv

    T = len(pp.query_pos_ids)
    q, k, v, dout = make_inputs(seed, 1, Hq, Hkv, T, D)
    qt, kt, vt = (torch.tensor(x, dtype=torch.float64, requires_grad=True) for x in (q, k, v))
    G = Hq // Hkv
    out, _ = ref.chain_of_edits_attn_ref(rotary_emb, qt, repeat_kv(kt, G), repeat_kv(vt, G), pp)
    out.backward(torch.tensor(dout, dtype=torch.float64))
    with torch.no_grad():
        # fresh layout caches: get_rotary_pos_emb memoises on the list
        w = ref.compute_attn_weights_ref(rotary_emb, qt.detach(), repeat_kv(kt.detach(), G), pp)
        lse = torch.logsumexp(w, dim=-1)
    return dict(
        seed=np.int64(seed), Hq=np.int64(Hq), Hkv=np.int64(Hkv), D=np.int64(D), T=np.int64(T),
        inv_freq=rotary_emb.inv_freq.detach().cpu().numpy().astype(np.float32),
        out=out.detach().numpy().astype(np.float32),
        lse=lse.numpy().astype(np.float32),
        dq=qt.grad.numpy().astype(np.float32),
        dk=kt.grad.numpy().astype(np.float32),
        dv=vt.grad.numpy().astype(np.float32),
    )


def main(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "src"))
    import torch
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding

    from autoindexer.models.autoindexer.attention import reference as ref
    from autoindexer.models.autoindexer.config import AutoIndexerConfig
    from autoindexer.models.autoindexer.perturb_labels import (get_parsed_positions_from_perturbations,
                                                                perturb_labels_per_sequence, to_operations)
    from autoindexer.models.autoindexer.perturb_labels import PositionBlockList as RefList
    from autoindexer.models.autoindexer.tests.generate_sequences import OPERATION_CASES, get_parsed_positions_from_case
    from autoindexer.models.autoindexer.type_utils import PositionBlock as RefBlock

    from autoindexer_b200.positions import cursor_stream, document_blocks
    from autoindexer_b200.rope import SectionedRope

    out_dir = HERE
    torch.set_num_threads(8)

    # Known-answer test of the reference (tests/test_generalized_rope.py:47-64).
    ops = to_operations([(0, 0, 0, 0, 5), (9, 0, 2, 2, 0), (4, 2, 0, 2, 4), (5, 1, 19, 20, 0), (5, 3, 6, 9, 0)])
    perts = perturb_labels_per_sequence(ops)
    n = perts[-1].curr_seq_idx
    pp = get_parsed_positions_from_perturbations(perts, None)
    with open(os.path.join(ref_root, "src/autoindexer/models/autoindexer/tests/labels/position_matrix.json")) as f:
        kat = json.load(f)
    np.savez_compressed(
        os.path.join(out_dir, "kat_position_matrix.npz"),
        position_matrix=np.asarray(kat["position_matrix"], dtype=np.int16)[0, :n, :n],
        attention_mask=np.asarray(kat["attention_mask"], dtype=np.int8)[0, :n, :n],
        **_layout_dict(pp))

    for i, oc in enumerate(OPERATION_CASES):
        for D in ((32, 64) if i in (3, 7) else (32,)):
            pp = get_parsed_positions_from_case(oc, None)
            rot = LlamaRotaryEmbedding(AutoIndexerConfig(num_heads=2, head_dim=D))
            res = run_reference(ref, rot, pp, seed=1000 + i, Hq=2, Hkv=1, D=D)
            name = f"op{i}_d{D}.npz"
            np.savez_compressed(os.path.join(out_dir, name), **res, **_layout_dict(pp))
            print(name, int(res["T"]))

    rng = np.random.Generator(np.random.PCG64(7))
    for name, S, sections, lens in (("sec2", 2, [(0, 16), (16, 32)], [30, 50]),
                                    ("sec3", 3, [(0, 12), (12, 24), (24, 32)], [20, 41, 19])):
        T = sum(lens)
        streams = [np.arange(T)] + [cursor_stream(T, rng) for _ in range(S - 1)]
        ours = document_blocks(lens, position_ids=np.arange(T))
        pp = RefList([RefBlock(key_pos_ids=b.key_pos_ids, query_pos_ids=b.query_pos_ids, abs_pos_mask=None,
                               attn_mask=b.attn_mask, start_idx=b.start_idx, end_idx=b.end_idx,
                               block_type=b.block_type) for b in ours])
        pp.concat()
        rot = SectionedRope(64, 1e6, [torch.as_tensor(s) for s in streams], sections)
        res = run_reference(ref, rot, pp, seed=2000 + S, Hq=4, Hkv=2, D=64)
        np.savez_compressed(os.path.join(out_dir, f"{name}.npz"), **res, **_layout_dict(pp),
                            streams=np.stack(streams).astype(np.int64),
                            sections=np.asarray(sections, dtype=np.int64), theta=np.float64(1e6))
        print(name, T)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <reference checkout>")
    main(sys.argv[1])
