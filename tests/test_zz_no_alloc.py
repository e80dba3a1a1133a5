"""ai_attn_bwd_noalloc: the backward entry point for callers that cannot
allocate device memory (a host whose memory pool belongs to another component,
a plugin that may only touch the buffers it is handed, code that must not call
cudaMalloc after start-up).  It takes its scratch from a fixed array inside the
library instead of a caller workspace.

The GPU tests call it through the C ABI, twice in a row each, and compare with
ai_attn_bwd given a workspace that holds the same things the fixed array
holds (the same kernels then run on the same data, so the results must be
bitwise equal):

* a small edit chain, where the array holds the row sums and the rotated Q/K
  copies;
* the same call with fwd_rotated = 1 (the forward's copies passed in), where
  the array holds only the row sums;
* a packed-documents batch at exactly AI_ATTN_NOALLOC_MAX_ROWS query rows,
  where the copies no longer fit and every tile is rotated in shared memory;
  there some documents are also checked against the oracle.

This file is collected last so that a run stopping at the first failure has
run everything else; it also passes on its own in a fresh process.
"""

import ctypes

import numpy as np
import pytest
import torch

from autoindexer_b200 import _lib

MAX_ROWS = 1 << 22  # AI_ATTN_NOALLOC_MAX_ROWS


def test_noalloc_rejects_sizes_beyond_its_scratch():
    a = _lib.AiAttnBwdArgs()
    a.fwd.batch, a.fwd.num_q_heads, a.fwd.seq_len = 8, 32, MAX_ROWS // 256 + 1  # one row over the limit
    rc = _lib.lib().ai_attn_bwd_noalloc(ctypes.byref(a), None)
    assert rc == 12
    assert "AI_ATTN_NOALLOC_MAX_ROWS" in _lib.strerror(rc)


def _bwd_args(q, k, v, out, lse, dout, layout, dq, dk, dv):
    from autoindexer_b200.attention import _fwd_args, _t4

    D = q.shape[-1]
    a = _lib.AiAttnBwdArgs()
    a.fwd = _fwd_args(q, k, v, out.permute(0, 2, 1, 3), lse, layout, D ** -0.5)
    a.dout = _t4(dout.permute(0, 2, 1, 3))
    a.dq, a.dk, a.dv = _t4(dq), _t4(dk), _t4(dv)
    return a


def _compare_two_noalloc_calls(q, k, v, out, lse, dout, layout, ws_bytes, fwd_ws, device):
    """ai_attn_bwd with a workspace of ``ws_bytes`` (and the forward's copies
    when ``fwd_ws`` is given), then two ai_attn_bwd_noalloc calls on fresh
    NaN-filled outputs; each must equal the first bit for bit."""
    from autoindexer_b200.attention import read_status

    lib = _lib.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
    ref = [torch.empty_like(x) for x in (q, k, v)]
    a = _bwd_args(q, k, v, out, lse, dout, layout, *ref)
    if fwd_ws is not None:
        a.fwd.workspace, a.fwd.workspace_bytes, a.fwd_rotated = fwd_ws.data_ptr(), fwd_ws.numel(), 1
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=device)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    assert lib.ai_attn_bwd(ctypes.byref(a), stream) == 0
    for call in range(2):
        got = [torch.full_like(x, float("nan")) for x in (q, k, v)]
        b = _bwd_args(q, k, v, out, lse, dout, layout, *got)
        if fwd_ws is not None:
            b.fwd.workspace, b.fwd.workspace_bytes, b.fwd_rotated = fwd_ws.data_ptr(), fwd_ws.numel(), 1
        b.workspace, b.workspace_bytes = None, 0  # ignored by the no-alloc entry point
        assert lib.ai_attn_bwd_noalloc(ctypes.byref(b), stream) == 0
        torch.cuda.synchronize(device)
        assert read_status(device) == 0
        for name, x, y in zip(("dq", "dk", "dv"), got, ref):
            assert torch.equal(x, y), (call, name)
    return ref


@pytest.mark.gpu
@pytest.mark.parametrize("reuse_forward_copies", [False, True])
def test_noalloc_backward_matches_workspace_backward(reuse_forward_copies, cuda_device):
    from conftest import ArrayLayout, HFRope, load_golden
    from autoindexer_b200.attention import attn_fwd
    from autoindexer_b200.meta import compile_layout
    from oracle import attn_oracle as O

    g = load_golden("op0_d32")
    lay = ArrayLayout.from_golden(g)
    B, Hq, Hkv, T, D = 2, 4, 2, int(g["T"]), 128
    gen = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(s, generator=gen).to(cuda_device, torch.bfloat16)
               for s in ((B, Hq, T, D), (B, Hkv, T, D), (B, Hkv, T, D)))
    dout = torch.randn(B, T, Hq, D, generator=gen).to(cuda_device, torch.bfloat16)
    rope = HFRope(O.default_inv_freq(D, 1e4)).to(cuda_device)
    layout = compile_layout(lay, B, T, D, torch.bfloat16, rope, cuda_device)
    out, lse, fwd_ws = attn_fwd(q, k, v, layout, D ** -0.5, keep_workspace=True)
    # At this size the fixed array holds the row sums and, without the
    # forward's copies, the rotated copies too: the same as a 16 MiB workspace.
    _compare_two_noalloc_calls(q, k, v, out, lse, dout, layout, 4 * MAX_ROWS,
                               fwd_ws if reuse_forward_copies else None, cuda_device)


@pytest.mark.gpu
def test_noalloc_backward_at_the_row_limit(cuda_device):
    """B * Hq * T = AI_ATTN_NOALLOC_MAX_ROWS (1 x 32 x 131072, packed
    documents of 128-256 tokens): the row sums fill the whole array, the
    rotated copies do not fit and every tile is rotated in shared memory.
    Equal bit for bit to ai_attn_bwd with a row-sums-only workspace, and
    within the bf16 tolerances of the oracle on a few documents."""
    from conftest import rel_l2
    from autoindexer_b200 import SectionedRope, document_blocks
    from autoindexer_b200.attention import attn_fwd
    from autoindexer_b200.meta import compile_layout
    from autoindexer_b200.positions import split_documents
    from oracle import attn_oracle as O

    B, Hq, Hkv, D = 1, 32, 8, 128
    T = MAX_ROWS // (B * Hq)
    rng = np.random.default_rng(12)
    lens = split_documents(T, 128, 256, rng)
    lay = document_blocks(lens, position_ids=np.arange(T))
    mod = SectionedRope(D, 1e6, [torch.arange(T)], [(0, D // 2)])
    gen = torch.Generator().manual_seed(12)
    q, k, v = (torch.randn(s, generator=gen).to(torch.bfloat16) for s in ((B, Hq, T, D), (B, Hkv, T, D), (B, Hkv, T, D)))
    dout = torch.randn(B, T, Hq, D, generator=gen).to(torch.bfloat16)
    tq, tk, tv, tdo = (x.to(cuda_device) for x in (q, k, v, dout))
    layout = compile_layout(lay, B, T, D, torch.bfloat16, mod.to(cuda_device), cuda_device)
    out, lse = attn_fwd(tq, tk, tv, layout, D ** -0.5)
    dq, dk, dv = _compare_two_noalloc_calls(tq, tk, tv, out, lse, tdo, layout, 4 * MAX_ROWS, None, cuda_device)
    rope = O.make_sectioned_rope(mod.inv_freq.cpu().numpy(), [np.arange(T)], [(0, D // 2)])
    bounds = lay.boundary_indices
    G = Hq // Hkv
    for di in (0, 1, len(bounds) // 2, len(bounds) - 1):
        s, e = int(bounds[di][0]), int(bounds[di][1])
        sub = document_blocks([e - s], position_ids=np.arange(s, e))
        hq, hk = slice(0, G), slice(0, 1)
        want = O.attn_chunked(q[:, hq, s:e].double().numpy(), k[:, hk, s:e].double().numpy(),
                              v[:, hk, s:e].double().numpy(), dout[:, s:e, hq].double().numpy(), sub, rope)
        got = [t.double().cpu().numpy() for t in (dq[:, hq, s:e], dk[:, hk, s:e], dv[:, hk, s:e])]
        for name, a_, b_ in zip(("dq", "dk", "dv"), got, want[2:]):
            assert rel_l2(a_, b_) <= 1e-2, (di, name, rel_l2(a_, b_))
