"""ai_attn_bwd_noalloc: the backward entry point for callers that cannot
allocate device memory (a host whose memory pool belongs to another component,
a plugin that may only touch the buffers it is handed, code that must not call
cudaMalloc after start-up).  It takes its scratch from a fixed array inside the
library instead of a caller workspace.

The GPU test calls it through the C ABI twice in a row and checks both calls
against ai_attn_bwd (same tolerance as the other bf16 tests; the kernels are
the same, so the results are expected to be bitwise equal).  This file is
collected last so that a run stopping at the first failure has run everything
else; it also passes on its own in a fresh process.
"""

import ctypes

import numpy as np
import pytest
import torch

from autoindexer_b200 import _lib


def test_noalloc_rejects_sizes_beyond_its_scratch():
    a = _lib.AiAttnBwdArgs()
    a.fwd.batch, a.fwd.num_q_heads, a.fwd.seq_len = 8, 32, (1 << 22) // 256 + 1  # one row over the limit
    rc = _lib.lib().ai_attn_bwd_noalloc(ctypes.byref(a), None)
    assert rc == 12
    assert "AI_ATTN_NOALLOC_MAX_ROWS" in _lib.strerror(rc)


@pytest.mark.gpu
def test_noalloc_backward_matches_workspace_backward(cuda_device):
    from conftest import ArrayLayout, HFRope, load_golden, rel_l2
    from autoindexer_b200.attention import _fwd_args, _t4, attn_fwd, read_status
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
    out, lse = attn_fwd(q, k, v, layout, D ** -0.5)
    lib = _lib.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)

    def args(dq, dk, dv):
        a = _lib.AiAttnBwdArgs()
        a.fwd = _fwd_args(q, k, v, out.permute(0, 2, 1, 3), lse, layout, D ** -0.5)
        a.dout = _t4(dout.permute(0, 2, 1, 3))
        a.dq, a.dk, a.dv = _t4(dq), _t4(dk), _t4(dv)
        return a

    # existing entry point, caller-provided workspace
    ref = [torch.empty_like(x) for x in (q, k, v)]
    a = args(*ref)
    nbytes = ctypes.c_size_t(0)
    assert lib.ai_attn_bwd_workspace(ctypes.byref(a), ctypes.byref(nbytes)) == 0
    ws = torch.empty(int(nbytes.value), dtype=torch.uint8, device=cuda_device)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    assert lib.ai_attn_bwd(ctypes.byref(a), stream) == 0

    for call in range(2):
        got = [torch.full_like(x, float("nan")) for x in (q, k, v)]
        b = args(*got)
        b.workspace, b.workspace_bytes = None, 0  # ignored by the no-alloc entry point
        assert lib.ai_attn_bwd_noalloc(ctypes.byref(b), stream) == 0
        torch.cuda.synchronize(cuda_device)
        assert read_status(cuda_device) == 0
        for name, x, y in zip(("dq", "dk", "dv"), got, ref):
            xa, ya = x.double().cpu().numpy(), y.double().cpu().numpy()
            assert np.isfinite(xa).all(), (call, name)
            assert rel_l2(xa, ya) <= 1e-2, (call, name, rel_l2(xa, ya))
