"""The C-ABI library: it loads without a GPU, exports every function that
``include/ai_attn.h`` declares, and rejects bad arguments on the host
(before any CUDA call) with the documented status codes."""

import ctypes
import os
import re

import pytest

from conftest import ROOT
from autoindexer_b200 import _lib

HEADER = os.path.join(ROOT, "include", "ai_attn.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(ai_\w+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_function():
    names = declared_functions()
    assert len(names) >= 8
    assert set(names) == set(_lib.EXPORTED_SYMBOLS)
    handle = ctypes.CDLL(_lib.LIB_PATH)
    for n in names:
        assert hasattr(handle, n), n


def test_abi_version_and_tiles():
    L = _lib.lib()
    assert L.ai_attn_abi_version() == 9 == _lib.ABI_VERSION
    assert L.ai_attn_fwd_tile_rows(_lib.DTYPE_BF16, 128) == 128
    assert L.ai_attn_fwd_tile_rows(_lib.DTYPE_F32, 64) == 32
    assert L.ai_attn_kv_tile_rows(_lib.DTYPE_F32, 64) > 0


def test_strerror_covers_codes():
    for code in (0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, -1, -2):
        s = _lib.strerror(code)
        assert s and s != "unknown status"
    assert _lib.strerror(12345) == "unknown status"


def _args(**over):
    a = _lib.AiAttnFwdArgs()
    a.batch, a.seq_len, a.num_q_heads, a.num_kv_heads, a.head_dim = 1, 16, 4, 2, 64
    a.dtype = _lib.DTYPE_F32
    a.scale = 0.125
    for t in ("q", "k", "v", "out"):
        getattr(a, t).ptr = 256
    a.lse = 256
    L = a.layout
    L.blocks = L.row_blocks = L.row_cov = L.key_info = L.q_pos = L.k_own = L.rope_cos = L.rope_sin = L.rope_cs16 = 256
    L.n_pos = 1
    L.fwd_tile = 32
    L.kv_tile = 64
    for k, v in over.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("field,value,code", [
    ("batch", 0, 2), ("num_kv_heads", 3, 2), ("head_dim", 96, 3), ("dtype", 7, 4),
])
def test_host_validation(field, value, code):
    a = _args(**{field: value})
    assert _lib.lib().ai_attn_fwd(ctypes.byref(a), None) == code


def test_host_validation_null_and_layout():
    L = _lib.lib()
    assert L.ai_attn_fwd(None, None) == 1
    a = _args()
    a.lse = None
    assert L.ai_attn_fwd(ctypes.byref(a), None) == 1
    a = _args()
    a.layout.fwd_tile = 17
    assert L.ai_attn_fwd(ctypes.byref(a), None) == 7
    b = _lib.AiAttnBwdArgs()
    b.fwd = _args()
    for t in ("dout", "dq", "dk", "dv"):
        getattr(b, t).ptr = 256
    nbytes = ctypes.c_size_t(0)
    assert L.ai_attn_bwd_workspace(ctypes.byref(b), ctypes.byref(nbytes)) == 0
    assert nbytes.value >= 1 * 4 * 16 * 4
    b.workspace = None
    assert L.ai_attn_bwd(ctypes.byref(b), None) == 8


def test_profile_entry_points_without_gpu():
    """Profiling: NULL outputs are rejected; enabling, reading with nothing
    recorded (no GPU here) and disabling succeed and report zeros."""
    L = _lib.lib()
    n = len(_lib.PROF_KINDS)
    ms = (ctypes.c_float * n)()
    cnt = (ctypes.c_int32 * n)()
    assert L.ai_attn_profile_read(None, cnt) == 1  # AI_ERR_NULL
    assert L.ai_attn_profile_enable(1) == 0
    assert L.ai_attn_profile_read(ms, cnt) == 0
    assert L.ai_attn_profile_enable(0) == 0
    assert list(cnt) == [0] * n and list(ms) == [0.0] * n
    header = open(HEADER).read()
    assert f"AI_PROF_KINDS = {n}" in header


def test_selftest_wait_rejects_bad_arguments():
    L = _lib.lib()
    assert L.ai_attn_selftest_wait(None, 1000, None) == 1
    assert L.ai_attn_selftest_wait(ctypes.c_void_p(256), 0, None) == 2
    assert L.ai_attn_selftest_wait(ctypes.c_void_p(256), 3_000_000_000, None) == 2


@pytest.mark.gpu
def test_bounded_wait_expiry_reports_timeout(cuda_device):
    """A bounded mbarrier wait that nothing completes gives up after its
    limit and records AI_ERR_DEV_TIMEOUT (-1) in the status word; reading the
    word back clears it, and the context stays usable."""
    import torch

    from autoindexer_b200.attention import read_status, status_word

    L = _lib.lib()
    w = status_word(cuda_device)
    assert read_status(cuda_device) == 0
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    assert L.ai_attn_selftest_wait(ctypes.c_void_p(w.data_ptr()), 2_000_000, stream) == 0
    assert read_status(cuda_device) == -1
    assert read_status(cuda_device) == 0
    x = torch.ones(1024, device=cuda_device)
    assert float(x.sum()) == 1024.0
