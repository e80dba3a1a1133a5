"""The attention function and its registration as a transformers attention
implementation.

Mirrors the reference's plugin boundary (AutodeskAILab/autoindexer,
``src/autoindexer/models/autoindexer/attention/__init__.py:18-100``):

* ``fused_chain_of_edits_attn_b200`` has the inner backend signature of
  ``fused_chain_of_edits_attn_triton`` (``attention/triton_wrapper.py:57-101``)
  and ``fused_chain_of_edits_attn_cutedsl`` (``attention/cutedsl/wrapper.py:127-170``):
  ``(rotary_emb, query, keys, values, parsed_positions, attention_mask=None,
  dropout_p=0.0, scaling=None) -> (out (B, T, Hq, D), None)``.  ``keys`` and
  ``values`` may be un-expanded (``Hkv < Hq``, GQA) or already expanded.
* ``attention_interface`` has the outer signature of the reference's wrapper
  (``__init__.py:19-30``) but passes K/V un-expanded (no ``repeat_kv`` copy);
  the decode-time ``IterPositions`` branch keeps the reference's eager math
  (``__init__.py:39-51``, ``attn_layers.py:15-27``).
* ``register_autoindexer_b200_attention`` registers it into
  ``ALL_ATTENTION_FUNCTIONS`` (``__init__.py:71-91``).

Every call runs the CUDA library; there is no CPU or eager fallback for the
chain-of-edits path.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch
from torch import Tensor, nn

from . import _lib
from .meta import CompiledLayout, compile_layout

__all__ = [
    "AttentionFn",
    "attn_fwd",
    "attn_bwd",
    "fused_chain_of_edits_attn_b200",
    "attention_interface",
    "register_autoindexer_b200_attention",
    "resolve_available_attn_implementation",
    "B200_ATTN_KEY",
]

B200_ATTN_KEY = "autoindexer_b200"

_status_words = {}


def status_word(device: torch.device) -> Tensor:
    """Per-device int32 status word the kernels report device-side errors into."""
    key = (device.type, device.index)
    t = _status_words.get(key)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        _status_words[key] = t
    return t


def read_status(device: torch.device) -> int:
    """Synchronises, returns and clears the device status word (0 = ok)."""
    w = status_word(device)
    out = ctypes.c_int32(0)
    stream = torch.cuda.current_stream(device).cuda_stream
    _lib.check(_lib.lib().ai_attn_read_status(ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(stream), ctypes.byref(out)),
               "ai_attn_read_status")
    return int(out.value)


def _t4(x: Tensor) -> "_lib.AiTensor4":
    assert x.dim() == 4 and x.stride(3) == 1
    t = _lib.AiTensor4()
    t.ptr = x.data_ptr()
    t.stride_b, t.stride_h, t.stride_t = x.stride(0), x.stride(1), x.stride(2)
    return t


def _dense_d(x: Tensor) -> Tensor:
    return x if x.stride(-1) == 1 else x.contiguous()


def _fwd_args(q: Tensor, k: Tensor, v: Tensor, out_bhtd: Tensor, lse: Tensor, layout: CompiledLayout,
              scale: float) -> "_lib.AiAttnFwdArgs":
    a = _lib.AiAttnFwdArgs()
    a.batch, a.num_q_heads, a.seq_len, a.head_dim = q.shape
    a.num_kv_heads = k.shape[1]
    a.dtype = layout.dtype
    a.scale = float(scale)
    a.q, a.k, a.v, a.out = _t4(q), _t4(k), _t4(v), _t4(out_bhtd)
    a.lse = lse.data_ptr()
    a.layout = layout.c_struct()
    a.status = status_word(q.device).data_ptr()
    return a


def attn_fwd(q: Tensor, k: Tensor, v: Tensor, layout: CompiledLayout, scale: float,
             rotated_copies: bool = True, keep_workspace: bool = False, out_bhtd: Optional[Tensor] = None):
    """Launches ``ai_attn_fwd``: returns ``out (B, T, Hq, D)`` and ``lse (B, Hq, T)`` fp32.

    ``rotated_copies``: give the kernels scratch for once-rotated Q/K copies
    (faster; ``ai_attn_fwd_workspace`` bytes); without it every tile is
    rotated in shared memory.  ``keep_workspace``: also return that scratch
    (or ``None``) so that ``attn_bwd(..., fwd_workspace=...)`` reads the
    rotated copies instead of rotating again.  ``out_bhtd``: a ``(B, Hq, T,
    D)`` view (d contiguous, any other strides) the kernels write the output
    into; the returned ``out`` is then its ``(B, T, Hq, D)`` permutation."""
    B, Hq, T, D = q.shape
    if out_bhtd is None:
        out = torch.empty((B, T, Hq, D), dtype=q.dtype, device=q.device)
        out_bhtd = out.permute(0, 2, 1, 3)
    else:
        if tuple(out_bhtd.shape) != (B, Hq, T, D) or out_bhtd.stride(-1) != 1 or out_bhtd.dtype != q.dtype:
            raise ValueError("out_bhtd must be a (B, Hq, T, D) view of q's dtype with d contiguous")
        out = out_bhtd.permute(0, 2, 1, 3)
    lse = torch.empty((B, Hq, T), dtype=torch.float32, device=q.device)
    a = _fwd_args(q, k, v, out_bhtd, lse, layout, scale)
    lib = _lib.lib()
    nbytes = ctypes.c_size_t(0)
    _lib.check(lib.ai_attn_fwd_workspace(ctypes.byref(a), ctypes.byref(nbytes)), "ai_attn_fwd_workspace")
    ws = None
    if nbytes.value and rotated_copies:
        ws = torch.empty(int(nbytes.value), dtype=torch.uint8, device=q.device)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    stream = torch.cuda.current_stream(q.device).cuda_stream
    _lib.check(lib.ai_attn_fwd(ctypes.byref(a), ctypes.c_void_p(stream)), "ai_attn_fwd")
    if keep_workspace:
        return out, lse, ws
    del ws
    return out, lse


def attn_bwd(q, k, v, out, lse, dout, layout: CompiledLayout, scale: float, rotated_copies: bool = True,
             fwd_workspace: Optional[Tensor] = None, grads: Optional[Tuple[Tensor, Tensor, Tensor]] = None,
             after_dq=None):
    """Launches ``ai_attn_bwd``: returns ``dq, dk, dv`` shaped like ``q, k, v``
    (``rotated_copies`` as for ``attn_fwd``; without it the workspace holds
    only the row sums of dO.O).  ``fwd_workspace``: the scratch that
    ``attn_fwd(..., keep_workspace=True)`` returned for these q, k and layout;
    its rotated Q/K copies are reused (``fwd_rotated`` in the C ABI).
    ``grads``: ``(dq, dk, dv)`` views (shaped like q, k, v, d contiguous) the
    kernels write into instead of new tensors.  ``after_dq``: called between
    the dQ launches and the dK/dV launches (two ``ai_attn_bwd`` calls,
    ``parts`` = dQ then dK/dV), when dQ is complete in stream order."""
    if grads is not None:
        dq, dk, dv = grads
        for g, x in ((dq, q), (dk, k), (dv, v)):
            if g.shape != x.shape or g.stride(-1) != 1 or g.dtype != x.dtype:
                raise ValueError("grads must be shaped like q, k, v with d contiguous")
    else:
        dq = torch.empty_like(q)
        dk = torch.empty_like(k)
        dv = torch.empty_like(v)
        if dq.stride(-1) != 1:
            dq = torch.empty(q.shape, dtype=q.dtype, device=q.device)
        if dk.stride(-1) != 1:
            dk = torch.empty(k.shape, dtype=k.dtype, device=k.device)
        if dv.stride(-1) != 1:
            dv = torch.empty(v.shape, dtype=v.dtype, device=v.device)
    a = _lib.AiAttnBwdArgs()
    a.fwd = _fwd_args(q, k, v, out.permute(0, 2, 1, 3), lse, layout, scale)
    dout_keep = _dense_d(dout)
    a.dout = _t4(dout_keep.permute(0, 2, 1, 3))
    a.dq, a.dk, a.dv = _t4(dq), _t4(dk), _t4(dv)
    if fwd_workspace is not None and rotated_copies:
        a.fwd.workspace, a.fwd.workspace_bytes = fwd_workspace.data_ptr(), fwd_workspace.numel()
        a.fwd_rotated = 1
    lib = _lib.lib()
    nbytes = ctypes.c_size_t(0)
    _lib.check(lib.ai_attn_bwd_workspace(ctypes.byref(a), ctypes.byref(nbytes)), "ai_attn_bwd_workspace")
    want = int(nbytes.value)
    if not rotated_copies:
        want = (q.shape[0] * q.shape[1] * q.shape[2] * 4 + 255) // 256 * 256
    ws = torch.empty(max(want, 256), dtype=torch.uint8, device=q.device)
    a.workspace = ws.data_ptr()
    a.workspace_bytes = ws.numel()
    stream = torch.cuda.current_stream(q.device).cuda_stream
    if after_dq is None:
        _lib.check(lib.ai_attn_bwd(ctypes.byref(a), ctypes.c_void_p(stream)), "ai_attn_bwd")
    else:
        a.parts = _lib.BWD_DQ
        _lib.check(lib.ai_attn_bwd(ctypes.byref(a), ctypes.c_void_p(stream)), "ai_attn_bwd")
        after_dq()
        a.parts = _lib.BWD_DKDV
        _lib.check(lib.ai_attn_bwd(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream(q.device).cuda_stream)),
                   "ai_attn_bwd")
    del dout_keep, ws
    return dq, dk, dv


class KernelTimes:
    """Per-kernel device times of this library's launches (CUDA events on the
    launch streams; ``ai_attn_profile_enable`` / ``ai_attn_profile_read``)::

        with KernelTimes() as kt:
            ...  # calls into the library
        kt.ms["dkdv"], kt.launches["dkdv"]
    """

    def __enter__(self):
        _lib.check(_lib.lib().ai_attn_profile_enable(1), "ai_attn_profile_enable")
        return self

    def __exit__(self, *exc):
        lib = _lib.lib()
        n = len(_lib.PROF_KINDS)
        ms = (ctypes.c_float * n)()
        cnt = (ctypes.c_int32 * n)()
        rc = lib.ai_attn_profile_read(ms, cnt)
        lib.ai_attn_profile_enable(0)
        _lib.check(rc, "ai_attn_profile_read")
        self.ms = {k: float(ms[i]) for i, k in enumerate(_lib.PROF_KINDS)}
        self.launches = {k: int(cnt[i]) for i, k in enumerate(_lib.PROF_KINDS)}
        return False


class AttentionFn(torch.autograd.Function):
    """Autograd wrapper: saves q, k, v, out and lse; backward is ``ai_attn_bwd``."""

    @staticmethod
    def forward(ctx, q, k, v, layout: CompiledLayout, scale: float):
        q, k, v = _dense_d(q), _dense_d(k), _dense_d(v)
        out, lse, ws = attn_fwd(q, k, v, layout, scale, keep_workspace=True)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.layout = layout
        ctx.scale = scale
        ctx.fwd_ws = ws  # rotated Q/K copies, reused by the backward
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse = ctx.saved_tensors
        dq, dk, dv = attn_bwd(q, k, v, out, lse, dout, ctx.layout, ctx.scale, fwd_workspace=ctx.fwd_ws)
        ctx.fwd_ws = None
        return dq, dk, dv, None, None


_MASK_CHECK_ELEMS = 1 << 26  # mask entries examined per chunk of rows


def _check_mask_is_causal(attention_mask: Tensor, T: int) -> None:
    """The kernels apply the block masks plus the global causal mask.  An
    external mask is accepted only when it removes nothing inside the causal
    triangle (HF injects a plain causal mask); anything else raises.

    The check runs once per mask tensor and version (every layer of a
    forward gets the same mask object), over chunks of rows so that no T x T
    temporary is built, with a single device-to-host read at the end."""
    m = attention_mask
    if m.dim() != 4 or m.shape[-1] != T or m.shape[-2] != T:
        raise NotImplementedError(f"attention_mask of shape {tuple(m.shape)} is not supported")
    stamp = (m._version, m.data_ptr(), tuple(m.shape), m.dtype)
    if getattr(m, "_b200_causal_ok", None) == stamp:
        return
    lead = max(1, m.shape[0] * m.shape[1])
    rows = max(1, _MASK_CHECK_ELEMS // (lead * T))
    cols = torch.arange(T, device=m.device)
    bad = torch.zeros((), dtype=torch.bool, device=m.device)
    for r0 in range(0, T, rows):
        r1 = min(T, r0 + rows)
        lower = cols[None, :] <= torch.arange(r0, r1, device=m.device)[:, None]  # causal triangle of these rows
        sub = m[..., r0:r1, :]
        removed = ~sub if m.dtype == torch.bool else sub != 0
        bad |= (removed & lower).any()
    if bool(bad):
        raise NotImplementedError("attention_mask masks entries inside the causal triangle; not supported")
    try:
        m._b200_causal_ok = stamp
    except (AttributeError, RuntimeError):
        pass


def fused_chain_of_edits_attn_b200(
    rotary_emb,
    query: Tensor,
    keys: Tensor,
    values: Tensor,
    parsed_positions,
    attention_mask: Optional[Tensor] = None,
    dropout_p: float = 0.0,
    scaling: Optional[float] = None,
) -> Tuple[Tensor, None]:
    """Chain-of-edits attention on the B200 kernels; same contract as the
    reference's Triton / CuTeDSL backends (see module docstring).

    ``parsed_positions`` is a concat()-ed ``PositionBlockList`` shared by all
    rows, or a ``RowLayouts`` with one per row."""
    if not isinstance(parsed_positions, list):
        raise TypeError("parsed_positions must be a PositionBlockList (or RowLayouts)")
    B, Hq, T, D = query.shape
    if keys.shape[2] != T:
        raise AssertionError("q_len must equal kv_len")
    if keys.shape[1] == 0 or Hq % keys.shape[1] != 0:
        raise ValueError(f"num_q_heads {Hq} is not a multiple of num_kv_heads {keys.shape[1]}")
    if dropout_p:
        raise NotImplementedError("autoindexer_b200 attention has no dropout")
    if not query.is_cuda:
        raise RuntimeError("autoindexer_b200 attention runs on CUDA tensors only")
    if attention_mask is not None:
        _check_mask_is_causal(attention_mask, T)
    scale = float(scaling) if scaling is not None else D ** -0.5
    layout = compile_layout(parsed_positions, B, T, D, query.dtype, rotary_emb, query.device)
    out = AttentionFn.apply(query, keys, values, layout, scale)
    return out, None


def _iter_positions_attention(module, query, key, value, attention_mask, dropout, scaling, rotary_emb,
                              parsed_positions):
    """Decode step (one query token).  On the kernel's domain (CUDA bf16,
    head_dim 128, <= 8 query heads per KV head, boolean or 0/-inf mask) the
    ``ai_attn_decode`` kernels (``autoindexer_b200.decode``), returning no
    attention weights, as the SDPA and flash backends of transformers do;
    otherwise the reference's eager math (``attn_layers.py:15-27`` then
    ``__init__.py:41-51``), weights included."""
    from .decode import decode_attention, decode_supported

    if decode_supported(query, key, attention_mask):
        return decode_attention(query, key, value, parsed_positions, rotary_emb, scaling, attention_mask), None
    groups = query.shape[1] // key.shape[1]
    if groups > 1:
        key = key.repeat_interleave(groups, dim=1)
        value = value.repeat_interleave(groups, dim=1)
    assert query.shape[2] == 1
    cos, sin = parsed_positions.get_rotary_pos_emb(rotary_emb, key)
    cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
    half = key.shape[-1] // 2
    rot = torch.cat((-key[..., half:], key[..., :half]), dim=-1)
    key_with_pos = key * cos + rot * sin
    w = query @ key_with_pos.transpose(-1, -2)
    w.masked_fill_(~parsed_positions.attn_mask.view(-1, 1, 1, key.shape[-2]), float("-inf"))
    w = w * (scaling if scaling is not None else query.shape[-1] ** -0.5)
    if attention_mask is not None:
        if attention_mask.dtype == torch.bool:
            w.masked_fill_(attention_mask.logical_not(), float("-inf"))
        else:
            w = w + attention_mask
    w = nn.functional.softmax(w, dim=-1, dtype=torch.float32).to(query.dtype)
    w = nn.functional.dropout(w, p=dropout, training=False)
    return torch.matmul(w, value), w


def attention_interface(
    module: nn.Module,
    query: Tensor,
    key: Tensor,
    value: Tensor,
    attention_mask: Optional[Tensor],
    dropout: float = 0.0,
    scaling: Optional[float] = None,
    rotary_emb=None,
    parsed_positions=None,
    **kwargs,
) -> Tuple[Tensor, Optional[Tensor]]:
    """transformers attention function (``ALL_ATTENTION_FUNCTIONS`` signature)."""
    if parsed_positions is not None and hasattr(parsed_positions, "key_pos_ids") and not isinstance(parsed_positions, list):
        return _iter_positions_attention(module, query, key, value, attention_mask, dropout, scaling, rotary_emb,
                                         parsed_positions)
    return fused_chain_of_edits_attn_b200(rotary_emb, query, key, value, parsed_positions,
                                          attention_mask=attention_mask, dropout_p=dropout, scaling=scaling)


def register_autoindexer_b200_attention(keys=(B200_ATTN_KEY,)) -> None:
    """Registers ``attention_interface`` under each key (default
    ``"autoindexer_b200"``; pass ``("autoindexer_b200", "autoindexer_cutedsl")``
    to make existing configs pick it up)."""
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    for k in keys:
        ALL_ATTENTION_FUNCTIONS.register(k, attention_interface)


def resolve_available_attn_implementation(requested: str) -> str:
    """Maps the reference's fused-kernel keys onto this backend (the reference
    downgrades cutedsl -> triton -> eager when a kernel package is missing,
    ``__init__.py:94-100``; here the CUDA library is required and a missing
    library raises instead of downgrading)."""
    if requested in ("autoindexer_cutedsl", "autoindexer_triton", B200_ATTN_KEY):
        _lib.lib()
        return B200_ATTN_KEY
    return requested
