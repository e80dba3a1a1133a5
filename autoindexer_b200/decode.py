"""Decode step on the B200 kernels (``ai_attn_decode``).

The reference's registered interface answers a one-token decode step
(``parsed_positions`` an ``IterPositions``) with eager math
(``attention/__init__.py:36-51`` and ``attn_layers.py:15-27``): it expands K/V
for GQA, rotates the whole key cache by ``key_pos_ids`` (relative position
ids), takes ``q . k_rot``, masks, scales, softmaxes in fp32 and multiplies by
V.  ``decode_attention`` computes the same in one pass over the unrotated
cache: every key is rotated as the kernel reads it, with the cos/sin the
rotary module gives for ``key_pos_ids`` (``IterPositions.get_rotary_pos_emb``,
``type_utils.py:62-67``, the reference's own call, so no host sync).
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch
from torch import Tensor

from . import _lib
from .attention import _t4, status_word

_MAX_GROUP = 8


def decode_supported(query: Tensor, key: Tensor, attention_mask: Optional[Tensor]) -> bool:
    """The kernel's domain: CUDA bf16, head_dim 128, one query token, at most
    8 query heads per KV head, and a boolean (or 0 / -inf additive) mask."""
    if not (query.is_cuda and query.dtype == torch.bfloat16 and key.dtype == torch.bfloat16):
        return False
    if query.shape[-1] != 128 or query.shape[2] != 1 or query.shape[1] % key.shape[1]:
        return False
    if query.shape[1] // key.shape[1] > _MAX_GROUP:
        return False
    if attention_mask is not None and attention_mask.dtype != torch.bool:
        finite = torch.isfinite(attention_mask)
        if bool((attention_mask[finite] != 0).any()):
            return False
    return True


def _key_ok(attn_mask: Optional[Tensor], attention_mask: Optional[Tensor], B: int, L: int, device):
    """uint8 (rows, L) attended flags and their row stride (0 = shared)."""
    keep = None
    if attn_mask is not None:
        keep = attn_mask.to(device=device, dtype=torch.bool).reshape(-1, L)
    if attention_mask is not None:
        m = attention_mask if attention_mask.dtype == torch.bool else torch.isfinite(attention_mask)
        m = m.to(device).reshape(m.shape[0], -1)[:, -L:].reshape(-1, L)
        keep = m if keep is None else (keep & m)
    if keep is None:
        return None, 0
    if keep.shape[0] not in (1, B):
        raise ValueError(f"mask rows {keep.shape[0]} match neither 1 nor batch {B}")
    keep = keep.to(torch.uint8).contiguous()
    return keep, (L if keep.shape[0] == B else 0)


def decode_attention(query: Tensor, key: Tensor, value: Tensor, parsed_positions, rotary_emb,
                     scaling: Optional[float] = None, attention_mask: Optional[Tensor] = None) -> Tensor:
    """One decode step: ``query`` ``(B, Hq, 1, D)``, ``key`` / ``value`` the
    unrotated ``(B, Hkv, L, D)`` cache (not expanded), ``parsed_positions``
    an ``IterPositions``-like object (``key_pos_ids`` ``(L,)`` or ``(B, L)``,
    ``attn_mask`` or ``None``, ``get_rotary_pos_emb``).  Returns ``(B, Hq, 1,
    D)``; a row whose keys are all masked gives zeros."""
    B, Hq, q_len, D = query.shape
    Hkv, L = key.shape[1], key.shape[2]
    if q_len != 1:
        raise AssertionError("decode_attention takes one query token")
    dev = query.device
    cos, sin = parsed_positions.get_rotary_pos_emb(rotary_emb, key)  # (1 or B, L, D)
    rows = cos.shape[0]
    if rows not in (1, B) or cos.shape[1] != L:
        raise ValueError(f"rotary cos/sin of shape {tuple(cos.shape)} for a batch of {B} x {L} keys")
    half = D // 2
    cs16 = torch.stack([cos[..., :half].float(), sin[..., :half].float()], dim=-1).to(torch.float16)
    cs16 = cs16.reshape(rows * L, half, 2).contiguous()
    key_rows = torch.arange(rows * L, device=dev, dtype=torch.int32).reshape(rows, L)
    key_ok, ok_stride = _key_ok(getattr(parsed_positions, "attn_mask", None), attention_mask, B, L, dev)
    q = query if query.stride(-1) == 1 else query.contiguous()
    k = key if key.stride(-1) == 1 else key.contiguous()
    v = value if value.stride(-1) == 1 else value.contiguous()
    out = torch.empty(B, Hq, 1, D, device=dev, dtype=query.dtype)
    a = _lib.AiAttnDecodeArgs()
    a.batch, a.kv_len, a.num_q_heads, a.num_kv_heads, a.head_dim = B, L, Hq, Hkv, D
    a.dtype = _lib.DTYPE_BF16
    a.scale = float(scaling) if scaling is not None else D ** -0.5
    a.q, a.k, a.v, a.out = _t4(q), _t4(k), _t4(v), _t4(out)
    a.key_rows = key_rows.data_ptr()
    a.key_rows_stride_b = L if rows == B and B > 1 else 0
    a.key_ok = key_ok.data_ptr() if key_ok is not None else None
    a.key_ok_stride_b = ok_stride
    a.rope_cs16 = cs16.data_ptr()
    a.n_pos = rows * L
    a.status = status_word(dev).data_ptr()
    lib = _lib.lib()
    nbytes = ctypes.c_size_t(0)
    _lib.check(lib.ai_attn_decode_workspace(ctypes.byref(a), ctypes.byref(nbytes)), "ai_attn_decode_workspace")
    ws = torch.empty(int(nbytes.value), dtype=torch.uint8, device=dev)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    _lib.check(lib.ai_attn_decode(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)),
               "ai_attn_decode")
    return out
