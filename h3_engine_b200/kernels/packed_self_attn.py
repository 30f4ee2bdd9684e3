"""Packed self-attention row shim (h3_inference/kernels/packed_self_attn.py:8-37).

``packed_self_attention(query, key, value, attention_mask=None)`` with
``(B, T, H, D)`` tensors: under H3_TL_ATTN and without a mask, the tcgen05
attention kernel, each batch element one document of the packed launch;
otherwise (or for a call the kernel does not take: head_dim other than 128,
more than 64 batch elements, CPU tensors) ``F.scaled_dot_product_attention``
as in the reference.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from h3_engine_b200.kernels._dispatch import MISS, enabled, note_miss

_MAX_DOCS = 64


def attention_kernel(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor):
    """softmax(Q K^T / sqrt(D)) V per batch element, (B, T, H, D) -> (B, T, H, D), or MISS."""
    from h3_engine_b200 import ops
    if not all(t.is_cuda and t.dtype == torch.bfloat16 and t.dim() == 4
               for t in (query, key, value)):
        return MISS
    B, T, H, D = query.shape
    if key.shape != query.shape or value.shape != query.shape or D != 128 or B > _MAX_DOCS:
        return MISS
    rows, hd = B * T, H * D
    q2 = query.reshape(rows, hd)
    if q2.stride(-1) != 1 or q2.stride(0) % 8 or q2.data_ptr() % 16:
        q2 = q2.contiguous()
    # keys and values side by side in one [rows, 2*H*D] buffer (the kernel's
    # K|V operand; in the model they come from different tensors anyway:
    # the keys out of qk-norm + RoPE, the values out of the projection)
    kv = torch.cat([key.reshape(rows, hd), value.reshape(rows, hd)], dim=1)
    cu = [b * T for b in range(B + 1)]
    out = ops.attention_varlen(q2, H, D, cu, q_off=0, k_off=0, v_off=hd, kv=kv)
    return out.view(B, T, H, D)


def attention_kernel_flat(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                          heads: int):
    """The plug-point form: ``(B, T, H*D)`` tensors and the head count."""
    b, t, hd = query.shape
    if hd % heads:
        return MISS
    d = hd // heads
    out = attention_kernel(query.view(b, t, heads, d), key.view(b, t, heads, d),
                           value.view(b, t, heads, d))
    return out if out is MISS else out.view(b, t, hd)


def packed_self_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                          attention_mask: torch.Tensor | None = None) -> torch.Tensor:
    """Full self-attention over the packed sequence; ``(B, T, H, D)`` in and out."""
    if attention_mask is None and enabled("H3_TL_ATTN"):
        out = attention_kernel(query, key, value)
        if out is not MISS:
            return out
        note_miss("attention")
    out = F.scaled_dot_product_attention(query.transpose(1, 2), key.transpose(1, 2),
                                         value.transpose(1, 2), attn_mask=attention_mask,
                                         dropout_p=0.0, is_causal=False)
    return out.transpose(1, 2)
