"""Packed self-attention row shim (h3_inference/kernels/packed_self_attn.py:8-37).

``packed_self_attention(query, key, value, attention_mask=None)`` with
``(B, T, H, D)`` tensors: under H3_TL_ATTN, the tcgen05 attention kernel with
each batch element one document of a packed launch, reading the query, key
and value tensors where they lie (strided views of one projection output
need no copy).

An attention mask is taken when it is the one the reference model builds
for padded sequences (h3_inference/transformer/model.py:326-329): ``mask =
is_pad[None, :] == is_pad[:, None]``, i.e. pad rows attend to pad rows and
the others to the others -- two documents of a permuted sequence.  The rows
are gathered into [non-pad | pad] order, attended as two documents per batch
element and scattered back; the permutation is derived once per mask tensor.
Any other mask (or a call the kernel does not take: head_dim other than 128,
more than 64 documents, CPU tensors) runs ``F.scaled_dot_product_attention``
as in the reference.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from h3_engine_b200.kernels._dispatch import MISS, enabled, note_miss

_MAX_DOCS = 64
_MASK_CACHE: dict = {}


def _mask_documents(mask: torch.Tensor, T: int):
    """(perm, n_first) when ``mask`` (bool (T, T), True = attend) is the
    two-class document mask ``c[:, None] == c[None, :]``; None otherwise.
    ``perm`` lists the rows of row 0's class first (n_first of them), then the
    others.  One host sync per mask tensor (cached on its identity)."""
    if mask.dtype != torch.bool or mask.shape != (T, T) or not mask.is_cuda:
        return None
    key = (mask.data_ptr(), mask._version, T)
    hit = _MASK_CACHE.get(key)
    if hit is not None and hit[0] is mask:
        return hit[1]
    cls = mask[0]
    res = None
    if bool(torch.equal(mask, cls[:, None] == cls[None, :])):
        first = torch.nonzero(cls).flatten()
        rest = torch.nonzero(~cls).flatten()
        res = (torch.cat([first, rest]), int(first.numel()))
    if len(_MASK_CACHE) > 8:
        _MASK_CACHE.clear()
    _MASK_CACHE[key] = (mask, res)
    return res


def _covered(query, key, value) -> bool:
    if not all(t.is_cuda and t.dtype == torch.bfloat16 and t.dim() == 4
               for t in (query, key, value)):
        return False
    B, T, H, D = query.shape
    return key.shape == query.shape and value.shape == query.shape and D == 128


def attention_kernel(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                     attention_mask: torch.Tensor | None = None):
    """softmax(Q K^T / sqrt(D)) V per batch element (and per mask document),
    (B, T, H, D) -> (B, T, H, D), or MISS."""
    from h3_engine_b200 import ops
    if not _covered(query, key, value):
        return MISS
    B, T, H, D = query.shape
    rows, hd = B * T, H * D
    if attention_mask is None:
        if B > _MAX_DOCS:
            return MISS
        cu = [b * T for b in range(B + 1)]
        out = ops.attention_qkv(query.reshape(rows, hd), key.reshape(rows, hd),
                                value.reshape(rows, hd), H, D, cu)
        return out.view(B, T, H, D)
    docs = _mask_documents(attention_mask, T)
    if docs is None or 2 * B > _MAX_DOCS:
        return MISS
    perm, n0 = docs
    cu = [0]
    for _ in range(B):
        cu += [cu[-1] + n0, cu[-1] + T]
    cu = sorted(set(cu))                  # an empty class adds no document
    qp, kp, vp = (t.index_select(1, perm).reshape(rows, hd) for t in (query, key, value))
    o = ops.attention_qkv(qp, kp, vp, H, D, cu).view(B, T, H, D)
    out = torch.empty_like(o)
    out.index_copy_(1, perm, o)
    return out


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
    if enabled("H3_TL_ATTN"):
        out = attention_kernel(query, key, value, attention_mask)
        if out is not MISS:
            return out
        note_miss("attention")
    out = F.scaled_dot_product_attention(query.transpose(1, 2), key.transpose(1, 2),
                                         value.transpose(1, 2), attn_mask=attention_mask,
                                         dropout_p=0.0, is_causal=False)
    return out.transpose(1, 2)
