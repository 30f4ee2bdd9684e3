"""Elementwise + norm + RoPE row shims (h3_inference/kernels/elementwise_norm_rope.py).

Same functions, signatures and env flags as the reference:

* ``rms_norm`` / ``qk_norm``      -- the module itself (reference :19-23)
* ``apply_rotary_emb``           -- H3_FUSED_ROPE: rotate-half RoPE kernel (:25-40)
* ``norm_modulate``              -- H3_FUSED_MODULATE: RMSNorm + gathered
                                    shift / scale in the RMSNorm -> NVFP4 kernel (:69-88)
* ``ada_modulate``               -- H3_FUSED_MODULATE: gathered modulation kernel (:90-102)
* ``norm_rope``                  -- H3_FUSED_ROPE: per-head RMSNorm + RoPE kernel (:104-148)
* ``gate_residual``              -- H3_FUSED_GATE: gathered gate + residual kernel (:150-163)

The gather kernels round to bf16 after every op as torch's bf16 expression
does, so their results equal the stock expression's bit for bit.  The RoPE
kernels write a new tensor (out of place) and leave the input untouched.
Where the reference falls back to ``torch.compile`` of its expression, these
shims run the same expression eagerly (calls the kernels do not cover).

``norm_modulate`` returns the normalized bf16 activation and keeps its
NVFP4 quantization (written by the same kernel) on the tensor, so the NVFP4
linear that consumes it next (``QuantizedActivation``) skips its own
quantization pass.
"""
from __future__ import annotations

import torch
from torch import nn

from h3_engine_b200.kernels._dispatch import MISS, enabled, note_miss


def rms_norm(norm_module: nn.RMSNorm, x: torch.Tensor) -> torch.Tensor:
    return norm_module(x)


def qk_norm(norm_module: nn.RMSNorm, x: torch.Tensor) -> torch.Tensor:
    return norm_module(x)


def _rope_covered(x: torch.Tensor, w, cos, sin) -> bool:
    if not (x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 4):
        return False
    D = x.shape[-1]
    if D not in (64, 128) or cos is None or sin is None or cos.dim() != 2:
        return False
    T, R = cos.shape
    if T != x.shape[1] or sin.shape != cos.shape or R % 2 or R > D or (R // 2) % 8:
        return False
    return w is None or (w.numel() == D and w.is_cuda)


def rope_kernel(x: torch.Tensor, w, eps: float, cos: torch.Tensor, sin: torch.Tensor):
    """Per-head RMSNorm (``w`` not None) + rotate-half RoPE of ``x`` (B, T, H, D)
    with tables ``cos`` / ``sin`` (T, R), into a new tensor, or MISS.  ``x``
    may be a strided view (the q / k slices of one projection output)."""
    from h3_engine_b200 import ops
    if not _rope_covered(x, w, cos, sin):
        return MISS
    B, T, H, D = x.shape
    try:
        x2 = x.view(B * T, H * D)       # rows of the projection output, no copy
    except RuntimeError:
        x2 = x.reshape(B * T, H * D)
    cs, sn = cos, sin
    if B > 1:                           # per-row tables for every batch element
        cs, sn = cs.repeat(B, 1), sn.repeat(B, 1)
    wq = None if w is None else (w if w.dtype == torch.bfloat16 and w.is_contiguous()
                                 else w.detach().to(torch.bfloat16).contiguous())
    out = ops.qk_norm_rope_out(x2, H, D, w=wq, eps=float(eps), cos=cs, sin=sn)
    return out.view(B, T, H, D)


def apply_rotary_emb(hidden_states: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    if enabled("H3_FUSED_ROPE"):
        out = rope_kernel(hidden_states, None, 0.0, cos, sin)
        if out is not MISS:
            return out
        note_miss("rope")
    rotary_dim = cos.shape[-1]
    rot, rest = hidden_states[..., :rotary_dim], hidden_states[..., rotary_dim:]
    c = cos.to(hidden_states.dtype)[None, :, None, :]
    s = sin.to(hidden_states.dtype)[None, :, None, :]
    x1, x2 = rot.chunk(2, dim=-1)
    rot = rot * c + torch.cat((-x2, x1), dim=-1) * s
    return torch.cat((rot, rest), dim=-1).contiguous()


def _norm_modulate_impl(x, norm_weight, eps, scale, shift, indices):
    xn = torch.nn.functional.rms_norm(x, (x.shape[-1],), weight=norm_weight, eps=eps)
    return xn * (1.0 + scale.index_select(0, indices)) + shift.index_select(0, indices)


def _gate_residual_impl(residual, y, gate, indices):
    return residual + gate.index_select(0, indices) * y


def norm_modulate_kernel(x: torch.Tensor, w: torch.Tensor, eps: float, scale: torch.Tensor,
                         shift: torch.Tensor, indices: torch.Tensor):
    """``rms_norm(x, w, eps) * (1 + scale[indices]) + shift[indices]`` (bf16)
    through the RMSNorm -> NVFP4 kernel, or MISS.  The NVFP4 codes, blocked
    scales and global scale of the result ride along on it for the next
    NVFP4 linear."""
    from h3_engine_b200 import ops
    if not (x.is_cuda and x.dtype == torch.bfloat16 and x.dim() >= 2):
        return MISS
    K = x.shape[-1]
    rows = x.numel() // K if K else 0
    if K % 256 or w is None or w.numel() != K or scale.dim() != 2 or scale.shape[-1] != K:
        return MISS
    if shift.shape != scale.shape or indices.dim() != 1 or rows == 0 or rows % indices.numel():
        return MISS
    if not (w.is_cuda and scale.is_cuda and shift.is_cuda and indices.is_cuda):
        return MISS
    idx = _row_indices(indices, rows)
    x2 = x.reshape(rows, K)
    # per-row scratch (rstd, amax) is reused across calls on the device's
    # stream; the outputs are fresh, they ride on the returned tensor
    scratch = _NORM_SCRATCH.setdefault(x.device, {})
    ws = dict(scratch)
    q, sf, gs, y = ops.rmsnorm_quantize(
        x2, _bf16(w), float(eps), shift=_bf16(shift), scale=_bf16(scale), mod_idx=idx,
        return_y=True, ws=ws)
    scratch["rstd"], scratch["amax"] = ws["rstd"], ws["amax"]
    y = y.view(x.shape)
    y._h3b_nvfp4 = (q, sf, gs, y._version)
    return y


_NORM_SCRATCH: dict = {}
_IDX_CACHE: dict = {}


def _bf16(t: torch.Tensor) -> torch.Tensor:
    """``t`` as contiguous bf16 (itself when it already is)."""
    t = t.detach()
    return t if t.dtype == torch.bfloat16 and t.is_contiguous() else t.to(torch.bfloat16).contiguous()


def _row_indices(indices: torch.Tensor, rows: int) -> torch.Tensor:
    """int32 table row per activation row (``indices`` repeated over the
    batch), converted once per indices tensor: the model passes the same
    per-token table indices to every block."""
    key = (indices.device, indices.data_ptr(), indices._version, indices.numel(), rows)
    hit = _IDX_CACHE.get(key)
    if hit is not None and hit[0] is indices:
        return hit[1]
    idx = indices.to(torch.int32)
    if idx.numel() != rows:
        idx = idx.repeat(rows // idx.numel())
    idx = idx.contiguous()
    if len(_IDX_CACHE) > 64:
        _IDX_CACHE.clear()
    _IDX_CACHE[key] = (indices, idx)
    return idx


def norm_modulate(norm_module: nn.RMSNorm, x: torch.Tensor, scale: torch.Tensor,
                  shift: torch.Tensor, indices: torch.Tensor) -> torch.Tensor | None:
    """Fused RMSNorm + gather-modulate, or ``None`` if not covered."""
    if not enabled("H3_FUSED_MODULATE"):
        return None
    w = getattr(norm_module, "weight", None)
    if w is None:
        return None
    out = norm_modulate_kernel(x, w, float(norm_module.eps), scale, shift, indices)
    if out is not MISS:
        return out
    note_miss("norm_modulate_h3")
    return _norm_modulate_impl(x, w, float(norm_module.eps), scale, shift, indices)


def _gather_covered(a: torch.Tensor, tables, indices: torch.Tensor) -> bool:
    if not all(isinstance(t, torch.Tensor) for t in (a, indices, *tables)):
        return False
    if not (a.is_cuda and a.dtype == torch.bfloat16 and a.dim() >= 2 and a.shape[-1] % 8 == 0):
        return False
    C = a.shape[-1]
    if not all(t.is_cuda and t.dtype == torch.bfloat16 and t.dim() == 2 and t.shape[-1] == C
               for t in tables):
        return False
    rows = a.numel() // C
    return (indices.is_cuda and indices.dim() == 1 and indices.numel() > 0
            and rows % indices.numel() == 0 and (a.dim() < 3 or a.shape[-2] == indices.numel()))


def ada_modulate_kernel(normed: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor,
                        indices: torch.Tensor):
    """``normed * (1 + scale[indices]) + shift[indices]`` (bf16 rounding after
    each op, as the stock expression), or MISS."""
    from h3_engine_b200 import ops
    if not _gather_covered(normed, (scale, shift), indices):
        return MISS
    return ops.ada_modulate(normed, scale, shift, indices)


def gate_residual_kernel(residual: torch.Tensor, y: torch.Tensor, gate: torch.Tensor,
                         indices: torch.Tensor):
    """``residual + gate[indices] * y`` (bf16 rounding after each op), or MISS."""
    from h3_engine_b200 import ops
    if not (isinstance(y, torch.Tensor) and isinstance(residual, torch.Tensor)):
        return MISS
    if y.shape != residual.shape or not (y.is_cuda and y.dtype == torch.bfloat16):
        return MISS
    if not _gather_covered(residual, (gate,), indices):
        return MISS
    return ops.gate_residual(residual, y, gate, indices)


def ada_modulate(normed: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor,
                 indices: torch.Tensor) -> torch.Tensor:
    """``normed * (1 + scale[indices]) + shift[indices]``."""
    if enabled("H3_FUSED_MODULATE"):
        out = ada_modulate_kernel(normed, scale, shift, indices)
        if out is not MISS:
            return out
        note_miss("ada_modulate_gather")
    return normed * (1.0 + scale.index_select(0, indices)) + shift.index_select(0, indices)


def _norm_rope_impl(x, weight, eps, cos, sin):
    rotary_dim = cos.shape[-1]
    half = rotary_dim // 2
    xn = torch.nn.functional.rms_norm(x, (x.shape[-1],), weight=weight, eps=eps)
    c1 = cos[None, :, None, :half].to(xn.dtype)
    c2 = cos[None, :, None, half:rotary_dim].to(xn.dtype)
    s1 = sin[None, :, None, :half].to(xn.dtype)
    s2 = sin[None, :, None, half:rotary_dim].to(xn.dtype)
    x1, x2 = xn[..., :half], xn[..., half:rotary_dim]
    return torch.cat((x1 * c1 - x2 * s1, x2 * c2 + x1 * s2, xn[..., rotary_dim:]), dim=-1)


def norm_rope(norm_module: nn.RMSNorm, x: torch.Tensor, cos: torch.Tensor,
              sin: torch.Tensor) -> torch.Tensor | None:
    """Fused qk_norm + RoPE, or ``None`` if this call is not covered."""
    if not enabled("H3_FUSED_ROPE"):
        return None
    w = getattr(norm_module, "weight", None)
    if w is None or cos is None:
        return None
    out = rope_kernel(x, w, float(norm_module.eps), cos, sin)
    if out is not MISS:
        return out
    note_miss("norm_rope_h3")
    return _norm_rope_impl(x, w, float(norm_module.eps), cos, sin)


def gate_residual(residual: torch.Tensor, y: torch.Tensor, gate: torch.Tensor,
                  indices: torch.Tensor) -> torch.Tensor:
    """``residual + gate[indices] * y``."""
    if enabled("H3_FUSED_GATE"):
        out = gate_residual_kernel(residual, y, gate, indices)
        if out is not MISS:
            return out
        note_miss("gate_residual_gather")
    return _gate_residual_impl(residual, y, gate, indices)
