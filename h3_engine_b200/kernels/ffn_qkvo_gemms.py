"""FFN + QKVO GEMM row shims (h3_inference/kernels/ffn_qkvo_gemms.py).

Same functions, signatures and env flags as the reference:

* ``qkv_projection``     -- H3_NVFP4: one activation quantization, one
                            N-concatenated NVFP4 GEMM for q | k | v (:10-22)
* ``out_projection``     -- H3_NVFP4: the NVFP4 GEMM of a quantized linear (:24-29)
* ``ffn``                -- H3_NVFP4: the SwiGLU feed-forward as two NVFP4
                            GEMMs, value * silu(gate) fused into the
                            up-projection's epilogue, its |max| feeding the
                            re-quantization (:45-54); H3_FUSED_SWIGLU alone: the
                            stock expression, eagerly
* ``context_projection`` -- the linear itself (:56-58)

"Quantized" means the linears carry an NVFP4 weight: this library's
``nvfp4._QuantLinear`` (``quantize_blocks`` / ``load_quantized``) or the
reference's own quantized linear (same packed format, read with global
scale 1); other linears take the reference's stock path.
"""
from __future__ import annotations

import torch
from torch import nn

from h3_engine_b200.kernels._dispatch import MISS, enabled, note_miss


def qkv_kernel(to_q, to_k, to_v, x: torch.Tensor):
    from h3_engine_b200 import nvfp4
    if not x.is_cuda:
        return MISS
    out = nvfp4.shared_qkv(to_q, to_k, to_v, x)
    return MISS if out is None else out


def out_kernel(to_out, x: torch.Tensor):
    from h3_engine_b200 import nvfp4
    if not (x.is_cuda and nvfp4._is_quant_linear(to_out)):
        return MISS
    if isinstance(to_out, nvfp4._QuantLinear):
        return to_out(x)
    # the reference's own quantized linear: same weight format, global scale 1
    to_out.calls = getattr(to_out, "calls", 0) + 1
    return nvfp4.QuantizedActivation(x).mm(to_out.weight_nvfp4)


def _swiglu_weight(lin):
    """The up-projection's packed weight with its rows in the order the
    SwiGLU epilogue reads (``ops.swiglu_rows``), cached on the module."""
    from h3_engine_b200 import nvfp4, ops
    w = nvfp4.as_nvfp4_weight(lin.weight_nvfp4)
    cached = getattr(lin, "_h3b_swiglu", None)
    if cached is not None and cached[0] is w:
        return cached[1]
    perm = ops.swiglu_rows(w.out_features // 2).to(w.qdata.device)
    q = w.qdata[perm].contiguous()
    sf_rows = nvfp4._unswizzle(w.scale_u8, w.out_features, w.in_features // nvfp4.FP4_BLOCK)
    sf = nvfp4._swizzle(sf_rows[perm].view(torch.float8_e4m3fn)).view(torch.uint8)
    res = (q, sf, w.global_scale)
    lin._h3b_swiglu = (w, res)
    return res


def ffn_kernel(ff: nn.Module, x: torch.Tensor):
    """``net.2(value * silu(gate))`` with ``value | gate = net.0.proj(x)`` in NVFP4, or MISS."""
    from h3_engine_b200 import nvfp4, ops
    net = getattr(ff, "net", None)
    if net is None or len(net) != 3 or not x.is_cuda or x.dtype != torch.bfloat16:
        return MISS
    gate_mod, down = net[0], net[2]
    up = getattr(gate_mod, "proj", None)
    act_fn = getattr(gate_mod, "activation", None)
    if not (nvfp4._is_quant_linear(up) and nvfp4._is_quant_linear(down)):
        return MISS
    if act_fn is not None and not isinstance(act_fn, nn.SiLU):
        return MISS
    f = up.out_features // 2
    # the GEMMs take K in whole 256-element k-blocks; the SwiGLU epilogue
    # whole 256-column tiles of [value | gate]
    if (up.out_features % 256 or f % 256 or up.in_features % 256 or down.in_features != f
            or up.in_features != x.shape[-1]):
        return MISS
    a = nvfp4.QuantizedActivation(x)
    wq, wsf, wgs = _swiglu_weight(up)
    amax = torch.zeros(1, dtype=torch.float32, device=x.device)
    h = ops.gemm(a.qdata.view(torch.uint8), a.scale_blocked.view(torch.uint8), a.global_scale,
                 a.rows, wq, wsf, wgs, 2 * f, up.in_features, act=ops.ACT_SWIGLU,
                 amax_out=amax)
    qh, sfh, gsh = ops.quantize(h, mpad=ops.pad_m(a.rows), amax_t=amax)
    wd = nvfp4.as_nvfp4_weight(down.weight_nvfp4)
    y = ops.gemm(qh, sfh, gsh, a.rows, wd.qdata, wd.scale_u8, wd.global_scale,
                 down.out_features, f)
    up.calls = getattr(up, "calls", 0) + 1
    down.calls = getattr(down, "calls", 0) + 1
    return y.reshape(*x.shape[:-1], down.out_features)


def qkv_projection(to_q: nn.Linear, to_k: nn.Linear, to_v: nn.Linear,
                   x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    if enabled("H3_NVFP4"):
        out = qkv_kernel(to_q, to_k, to_v, x)
        if out is not MISS:
            return out
        note_miss("qkv_projection")
    return to_q(x), to_k(x), to_v(x)


def out_projection(to_out: nn.Linear, x: torch.Tensor) -> torch.Tensor:
    if enabled("H3_NVFP4"):
        out = out_kernel(to_out, x)
        if out is not MISS:
            return out
        note_miss("out_projection")
    return to_out(x)


def _swiglu_impl(gate_up: torch.Tensor) -> torch.Tensor:
    """``value * silu(gate)`` from the fused ``(T, 2*ffn_dim)`` projection output."""
    value, gate = gate_up.chunk(2, dim=-1)
    return value * torch.nn.functional.silu(gate)


def _swiglu(gate_up: torch.Tensor) -> torch.Tensor:
    return _swiglu_impl(gate_up)


def ffn(ff: nn.Module, x: torch.Tensor) -> torch.Tensor:
    """The SwiGLU feed-forward: ``net.0`` (fused gate+up), ``net.2`` (down)."""
    if enabled("H3_NVFP4"):
        out = ffn_kernel(ff, x)
        if out is not MISS:
            return out
        note_miss("ffn")
    if enabled("H3_FUSED_SWIGLU"):
        return ff.net[2](_swiglu(ff.net[0].proj(x)))
    return ff(x)


def context_projection(linear: nn.Linear, x: torch.Tensor) -> torch.Tensor:
    """Text/video/audio input projections and the two output heads."""
    return linear(x)
