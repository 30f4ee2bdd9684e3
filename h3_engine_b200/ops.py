"""Tensor-level wrappers over the C ABI (torch owns the memory, the kernels
run on the current CUDA stream).

These are the building blocks the reference-shaped API in ``nvfp4.py`` and
the row shims in ``kernels/`` are written with.  Every function checks
dtype / device / contiguity on the host and raises on a non-zero status.
"""
from __future__ import annotations

import torch

from . import _lib  # noqa: F401  (loaded by the operators; kept for callers of ops._lib)
from . import torch_ops  # noqa: F401  (registers torch.ops.h3b.*)

_H3B = torch.ops.h3b

SF_ROWMAJOR = 0
SF_SWIZZLED = 1
ACT_NONE = 0
ACT_GELU_TANH = 1
ACT_SWIGLU = 2


def swiglu_rows(ffn_dim: int) -> torch.Tensor:
    """Row order of a fused SwiGLU up-projection weight ([value | gate], 2F
    rows, the reference's chunk order) that the ACT_SWIGLU epilogue reads:
    per 256 rows, value f..f+63, gate f..f+63, value f+64..f+127, gate
    f+64..f+127 (f = 128 t), so one epilogue warp holds a value column and its
    gate.  ``w[swiglu_rows(F)]`` permutes rows; NVFP4 block scales are per row
    and the global scale is the whole tensor's, so quantizing the permuted
    weight gives the permuted rows of the quantized weight."""
    if ffn_dim % 128:
        raise ValueError("SwiGLU ffn_dim must be a multiple of 128")
    idx = []
    for t in range(ffn_dim // 128):
        for half in range(2):
            base = 128 * t + 64 * half
            idx.extend(range(base, base + 64))
            idx.extend(range(ffn_dim + base, ffn_dim + base + 64))
    return torch.tensor(idx, dtype=torch.long)
M_ALIGN = 128


def _need_cuda(*ts: torch.Tensor | None) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("h3b ops take CUDA tensors (there is no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} vs {t.device}")
    assert dev is not None
    return dev


def pad_m(m: int) -> int:
    return ((m + M_ALIGN - 1) // M_ALIGN) * M_ALIGN


def swizzled_sf_bytes(rows: int, k: int) -> int:
    """Bytes of a swizzled scale buffer for ``rows`` x ``k`` values (rows padded to 128)."""
    return pad_m(rows) * (k // 16)


def amax(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 ``[1]`` tensor = max |x| (bf16 ``x``, last dim contiguous)."""
    dev = _need_cuda(x)
    if x.dtype != torch.bfloat16:
        raise TypeError("amax expects bf16")
    x2 = x.reshape(-1, x.shape[-1]) if x.dim() != 2 else x
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    if out is None:
        out = torch.empty(1, dtype=torch.float32, device=dev)
    _H3B.amax_bf16(x2, x2.shape[0], x2.shape[1], x2.stride(0), out)
    return out


def quantize(x: torch.Tensor, *, mpad: int | None = None, layout: int = SF_SWIZZLED,
             amax_t: torch.Tensor | None = None, gs: float | None = None,
             q_out: torch.Tensor | None = None, sf_out: torch.Tensor | None = None,
             gs_out: torch.Tensor | None = None):
    """bf16 ``[M, K]`` -> (q u8 ``[Mpad, K/2]``, sf u8 (layout), gs fp32 ``[1]``).

    The global scale comes from ``gs`` when given (``gs=1.0`` is the
    reference's two-level scheme), else from ``amax_t`` (a device scalar some
    producer already reduced), else from an amax pass over ``x``.
    """
    dev = _need_cuda(x)
    if x.dtype != torch.bfloat16:
        raise TypeError("quantize expects bf16")
    x2 = x.reshape(-1, x.shape[-1]) if x.dim() != 2 else x
    if x2.stride(-1) != 1 or x2.stride(0) % 8:
        x2 = x2.contiguous()
    M, K = x2.shape
    Mp = M if mpad is None else int(mpad)
    if layout == SF_SWIZZLED and Mp % M_ALIGN:
        Mp = pad_m(Mp)
    if q_out is None:
        q_out = torch.empty(Mp, K // 2, dtype=torch.uint8, device=dev)
    if sf_out is None:
        sf_out = torch.empty(Mp * (K // 16), dtype=torch.uint8, device=dev)
    if gs_out is None:
        gs_out = torch.empty(1, dtype=torch.float32, device=dev)
    if q_out.numel() < Mp * (K // 2) or sf_out.numel() < Mp * (K // 16):
        raise ValueError("output buffers too small")
    if gs is None and amax_t is None:
        amax_t = amax(x2)
    _H3B.nvfp4_quantize(x2, M, K, x2.stride(0), amax_t if gs is None else None,
                        float(gs if gs is not None else 0.0), q_out, sf_out, gs_out, layout, Mp)
    return q_out, sf_out, gs_out


def dequantize(q: torch.Tensor, sf: torch.Tensor, gs: torch.Tensor | None, M: int, K: int, *,
               layout: int = SF_SWIZZLED, sf_rows: int | None = None,
               out: torch.Tensor | None = None) -> torch.Tensor:
    dev = _need_cuda(q, sf, gs)
    rows = sf_rows if sf_rows is not None else (q.shape[0] if q.dim() == 2 else M)
    if out is None:
        out = torch.empty(M, K, dtype=torch.bfloat16, device=dev)
    _H3B.nvfp4_dequantize(q, sf, layout, rows, gs, M, K, out)
    return out


def gemm(qa: torch.Tensor, sfa: torch.Tensor, gsa: torch.Tensor | None, M: int,
         qb: torch.Tensor, sfb: torch.Tensor, gsb: torch.Tensor | None, N: int, K: int, *,
         gsb_seg: int = 0, bias: torch.Tensor | None = None,
         residual: torch.Tensor | None = None, act: int = ACT_NONE,
         gate: torch.Tensor | None = None, gate_idx: torch.Tensor | None = None,
         out: torch.Tensor | None = None, amax_out: torch.Tensor | None = None) -> torch.Tensor:
    """``out[M, N] = epilogue(gsa*gsb * deq(qa) @ deq(qb)^T)`` in bf16
    (``out[M, N/2]`` for ``act=ACT_SWIGLU`` with ``qb`` in ``swiglu_rows`` order).

    ``qa``: u8 ``[a_rows, K/2]`` (a_rows % 128 == 0) with swizzled ``sfa``;
    ``qb``: u8 ``[N, K/2]`` with swizzled ``sfb``.  ``amax_out`` (fp32 [1],
    zeroed by the caller) receives max |out| for a following re-quantization.
    """
    dev = _need_cuda(qa, sfa, gsa, qb, sfb, gsb, bias, residual, out, amax_out)
    if qa.dtype != torch.uint8 or qb.dtype != torch.uint8:
        raise TypeError("packed operands must be uint8")
    a_rows = qa.shape[0]
    n_out = N // 2 if act == ACT_SWIGLU else N
    if act == ACT_SWIGLU and (bias is not None or residual is not None or gate is not None):
        raise ValueError("the SwiGLU epilogue takes no bias, residual or gate")
    if out is None:
        out = torch.empty(M, n_out, dtype=torch.bfloat16, device=dev)
    if bias is not None and (bias.dtype != torch.bfloat16 or bias.numel() != N):
        raise ValueError("bias must be bf16 [N]")
    if residual is not None and (residual.dtype != torch.bfloat16 or residual.stride(-1) != 1):
        raise ValueError("residual must be bf16 with a contiguous last dim")
    ldr = residual.stride(0) if residual is not None else 0
    if gate is not None and (gate.dtype != torch.bfloat16 or gate.shape[-1] != N
                             or not gate.is_contiguous()):
        raise ValueError("gate must be a contiguous bf16 [rows, N] table")
    if gate_idx is not None and gate_idx.dtype != torch.int32:
        gate_idx = gate_idx.to(torch.int32)
    _H3B.nvfp4_gemm(qa, sfa, gsa, M, qb, sfb, gsb, gsb_seg, N, K, bias, residual, ldr, gate,
                    gate_idx, act, out, amax_out)
    return out


def rmsnorm_quantize(x: torch.Tensor, gamma: torch.Tensor, eps: float, *,
                     shift: torch.Tensor | None = None, scale: torch.Tensor | None = None,
                     mod_idx: torch.Tensor | None = None, mpad: int | None = None,
                     return_y: bool = False, ws: dict | None = None, amax_hook=None):
    """Fused RMSNorm(+modulation) -> NVFP4.  Returns (q, sf_swizzled, gs[, y]).

    ``ws`` optionally carries preallocated buffers (keys rstd, amax, q, sf, gs, y).
    ``amax_hook(amax)`` runs between the two passes (e.g. a max all-reduce so
    that token shards quantize with the global scale of the whole tensor).
    """
    dev = _need_cuda(x, gamma, shift, scale, mod_idx)
    x2 = x.reshape(-1, x.shape[-1]) if x.dim() != 2 else x
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    M, K = x2.shape
    Mp = pad_m(M if mpad is None else mpad)
    ws = {} if ws is None else ws

    def buf(name, n, dtype):
        t = ws.get(name)
        if t is None or t.numel() < n or t.dtype != dtype:
            t = torch.empty(n, dtype=dtype, device=dev)
            ws[name] = t
        return t[:n]

    rstd = buf("rstd", max(M, 1), torch.float32)
    am = buf("amax", 1, torch.float32)
    q = buf("q", Mp * (K // 2), torch.uint8).view(Mp, K // 2)
    sf = buf("sf", Mp * (K // 16), torch.uint8)
    gs = buf("gs", 1, torch.float32)
    y = buf("y", M * K, torch.bfloat16).view(M, K) if return_y else None
    if mod_idx is not None and mod_idx.dtype != torch.int32:
        mod_idx = mod_idx.to(torch.int32)
    _H3B.rmsnorm_stats(x2, M, K, x2.stride(0), gamma, float(eps), shift, scale, mod_idx, rstd,
                       am)
    if amax_hook is not None:
        amax_hook(am)
    _H3B.rmsnorm_quantize(x2, M, K, x2.stride(0), gamma, shift, scale, mod_idx, rstd, am, gs, q,
                          sf, Mp, y)
    return (q, sf, gs, y) if return_y else (q, sf, gs)


def qk_norm_rope(qkv: torch.Tensor, heads: int, head_dim: int, *, q_off: int, k_off: int,
                 wq: torch.Tensor | None, wk: torch.Tensor | None, eps: float,
                 cos: torch.Tensor | None = None, sin: torch.Tensor | None = None,
                 k_buf: torch.Tensor | None = None, heads_q: bool = True,
                 heads_k: bool = True) -> torch.Tensor:
    """In-place per-head RMSNorm + rotate-half RoPE on the query heads of
    ``qkv`` (at ``q_off``) and the key heads of ``k_buf`` (default ``qkv``, at
    ``k_off``), both bf16 ``[T, stride]``.  ``cos``/``sin``: fp32 ``[T, R]``.
    ``heads_q`` / ``heads_k`` False skips the query / key heads."""
    if not (heads_q or heads_k):
        raise ValueError("nothing to do: both query and key heads skipped")
    dev = _need_cuda(qkv, wq, wk, cos, sin, k_buf)
    q2 = qkv.reshape(-1, qkv.shape[-1]) if qkv.dim() != 2 else qkv
    k2 = q2 if k_buf is None else (k_buf.reshape(-1, k_buf.shape[-1]) if k_buf.dim() != 2 else k_buf)
    for t in (q2, k2):
        if t.dtype != torch.bfloat16 or t.stride(-1) != 1:
            raise ValueError("q / k buffers must be bf16 with a contiguous last dim")
    T = q2.shape[0]
    if k2.shape[0] != T:
        raise ValueError("q and k buffers must have the same number of rows")
    R, cs = 0, 0
    if cos is not None:
        if cos.dtype != torch.float32 or sin is None or sin.dtype != torch.float32:
            raise TypeError("cos/sin must be fp32")
        cos = cos.reshape(T, -1)
        sin = sin.reshape(T, -1)
        if (cos.stride(-1) != 1 or sin.stride(-1) != 1 or cos.stride(0) != sin.stride(0)
                or cos.stride(0) % 4 or cos.storage_offset() % 4 or sin.storage_offset() % 4):
            cos, sin = cos.contiguous().clone(), sin.contiguous().clone()
        R, cs = cos.shape[1], cos.stride(0)
    _H3B.qk_norm_rope(q2, q2.stride(0), q_off, None if k2 is q2 else k2, k2.stride(0), k_off, T,
                      heads, head_dim, wq, wk, float(eps), cos, sin, R, cs, heads_q, heads_k)
    return qkv


def attention_varlen(qkv: torch.Tensor, heads: int, head_dim: int, cu_seqlens, *, q_off: int,
                     k_off: int, v_off: int, scale: float | None = None,
                     out: torch.Tensor | None = None, kv: torch.Tensor | None = None,
                     q_row0: int = 0) -> torch.Tensor:
    """Non-causal attention per document of a packed sequence.

    ``qkv``: bf16 ``[rows, stride]`` holding the query heads at ``q_off``
    (and, when ``kv`` is None, the key / value heads at ``k_off`` / ``v_off``).
    ``kv``: optional bf16 ``[T, stride]`` with the keys / values of the whole
    sequence (token-sharded runs: ``qkv`` is the local shard whose first row is
    global row ``q_row0``).  ``cu_seqlens``: host sequence of global document
    boundaries.  Returns ``[rows, heads*head_dim]`` bf16."""
    dev = _need_cuda(qkv, out, kv)
    q2 = qkv.reshape(-1, qkv.shape[-1]) if qkv.dim() != 2 else qkv
    kv2 = q2 if kv is None else (kv.reshape(-1, kv.shape[-1]) if kv.dim() != 2 else kv)
    for t in (q2, kv2):
        if t.dtype != torch.bfloat16 or t.stride(-1) != 1:
            raise ValueError("q / kv buffers must be bf16 with a contiguous last dim")
    rows = q2.shape[0]
    cu = [int(v) for v in (cu_seqlens.tolist() if hasattr(cu_seqlens, "tolist") else cu_seqlens)]
    if out is None:
        out = torch.empty(rows, heads * head_dim, dtype=torch.bfloat16, device=dev)
    sc = float(scale) if scale is not None else head_dim ** -0.5
    _H3B.attention_varlen(q2, rows, q2.stride(0), q_off, q_row0, kv2, kv2.shape[0], kv2.stride(0),
                          k_off, v_off, heads, head_dim, cu, sc, out)
    return out


def _rows2d(t: torch.Tensor) -> torch.Tensor:
    """A [rows, C] view with a contiguous last dim and 8-element row stride
    (a copy only when the layout needs one)."""
    t2 = t.reshape(-1, t.shape[-1]) if t.dim() != 2 else t
    if t2.stride(-1) != 1 or t2.stride(0) % 8 or t2.storage_offset() % 8:
        t2 = t2.contiguous()
    return t2


def qk_norm_rope_out(x: torch.Tensor, heads: int, head_dim: int, *, w: torch.Tensor | None,
                     eps: float, cos: torch.Tensor | None, sin: torch.Tensor | None,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """Per-head RMSNorm (``w``) + rotate-half RoPE of ``x`` [rows, heads*head_dim]
    (any row stride) into a new contiguous ``out``; ``x`` is left untouched.
    ``cos``/``sin``: fp32 [rows, R]."""
    dev = _need_cuda(x, w, cos, sin, out)
    x2 = _rows2d(x)
    if x2.dtype != torch.bfloat16 or x2.shape[1] != heads * head_dim:
        raise ValueError("x must be bf16 [rows, heads * head_dim]")
    T = x2.shape[0]
    if out is None:
        out = torch.empty(T, heads * head_dim, dtype=torch.bfloat16, device=dev)
    R, cs = 0, 0
    if cos is not None:
        cos, sin = cos.reshape(T, -1), sin.reshape(T, -1)
        if cos.dtype != torch.float32 or sin.dtype != torch.float32:
            cos, sin = cos.float(), sin.float()
        if (cos.stride(-1) != 1 or sin.stride(-1) != 1 or cos.stride(0) != sin.stride(0)
                or cos.stride(0) % 4 or cos.storage_offset() % 4 or sin.storage_offset() % 4):
            cos, sin = cos.contiguous(), sin.contiguous()
        R, cs = cos.shape[1], cos.stride(0)
    _H3B.qk_norm_rope_out(x2, x2.stride(0), None, 0, out, out.stride(0), None, 0, T, heads,
                          head_dim, w, None, float(eps), cos, sin, R, cs)
    return out


def attention_qkv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int, head_dim: int,
                  cu_seqlens, *, scale: float | None = None,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """Attention per document over separate q, k, v activations
    [rows, heads*head_dim] (any row strides): no concatenation of k and v."""
    dev = _need_cuda(q, k, v, out)
    q2, k2, v2 = _rows2d(q), _rows2d(k), _rows2d(v)
    for t in (q2, k2, v2):
        if t.dtype != torch.bfloat16 or t.shape != q2.shape:
            raise ValueError("q, k, v must be bf16 [rows, heads * head_dim] of one shape")
    rows = q2.shape[0]
    cu = [int(c) for c in (cu_seqlens.tolist() if hasattr(cu_seqlens, "tolist") else cu_seqlens)]
    if out is None:
        out = torch.empty(rows, heads * head_dim, dtype=torch.bfloat16, device=dev)
    sc = float(scale) if scale is not None else head_dim ** -0.5
    _H3B.attention_qkv(q2, q2.stride(0), k2, k2.stride(0), v2, v2.stride(0), rows, heads,
                       head_dim, cu, sc, out)
    return out


def _table_rows(idx: torch.Tensor | None, dev) -> tuple[torch.Tensor | None, int]:
    if idx is None:
        return None, 0
    if idx.dtype != torch.int32 or not idx.is_contiguous():
        idx = idx.to(torch.int32).contiguous()
    return idx, idx.numel()


def gate_residual(residual: torch.Tensor, y: torch.Tensor, gate: torch.Tensor,
                  idx: torch.Tensor | None, out: torch.Tensor | None = None) -> torch.Tensor:
    """``residual + gate[idx] * y`` with torch's bf16 rounding after each op;
    ``residual``/``y`` [..., C] bf16, ``gate`` bf16 [n, C], ``idx`` per row,
    repeating over leading dims (row r uses ``idx[r % len(idx)]``)."""
    dev = _need_cuda(residual, y, gate, idx, out)
    r2, y2 = _rows2d(residual), _rows2d(y)
    g2 = gate.reshape(-1, gate.shape[-1]).contiguous()
    rows, C = r2.shape
    if y2.shape != r2.shape or g2.shape[1] != C:
        raise ValueError("residual, y and gate must agree on [rows, C]")
    i2, n = _table_rows(idx, dev)
    if out is None:
        out = torch.empty(residual.shape, dtype=torch.bfloat16, device=dev)
    o2 = out.view(rows, C)
    _H3B.gate_residual(r2, r2.stride(0), y2, y2.stride(0), g2, i2, n, rows, C, o2, o2.stride(0))
    return out


def ada_modulate(x: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor,
                 idx: torch.Tensor | None, out: torch.Tensor | None = None) -> torch.Tensor:
    """``x * (1 + scale[idx]) + shift[idx]`` with torch's bf16 rounding after
    each op (tables bf16 [n, C], row r uses ``idx[r % len(idx)]``)."""
    dev = _need_cuda(x, scale, shift, idx, out)
    x2 = _rows2d(x)
    rows, C = x2.shape
    sc = scale.reshape(-1, C).contiguous()
    sh = shift.reshape(-1, C).contiguous()
    i2, n = _table_rows(idx, dev)
    if out is None:
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=dev)
    o2 = out.view(rows, C)
    _H3B.ada_modulate(x2, x2.stride(0), sc, sh, i2, n, rows, C, o2, o2.stride(0))
    return out
