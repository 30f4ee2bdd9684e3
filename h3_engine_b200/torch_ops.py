"""torch custom operators over the C ABI of libh3b.so (namespace ``h3b``).

Each operator launches one C-ABI entry point (include/h3b.h) on the current
CUDA stream of its tensors' device, under a device guard taken from those
tensors (never from whatever device happens to be current), and raises on a
non-zero status.  Outputs are caller-allocated tensors declared as mutated
arguments, so the operators are functional-safe for ``torch.compile`` /
``torch.export``: each has a fake (meta) implementation that does nothing but
declare the mutation, and tracing a caller records ``torch.ops.h3b.*`` nodes
instead of breaking the graph at a foreign call.

Only CUDA implementations are registered: a CPU tensor reaching an operator
is a dispatch error, never a silent fallback.  The tensor-level wrappers in
``ops.py`` allocate outputs, check shapes and call these operators; they are
the functions the rest of the package uses.
"""
from typing import Optional

import torch

from . import _lib


def _p(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _run(t: torch.Tensor, name: str, *args) -> None:
    with torch.cuda.device(t.device):
        st = getattr(_lib.lib(), name)(*args, _stream(t))
    _lib.check(st, name)


def _no_output(*_args, **_kwargs) -> None:
    return None


def _op(name: str, mutates: tuple[str, ...]):
    """Register ``fn`` as ``h3b::name`` (CUDA only) with a fake implementation
    that only declares the mutated outputs."""
    def wrap(fn):
        op = torch.library.custom_op(f"h3b::{name}", mutates_args=mutates, device_types="cuda")(fn)
        op.register_fake(_no_output)
        return op
    return wrap


@_op("amax_bf16", ("out",))
def amax_bf16(x: torch.Tensor, rows: int, cols: int, ldx: int, out: torch.Tensor) -> None:
    """out[0] = max |x| over a [rows, cols] bf16 view with row stride ldx
    (h3b_amax_bf16)."""
    _run(x, "h3b_amax_bf16", _p(x), rows, cols, ldx, _p(out))


@_op("nvfp4_quantize", ("q", "sf", "gs_out"))
def nvfp4_quantize(x: torch.Tensor, rows: int, cols: int, ldx: int, amax: Optional[torch.Tensor],
                   gs_in: float, q: torch.Tensor, sf: torch.Tensor, gs_out: torch.Tensor,
                   layout: int, mpad: int) -> None:
    """E2M1 codes, e4m3 block scales and the fp32 global scale of a bf16
    [rows, cols] view (h3b_nvfp4_quantize); ``amax`` None uses ``gs_in``."""
    _run(q, "h3b_nvfp4_quantize", _p(x) if rows else None, rows, cols, ldx, _p(amax),
         float(gs_in), _p(gs_out), _p(q), _p(sf), layout, mpad)


@_op("nvfp4_dequantize", ("out",))
def nvfp4_dequantize(q: torch.Tensor, sf: torch.Tensor, layout: int, sf_rows: int,
                     gs: Optional[torch.Tensor], rows: int, cols: int, out: torch.Tensor) -> None:
    """bf16 [rows, cols] = (LUT[code] * scale) * gs (h3b_nvfp4_dequantize)."""
    _run(q, "h3b_nvfp4_dequantize", _p(q), _p(sf), layout, sf_rows, _p(gs), rows, cols, _p(out))


@_op("nvfp4_gemm", ("out", "amax_out"))
def nvfp4_gemm(qa: torch.Tensor, sfa: torch.Tensor, gsa: Optional[torch.Tensor], m: int,
               qb: torch.Tensor, sfb: torch.Tensor, gsb: Optional[torch.Tensor], gsb_seg: int,
               n: int, k: int, bias: Optional[torch.Tensor], residual: Optional[torch.Tensor],
               ldr: int, gate: Optional[torch.Tensor], gate_idx: Optional[torch.Tensor], act: int,
               out: torch.Tensor, amax_out: Optional[torch.Tensor]) -> None:
    """Block-scaled NVFP4 GEMM with the fused epilogue (h3b_nvfp4_gemm)."""
    _run(out, "h3b_nvfp4_gemm", _p(qa), _p(sfa), _p(gsa), m, qa.shape[0], _p(qb), _p(sfb),
         _p(gsb), gsb_seg, n, k, _p(bias), _p(residual), ldr, _p(gate), _p(gate_idx), act,
         _p(out), out.stride(0), _p(amax_out))


@_op("rmsnorm_stats", ("rstd", "amax"))
def rmsnorm_stats(x: torch.Tensor, rows: int, cols: int, ldx: int, gamma: torch.Tensor,
                  eps: float, shift: Optional[torch.Tensor], scale: Optional[torch.Tensor],
                  mod_idx: Optional[torch.Tensor], rstd: torch.Tensor,
                  amax: torch.Tensor) -> None:
    """Pass 1 of RMSNorm(+modulation) -> NVFP4: per-row rstd and max |y|
    (h3b_rmsnorm_stats)."""
    _run(gamma, "h3b_rmsnorm_stats", _p(x) if rows else None, rows, cols, ldx, _p(gamma),
         float(eps), _p(shift), _p(scale), _p(mod_idx), _p(rstd), _p(amax))


@_op("rmsnorm_quantize", ("gs_out", "q", "sf", "y_out"))
def rmsnorm_quantize(x: torch.Tensor, rows: int, cols: int, ldx: int, gamma: torch.Tensor,
                     shift: Optional[torch.Tensor], scale: Optional[torch.Tensor],
                     mod_idx: Optional[torch.Tensor], rstd: torch.Tensor, amax: torch.Tensor,
                     gs_out: torch.Tensor, q: torch.Tensor, sf: torch.Tensor, mpad: int,
                     y_out: Optional[torch.Tensor]) -> None:
    """Pass 2: the normalized (modulated) rows as NVFP4 (h3b_rmsnorm_quantize)."""
    _run(gamma, "h3b_rmsnorm_quantize", _p(x) if rows else None, rows, cols, ldx, _p(gamma),
         _p(shift), _p(scale), _p(mod_idx), _p(rstd), _p(amax), _p(gs_out), _p(q), _p(sf),
         mpad, _p(y_out))


@_op("qk_norm_rope", ("buf", "k_buf"))
def qk_norm_rope(buf: torch.Tensor, q_stride: int, q_off: int, k_buf: Optional[torch.Tensor],
                 k_stride: int, k_off: int, rows: int, heads: int, head_dim: int,
                 wq: Optional[torch.Tensor], wk: Optional[torch.Tensor], eps: float,
                 cos: Optional[torch.Tensor], sin: Optional[torch.Tensor], rot: int,
                 cs_stride: int, heads_q: bool, heads_k: bool) -> None:
    """In-place per-head RMSNorm + rotate-half RoPE (h3b_qk_norm_rope).  The
    query heads live in ``buf``; the key heads in ``k_buf``, or in ``buf``
    too when ``k_buf`` is None (one packed q|k|v activation)."""
    kb = buf if k_buf is None else k_buf
    _run(buf, "h3b_qk_norm_rope", _p(buf) if heads_q else None, q_stride, q_off,
         _p(kb) if heads_k else None, k_stride, k_off, rows, heads, head_dim, _p(wq), _p(wk),
         float(eps), _p(cos), _p(sin), rot, cs_stride)


@_op("attention_varlen", ("out",))
def attention_varlen(q_buf: torch.Tensor, q_rows: int, q_stride: int, q_off: int, q_row0: int,
                     kv_buf: torch.Tensor, kv_rows: int, kv_stride: int, k_off: int, v_off: int,
                     heads: int, head_dim: int, cu_seqlens: list[int], scale: float,
                     out: torch.Tensor) -> None:
    """Packed varlen attention per document (h3b_attention_varlen);
    ``cu_seqlens`` are host integers (the launch shape depends on them)."""
    import ctypes
    arr = (ctypes.c_int32 * len(cu_seqlens))(*cu_seqlens)
    _run(out, "h3b_attention_varlen", _p(q_buf), q_rows, q_stride, q_off, q_row0, _p(kv_buf),
         kv_rows, kv_stride, k_off, v_off, heads, head_dim, arr, len(cu_seqlens) - 1,
         float(scale), _p(out), out.stride(0))


@_op("qk_norm_rope_out", ("q_out", "k_out"))
def qk_norm_rope_out(q: Optional[torch.Tensor], q_stride: int, k: Optional[torch.Tensor],
                     k_stride: int, q_out: Optional[torch.Tensor], qo_stride: int,
                     k_out: Optional[torch.Tensor], ko_stride: int, rows: int, heads: int,
                     head_dim: int, wq: Optional[torch.Tensor], wk: Optional[torch.Tensor],
                     eps: float, cos: Optional[torch.Tensor], sin: Optional[torch.Tensor],
                     rot: int, cs_stride: int) -> None:
    """Per-head RMSNorm + RoPE from q / k into q_out / k_out (h3b_qk_norm_rope_out)."""
    ref = q_out if q_out is not None else k_out
    _run(ref, "h3b_qk_norm_rope_out", _p(q), q_stride, _p(k), k_stride, _p(q_out), qo_stride,
         _p(k_out), ko_stride, rows, heads, head_dim, _p(wq), _p(wk), float(eps), _p(cos),
         _p(sin), rot, cs_stride)


@_op("attention_qkv", ("out",))
def attention_qkv(q: torch.Tensor, q_stride: int, k: torch.Tensor, k_stride: int,
                  v: torch.Tensor, v_stride: int, rows: int, heads: int, head_dim: int,
                  cu_seqlens: list[int], scale: float, out: torch.Tensor) -> None:
    """Packed varlen attention over separate q, k, v rows (h3b_attention_qkv)."""
    import ctypes
    arr = (ctypes.c_int32 * len(cu_seqlens))(*cu_seqlens)
    _run(out, "h3b_attention_qkv", _p(q), q_stride, _p(k), k_stride, _p(v), v_stride, rows,
         heads, head_dim, arr, len(cu_seqlens) - 1, float(scale), _p(out), out.stride(0))


@_op("gate_residual", ("out",))
def gate_residual(residual: torch.Tensor, ldr: int, y: torch.Tensor, ldy: int,
                  gate: torch.Tensor, idx: Optional[torch.Tensor], n_idx: int, rows: int,
                  cols: int, out: torch.Tensor, ldo: int) -> None:
    """out = residual + gate[idx] * y, torch's bf16 rounding (h3b_gate_residual)."""
    _run(out, "h3b_gate_residual", _p(residual), ldr, _p(y), ldy, _p(gate), _p(idx), n_idx, rows,
         cols, _p(out), ldo)


@_op("ada_modulate", ("out",))
def ada_modulate(x: torch.Tensor, ldx: int, scale: torch.Tensor, shift: torch.Tensor,
                 idx: Optional[torch.Tensor], n_idx: int, rows: int, cols: int,
                 out: torch.Tensor, ldo: int) -> None:
    """out = x * (1 + scale[idx]) + shift[idx], torch's bf16 rounding (h3b_ada_modulate)."""
    _run(out, "h3b_ada_modulate", _p(x), ldx, _p(scale), _p(shift), _p(idx), n_idx, rows, cols,
         _p(out), ldo)


@_op("amax_exchange", ("amax",))
def amax_exchange(amax: torch.Tensor, slot_table: torch.Tensor, rank: int, world: int,
                  epoch: int, limit_us: int) -> None:
    """amax[0] = max over the ranks of each rank's amax[0], through peer
    memory (h3b_amax_exchange); slot_table: int64 [world] device pointers."""
    _run(amax, "h3b_amax_exchange", _p(amax), _p(slot_table), rank, world, epoch, limit_us)
