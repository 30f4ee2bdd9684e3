"""CPU oracle for the DiT sub-blocks -- TEST INFRASTRUCTURE ONLY (see
``oracle/nvfp4_ref.py`` for who may import it).

Restates, in numpy:
* RMSNorm as torch computes it for bf16 input (fp32 math, one bf16 rounding
  of ``x * rstd * gamma``): ``h3_inference/kernels/elementwise_norm_rope.py:19-23``;
  pinned against the reference's nn.RMSNorm by ``tests/golden/blocks_golden.npz``.
* adaLN modulation ``norm(x) * (1 + scale[idx]) + shift[idx]``:
  ``h3_inference/kernels/elementwise_norm_rope.py:42-52``.
* The FFN sub-block of the GELU/bias configuration: RMSNorm -> NVFP4 linear
  (+b1) -> GELU-tanh -> NVFP4 re-quantization -> NVFP4 linear (+b2) ->
  residual add (the row shim ``ffn`` at ``h3_inference/kernels/ffn_qkvo_gemms.py:45-54``
  plus ``gate_residual`` at ``h3_inference/kernels/elementwise_norm_rope.py:150-163``
  with gate 1).
Every NVFP4 step uses ``nvfp4_ref.quantize`` (bit-exact recipe) and
fp64-accumulated GEMMs rounded once to bf16.
"""
from __future__ import annotations

import numpy as np

from . import nvfp4_ref as R


def rmsnorm(x, gamma, eps: float, shift=None, scale=None, mod_idx=None) -> np.ndarray:
    """bf16 RMSNorm (+ optional modulation), returned as bf16 values in fp32."""
    x = R.bf16_round(x).astype(np.float64)
    g = R.bf16_round(gamma).astype(np.float64)
    ms = np.mean(x * x, axis=-1, keepdims=True)
    y = x / np.sqrt(ms + eps) * g
    if scale is not None:
        idx = np.zeros(x.shape[0], dtype=np.int64) if mod_idx is None else np.asarray(mod_idx)
        sc = R.bf16_round(scale).astype(np.float64)[idx]
        sh = R.bf16_round(shift).astype(np.float64)[idx]
        y = y * (1.0 + sc) + sh
    return R.bf16_round(y.astype(np.float32))


def nvfp4_linear_from_bf16(a_bf16, qw, sw, gw, bias=None, act=None, residual=None, gs_a=None):
    """Quantize bf16 activations with the recipe (optionally with a given gs),
    GEMM against a quantized weight, epilogue, bf16 out."""
    M = a_bf16.shape[0]
    qa, sa, ga = R.quantize(a_bf16, gs=gs_a)
    y = R.gemm_ref(qa, sa, ga, qw, sw, gw, M, qw.shape[0])
    if bias is not None:
        y = y + R.bf16_round(bias).astype(np.float64)[None, :]
    if act == "gelu_tanh":
        y = R.gelu_tanh(y)
    if residual is not None:
        y = y + R.bf16_round(residual).astype(np.float64)
    return R.bf16_round(y.astype(np.float32)), ga


def ffn_block(x, gamma, eps, w1q, b1, w2q, b2, gs_u=None):
    """FFN sub-block.  ``w1q``/``w2q`` are (q, sf_rowmajor, gs) triples of the
    quantized weights.  ``gs_u`` optionally forces the re-quantization global
    scale (used when checking a row sample of a tensor too large for the
    oracle, with the global scale taken from the full GPU run)."""
    h = rmsnorm(x, gamma, eps)
    u, _ = nvfp4_linear_from_bf16(h, *w1q, bias=b1, act="gelu_tanh")
    y, gu = nvfp4_linear_from_bf16(u, *w2q, bias=b2, residual=x, gs_a=gs_u)
    return y, h, u


def qk_norm_rope(x, w, eps, cos=None, sin=None) -> np.ndarray:
    """Per-head RMSNorm over the last dim then rotate-half RoPE over the first
    R = cos.shape[-1] dims (``h3_inference/kernels/elementwise_norm_rope.py:104-122``).
    ``x``: [T, H, D]; ``cos``/``sin``: [T, R] (rounded to bf16 like the
    reference's ``.to(xn.dtype)``).  fp64 math, one bf16 rounding."""
    x = R.bf16_round(x).astype(np.float64)
    if w is not None:
        ms = np.mean(x * x, axis=-1, keepdims=True)
        x = x / np.sqrt(ms + eps) * R.bf16_round(w).astype(np.float64)
    if cos is not None:
        rd = cos.shape[-1]
        half = rd // 2
        c = R.bf16_round(cos).astype(np.float64)[:, None, :]
        s = R.bf16_round(sin).astype(np.float64)[:, None, :]
        x1, x2 = x[..., :half], x[..., half:rd]
        out = x.copy()
        out[..., :half] = x1 * c[..., :half] - x2 * s[..., :half]
        out[..., half:rd] = x2 * c[..., half:rd] + x1 * s[..., half:rd]
        x = out
    return R.bf16_round(x.astype(np.float32))


def rope_tables(pos, dims, theta: float = 10000.0):
    """(T, 3) positions -> fp32 (cos, sin) of shape (T, sum(dims)) for the
    rotate-half layout ``H3RotaryPosEmbed`` builds
    (``h3_inference/transformer/model.py:23-38``): first half = [t-axis |
    h-axis | w-axis] angles, second half repeats it; generalised to per-axis
    widths with per-axis inv_freq = theta^(-2i/d_axis)."""
    pos = np.asarray(pos, dtype=np.float64)
    freqs = []
    for a, d in enumerate(dims):
        inv = 1.0 / (theta ** (np.arange(0, d, 2, dtype=np.float64) / d))
        freqs.append(pos[:, a:a + 1] * inv[None, :])
    f = np.concatenate(freqs, axis=1)
    f = np.concatenate([f, f], axis=1)
    return np.cos(f).astype(np.float32), np.sin(f).astype(np.float32)


def attention(q, k, v, cu_seqlens, scale: float | None = None, rows=None) -> np.ndarray:
    """Non-causal softmax(q k^T * scale) v per document of a packed sequence
    (``h3_inference/kernels/packed_self_attn.py:31-37`` with a per-document
    mask).  ``q, k, v``: [T, H, D] (bf16 values); fp64 math, fp64 out.
    ``rows`` optionally restricts the output to those query rows."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    T, H, D = q.shape
    sc = D ** -0.5 if scale is None else scale
    rows = np.arange(T) if rows is None else np.asarray(rows)
    out = np.zeros((len(rows), H, D))
    cu = list(cu_seqlens)
    for i, r in enumerate(rows):
        d = int(np.searchsorted(cu, r, side="right")) - 1
        a, b = cu[d], cu[d + 1]
        s = np.einsum("hd,jhd->hj", q[r], k[a:b]) * sc
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        out[i] = np.einsum("hj,jhd->hd", p, v[a:b])
    return out


def attn_block(x, gamma, eps, wq, wk, wv, wo, norm_q, norm_k, qk_eps, heads, cos, sin,
               cu_seqlens, bo=None, shift=None, scale=None, gate=None, mod_idx=None):
    """Attention half of a DiT block: ``x + gate * out_proj(attn(rope(qk_norm(
    qkv_proj(modulate(norm(x)))))))`` with every projection an NVFP4 linear
    (``h3_inference/transformer/model.py:81-106,191-198``).  ``w*`` are (q,
    sf_rowmajor, gs) triples of quantized weights; the projection input is
    quantized once and shared by q, k, v (``h3_inference/nvfp4.py:295-302``)."""
    x = R.bf16_round(x)
    T = x.shape[0]
    h = rmsnorm(x, gamma, eps, shift, scale, mod_idx)
    qa, sa, ga = R.quantize(h)
    outs = []
    for w in (wq, wk, wv):
        y = R.gemm_ref(qa, sa, ga, *w, M=T, N=w[0].shape[0])
        outs.append(R.bf16_round(y.astype(np.float32)))
    HD = outs[0].shape[1]
    D = HD // heads
    q = qk_norm_rope(outs[0].reshape(T, heads, D), norm_q, qk_eps, cos, sin)
    k = qk_norm_rope(outs[1].reshape(T, heads, D), norm_k, qk_eps, cos, sin)
    v = outs[2].reshape(T, heads, D)
    o = R.bf16_round(attention(q, k, v, cu_seqlens).astype(np.float32)).reshape(T, HD)
    qo, so, go = R.quantize(o)
    y = R.gemm_ref(qo, so, go, *wo, M=T, N=wo[0].shape[0])
    if bo is not None:
        y = y + R.bf16_round(bo).astype(np.float64)[None, :]
    if gate is not None:
        idx = np.zeros(T, dtype=np.int64) if mod_idx is None else np.asarray(mod_idx)
        y = y * R.bf16_round(gate).astype(np.float64)[idx]
    y = y + x.astype(np.float64)
    return R.bf16_round(y.astype(np.float32))


def ffn_block_mod(x, gamma, eps, w1q, b1, w2q, b2, shift=None, scale=None, gate=None,
                  mod_idx=None):
    """FFN half with adaLN modulation and gate."""
    x = R.bf16_round(x)
    h = rmsnorm(x, gamma, eps, shift, scale, mod_idx)
    u, _ = nvfp4_linear_from_bf16(h, *w1q, bias=b1, act="gelu_tanh")
    qa, sa, ga = R.quantize(u)
    y = R.gemm_ref(qa, sa, ga, *w2q, M=x.shape[0], N=w2q[0].shape[0])
    if b2 is not None:
        y = y + R.bf16_round(b2).astype(np.float64)[None, :]
    if gate is not None:
        idx = np.zeros(x.shape[0], dtype=np.int64) if mod_idx is None else np.asarray(mod_idx)
        y = y * R.bf16_round(gate).astype(np.float64)[idx]
    y = y + x.astype(np.float64)
    return R.bf16_round(y.astype(np.float32))


def silu_bf16(g):
    """silu of bf16 values computed in fp32 and rounded to bf16 (torch's bf16
    ``F.silu``), h3_inference/transformer/ops.py:62-73."""
    g = np.asarray(g, dtype=np.float32)
    return R.bf16_round((g / (np.float32(1.0) + np.exp(-g))).astype(np.float32))


def swiglu_ffn_block_mod(x, gamma, eps, wupq, wdownq, shift=None, scale=None, gate=None,
                         mod_idx=None):
    """FFN half of the reference-shape block: RMSNorm (+modulation) -> NVFP4
    up-projection to [value | gate] (2F, no bias) -> value * silu(gate), each
    op rounded to bf16 as the reference's bf16 modules do
    (h3_inference/kernels/ffn_qkvo_gemms.py:31-35) -> NVFP4 down-projection
    (no bias) -> adaLN gate and residual.  ``wupq`` is the (q, sf, gs) triple
    of the [2F, d] weight in the reference's [value | gate] row order."""
    x = R.bf16_round(x)
    h = rmsnorm(x, gamma, eps, shift, scale, mod_idx)
    u2, _ = nvfp4_linear_from_bf16(h, *wupq)
    F = u2.shape[1] // 2
    u = R.bf16_round((u2[:, :F] * silu_bf16(u2[:, F:])).astype(np.float32))
    qa, sa, ga = R.quantize(u)
    y = R.gemm_ref(qa, sa, ga, *wdownq, M=x.shape[0], N=wdownq[0].shape[0])
    if gate is not None:
        idx = np.zeros(x.shape[0], dtype=np.int64) if mod_idx is None else np.asarray(mod_idx)
        y = y * R.bf16_round(gate).astype(np.float64)[idx]
    y = y + x.astype(np.float64)
    return R.bf16_round(y.astype(np.float32)), u
