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


# ----------------------------------------------------------------------------- full-size row samples
# The configured sub-block sizes (33784 or 2 x 33784 tokens, hidden 3072) are
# too large for the fp64 helpers above on every row, but attention needs the
# keys and values of every row of a document.  These helpers compute the
# key / value projections of ALL rows (recipe-quantized activations and
# weights, decoded exactly to fp32, one fp32 GEMM on the host's cores --
# relative error ~1e-6 against the fp64 path, far inside the 1e-2 bar) and
# everything query-side only for a sample of rows, in fp64 as above.

def _row_chunks(n: int, chunk: int = 4096):
    for a in range(0, n, chunk):
        yield a, min(n, a + chunk)


def rmsnorm_all(x, gamma, eps, shift=None, scale=None, mod_idx=None) -> np.ndarray:
    """``rmsnorm`` over every row, in row chunks (bounded fp64 temporaries)."""
    out = np.empty(x.shape, dtype=np.float32)
    for a, b in _row_chunks(x.shape[0]):
        idx = None if mod_idx is None else np.asarray(mod_idx)[a:b]
        out[a:b] = rmsnorm(x[a:b], gamma, eps, shift, scale, idx)
    return out


def _decoded_weight_f32(w):
    """(q, sf_rowmajor, gs) -> fp32 torch [N, K] holding LUT[code] * s (exact),
    and gs separately."""
    import torch
    q, s, g = w
    return torch.from_numpy(R.dequantize_f32(q, s, np.float32(1.0))), np.float32(g)


def project_all_rows(h, gs_h, weights, chunk: int = 4096):
    """bf16 ``h`` [T, K] quantized with the fixed global scale ``gs_h`` (so
    row chunks quantize exactly as the whole tensor would), times each weight
    triple: returns one fp32 [T, N] array of bf16 values per weight."""
    import torch
    dec = [_decoded_weight_f32(w) for w in weights]
    outs = [np.empty((h.shape[0], d.shape[0]), dtype=np.float32) for d, _ in dec]
    for a, b in _row_chunks(h.shape[0], chunk):
        qa, sa, ga = R.quantize(h[a:b], gs=gs_h)
        A = torch.from_numpy(R.dequantize_f32(qa, sa, np.float32(1.0)))
        for o, (Wd, gw) in zip(outs, dec):
            y = (A @ Wd.T).numpy().astype(np.float64) * (float(ga) * float(gw))
            o[a:b] = R.bf16_round(y.astype(np.float32))
    return outs


def attention_rows(q_rows, rows, k, v, cu_seqlens, scale: float | None = None) -> np.ndarray:
    """``attention`` for the query rows ``rows`` (``q_rows`` [S, H, D]) against
    the full ``k``, ``v`` [T, H, D]: fp64, one BLAS product per head and row
    group of a document."""
    q_rows = np.asarray(q_rows, dtype=np.float64)
    S, H, D = q_rows.shape
    sc = D ** -0.5 if scale is None else scale
    out = np.zeros((S, H, D))
    cu = list(cu_seqlens)
    doc = np.searchsorted(cu, np.asarray(rows), side="right") - 1
    for d in np.unique(doc):
        sel = np.nonzero(doc == d)[0]
        a, b = cu[d], cu[d + 1]
        for hh in range(H):
            kh = np.asarray(k[a:b, hh], dtype=np.float64)
            vh = np.asarray(v[a:b, hh], dtype=np.float64)
            s = q_rows[sel, hh] @ kh.T * sc
            s -= s.max(axis=1, keepdims=True)
            p = np.exp(s)
            p /= p.sum(axis=1, keepdims=True)
            out[sel, hh] = p @ vh
    return out


def attn_block_rows(x, rows, gamma, eps, wq, wk, wv, wo, norm_q, norm_k, qk_eps, heads, cos,
                    sin, cu_seqlens, gs_o, shift=None, scale=None, gate=None, mod_idx=None):
    """``attn_block`` for the output rows ``rows`` of a full-size packed
    sequence ``x`` [T, d].  Keys and values are computed for every row (the
    norm's global scale is the whole tensor's, as in ``attn_block``); the
    attention output exists only for the sampled rows here, so its
    re-quantization uses the given global scale ``gs_o`` (the amax of the full
    output comes from the run being checked).  Returns the sampled rows."""
    x = R.bf16_round(x)
    rows = np.asarray(rows)
    T = x.shape[0]
    h = rmsnorm_all(x, gamma, eps, shift, scale, mod_idx)
    gs_h = R.global_scale(np.max(np.abs(h)))
    k, v = project_all_rows(h, gs_h, (wk, wv))
    HD = k.shape[1]
    D = HD // heads
    k = k.reshape(T, heads, D)
    for a, b in _row_chunks(T):
        k[a:b] = qk_norm_rope(k[a:b], norm_k, qk_eps, cos[a:b], sin[a:b])
    v = v.reshape(T, heads, D)
    hs = h[rows]
    qa, sa, ga = R.quantize(hs, gs=gs_h)
    qs = R.bf16_round(R.gemm_ref(qa, sa, ga, *wq, M=len(rows), N=HD).astype(np.float32))
    qs = qk_norm_rope(qs.reshape(len(rows), heads, D), norm_q, qk_eps, cos[rows], sin[rows])
    o = R.bf16_round(attention_rows(qs, rows, k, v, cu_seqlens).astype(np.float32))
    qo, so, go = R.quantize(o.reshape(len(rows), HD), gs=gs_o)
    y = R.gemm_ref(qo, so, go, *wo, M=len(rows), N=wo[0].shape[0])
    if gate is not None:
        idx = np.zeros(T, dtype=np.int64) if mod_idx is None else np.asarray(mod_idx)
        y = y * R.bf16_round(gate).astype(np.float64)[idx[rows]]
    y = y + x[rows].astype(np.float64)
    return R.bf16_round(y.astype(np.float32)), gs_h


def ffn_block_rows(x_rows, row_idx, gamma, eps, w1q, b1, w2q, b2, gs_h, gs_u, shift=None,
                   scale=None, gate=None):
    """``ffn_block_mod`` on a sample of rows (``row_idx`` their modulation
    rows), with both activation quantizations at given global scales (the
    amaxes of the full tensors come from the run being checked)."""
    x = R.bf16_round(x_rows)
    h = rmsnorm(x, gamma, eps, shift, scale, row_idx)
    u, _ = nvfp4_linear_from_bf16(h, *w1q, bias=b1, act="gelu_tanh", gs_a=gs_h)
    qa, sa, ga = R.quantize(u, gs=gs_u)
    y = R.gemm_ref(qa, sa, ga, *w2q, M=x.shape[0], N=w2q[0].shape[0])
    if b2 is not None:
        y = y + R.bf16_round(b2).astype(np.float64)[None, :]
    if gate is not None:
        idx = np.zeros(x.shape[0], dtype=np.int64) if row_idx is None else np.asarray(row_idx)
        y = y * R.bf16_round(gate).astype(np.float64)[idx]
    y = y + x.astype(np.float64)
    return R.bf16_round(y.astype(np.float32))


def drift(ref, cand) -> dict:
    """The trajectory drift metrics of ``h3_inference/tests/equiv.py:82-95``:
    max |d|, relative L2 (%), cosine, and PSNR with the reference's
    peak-to-peak range as the peak."""
    a = np.asarray(ref, dtype=np.float64).ravel()
    b = np.asarray(cand, dtype=np.float64).ravel()
    d = b - a
    mse = float(np.mean(d * d))
    peak = float(a.max() - a.min())
    psnr = float("inf") if mse == 0.0 else 20.0 * np.log10(peak) - 10.0 * np.log10(mse)
    return {"max_abs": float(np.abs(d).max()),
            "rel_l2_pct": 100.0 * float(np.linalg.norm(d) / np.linalg.norm(a)),
            "cosine": float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b))),
            "psnr_db": psnr}
