"""Multi-threaded torch-CPU port of the NVFP4 recipe and the FFN sub-block --
TEST / CPU-BASELINE INFRASTRUCTURE ONLY.

This is the timed CPU baseline (``bench.py --impl reference`` and the
``cpu_baseline`` object): the reference's NVFP4 path cannot run on a CPU
(its quantizer lives in the absent ``maiku`` package and CPU
``torch._scaled_mm`` rejects block scales), so the CPU path timed is the
reference's CPU decode (``h3_inference/render.py:174-183``: LUT[code] *
scale, then ``F.linear``) applied to operands quantized with the same
three-level recipe as ``oracle/nvfp4_ref.py``.  Vectorised torch ops on all
host threads; results agree with ``nvfp4_ref`` (checked in tests).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

_LUT = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                     -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=torch.float32)
_UP = (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)
_TIE_UP = (False, True, False, True, False, True, False)


def quantize(x: torch.Tensor, gs: float | None = None):
    """bf16/fp32 ``[M, K]`` (bf16 values) -> (codes u8 [M, K], scales u8 [M, K/16], gs)."""
    x = x.float()
    M, K = x.shape
    if gs is None:
        amax = float(x.abs().max()) if x.numel() else 0.0
        gs_t = torch.tensor(amax, dtype=torch.float32) / torch.tensor(2688.0)
        gs_t = gs_t if amax > 0 else torch.tensor(1.0)
    else:
        gs_t = torch.tensor(float(gs), dtype=torch.float32)
    d6 = torch.tensor(6.0, dtype=torch.float32) * gs_t
    xb = x.view(M, K // 16, 16)
    bmax = xb.abs().amax(-1)
    s = (bmax / d6).clamp(max=448.0).to(torch.float8_e4m3fn)
    d = s.float() * gs_t
    inv = torch.where(d > 0, 1.0 / d, torch.zeros_like(d))
    v = xb * inv.unsqueeze(-1)
    a = v.abs()
    code = torch.zeros_like(a, dtype=torch.uint8)
    for t, up in zip(_UP, _TIE_UP):
        code += (a >= t if up else a > t).to(torch.uint8)
    code |= (torch.signbit(v).to(torch.uint8) << 3)
    code = torch.where((d > 0).unsqueeze(-1), code, torch.zeros_like(code))
    return code.view(M, K), s.view(torch.uint8), float(gs_t)


def dequantize(codes: torch.Tensor, s: torch.Tensor, gs: float) -> torch.Tensor:
    M, K = codes.shape
    vals = _LUT[codes.long()].view(M, K // 16, 16)
    return ((vals * s.view(torch.float8_e4m3fn).float().unsqueeze(-1)) * gs).view(M, K)


def rmsnorm(x: torch.Tensor, gamma: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * gamma.float()
    return y.to(torch.bfloat16)


class FFNBlockCPU:
    """RMSNorm -> NVFP4 linear(+b1) -> GELU-tanh -> re-quant -> NVFP4 linear(+b2) + x;
    ``act="swiglu"``: w1 is the fused [value | gate] projection (2F rows, no
    biases) and the activation is bf16(value * bf16(silu(gate))), the
    reference's SwiGLU (h3_inference/transformer/ops.py:62-71)."""

    def __init__(self, w1, b1, w2, b2, gamma, eps, act: str = "gelu_tanh"):
        if act not in ("gelu_tanh", "swiglu"):
            raise ValueError(act)
        c1, s1, g1 = quantize(w1.to(torch.bfloat16).float())
        c2, s2, g2 = quantize(w2.to(torch.bfloat16).float())
        self.w1 = dequantize(c1, s1, g1)          # fp32, decoded once like a loaded checkpoint
        self.w2 = dequantize(c2, s2, g2)
        self.b1 = None if b1 is None else b1.to(torch.bfloat16).float()
        self.b2 = None if b2 is None else b2.to(torch.bfloat16).float()
        self.gamma = gamma.to(torch.bfloat16)
        self.eps = eps
        self.act = act

    def __call__(self, x: torch.Tensor, gs_h: float | None = None, gs_u: float | None = None):
        h = rmsnorm(x, self.gamma, self.eps)
        ch, sh, gh = quantize(h.float(), gs_h)
        u = F.linear(dequantize(ch, sh, gh), self.w1, self.b1)
        if self.act == "swiglu":
            val, gate = u.to(torch.bfloat16).float().chunk(2, dim=-1)
            u = val * F.silu(gate).to(torch.bfloat16).float()
        else:
            u = F.gelu(u, approximate="tanh")
        u = u.to(torch.bfloat16)
        cu, su, gu = quantize(u.float(), gs_u)
        y = F.linear(dequantize(cu, su, gu), self.w2, self.b2) + x.float()
        return y.to(torch.bfloat16)


def qk_norm_rope(x: torch.Tensor, w: torch.Tensor, eps: float, cos: torch.Tensor,
                 sin: torch.Tensor) -> torch.Tensor:
    """[S, H, D] bf16 -> per-head RMSNorm + rotate-half RoPE (reference formula,
    h3_inference/kernels/elementwise_norm_rope.py:104-122), bf16 out."""
    xf = x.float()
    xn = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    r = cos.shape[-1]
    half = r // 2
    c = cos.to(torch.bfloat16).float()[:, None, :]
    s = sin.to(torch.bfloat16).float()[:, None, :]
    x1, x2 = xn[..., :half], xn[..., half:r]
    out = torch.cat([x1 * c[..., :half] - x2 * s[..., :half],
                     x2 * c[..., half:] + x1 * s[..., half:], xn[..., r:]], dim=-1)
    return out.to(torch.bfloat16)


class AttnRowsCPU:
    """Attention half of a DiT block for a SAMPLE of query rows against keys /
    values of the full sequence: norm -> NVFP4 (decoded) QKV projection of the
    sample -> qk-norm + RoPE -> softmax attention over all T keys -> NVFP4
    out-projection + residual.  The keys / values of the other rows are random
    stand-ins: the cost per query row is that of the full computation."""

    def __init__(self, d: int, heads: int, head_dim: int, total: int, seed: int = 4):
        g = torch.Generator().manual_seed(seed)
        hd = heads * head_dim
        self.heads, self.head_dim = heads, head_dim
        w = lambda n, k: (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)  # noqa: E731
        self.wqkv = [dequantize(*quantize(w(hd, d).float())) for _ in range(3)]
        self.wo = dequantize(*quantize(w(d, hd).float()))
        self.gamma = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
        self.nq = (1 + 0.1 * torch.randn(head_dim, generator=g)).to(torch.bfloat16)
        self.nk = (1 + 0.1 * torch.randn(head_dim, generator=g)).to(torch.bfloat16)
        self.k_all = torch.randn(heads, total, head_dim, generator=g).to(torch.bfloat16).float()
        self.v_all = torch.randn(heads, total, head_dim, generator=g).to(torch.bfloat16).float()

    def __call__(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        S = x.shape[0]
        h = rmsnorm(x, self.gamma, 1e-6)
        c, s, g = quantize(h.float())
        hq = dequantize(c, s, g)
        q, k, v = (F.linear(hq, w).to(torch.bfloat16).view(S, self.heads, self.head_dim)
                   for w in self.wqkv)
        q = qk_norm_rope(q, self.nq, 1e-6, cos, sin)
        qf = q.float().transpose(0, 1)                                   # [H, S, D]
        p = torch.softmax(qf @ self.k_all.transpose(1, 2) * self.head_dim ** -0.5, dim=-1)
        o = (p @ self.v_all).transpose(0, 1).reshape(S, -1).to(torch.bfloat16)
        c, s, g = quantize(o.float())
        return (F.linear(dequantize(c, s, g), self.wo) + x.float()).to(torch.bfloat16)
