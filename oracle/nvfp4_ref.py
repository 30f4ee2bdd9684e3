"""CPU oracle for the NVFP4 hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this module, and only as
the checker or as the timed CPU baseline.  The product path (``h3_engine_b200``)
never imports it and fails loudly when its CUDA library is missing.

What it restates
----------------
The reference quantizes through an un-vendored package (``maiku``,
``quantize_nvfp4`` / ``_nvfp4_quant_fwd``; no version pin anywhere) at
``h3_inference/nvfp4.py:20-42`` and swizzles scales with torchao's
``to_blocked`` (``h3_inference/nvfp4.py:44-46``, also un-vendored).  Neither
can run here, and the reference holds no golden vectors for the packed bytes,
so byte-level parity is pinned by the facts the reference source fixes plus
the recipe written out below:

* E2M1 decode table and nibble order (low nibble = even K index):
  ``h3_inference/render.py:178-188``.
* Block of 16 along K, E2M1 max 6: ``h3_inference/nvfp4.py:9-10``.
* Shapes: packed u8 ``[M, K/2]``, e4m3 scales ``[M, K/16]``:
  ``h3_inference/nvfp4.py:21``; rows padded to 128: ``h3_inference/nvfp4.py:12,17-18``.
* Swizzled scale layout consumed by ``torch._scaled_mm``
  (``h3_inference/nvfp4.py:113-114``): 128x4 tiles of 512 bytes,
  element (r, c) at ``((r//128)*ceil(C/4) + c//4)*512 + (r%32)*16 + ((r%128)//32)*4 + c%4``.

The three-level recipe (fp32 global scale over e4m3 block scales over E2M1
codes), every step IEEE-754 fp32 round-to-nearest-even, in this order:

1. ``amax = max|x|``; ``gs = amax / 2688`` (2688 = 6 * 448); ``gs = 1`` when amax == 0.
2. ``d6 = 6 * gs``; per 16-block ``s = e4m3_rne_satfinite(bmax / d6)``.
3. ``d = float(s) * gs``; ``d == 0`` -> all 16 codes are 0x0.
4. ``inv = 1 / d``; ``v = x * inv``; ``code = e2m1_rne_satfinite(v)`` with the
   sign bit taken from ``v`` (a negative value that rounds to zero is 0x8).
5. ``byte = code[2j] | code[2j+1] << 4``.
6. dequantize: ``bf16( (LUT[code] * float(s)) * gs )``.

Step 4 multiplies by the reciprocal of the block scale (the usual NVFP4
recipe) rather than dividing every element; the CUDA kernel performs the
identical fp32 operations, so the packed bytes are bit-exact against this file.
With ``gs = 1`` the recipe reduces to the reference's two-level scheme.
"""
from __future__ import annotations

import numpy as np

FP4_BLOCK = 16          # h3_inference/nvfp4.py:9
FP4_MAX = 6.0           # h3_inference/nvfp4.py:10
E4M3_MAX = 448.0
M_ALIGN = 128           # h3_inference/nvfp4.py:12
GS_DENOM = np.float32(FP4_MAX * E4M3_MAX)   # 2688

# h3_inference/render.py:185-188
E2M1_LUT = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                     -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=np.float32)


def pad_m(m: int) -> int:
    """``h3_inference/nvfp4.py:17-18``."""
    return ((m + M_ALIGN - 1) // M_ALIGN) * M_ALIGN


# ----------------------------------------------------------------------------- bf16
def bf16_round(a) -> np.ndarray:
    """fp32 -> nearest-even bf16, returned as the fp32 value it represents."""
    f = np.ascontiguousarray(a, dtype=np.float32)
    u = f.view(np.uint32)
    # uint32 arithmetic: finite values and infinities never carry out of 32
    # bits (at most 0xFF7FFFFF + 0x8000); only NaN payloads can, and those are
    # restored below
    r = (u >> np.uint32(16)) & np.uint32(1)
    r += np.uint32(0x7FFF)
    r += u
    r &= np.uint32(0xFFFF0000)
    out = r.view(np.float32)
    nan = np.isnan(f)
    return np.where(nan, f, out) if nan.any() else out


def bf16_bits(a) -> np.ndarray:
    """fp32 values already representable in bf16 -> raw uint16 bits."""
    f = np.ascontiguousarray(bf16_round(a), dtype=np.float32)
    return (f.view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(b) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ----------------------------------------------------------------------------- e4m3
def e4m3_rne_satfinite(v) -> np.ndarray:
    """fp32 -> e4m3fn bits, round-to-nearest-even, saturating to +-448.

    Restated from the OCP FP8 definition (bias 7, 3 mantissa bits, subnormal
    quantum 2**-9, no infinities, 0x7F = NaN).  Exact: the work is done in
    float64 on fp32 inputs, where every step below is exact.
    """
    v = np.asarray(v, dtype=np.float32).astype(np.float64)
    sign = np.signbit(v)
    a = np.abs(v)
    out = np.zeros(a.shape, dtype=np.uint8)
    nz = a > 0
    e = np.zeros(a.shape, dtype=np.int64)
    e[nz] = np.floor(np.log2(a[nz])).astype(np.int64)
    # guard log2 rounding at exact powers of two
    e = np.where(nz & (np.ldexp(1.0, e) > a), e - 1, e)
    e = np.where(nz & (np.ldexp(1.0, e + 1) <= a), e + 1, e)
    qexp = np.maximum(e, -6) - 3                       # quantum exponent
    r = np.rint(np.ldexp(a, -qexp))                    # ties-to-even
    val = np.ldexp(r, qexp)
    val = np.minimum(val, E4M3_MAX)                    # satfinite
    # encode
    sub = val < 2.0 ** -6
    m_sub = np.rint(np.ldexp(val, 9)).astype(np.int64)
    ev = np.zeros(val.shape, dtype=np.int64)
    pos = val > 0
    ev[pos] = np.floor(np.log2(val[pos])).astype(np.int64)
    ev = np.where(pos & (np.ldexp(1.0, ev) > val), ev - 1, ev)
    mant = np.rint(np.ldexp(val, -ev) * 8 - 8).astype(np.int64)
    enc_norm = ((ev + 7) << 3) | mant
    enc = np.where(sub, m_sub, enc_norm)
    enc = np.where(val == 0, 0, enc)
    out = enc.astype(np.uint8)
    out = np.where(np.isnan(v), np.uint8(0x7F), out)
    out = out | (sign.astype(np.uint8) << 7)
    return out.astype(np.uint8)


def e4m3_to_f32(bits) -> np.ndarray:
    b = np.asarray(bits, dtype=np.uint8).astype(np.int64)
    s = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = b & 0x7
    val = np.where(e == 0, m * 2.0 ** -9, (8 + m) * np.ldexp(1.0, e - 10))
    val = np.where((b & 0x7F) == 0x7F, np.nan, val)
    return (s * val).astype(np.float32)


# ----------------------------------------------------------------------------- e2m1
_E2M1_UP = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], dtype=np.float32)
# a magnitude equal to a midpoint rounds up only when the upper neighbour has an
# even mantissa: 0.75->1.0, 1.75->2.0, 3.5->4.0 (ties-to-even on the code LSB)
_E2M1_TIE_UP = np.array([False, True, False, True, False, True, False])


def e2m1_rne_satfinite(v) -> np.ndarray:
    """fp32 -> 4-bit E2M1 code (sign in bit 3), round-to-nearest-even, |v|>6 -> 6."""
    v = np.asarray(v, dtype=np.float32)
    a = np.abs(v)
    code = np.zeros(v.shape, dtype=np.uint8)
    for t, up in zip(_E2M1_UP, _E2M1_TIE_UP):
        code += ((a >= t) if up else (a > t)).astype(np.uint8)
    return code | (np.signbit(v).astype(np.uint8) << 3)


def e2m1_decode(codes) -> np.ndarray:
    return E2M1_LUT[np.asarray(codes, dtype=np.uint8) & 0xF]


# ----------------------------------------------------------------------------- swizzle
def swizzled_offset(r, c, cols: int):
    """Byte offset of scale (r, c) in the 128x4-tile layout of a ``[R, cols]`` scale matrix."""
    c4 = (cols + 3) // 4
    r = np.asarray(r, dtype=np.int64)
    c = np.asarray(c, dtype=np.int64)
    return ((r // 128) * c4 + c // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + (c % 4)


def swizzle(sf_rowmajor) -> np.ndarray:
    """``[R, C]`` scale bytes -> flat blocked layout (torchao ``to_blocked`` semantics).

    R is padded to a multiple of 128 and C to a multiple of 4 with zeros.
    """
    sf = np.asarray(sf_rowmajor, dtype=np.uint8)
    R, C = sf.shape
    Rp, Cp = pad_m(R), ((C + 3) // 4) * 4
    out = np.zeros(Rp * Cp, dtype=np.uint8)
    rr, cc = np.meshgrid(np.arange(R), np.arange(C), indexing="ij")
    out[swizzled_offset(rr, cc, C)] = sf
    return out


def unswizzle(flat, rows: int, cols: int) -> np.ndarray:
    flat = np.asarray(flat, dtype=np.uint8).reshape(-1)
    rr, cc = np.meshgrid(np.arange(rows), np.arange(cols), indexing="ij")
    return flat[swizzled_offset(rr, cc, cols)]


# ----------------------------------------------------------------------------- recipe
def global_scale(amax) -> np.float32:
    amax = np.float32(amax)
    if amax == 0:
        return np.float32(1.0)
    return np.float32(amax / GS_DENOM)


def quantize(x, mpad: int | None = None, gs=None, amax=None):
    """bf16 ``[M, K]`` (given as fp32 values) -> (q u8 ``[Mpad, K/2]``,
    sf e4m3 bits ``[Mpad, K/16]`` row-major, gs fp32).

    ``gs`` may be forced (e.g. 1.0 for the two-level scheme); else it comes
    from ``amax`` (else from the data).  Rows ``M..Mpad-1`` are zero codes and
    zero scales.
    """
    x = bf16_round(np.asarray(x, dtype=np.float32))
    M, K = x.shape
    assert K % FP4_BLOCK == 0
    if gs is None:
        if amax is None:
            amax = np.float32(np.max(np.abs(x))) if x.size else np.float32(0)
        gs = global_scale(amax)
    gs = np.float32(gs)
    d6 = np.float32(np.float32(6.0) * gs)
    xb = x.reshape(M, K // FP4_BLOCK, FP4_BLOCK)
    bmax = np.max(np.abs(xb), axis=2).astype(np.float32)
    s = e4m3_rne_satfinite((bmax / d6).astype(np.float32))
    d = (e4m3_to_f32(s) * gs).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        inv = (np.float32(1.0) / d).astype(np.float32)
        v = (xb * inv[:, :, None]).astype(np.float32)
    codes = e2m1_rne_satfinite(v)
    codes = np.where((d == 0)[:, :, None], np.uint8(0), codes).reshape(M, K)
    q = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    Mp = M if mpad is None else mpad
    assert Mp >= M
    qp = np.zeros((Mp, K // 2), dtype=np.uint8)
    sp = np.zeros((Mp, K // FP4_BLOCK), dtype=np.uint8)
    qp[:M] = q
    sp[:M] = s
    return qp, sp, gs


def unpack_codes(q) -> np.ndarray:
    q = np.asarray(q, dtype=np.uint8)
    M, Kh = q.shape
    codes = np.empty((M, Kh * 2), dtype=np.uint8)
    codes[:, 0::2] = q & 0xF      # low nibble = even K index (h3_inference/render.py:178-180)
    codes[:, 1::2] = q >> 4
    return codes


def dequantize_f32(q, sf_rowmajor, gs) -> np.ndarray:
    """fp32 dequantized values ``(LUT[code] * s) * gs`` (no bf16 rounding)."""
    codes = unpack_codes(q)
    M, K = codes.shape
    vals = e2m1_decode(codes).reshape(M, K // FP4_BLOCK, FP4_BLOCK)
    s = e4m3_to_f32(np.asarray(sf_rowmajor, dtype=np.uint8))[:M, :K // FP4_BLOCK]
    prod = (vals * s[:, :, None]).astype(np.float32)         # exact
    return (prod * np.float32(gs)).astype(np.float32).reshape(M, K)


def dequantize(q, sf_rowmajor, gs) -> np.ndarray:
    """bf16 dequantization (as fp32 values), ``h3_inference/render.py:178-183`` plus gs."""
    return bf16_round(dequantize_f32(q, sf_rowmajor, gs))


def gemm_ref(qa, sfa, gsa, qb, sfb, gsb, M: int, N: int) -> np.ndarray:
    """``bf16(deq(A) @ deq(B)^T)`` with float64 accumulation, fp32 values out."""
    a = dequantize_f32(qa[:M], sfa[:M], np.float32(1.0)).astype(np.float64)
    b = dequantize_f32(qb[:N], sfb[:N], np.float32(1.0)).astype(np.float64)
    y = (a @ b.T) * (float(gsa) * float(gsb))
    return y


def linear_ref(x, w, bias=None, act: str | None = None, residual=None):
    """NVFP4 linear: quantize x and w with the recipe, dequantize, fp64 GEMM,
    optional bias / GELU-tanh / residual, bf16 out (as fp32 values)."""
    x = bf16_round(x)
    w = bf16_round(w)
    M, K = x.shape
    N = w.shape[0]
    qa, sa, ga = quantize(x)
    qb, sb, gb = quantize(w)
    y = gemm_ref(qa, sa, ga, qb, sb, gb, M, N)
    if bias is not None:
        y = y + bf16_round(bias).astype(np.float64)[None, :]
    if act == "gelu_tanh":
        y = gelu_tanh(y)
    if residual is not None:
        y = y + bf16_round(residual).astype(np.float64)
    return bf16_round(y.astype(np.float32))


def gelu_tanh(y):
    y = np.asarray(y, dtype=np.float64)
    return 0.5 * y * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (y + 0.044715 * y ** 3)))


def max_rel_err(got, ref) -> float:
    """``max|got - ref| / max|ref|`` -- the tolerance metric of the parity tests."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.max(np.abs(ref))
    return float(np.max(np.abs(got - ref)) / (den if den > 0 else 1.0))
