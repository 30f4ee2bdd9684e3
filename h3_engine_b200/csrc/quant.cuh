// NVFP4 quantize / pack / unpack kernels (HBM-bound).
//
// Replaces the maiku quantizer behind h3_inference/nvfp4.py:20-42 and the
// torchao scale swizzle at h3_inference/nvfp4.py:44-46.  The arithmetic is
// the three-level recipe, every step an IEEE fp32 round-to-nearest-even op
// in a fixed order, so the packed bytes and scales are bit-exact against the
// CPU oracle:
//   gs  = amax / 2688            (gs = 1 when amax == 0)
//   s   = e4m3_rne_sat(bmax / (6*gs))         per 16 elements along K
//   d   = float(s) * gs;  inv = 1/d
//   code= e2m1_rne_sat(x * inv), sign from x  (all-zero when d == 0)
//   byte= code[2j] | code[2j+1] << 4          (h3_inference/render.py:178-180)
#pragma once

#include "common.cuh"

namespace h3b {

constexpr float kGsDenom = 2688.0f;  // 6 (E2M1 max) * 448 (E4M3 max)

__device__ __forceinline__ float global_scale_from_amax(float amax) {
  return amax > 0.f ? __fdiv_rn(amax, kGsDenom) : 1.0f;
}

// fp32 (>= 0) -> e4m3fn bits, round-to-nearest-even, saturating at 448.
__device__ __forceinline__ uint32_t f32_to_e4m3_sat(float v) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(v));
  return r & 0xFFu;
}

// e4m3fn bits -> fp32, exact.
__device__ __forceinline__ float e4m3_to_f32(uint32_t b) {
  const uint32_t e = (b >> 3) & 15u, m = b & 7u;
  float v = e ? __uint_as_float(((e + 120u) << 23) | (m << 20)) : float(m) * 0.001953125f;
  return (b & 0x80u) ? -v : v;
}

// e4m3fn bits (finite) -> fp32 through the hardware e4m3x2 -> f16x2 decode
// (every finite e4m3 value is exact in f16; checked against e4m3_to_f32 on
// all codes).
__device__ __forceinline__ float e4m3_to_f32_hw(uint32_t b) {
  uint32_t h2;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"((uint16_t)b));
  return __half2float(__ushort_as_half((unsigned short)(h2 & 0xFFFFu)));
}

// Two fp32 -> one byte of E2M1 codes: lo -> low nibble, hi -> high nibble,
// round-to-nearest-even with saturation.  The conversion keeps the sign of a
// negative value that rounds to zero (0x8), as the recipe requires.
__device__ __forceinline__ uint32_t f32x2_to_e2m1x2(float lo, float hi) {
  uint32_t r;
  asm("{\n\t.reg .b8 t;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\t"
      "cvt.u32.u8 %0, t;\n\t}"
      : "=r"(r)
      : "f"(hi), "f"(lo));
  return r;
}

// Two IEEE round-to-nearest fp32 products in one instruction.
__device__ __forceinline__ void mul_rn_f32x2(float a0, float a1, float b, float& d0, float& d1) {
  asm("{\n\t.reg .b64 a, b, d;\n\tmov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %4};\n\t"
      "mul.rn.f32x2 d, a, b;\n\tmov.b64 {%0, %1}, d;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b));
}

// Byte offset of scale (r, c) in the 128x4-tile layout (c4 = C/4 tiles per row block).
__device__ __forceinline__ int64_t sf_swizzled_offset(int64_t r, int64_t c, int64_t c4) {
  return ((r >> 7) * c4 + (c >> 2)) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4 + (c & 3);
}

// Per-tensor table of the reciprocal each block multiplies by: entry s holds
// __frcp_rn(d) with d = float(s) * gs, or 0 where d == 0 (the block's codes
// are then all +0).  A block scale is never negative (it is the saturating
// e4m3 conversion of |x|max / (6 gs) >= 0), so its byte indexes 128 entries.
// Each CTA of a quantizing kernel fills its own copy in shared memory once:
// 128 reciprocals instead of one decode, multiply and IEEE reciprocal per
// 16-element block.
constexpr int kInvTableSize = 128;

__device__ __forceinline__ void fill_inv_table(float* tab, float gs) {
  for (int s = threadIdx.x; s < kInvTableSize; s += blockDim.x) {
    const float d = __fmul_rn(e4m3_to_f32_hw((uint32_t)s), gs);
    tab[s] = d != 0.f ? __frcp_rn(d) : 0.f;
  }
  __syncthreads();
}

// Quantize 8 consecutive bf16 values (one lane's half of a 16-block; the
// partner half sits in the neighbouring lane).  Returns 4 packed code bytes
// and the block's scale byte.  The block max is taken on the bf16 bit
// patterns: |x| of a bf16 is its bits & 0x7FFF, and non-negative bf16 values
// order like their 16-bit integers (NaN inputs are outside the recipe).
// inv_tab: the tensor's reciprocal table (fill_inv_table).
__device__ __forceinline__ uint32_t quantize_half_block(const uint4& raw, const float* inv_tab,
                                                        float d6, uint32_t& s8_out) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
  uint32_t m2 = __vmaxu2(w[0] & 0x7FFF7FFFu, w[1] & 0x7FFF7FFFu);
  m2 = __vmaxu2(m2, __vmaxu2(w[2] & 0x7FFF7FFFu, w[3] & 0x7FFF7FFFu));
  uint32_t mb = max(m2 & 0xFFFFu, m2 >> 16);
  mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, 1));
  const float m = __uint_as_float(mb << 16);
  const uint32_t s8 = f32_to_e4m3_sat(__fdiv_rn(m, d6));
  const float inv = inv_tab[s8 & (kInvTableSize - 1)];
  uint32_t packed = 0;
  if (inv != 0.f) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float a, b;
      mul_rn_f32x2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xFFFF0000u), inv, a, b);
      packed |= f32x2_to_e2m1x2(a, b) << (8 * i);
    }
  }
  s8_out = s8;
  return packed;
}

constexpr int kQuantThreads = 256;

// One warp per row (grid-stride over rows), two lanes per 16-element block,
// each lane one 16-byte load; UNROLL loads in flight per lane (6 or 7 where
// the row is a whole number of such steps of 32 loads, else 4: measured on
// the DiT and FFN-hidden rows, 6 is 4 % faster there and slower where the
// last step would be partly idle).  Reads and code writes of a warp are contiguous
// 512-byte / 128-byte runs.  Rows in [M, Mpad) are padding: they quantize
// zeros (codes and scales 0).
template <int LAYOUT, int UNROLL>
__global__ void __launch_bounds__(kQuantThreads)
    k_nvfp4_quantize(const __nv_bfloat16* __restrict__ x, int64_t M, int64_t K, int64_t ldx,
                     const float* __restrict__ amax, float gs_in, float* __restrict__ gs_out,
                     uint8_t* __restrict__ q, uint8_t* __restrict__ sf, int64_t Mpad) {
  const float gs = amax ? global_scale_from_amax(__ldg(amax)) : gs_in;
  const float d6 = __fmul_rn(6.0f, gs);
  if (gs_out != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *gs_out = gs;
  __shared__ float inv_tab[kInvTableSize];
  fill_inv_table(inv_tab, gs);

  const int lane = threadIdx.x & 31;
  const int hpr = (int)(K >> 3);              // 8-element halves per row (even)
  const int64_t kq = K >> 1;                  // code bytes per row
  const int64_t c_row = K >> 4;               // scales per row
  const int64_t c4 = K >> 6;
  const int64_t warps = (int64_t)gridDim.x * (kQuantThreads / 32);
  for (int64_t r = (int64_t)blockIdx.x * (kQuantThreads / 32) + (threadIdx.x >> 5); r < Mpad;
       r += warps) {
    const bool real = r < M;
    const __nv_bfloat16* xr = x + r * ldx;
    uint8_t* qr = q + r * kq;
    for (int h0 = 0; h0 < hpr; h0 += 32 * UNROLL) {
      uint4 raw[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const int h = h0 + u * 32 + lane;
        raw[u] = make_uint4(0, 0, 0, 0);
        if (real && h < hpr) raw[u] = ld_nc_v4(xr + (int64_t)h * 8);
      }
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const int h = h0 + u * 32 + lane;
        uint32_t s8;
        const uint32_t packed = quantize_half_block(raw[u], inv_tab, d6, s8);
        if (h < hpr) {
          *reinterpret_cast<uint32_t*>(qr + (int64_t)h * 4) = packed;
          if ((lane & 1) == 0) {
            const int64_t c = h >> 1;
            const int64_t off = LAYOUT == H3B_SF_SWIZZLED ? sf_swizzled_offset(r, c, c4)
                                                          : r * c_row + c;
            sf[off] = static_cast<uint8_t>(s8);
          }
        }
      }
    }
  }
}

constexpr int kAmaxThreads = 256;

__device__ __forceinline__ float absmax_bf16x8(const uint4& r, float m) {
  const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m = fmaxf(m, fabsf(__uint_as_float(w[i] << 16)));
    m = fmaxf(m, fabsf(__uint_as_float(w[i] & 0xFFFF0000u)));
  }
  return m;
}

__device__ __forceinline__ void block_atomic_max(float m, float* out) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ float red[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (warp == 0) {
    m = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0 && m > 0.f) atomicMax(reinterpret_cast<unsigned int*>(out), __float_as_uint(m));
  }
}

// max |x| of a [rows, cols] bf16 matrix (cols % 8 == 0), 16-byte loads.
__global__ void __launch_bounds__(kAmaxThreads)
    k_amax_bf16(const __nv_bfloat16* __restrict__ x, int64_t rows, int64_t cols, int64_t ldx,
                float* __restrict__ out) {
  const int64_t cpr = cols >> 3;
  const int64_t total = rows * cpr;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const bool dense = ldx == cols;
  float m = 0.f;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < total; i += 4 * stride) {
    uint4 r[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t c = i + u * stride;
      const int64_t off = dense ? c * 8 : (c / cpr) * ldx + (c % cpr) * 8;
      r[u] = ld_nc_v4(x + off);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) m = absmax_bf16x8(r[u], m);
  }
  for (; i < total; i += stride) {
    const int64_t off = dense ? i * 8 : (i / cpr) * ldx + (i % cpr) * 8;
    m = absmax_bf16x8(ld_nc_v4(x + off), m);
  }
  block_atomic_max(m, out);
}

// Unpack: E2M1 codes (4 bytes per 8 values) and their e4m3 block scale -> 8
// bf16 values (16 bytes), bf16((LUT[code] * s) * gs).
template <int LAYOUT>
__global__ void __launch_bounds__(256)
    k_nvfp4_dequantize(const uint8_t* __restrict__ q, const uint8_t* __restrict__ sf,
                       const float* __restrict__ gs_ptr, int64_t M, int64_t K,
                       __nv_bfloat16* __restrict__ out) {
  // One warp per row (grid-stride over rows); lane l takes the 8-value halves
  // l, l + 32, ... of the row, four in flight: 128 contiguous bytes of codes
  // read and 512 bytes written per warp instruction, no per-element division.
  const float gs = gs_ptr ? __ldg(gs_ptr) : 1.0f;
  const int lane = threadIdx.x & 31;
  const int hpr = (int)(K >> 3);              // 8-value halves per row
  const int64_t c_row = K >> 4, c4 = K >> 6;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  constexpr int U = 4;
  for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < M;
       row += nwarps) {
    const uint32_t* qrow = reinterpret_cast<const uint32_t*>(q + row * (K >> 1));
    __nv_bfloat16* orow = out + row * K;
    for (int h0 = lane; h0 < hpr; h0 += 32 * U) {
      uint32_t codes[U];
      uint8_t s8[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int hc = h0 + u * 32;
        codes[u] = 0;
        s8[u] = 0;
        if (hc < hpr) {
          codes[u] = __ldg(qrow + hc);
          const int64_t c = hc >> 1;
          s8[u] = __ldg(sf + (LAYOUT == H3B_SF_SWIZZLED ? sf_swizzled_offset(row, c, c4)
                                                         : row * c_row + c));
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int hc = h0 + u * 32;
        if (hc >= hpr) break;
        const float s = e4m3_to_f32(s8[u]);
        uint32_t hx2[4];
        asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
            "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
            "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
            "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
            "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
            "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
            : "=r"(hx2[0]), "=r"(hx2[1]), "=r"(hx2[2]), "=r"(hx2[3])
            : "r"(codes[u]));
        uint32_t o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hx2[i]));
          const float lo = __fmul_rn(__fmul_rn(f.x, s), gs);
          const float hi = __fmul_rn(__fmul_rn(f.y, s), gs);
          o[i] = pack_bf16x2(lo, hi);
        }
        *reinterpret_cast<uint4*>(orow + (int64_t)hc * 8) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
}

}  // namespace h3b
