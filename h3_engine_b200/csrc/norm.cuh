// RMSNorm feeding an NVFP4 GEMM (HBM-bound).
//
// Replaces nn.RMSNorm / the fused norm_modulate row shim
// (h3_inference/kernels/elementwise_norm_rope.py:19-23,42-52,69-88) followed
// by the activation quantization of QuantizedActivation
// (h3_inference/nvfp4.py:92-110).  The normalized bf16 activation is never
// written to HBM: pass 1 computes per-row rstd and the global amax of
//   y = bf16( (x * rstd * gamma) * (1 + scale[idx]) + shift[idx] )
// (modulation optional), pass 2 recomputes y and quantizes it with the
// global scale amax / 2688 -- 2 + 2 + 0.5625 bytes per element instead of
// 2 + 2 + 2 + 2 + 0.5625 for norm -> bf16 -> amax -> quantize.
// rstd = 1 / sqrt(mean(x^2) + eps), fp32, one bf16 rounding of y (torch's
// rms_norm rounding).
#pragma once

#include "common.cuh"
#include "quant.cuh"

namespace h3b {

struct NormArgs {
  const __nv_bfloat16* x;      // [M, K], row stride ldx
  const __nv_bfloat16* gamma;  // [K]
  const __nv_bfloat16* shift;  // [num_mod, K] or null (adaLN modulation)
  const __nv_bfloat16* scale;  // [num_mod, K] or null
  const int32_t* mod_idx;      // [M] row -> modulation row, or null (row 0)
  long long ldx;
  long long M, K;
  float eps;
};

constexpr int kNormWarps = 8;   // rows per CTA, one warp per row
constexpr int kNormCacheChunks = 12;   // rows of K <= 3072 stay in registers

// y[0..8) of row `row`, columns chunk*256 + lane*8 ..: (x * rstd) * gamma,
// then * (1 + scale) + shift (one fma) when modulated -- packed two-lane
// fp32 ops, each lane rounded as the scalar op.
__device__ __forceinline__ void norm_row_values(const NormArgs& a, long long row, int lane,
                                                int chunk, const uint4& xr, float rstd,
                                                float (&y)[8]) {
  const long long col = (long long)chunk * 256 + lane * 8;
  const uint4 g = __ldg(reinterpret_cast<const uint4*>(a.gamma + col));
  const uint32_t xw[4] = {xr.x, xr.y, xr.z, xr.w};
  const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
  const float2 r2 = make_float2(rstd, rstd);
  float2 v[4];
#pragma unroll
  for (int t = 0; t < 4; ++t) v[t] = mul2(mul2(bf16x2_to_f2(xw[t]), r2), bf16x2_to_f2(gw[t]));
  if (a.scale != nullptr) {
    const long long mrow = a.mod_idx ? a.mod_idx[row] : 0;
    const uint4 sc = __ldg(reinterpret_cast<const uint4*>(a.scale + mrow * a.K + col));
    const uint4 sh = __ldg(reinterpret_cast<const uint4*>(a.shift + mrow * a.K + col));
    const uint32_t cw[4] = {sc.x, sc.y, sc.z, sc.w};
    const uint32_t hw[4] = {sh.x, sh.y, sh.z, sh.w};
    const float2 one = make_float2(1.0f, 1.0f);
#pragma unroll
    for (int t = 0; t < 4; ++t)
      v[t] = fma2(v[t], add2(one, bf16x2_to_f2(cw[t])), bf16x2_to_f2(hw[t]));
  }
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    y[2 * t] = v[t].x;
    y[2 * t + 1] = v[t].y;
  }
}

// Pass 1: one warp per row.  With CACHE > 0 the row (K <= CACHE * 256) stays
// in registers between the sum of squares and the amax of y; otherwise the
// second traversal re-reads it (an L2 hit: the row was read microseconds ago).
template <int CACHE>
__global__ void __launch_bounds__(kNormWarps * 32)
    k_rmsnorm_stats(const NormArgs a, float* __restrict__ rstd_out, float* __restrict__ amax_out) {
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * kNormWarps + (threadIdx.x >> 5);
  const int chunks = (int)(a.K / 256);
  float m = 0.f;
  if (row < a.M) {
    constexpr int NR = CACHE > 0 ? CACHE : 1;
    uint4 xr[NR];
    const __nv_bfloat16* xp = a.x + row * a.ldx + lane * 8;
    float ss = 0.f;
    auto accum = [&](const uint4& v) {
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float lo = __uint_as_float(w[t] << 16), hi = __uint_as_float(w[t] & 0xFFFF0000u);
        ss = fmaf(lo, lo, ss);
        ss = fmaf(hi, hi, ss);
      }
    };
    if (CACHE > 0) {
#pragma unroll
      for (int c = 0; c < NR; ++c) {
        if (c < chunks) {
          xr[c] = ld_nc_v4(xp + c * 256);
          accum(xr[c]);
        }
      }
    } else {
#pragma unroll 4
      for (int c = 0; c < chunks; ++c) accum(__ldg(reinterpret_cast<const uint4*>(xp + c * 256)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rstd = rsqrtf(ss / (float)a.K + a.eps);
    if (lane == 0) rstd_out[row] = rstd;
    // |bf16(y)| max on packed bit patterns (non-negative bf16 values order
    // like their 16-bit integers)
    uint32_t mb2 = 0;
    auto amax_y = [&](int c, const uint4& v) {
      float y[8];
      norm_row_values(a, row, lane, c, v, rstd, y);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        mb2 = __vmaxu2(mb2, pack_bf16x2(y[2 * i], y[2 * i + 1]) & 0x7FFF7FFFu);
    };
    if (CACHE > 0) {
#pragma unroll
      for (int c = 0; c < NR; ++c)
        if (c < chunks) amax_y(c, xr[c]);
    } else {
      for (int c = 0; c < chunks; ++c)
        amax_y(c, __ldg(reinterpret_cast<const uint4*>(xp + c * 256)));
    }
    m = __uint_as_float(max(mb2 & 0xFFFFu, mb2 >> 16) << 16);
  }
  // CTA-wide max then one atomic
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ float red[kNormWarps];
  if (lane == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = 0.f;
    for (int i = 0; i < kNormWarps; ++i) v = fmaxf(v, red[i]);
    if (v > 0.f) atomicMax(reinterpret_cast<unsigned int*>(amax_out), __float_as_uint(v));
  }
}

// Pass 2: one warp per row; lanes (2j, 2j+1) share a 16-element block.
// Writes E2M1 codes [Mpad, K/2], swizzled scales, and optionally y (bf16).
// (4 CTAs per SM: at the 69 registers ptxas picks unbounded, 3 CTAs fit and
// the pass runs 13 % slower)
__global__ void __launch_bounds__(kNormWarps * 32, 4)
    k_rmsnorm_quant(const NormArgs a, const float* __restrict__ rstd_in,
                    const float* __restrict__ amax_in, float* __restrict__ gs_out,
                    uint8_t* __restrict__ q, uint8_t* __restrict__ sf, long long Mpad,
                    __nv_bfloat16* __restrict__ y_out) {
  const float gs = global_scale_from_amax(__ldg(amax_in));
  const float d6 = __fmul_rn(6.0f, gs);
  if (gs_out != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *gs_out = gs;
  __shared__ float inv_tab[kInvTableSize];
  fill_inv_table(inv_tab, gs);
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * kNormWarps + (threadIdx.x >> 5);
  if (row >= Mpad) return;   // warp-uniform
  const int chunks = (int)(a.K / 256);
  const long long c4 = a.K >> 6;
  const bool live = row < a.M;
  const float rstd = live ? __ldg(rstd_in + row) : 0.f;
  constexpr int U = 4;                         // 16-byte loads in flight per lane
  for (int c0 = 0; c0 < chunks; c0 += U) {
    uint4 xr[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      xr[u] = make_uint4(0, 0, 0, 0);
      if (live && c0 + u < chunks) xr[u] = ld_nc_v4(a.x + row * a.ldx + (c0 + u) * 256 + lane * 8);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + u;
      if (c >= chunks) break;                    // warp-uniform
      uint4 yr = make_uint4(0, 0, 0, 0);
      if (live) {
        float y[8];
        norm_row_values(a, row, lane, c, xr[u], rstd, y);
        yr = make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]),
                        pack_bf16x2(y[6], y[7]));
        if (y_out) *reinterpret_cast<uint4*>(y_out + row * a.K + c * 256 + lane * 8) = yr;
      }
      uint32_t s8;
      const uint32_t packed = quantize_half_block(yr, inv_tab, d6, s8);
      const long long hc = (long long)c * 32 + lane;        // 8-element half index in the row
      *reinterpret_cast<uint32_t*>(q + row * (a.K >> 1) + hc * 4) = packed;
      if ((lane & 1) == 0) sf[sf_swizzled_offset(row, hc >> 1, c4)] = static_cast<uint8_t>(s8);
    }
  }
}

}  // namespace h3b
