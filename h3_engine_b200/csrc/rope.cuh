// Per-head RMSNorm + rotate-half RoPE on q and k, in place in the projected
// query / key activations (HBM-bound).
//
// Replaces qk_norm + apply_rotary_emb / norm_rope
// (h3_inference/kernels/elementwise_norm_rope.py:19-40,104-148) applied to the
// query and key heads that H3Attention.forward produces
// (h3_inference/transformer/model.py:89-102).  For a head vector x (D values):
//   xn  = x * rsqrt(mean(x^2) + eps) * w              (fp32)
//   out[j] = xn[j]*cos[j] - xn[j+R/2]*sin[j]           j <  R/2
//   out[j] = xn[j]*cos[j] + xn[j-R/2]*sin[j]           R/2 <= j < R
//   out[j] = xn[j]                                      j >= R  (pass-through)
// with cos/sin rounded to bf16 first (the reference casts them to the
// activation dtype), one bf16 rounding of out.  cos/sin are the (T, R) fp32
// tables the reference's rotary module produces; w may be NULL (RoPE only)
// and cos may be NULL (norm only).
#pragma once

#include "common.cuh"

namespace h3b {

struct RopeArgs {
  __nv_bfloat16* q;        // [T, q_stride], q heads at column q_off + h*D
  __nv_bfloat16* k;        // [T, k_stride], k heads at column k_off + h*D
  long long T, q_stride, k_stride;
  long long q_off, k_off;
  int H;                   // heads per block
  int hq, hk;              // query / key heads processed (H or 0)
  int R;                   // rotary dims (even, <= D)
  const __nv_bfloat16* wq; // [D] or null
  const __nv_bfloat16* wk; // [D] or null
  const float* cos;        // [T, R] (row stride cs_stride) or null
  const float* sin;
  long long cs_stride;
  float eps;
};

constexpr int kRopeWarps = 8;
// 16-byte loads in flight per lane (UNROLL): 6 (12 head vectors of 128 per
// warp iteration, 2 CTAs per SM) measured 10 % faster than 4 on the DiT rows
// (24 + 24 heads); 8 and 12 drop to one CTA per SM and are slower.  The host
// takes 7 where a row's head vectors are a whole number of 7-deep steps and
// not of 6-deep ones (56 + 56 heads), so no step runs partly idle.

// One warp per token row (grid-stride over rows).  A head vector of D values
// is spread over LPH = D/8 lanes, 8 consecutive values (one 16-byte load) per
// lane, so one warp instruction covers 32/LPH head vectors of the row's 2H
// (q heads then k heads).  The row's cos / sin values of a lane's 8 columns
// (bf16-rounded) and its norm weights are loaded once per row / once per
// warp.  The sum of squares reduces over the LPH lanes of a head; the
// rotate-half partner of column j (j +- R/2, R/2 a multiple of 8) is the
// lane (R/2)/8 away in the same head, fetched with shuffles.
template <int D, int UNROLL>
__global__ void __launch_bounds__(kRopeWarps * 32) k_qk_norm_rope(const RopeArgs a) {
  constexpr int LPH = D / 8;                 // lanes per head vector
  constexpr int HPW = 32 / LPH;              // head vectors per warp instruction
  const int lane = threadIdx.x & 31;
  const int sub = lane % LPH;
  const int j0 = sub * 8;                    // first column of this lane
  const int half = a.R >> 1;
  const bool rot = a.cos != nullptr && j0 < a.R;
  const int partner = (lane - sub) + (j0 < half ? (j0 + half) >> 3 : (j0 - half) >> 3);
  float gq[8], gk[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    gq[e] = a.wq ? __bfloat162float(a.wq[j0 + e]) : 1.f;
    gk[e] = a.wk ? __bfloat162float(a.wk[j0 + e]) : 1.f;
  }
  const int nv = a.hq + a.hk;                // head vectors per row (q heads, then k heads)
  const long long warp_id = (long long)blockIdx.x * kRopeWarps + (threadIdx.x >> 5);
  const long long nwarps = (long long)gridDim.x * kRopeWarps;
  for (long long t = warp_id; t < a.T; t += nwarps) {
    float c[8], s[8];
    if (rot) {
      const float4* cp = reinterpret_cast<const float4*>(a.cos + t * a.cs_stride + j0);
      const float4* sp = reinterpret_cast<const float4*>(a.sin + t * a.cs_stride + j0);
      const float4 c0 = __ldg(cp), c1 = __ldg(cp + 1), s0 = __ldg(sp), s1 = __ldg(sp + 1);
      const float cv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
      const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        c[e] = __bfloat162float(__float2bfloat16_rn(cv[e]));
        s[e] = __bfloat162float(__float2bfloat16_rn(sv[e]));
      }
    }
    __nv_bfloat16* qrow = a.hq ? a.q + t * a.q_stride + a.q_off : nullptr;
    __nv_bfloat16* krow = a.hk ? a.k + t * a.k_stride + a.k_off : nullptr;
    for (int v0 = 0; v0 < nv; v0 += HPW * UNROLL) {
      uint4 raw[UNROLL];
      __nv_bfloat16* ptr[UNROLL];
      bool is_k[UNROLL], valid[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const int v = v0 + u * HPW + lane / LPH;
        valid[u] = v < nv;
        is_k[u] = v >= a.hq;
        const int h = is_k[u] ? v - a.hq : v;
        ptr[u] = (is_k[u] ? krow : qrow) + (long long)h * D + j0;
        raw[u] = valid[u] ? *reinterpret_cast<const uint4*>(ptr[u]) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const uint32_t w[4] = {raw[u].x, raw[u].y, raw[u].z, raw[u].w};
        float x[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          x[2 * i] = __uint_as_float(w[i] << 16);
          x[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
        }
        // the reduction runs on every lane (the head vectors of one warp
        // instruction may mix q and k heads, with and without a norm weight)
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(x[e], x[e], ss);
#pragma unroll
        for (int o = LPH / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (is_k[u] ? a.wk != nullptr : a.wq != nullptr) {
          const float rstd = rsqrtf(ss / (float)D + a.eps);
#pragma unroll
          for (int e = 0; e < 8; ++e) x[e] = x[e] * rstd * (is_k[u] ? gk[e] : gq[e]);
        }
        if (a.cos != nullptr) {
          float xp[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) xp[e] = __shfl_sync(0xffffffffu, x[e], partner);
          if (rot) {
#pragma unroll
            for (int e = 0; e < 8; ++e)
              x[e] = j0 < half ? fmaf(x[e], c[e], -xp[e] * s[e]) : fmaf(x[e], c[e], xp[e] * s[e]);
          }
        }
        if (valid[u]) {
          *reinterpret_cast<uint4*>(ptr[u]) =
              make_uint4(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]),
                         pack_bf16x2(x[4], x[5]), pack_bf16x2(x[6], x[7]));
        }
      }
    }
  }
}

}  // namespace h3b
