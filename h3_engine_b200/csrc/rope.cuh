// Per-head RMSNorm + rotate-half RoPE on q and k, in place in the projected
// query / key activations or into separate output rows (HBM-bound).
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
  const __nv_bfloat16* q;  // [T, q_stride], q heads at column q_off + h*D
  const __nv_bfloat16* k;  // [T, k_stride], k heads at column k_off + h*D
  __nv_bfloat16* qo;       // results: [T, qo_stride] at column qo_off + h*D (== q: in place)
  __nv_bfloat16* ko;       // [T, ko_stride] at column ko_off + h*D (== k: in place)
  long long T, q_stride, k_stride;
  long long q_off, k_off;
  long long qo_stride, ko_stride, qo_off, ko_off;
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
    const __nv_bfloat16* qrow = a.hq ? a.q + t * a.q_stride + a.q_off : nullptr;
    const __nv_bfloat16* krow = a.hk ? a.k + t * a.k_stride + a.k_off : nullptr;
    __nv_bfloat16* qorow = a.hq ? a.qo + t * a.qo_stride + a.qo_off : nullptr;
    __nv_bfloat16* korow = a.hk ? a.ko + t * a.ko_stride + a.ko_off : nullptr;
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
        const __nv_bfloat16* src = (is_k[u] ? krow : qrow) + (long long)h * D + j0;
        ptr[u] = (is_k[u] ? korow : qorow) + (long long)h * D + j0;
        raw[u] = valid[u] ? *reinterpret_cast<const uint4*>(src) : make_uint4(0, 0, 0, 0);
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

// Full-width rotary (R == D, the rotate-half partner of every column inside
// the head): lane s of a head's LPH = D/16 lanes holds columns [8s, 8s+8)
// AND their partners [8s + D/2, 8s + D/2 + 8), two 16-byte loads, so the
// rotation needs no shuffles and the sum of squares reduces over LPH lanes.
// Same arithmetic, in the same order, as k_qk_norm_rope: bit-identical.
template <int D, int UNROLL>
__global__ void __launch_bounds__(kRopeWarps * 32, 2) k_qk_norm_rope_full(const RopeArgs a) {
  constexpr int LPH = D / 16;                // lanes per head vector
  constexpr int HPW = 32 / LPH;              // head vectors per warp instruction
  constexpr int HALF = D / 2;
  const int lane = threadIdx.x & 31;
  const int sub = lane % LPH;
  const int j0 = sub * 8;                    // first column of the lower half
  float gq[16], gk[16];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    gq[e] = a.wq ? __bfloat162float(a.wq[j0 + e]) : 1.f;
    gq[8 + e] = a.wq ? __bfloat162float(a.wq[HALF + j0 + e]) : 1.f;
    gk[e] = a.wk ? __bfloat162float(a.wk[j0 + e]) : 1.f;
    gk[8 + e] = a.wk ? __bfloat162float(a.wk[HALF + j0 + e]) : 1.f;
  }
  const int nv = a.hq + a.hk;
  const long long warp_id = (long long)blockIdx.x * kRopeWarps + (threadIdx.x >> 5);
  const long long nwarps = (long long)gridDim.x * kRopeWarps;
  for (long long t = warp_id; t < a.T; t += nwarps) {
    float c[16], s[16];
    {
      const float* cr = a.cos + t * a.cs_stride;
      const float* sr = a.sin + t * a.cs_stride;
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        const float4* cp = reinterpret_cast<const float4*>(cr + part * HALF + j0);
        const float4* sp = reinterpret_cast<const float4*>(sr + part * HALF + j0);
        const float4 c0 = __ldg(cp), c1 = __ldg(cp + 1), s0 = __ldg(sp), s1 = __ldg(sp + 1);
        const float cv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
        const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          c[part * 8 + e] = __bfloat162float(__float2bfloat16_rn(cv[e]));
          s[part * 8 + e] = __bfloat162float(__float2bfloat16_rn(sv[e]));
        }
      }
    }
    const __nv_bfloat16* qrow = a.hq ? a.q + t * a.q_stride + a.q_off : nullptr;
    const __nv_bfloat16* krow = a.hk ? a.k + t * a.k_stride + a.k_off : nullptr;
    __nv_bfloat16* qorow = a.hq ? a.qo + t * a.qo_stride + a.qo_off : nullptr;
    __nv_bfloat16* korow = a.hk ? a.ko + t * a.ko_stride + a.ko_off : nullptr;
    for (int v0 = 0; v0 < nv; v0 += HPW * UNROLL) {
      uint4 lo[UNROLL], hi[UNROLL];
      __nv_bfloat16* ptr[UNROLL];
      bool is_k[UNROLL], valid[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const int v = v0 + u * HPW + lane / LPH;
        valid[u] = v < nv;
        is_k[u] = v >= a.hq;
        const int h = is_k[u] ? v - a.hq : v;
        const __nv_bfloat16* src = (is_k[u] ? krow : qrow) + (long long)h * D + j0;
        ptr[u] = (is_k[u] ? korow : qorow) + (long long)h * D + j0;
        lo[u] = valid[u] ? *reinterpret_cast<const uint4*>(src) : make_uint4(0, 0, 0, 0);
        hi[u] = valid[u] ? *reinterpret_cast<const uint4*>(src + HALF) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const uint32_t w[8] = {lo[u].x, lo[u].y, lo[u].z, lo[u].w, hi[u].x, hi[u].y, hi[u].z, hi[u].w};
        float x[16];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          x[2 * i] = __uint_as_float(w[i] << 16);
          x[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
        }
        // the sum of squares in k_qk_norm_rope's order: per 8 columns, then
        // lower + upper half (its first butterfly step, lanes D/16 apart),
        // then the remaining butterfly over the head's lanes: same rounding
        float sa = 0.f, sb = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) sa = fmaf(x[e], x[e], sa);
#pragma unroll
        for (int e = 0; e < 8; ++e) sb = fmaf(x[8 + e], x[8 + e], sb);
        float ss = sa + sb;
#pragma unroll
        for (int o = LPH / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float* g = is_k[u] ? gk : gq;
        if (is_k[u] ? a.wk != nullptr : a.wq != nullptr) {
          const float rstd = rsqrtf(ss / (float)D + a.eps);
#pragma unroll
          for (int e = 0; e < 16; ++e) x[e] = x[e] * rstd * g[e];
        }
        float y[16];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          y[e] = fmaf(x[e], c[e], -x[8 + e] * s[e]);
          y[8 + e] = fmaf(x[8 + e], c[8 + e], x[e] * s[8 + e]);
        }
        if (valid[u]) {
          *reinterpret_cast<uint4*>(ptr[u]) =
              make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]),
                         pack_bf16x2(y[4], y[5]), pack_bf16x2(y[6], y[7]));
          *reinterpret_cast<uint4*>(ptr[u] + HALF) =
              make_uint4(pack_bf16x2(y[8], y[9]), pack_bf16x2(y[10], y[11]),
                         pack_bf16x2(y[12], y[13]), pack_bf16x2(y[14], y[15]));
        }
      }
    }
  }
}

}  // namespace h3b
