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
  int R;                   // rotary dims (even, <= D)
  const __nv_bfloat16* wq; // [D] or null
  const __nv_bfloat16* wk; // [D] or null
  const float* cos;        // [T, R] (row stride cs_stride) or null
  const float* sin;
  long long cs_stride;
  float eps;
};

constexpr int kRopeWarps = 8;

// One warp per head vector; lane l holds elements [l*D/32, (l+1)*D/32).
// The rotate-half partner of element j (j +- R/2) lives in another lane and
// is fetched with a shuffle (R/2 is a multiple of D/32, so slots line up).
template <int D>
__global__ void __launch_bounds__(kRopeWarps * 32) k_qk_norm_rope(const RopeArgs a) {
  constexpr int EPL = D / 32;     // elements per lane (2 or 4)
  const int lane = threadIdx.x & 31;
  const long long total = a.T * 2 * a.H;
  const long long warp_id = (long long)blockIdx.x * kRopeWarps + (threadIdx.x >> 5);
  const long long nwarps = (long long)gridDim.x * kRopeWarps;
  const int half = a.R >> 1;
  for (long long w = warp_id; w < total; w += nwarps) {
    const long long t = w / (2 * a.H);
    const int v = (int)(w - t * 2 * a.H);
    const bool is_k = v >= a.H;
    const int h = is_k ? v - a.H : v;
    __nv_bfloat16* p = (is_k ? a.k + t * a.k_stride + a.k_off : a.q + t * a.q_stride + a.q_off) +
                       (long long)h * D + lane * EPL;
    float x[EPL];
    if (EPL == 4) {
      const uint2 r = *reinterpret_cast<const uint2*>(p);
      x[0] = __uint_as_float(r.x << 16);
      x[1] = __uint_as_float(r.x & 0xFFFF0000u);
      x[2] = __uint_as_float(r.y << 16);
      x[3] = __uint_as_float(r.y & 0xFFFF0000u);
    } else {
      const uint32_t r = *reinterpret_cast<const uint32_t*>(p);
      x[0] = __uint_as_float(r << 16);
      x[1] = __uint_as_float(r & 0xFFFF0000u);
    }
    const __nv_bfloat16* wp = is_k ? a.wk : a.wq;
    if (wp != nullptr) {
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) ss = fmaf(x[e], x[e], ss);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float rstd = rsqrtf(ss / (float)D + a.eps);
#pragma unroll
      for (int e = 0; e < EPL; ++e) x[e] = x[e] * rstd * __bfloat162float(wp[lane * EPL + e]);
    }
    if (a.cos != nullptr) {
      const int j0 = lane * EPL;
      const int plane = j0 < half ? (j0 + half) / EPL : (j0 - half) / EPL;
      float xp[EPL];
#pragma unroll
      for (int e = 0; e < EPL; ++e) xp[e] = __shfl_sync(0xffffffffu, x[e], plane & 31);
      if (j0 < a.R) {
        const float* cp = a.cos + t * a.cs_stride + j0;
        const float* sp = a.sin + t * a.cs_stride + j0;
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          const float c = __bfloat162float(__float2bfloat16_rn(__ldg(cp + e)));
          const float s = __bfloat162float(__float2bfloat16_rn(__ldg(sp + e)));
          x[e] = j0 < half ? fmaf(x[e], c, -xp[e] * s) : fmaf(x[e], c, xp[e] * s);
        }
      }
    }
    if (EPL == 4) {
      *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]));
    } else {
      *reinterpret_cast<uint32_t*>(p) = pack_bf16x2(x[0], x[1]);
    }
  }
}

}  // namespace h3b
