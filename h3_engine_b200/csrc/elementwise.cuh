// Gathered adaLN elementwise ops of the reference block's row shims
// (HBM-bound), with torch's bf16 rounding after every op so the results
// equal the reference's stock expressions bit for bit:
//
//   gate_residual (h3_inference/kernels/elementwise_norm_rope.py:150-163):
//     out = bf16( residual + bf16( gate[idx[t]] * y ) )
//   ada_modulate  (h3_inference/kernels/elementwise_norm_rope.py:90-102):
//     out = bf16( bf16( x * bf16(1 + scale[idx[t]]) ) + shift[idx[t]] )
//
// Rows are (batch, token) pairs of a [rows, cols] bf16 activation; the table
// row of row r is idx[r % n_idx] (the reference's indices are per token,
// broadcast over the batch).  One warp per row (grid-stride), 16-byte lanes,
// four in flight.
#pragma once

#include "common.cuh"

namespace h3b {

struct EwArgs {
  const __nv_bfloat16* a;      // residual (gate_residual) or x (ada_modulate)
  const __nv_bfloat16* b;      // y (gate_residual) or unused
  const __nv_bfloat16* t0;     // gate table, or the scale table
  const __nv_bfloat16* t1;     // unused, or the shift table
  const int32_t* idx;          // [n_idx] table rows (NULL: row 0)
  __nv_bfloat16* out;
  long long rows, cols, lda, ldb, ldo, n_idx;
};

__device__ __forceinline__ float bf16r(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

template <bool GATE>
__global__ void __launch_bounds__(256) k_gather_elementwise(const EwArgs p) {
  const int lane = threadIdx.x & 31;
  const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
  const long long c8 = p.cols >> 3;
  constexpr int U = 4;
  for (long long r = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < p.rows; r += nw) {
    const long long m = p.idx ? (long long)__ldg(p.idx + (p.n_idx > 0 ? r % p.n_idx : 0)) : 0;
    const __nv_bfloat16* ar = p.a + r * p.lda;
    const __nv_bfloat16* br = GATE ? p.b + r * p.ldb : nullptr;
    const __nv_bfloat16* t0 = p.t0 + m * p.cols;
    const __nv_bfloat16* t1 = GATE ? nullptr : p.t1 + m * p.cols;
    __nv_bfloat16* orow = p.out + r * p.ldo;
    for (long long c0 = lane; c0 < c8; c0 += 32 * U) {
      uint4 av[U], bv[U], tv[U], sv[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const long long c = c0 + (long long)u * 32;
        if (c < c8) {
          av[u] = ld_nc_v4(ar + c * 8);
          bv[u] = GATE ? ld_nc_v4(br + c * 8) : make_uint4(0, 0, 0, 0);
          tv[u] = __ldg(reinterpret_cast<const uint4*>(t0) + c);
          sv[u] = GATE ? make_uint4(0, 0, 0, 0) : __ldg(reinterpret_cast<const uint4*>(t1) + c);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const long long c = c0 + (long long)u * 32;
        if (c >= c8) break;
        const uint32_t aw[4] = {av[u].x, av[u].y, av[u].z, av[u].w};
        const uint32_t bw[4] = {bv[u].x, bv[u].y, bv[u].z, bv[u].w};
        const uint32_t tw[4] = {tv[u].x, tv[u].y, tv[u].z, tv[u].w};
        const uint32_t sw[4] = {sv[u].x, sv[u].y, sv[u].z, sv[u].w};
        uint32_t o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 a2 = bf16x2_to_f2(aw[i]), t2 = bf16x2_to_f2(tw[i]);
          float lo, hi;
          if (GATE) {
            const float2 y2 = bf16x2_to_f2(bw[i]);
            lo = __fadd_rn(a2.x, bf16r(__fmul_rn(t2.x, y2.x)));
            hi = __fadd_rn(a2.y, bf16r(__fmul_rn(t2.y, y2.y)));
          } else {
            const float2 s2 = bf16x2_to_f2(sw[i]);
            lo = __fadd_rn(bf16r(__fmul_rn(a2.x, bf16r(__fadd_rn(1.0f, t2.x)))), s2.x);
            hi = __fadd_rn(bf16r(__fmul_rn(a2.y, bf16r(__fadd_rn(1.0f, t2.y)))), s2.y);
          }
          o[i] = pack_bf16x2(lo, hi);
        }
        *reinterpret_cast<uint4*>(orow + c * 8) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
}

}  // namespace h3b
