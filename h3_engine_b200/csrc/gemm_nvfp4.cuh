// NVFP4 x NVFP4 -> bf16 GEMM on the 5th-generation tensor cores (sm_100a).
//
// Replaces torch._scaled_mm(fp4, fp4^T, blocked scales) at
// h3_inference/nvfp4.py:112-115 together with the bias / GELU / residual work
// that follows it in the row shims (h3_inference/kernels/ffn_qkvo_gemms.py).
//
#pragma once

#include "common.cuh"

namespace h3b {

// ============================================================================
// Persistent variant (the production kernel).
//
// grid = min(#tiles, #SMs); CTA b processes tiles b, b+grid, ... in M-major
// raster (consecutive tiles share the A row-block, so concurrently running
// CTAs reuse it from L2).  The producer and the MMA issuer run ahead across
// tile boundaries, so the operand pipeline never drains between tiles.
//   warp 0     TMA producer (3-stage ring, 54 KiB per stage)
//   warp 1     TMEM allocator + MMA issuer: the whole warp runs the issue loop
//              and one elected lane issues each tcgen05.cp / mma / commit
//   warps 2-9  epilogue, two warps per TMEM lane quadrant (128 columns each):
//              they pull the whole 128x256 fp32 accumulator into registers,
//              hand TMEM back to the MMA warp (acc_empty, 8 arrivals), then
//              apply alpha / bias / GELU (or SwiGLU) / gate / residual,
//              convert to bf16, stage 64-column chunks in a 128B-swizzled
//              4 KiB buffer per warp and write them with TMA stores (which
//              clip rows >= M), while the next tile's mainloop runs.
// Every wait is bounded; there is no barrier among the epilogue warps, so a
// timeout in one role always unwinds the whole CTA.
// ============================================================================
namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int KB_ELEMS = 256;
constexpr int KB_BYTES = KB_ELEMS / 2;
constexpr int STAGES = 3;
constexpr int A_BYTES = BM * KB_BYTES;
constexpr int B_BYTES = BN * KB_BYTES;
constexpr int SF_ATOM = 512;
constexpr int SFA_BYTES = (BM / 128) * 4 * SF_ATOM;
constexpr int SFB_BYTES = (BN / 128) * 4 * SF_ATOM;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
constexpr int EPI_WARPS = 8;
constexpr int OUT_CHUNK_COLS = 64;                       // bf16 columns per TMA store
constexpr int OUT_WARP_BYTES = 32 * OUT_CHUNK_COLS * 2;  // 4 KiB, one 128B-swizzled box
constexpr int OUT_OFFSET = STAGES * STAGE_BYTES;
constexpr int BAR_OFFSET = OUT_OFFSET + EPI_WARPS * OUT_WARP_BYTES;
constexpr int SMEM_BYTES = BAR_OFFSET + 256 + 1024;
constexpr int THREADS = 64 + EPI_WARPS * 32;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t ACC_COL = 0;
constexpr uint32_t SF_COL = 256;
constexpr uint32_t SF_STAGE_COLS = 4 * 4 + 4 * 8;
constexpr uint32_t IDESC = (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                           ((uint32_t)(BM >> 4) << 24);

static_assert(STAGE_BYTES % 1024 == 0 && OUT_OFFSET % 1024 == 0, "swizzle alignment");
static_assert(SF_COL + STAGES * SF_STAGE_COLS <= TMEM_COLS, "TMEM budget");
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

struct Args {
  CUtensorMap tmap_a;      // u8 [a_rows, K/2],  box 128 B x 128 rows, 128B swizzle
  CUtensorMap tmap_b;      // u8 [N, K/2],       box 128 B x 256 rows, 128B swizzle
  CUtensorMap tmap_d;      // bf16 [M, N] (pitch ldd), box 64 x 32, 128B swizzle
  const uint8_t* sfa;
  const uint8_t* sfb;
  const float* gs_a;
  const float* gs_b;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* residual;
  const __nv_bfloat16* gate;   // [rows, N]: v *= gate[gate_idx[m], n] (adaLN-zero gate)
  const int32_t* gate_idx;     // [M] or null (row 0)
  float* amax_out;
  long long ldr;
  int M, N, K;
  int sf_atoms_k;
  int act;
  int gsb_seg;
  int n_tiles;
  int num_tiles;
};

__device__ __forceinline__ float gelu_tanh(float v) {
  // 0.5 v (1 + tanh(sqrt(2/pi) (v + 0.044715 v^3))), tanh from the hardware
  // tanh.approx.f32 instruction (max relative error ~2^-11, below bf16 ulp).
  const float u = 0.7978845608028654f * fmaf(0.044715f * v, v * v, v);
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
  return 0.5f * v * (1.0f + t);
}
// The same for two lanes with packed fp32 ops (each lane the scalar op above,
// in the same order: the same bits).
__device__ __forceinline__ float2 gelu_tanh2(float2 v) {
  const float2 inner = fma2(mul2(make_float2(0.044715f, 0.044715f), v), mul2(v, v), v);
  const float2 u = mul2(make_float2(0.7978845608028654f, 0.7978845608028654f), inner);
  float2 t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t.x) : "f"(u.x));
  asm("tanh.approx.f32 %0, %1;" : "=f"(t.y) : "f"(u.y));
  return mul2(mul2(make_float2(0.5f, 0.5f), v), add2(make_float2(1.0f, 1.0f), t));
}

// The epilogue of one warp's 32 rows x 128 accumulator columns (columns
// n0 + 128 * half ..) of a tile whose rows start at m0: alpha, bias, GELU or
// SwiGLU, gate, residual, bf16, |D| max, staged in the warp's 4 KiB buffer and
// written by TMA stores (rows >= M clipped).  Shared by the single-CTA and
// the CTA-pair kernels.  Elementwise steps run as packed two-lane fp32 ops
// (each lane the IEEE op the scalar form does); |D| max is kept on the bf16
// bit patterns of |D| (non-negative bf16 values order like their 16-bit
// integers), two per 32-bit word, and only when the caller asked for it.
__device__ __forceinline__ void amax_bf16x2(uint32_t& amax2, uint32_t o) {
  amax2 = __vmaxu2(amax2, o & 0x7FFF7FFFu);
}
__device__ __forceinline__ float amax_bf16x2_value(uint32_t amax2) {
  return __uint_as_float(max(amax2 & 0xFFFFu, amax2 >> 16) << 16);
}

template <bool SWIGLU>
__device__ __forceinline__ void epilogue_rows(const Args& p, const uint32_t (&acc)[128], int m0,
                                              int n0, int half, int qd, int lane, uint8_t* stage,
                                              uint32_t stage_s, float gsa, uint32_t& amax2) {
  const int n_base = n0 + half * 128;
  const bool want_amax = p.amax_out != nullptr;
  if (SWIGLU) {
    if (m0 + qd * 32 >= p.M) return;
    const int row = m0 + qd * 32 + lane;
    const bool row_ok = row < p.M;
    const float alpha = gsa * (p.gs_b ? __ldg(p.gs_b) : 1.f);
    if (lane == 0) bulk_wait_read0();
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float r[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float v = __bfloat162float(
              __float2bfloat16_rn(__uint_as_float(acc[j * 8 + 2 * e + h]) * alpha));
          const float g = __bfloat162float(
              __float2bfloat16_rn(__uint_as_float(acc[64 + j * 8 + 2 * e + h]) * alpha));
          const float sg = __bfloat162float(__float2bfloat16_rn(g / (1.0f + __expf(-g))));
          r[h] = v * sg;
        }
        o[e] = pack_bf16x2(r[0], r[1]);
        if (want_amax && row_ok) amax_bf16x2(amax2, o[e]);
      }
      *reinterpret_cast<uint4*>(stage + lane * 128 + ((j ^ (lane & 7)) << 4)) =
          make_uint4(o[0], o[1], o[2], o[3]);
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(&p.tmap_d, stage_s, (n0 >> 1) + half * 64, m0 + qd * 32);
      bulk_commit();
    }
    return;
  }
  if (n_base >= p.N || m0 + qd * 32 >= p.M) return;   // warp-uniform
  const int row = m0 + qd * 32 + lane;
  const bool row_ok = row < p.M;
  const float alpha = gsa * (p.gs_b ? __ldg(p.gs_b + (p.gsb_seg ? n_base / p.gsb_seg : 0)) : 1.f);
  const float2 a2 = make_float2(alpha, alpha);
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    if (lane == 0) bulk_wait_read0();   // staging buffer free again
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int col = n_base + c * 64 + j * 8;
      float2 v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        v[e] = mul2(make_float2(__uint_as_float(acc[c * 64 + j * 8 + 2 * e]),
                                __uint_as_float(acc[c * 64 + j * 8 + 2 * e + 1])), a2);
      if (p.bias) {
        const uint4 b = __ldg(reinterpret_cast<const uint4*>(p.bias + col));
        const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = add2(v[e], bf16x2_to_f2(bw[e]));
      }
      if (p.act == H3B_ACT_GELU_TANH) {
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = gelu_tanh2(v[e]);
      }
      if (p.gate) {
        const long long grow = p.gate_idx ? (row_ok ? __ldg(p.gate_idx + row) : 0) : 0;
        const uint4 b = __ldg(reinterpret_cast<const uint4*>(p.gate + grow * p.N + col));
        const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = mul2(v[e], bf16x2_to_f2(bw[e]));
      }
      if (p.residual && row_ok) {
        const uint4 b =
            __ldg(reinterpret_cast<const uint4*>(p.residual + (size_t)row * p.ldr + col));
        const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = add2(v[e], bf16x2_to_f2(bw[e]));
      }
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        o[e] = pack_bf16x2(v[e].x, v[e].y);
        if (want_amax && row_ok) amax_bf16x2(amax2, o[e]);
      }
      // 128B swizzle: 16-byte chunk j of row `lane` sits at chunk j ^ (lane % 8)
      *reinterpret_cast<uint4*>(stage + lane * 128 + ((j ^ (lane & 7)) << 4)) =
          make_uint4(o[0], o[1], o[2], o[3]);
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(&p.tmap_d, stage_s, n_base + c * OUT_CHUNK_COLS, m0 + qd * 32);
      bulk_commit();
    }
  }
}

// SWIGLU: the fused up-projection epilogue (act == H3B_ACT_SWIGLU), a separate
// instantiation so the other epilogues keep their register allocation.
template <bool SWIGLU>
__global__ void __launch_bounds__(THREADS, 1) k_gemm_nvfp4(const __grid_constant__ Args p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFFSET);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = bars + 2 * STAGES;
  uint64_t* acc_empty = bars + 2 * STAGES + 1;
  uint64_t* drain = bars + 2 * STAGES + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 3);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_kb = p.K / KB_ELEMS;

  auto sA = [&](int s) { return smem + s * STAGE_BYTES; };
  auto sB = [&](int s) { return smem + s * STAGE_BYTES + A_BYTES; };
  auto sSFA = [&](int s) { return smem + s * STAGE_BYTES + A_BYTES + B_BYTES; };
  auto sSFB = [&](int s) { return smem + s * STAGE_BYTES + A_BYTES + B_BYTES + SFA_BYTES; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    mbar_init(smem_u32(acc_full), 1);
    mbar_init(smem_u32(acc_empty), EPI_WARPS);
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&p.tmap_a);
      prefetch_tmap(&p.tmap_b);
      uint32_t g = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        const int m0 = (t / p.n_tiles) * BM, n0 = (t % p.n_tiles) * BN;
        const bool b_hi = (n0 + 128) < p.N;
        const uint32_t tx = A_BYTES + B_BYTES + SFA_BYTES + (b_hi ? 2 : 1) * 4 * SF_ATOM;
        const uint8_t* sfa_row = p.sfa + (size_t)(m0 / 128) * p.sf_atoms_k * SF_ATOM;
        const uint8_t* sfb_row0 = p.sfb + (size_t)(n0 / 128) * p.sf_atoms_k * SF_ATOM;
        const uint8_t* sfb_row1 = sfb_row0 + (size_t)p.sf_atoms_k * SF_ATOM;
        for (int kb = 0; kb < num_kb; ++kb, ++g) {
          const int s = g % STAGES;
          const uint32_t ph = (g / STAGES) & 1;
          if (g >= STAGES && !mbar_wait(smem_u32(&empty[s]), ph ^ 1, abort_flag)) {
            record_error(H3B_ERR_TIMEOUT);
            *abort_flag = 1;
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&full[s]);
          mbar_expect_tx(fb, tx);
          tma_load_2d(smem_u32(sA(s)), &p.tmap_a, kb * KB_BYTES, m0, fb);
          tma_load_2d(smem_u32(sB(s)), &p.tmap_b, kb * KB_BYTES, n0, fb);
          bulk_load(smem_u32(sSFA(s)), sfa_row + (size_t)kb * 4 * SF_ATOM, 4 * SF_ATOM, fb);
          bulk_load(smem_u32(sSFB(s)), sfb_row0 + (size_t)kb * 4 * SF_ATOM, 4 * SF_ATOM, fb);
          if (b_hi)
            bulk_load(smem_u32(sSFB(s)) + 4 * SF_ATOM, sfb_row1 + (size_t)kb * 4 * SF_ATOM,
                      4 * SF_ATOM, fb);
        }
      }
      if (!ok || *abort_flag) {
        // Let every copy already in flight land before the CTA can exit.
        for (uint32_t q = g > (uint32_t)STAGES ? g - STAGES : 0; q < g; ++q)
          mbar_wait(smem_u32(&full[q % STAGES]), (q / STAGES) & 1, nullptr);
      }
    }
  } else if (warp == 1) {
    // The whole warp runs the issue loop on warp-uniform values; per MMA
    // k-step one elected lane issues the three scale copies and the MMA back
    // to back (a converged issuer keeps pace beside the busy epilogue warps,
    // and one election per k-step instead of one per op takes the issue
    // stream, the kernel's limit, from ~40 cycles per op down).  Descriptors
    // advance by adding (offset >> 4) to the start-address field.
    auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(smem_u32(bar), parity, abort_flag));
    };
    uint32_t g = 0, i = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x, ++i) {
      if (i > 0 && !wait(acc_empty, (i - 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      for (int kb = 0; kb < num_kb; ++kb, ++g) {
        const int s = g % STAGES;
        const uint32_t ph = (g / STAGES) & 1;
        if (!wait(&full[s], ph)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // Scale atoms of this k-block -> tensor memory (one 32x128b.warpx4
        // copy per 128 rows per MMA k-step), then the four MMAs that read them.
        const uint32_t sf_t = tmem + SF_COL + s * SF_STAGE_COLS;
        const uint64_t sfa_d = desc_sf_atom(smem_u32(sSFA(s)));
        const uint64_t sfb_d = desc_sf_atom(smem_u32(sSFB(s)));
        const uint64_t a_d = desc_kmajor_sw128(smem_u32(sA(s)));
        const uint64_t b_d = desc_kmajor_sw128(smem_u32(sB(s)));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          tc_kstep_nvf4_elect(sf_t + kk * 4, sfa_d + ((kk * SF_ATOM) >> 4), sf_t + 16 + kk * 8,
                              sfb_d + ((kk * SF_ATOM) >> 4), sf_t + 16 + kk * 8 + 4,
                              sfb_d + (((4 + kk) * SF_ATOM) >> 4), tmem + ACC_COL,
                              a_d + ((kk * 32) >> 4), b_d + ((kk * 32) >> 4), IDESC,
                              (kb | kk) != 0);
        }
        tc_commit_elect(smem_u32(&empty[s]));
      }
      if (!ok) break;
      tc_commit_elect(smem_u32(acc_full));
    }
    if (!ok) {
      if (lane == 0 && !*abort_flag) {
        record_error(H3B_ERR_TIMEOUT);
        *abort_flag = 1;
      }
      tc_commit_elect(smem_u32(drain));
      mbar_wait(smem_u32(drain), 0, nullptr);
    }
  } else {
    const int ew = warp - 2;
    const int qd = warp & 3;          // TMEM lane quadrant this warp may access
    const int half = ew >> 2;         // which 128 of the 256 accumulator columns
    uint8_t* stage = smem + OUT_OFFSET + ew * OUT_WARP_BYTES;
    const uint32_t stage_s = smem_u32(stage);
    const float gsa = p.gs_a ? __ldg(p.gs_a) : 1.f;
    uint32_t amax2 = 0;                  // packed |bf16(D)| max of this warp's rows
    uint32_t i = 0;
    if (lane == 0) prefetch_tmap(&p.tmap_d);
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++i) {
      const int m0 = (t / p.n_tiles) * BM, n0 = (t % p.n_tiles) * BN;
      const bool ready = __all_sync(0xffffffffu, mbar_wait(smem_u32(acc_full), i & 1, abort_flag));
      if (!ready) {
        if (!*abort_flag) {
          record_error(H3B_ERR_TIMEOUT);
          *abort_flag = 1;
        }
        break;
      }
      tc_fence_after();
      uint32_t acc[128];
      const uint32_t taddr = tmem + ACC_COL + ((uint32_t)(qd * 32) << 16) + half * 128;
      tmem_ld_32x32b_x64(taddr, acc);
      tmem_ld_32x32b_x64(taddr + 64, acc + 64);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(acc_empty));

      epilogue_rows<SWIGLU>(p, acc, m0, n0, half, qd, lane, stage, stage_s, gsa, amax2);
    }
    if (lane == 0) bulk_wait0();
    if (p.amax_out) {
      float amax = amax_bf16x2_value(amax2);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      if (lane == 0 && amax > 0.f)
        atomicMax(reinterpret_cast<unsigned int*>(p.amax_out), __float_as_uint(amax));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ============================================================================
// CTA-pair variant (cluster of 2): one 256 x 256 output tile per pair, the
// tcgen05 MMA in its cta_group::2 form (M = 256 over the two CTAs' tensor
// memory).  CTA r of the pair TMA-loads, into its own shared memory, rows
// m0 + 128 r .. of A with their scale atoms, rows n0 + 128 r .. of B (its half
// of the tile's N), and the scale atoms of all 256 B rows; every load counts
// its bytes on the leader CTA's full barrier (cta_group::2 form, no
// multicast).  Only the leader's MMA warp issues: per k-block 4 scale copies
// for A and 8 for B (each moving both CTAs' atoms) and 4 MMAs for 2 x the work
// of the single-CTA kernel's 4, so the per-SM tcgen05 issue and the per-SM B
// traffic through shared memory halve.  Commits reach both CTAs' barriers
// (tcgen05.commit multicast).  Each CTA's 8 epilogue warps drain its 128
// accumulator rows exactly as the single-CTA kernel does and arrive on the
// leader's acc_empty.  Every wait is bounded; the pair meets once after
// initialisation and once before tensor memory is freed.
// ============================================================================
constexpr int P_STAGES = 4;
constexpr int P_A_BYTES = 128 * KB_BYTES;            // this CTA's 128 rows of A
constexpr int P_B_BYTES = 128 * KB_BYTES;            // this CTA's half of B
constexpr int P_SFA_BYTES = 4 * SF_ATOM;
constexpr int P_SFB_BYTES = 8 * SF_ATOM;             // all 256 B rows
constexpr int P_STAGE_BYTES = P_A_BYTES + P_B_BYTES + P_SFA_BYTES + P_SFB_BYTES;
constexpr int P_OUT_OFFSET = P_STAGES * P_STAGE_BYTES;
constexpr int P_BAR_OFFSET = P_OUT_OFFSET + EPI_WARPS * OUT_WARP_BYTES;
constexpr int P_SMEM_BYTES = P_BAR_OFFSET + 256 + 1024;
constexpr uint32_t P_IDESC = (1u << 7) | (1u << 10) | ((uint32_t)(256 >> 3) << 17) |
                             ((uint32_t)(256 >> 4) << 24);
static_assert(P_STAGE_BYTES % 1024 == 0 && P_OUT_OFFSET % 1024 == 0, "swizzle alignment");
static_assert(SF_COL + P_STAGES * SF_STAGE_COLS <= TMEM_COLS, "TMEM budget");
static_assert(P_SMEM_BYTES <= 232448, "shared memory budget");

struct PairArgs {
  Args base;               // tmap_a box 128 B x 128 rows; tmap_b box 128 B x 128 rows
  CUtensorMap tmap_sfa;    // u64 [a_rows / 128, K / 64 * 64], box 256 x 1 (one k-block)
  CUtensorMap tmap_sfb;    // u64 [N / 128, K / 64 * 64], box 256 x 2
  int m_tiles;             // 256-row tiles
};

template <bool SWIGLU>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    k_gemm_nvfp4_pair(const __grid_constant__ PairArgs pa) {
  const Args& p = pa.base;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P_BAR_OFFSET);
  uint64_t* full = bars;                       // leader: both CTAs' loads of a stage
  uint64_t* empty = bars + P_STAGES;           // both: stage consumed (leader's commit)
  uint64_t* acc_full = bars + 2 * P_STAGES;    // both: accumulator ready
  uint64_t* acc_empty = bars + 2 * P_STAGES + 1;   // leader: both CTAs drained it
  uint64_t* drain = bars + 2 * P_STAGES + 2;
  uint64_t* bye = bars + 2 * P_STAGES + 3;     // both: the peer is done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * P_STAGES + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int num_kb = p.K / KB_ELEMS;
  const int pair_id = (int)(blockIdx.x >> 1);
  const int num_pairs = (int)(gridDim.x >> 1);
  const int num_tiles = pa.m_tiles * p.n_tiles;

  auto sA = [&](int s) { return smem + s * P_STAGE_BYTES; };
  auto sB = [&](int s) { return smem + s * P_STAGE_BYTES + P_A_BYTES; };
  auto sSFA = [&](int s) { return smem + s * P_STAGE_BYTES + P_A_BYTES + P_B_BYTES; };
  auto sSFB = [&](int s) {
    return smem + s * P_STAGE_BYTES + P_A_BYTES + P_B_BYTES + P_SFA_BYTES;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    mbar_init(smem_u32(acc_full), 1);
    mbar_init(smem_u32(acc_empty), 2 * EPI_WARPS);
    mbar_init(smem_u32(drain), 1);
    mbar_init(smem_u32(bye), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  // both CTAs' barriers exist before any load or arrival reaches them
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto fail = [&]() {
    if (!*abort_flag) {
      record_error(H3B_ERR_TIMEOUT);
      *abort_flag = 1;
    }
  };

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&p.tmap_a);
      prefetch_tmap(&p.tmap_b);
      prefetch_tmap(&pa.tmap_sfa);
      prefetch_tmap(&pa.tmap_sfb);
      uint32_t g = 0;
      bool ok = true;
      for (int t = pair_id; t < num_tiles && ok; t += num_pairs) {
        const int m0 = (t / p.n_tiles) * 256, n0 = (t % p.n_tiles) * BN;
        for (int kb = 0; kb < num_kb; ++kb, ++g) {
          const int s = g % P_STAGES;
          const uint32_t ph = (g / P_STAGES) & 1;
          if (g >= P_STAGES && !mbar_wait(smem_u32(&empty[s]), ph ^ 1, abort_flag)) {
            fail();
            ok = false;
            break;
          }
          const uint32_t lb = mapa_shared(smem_u32(&full[s]), 0);
          if (rank == 0) mbar_expect_tx(smem_u32(&full[s]), 2 * P_STAGE_BYTES);
          tma_load_2d_pair(smem_u32(sA(s)), &p.tmap_a, kb * KB_BYTES, m0 + 128 * (int)rank, lb);
          tma_load_2d_pair(smem_u32(sB(s)), &p.tmap_b, kb * KB_BYTES, n0 + 128 * (int)rank, lb);
          tma_load_2d_pair(smem_u32(sSFA(s)), &pa.tmap_sfa, kb * 256, m0 / 128 + (int)rank, lb);
          tma_load_2d_pair(smem_u32(sSFB(s)), &pa.tmap_sfb, kb * 256, n0 / 128, lb);
        }
      }
      // tail: the release of every stage this CTA filled has arrived (the
      // leader's last commits reach this CTA's barriers before it can exit)
      for (uint32_t q = g > (uint32_t)P_STAGES ? g - P_STAGES : 0; q < g && ok; ++q) {
        if (!mbar_wait(smem_u32(&empty[q % P_STAGES]), (q / P_STAGES) & 1, abort_flag)) {
          fail();
          ok = false;
        }
      }
    }
  } else if (warp == 1) {
    if (rank == 0) {
      auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
        return __all_sync(0xffffffffu, mbar_wait(smem_u32(bar), parity, abort_flag));
      };
      uint32_t g = 0, i = 0;
      bool ok = true;
      for (int t = pair_id; t < num_tiles && ok; t += num_pairs, ++i) {
        if (i > 0 && !wait(acc_empty, (i - 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kb = 0; kb < num_kb; ++kb, ++g) {
          const int s = g % P_STAGES;
          const uint32_t ph = (g / P_STAGES) & 1;
          if (!wait(&full[s], ph)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sf_t = tmem + SF_COL + s * SF_STAGE_COLS;
          const uint64_t sfa_d = desc_sf_atom(smem_u32(sSFA(s)));
          const uint64_t sfb_d = desc_sf_atom(smem_u32(sSFB(s)));
          const uint64_t a_d = desc_kmajor_sw128(smem_u32(sA(s)));
          const uint64_t b_d = desc_kmajor_sw128(smem_u32(sB(s)));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            tc_kstep_nvf4_pair_elect(sf_t + kk * 4, sfa_d + ((kk * SF_ATOM) >> 4),
                                     sf_t + 16 + kk * 8, sfb_d + ((kk * SF_ATOM) >> 4),
                                     sf_t + 16 + kk * 8 + 4, sfb_d + (((4 + kk) * SF_ATOM) >> 4),
                                     tmem + ACC_COL, a_d + ((kk * 32) >> 4),
                                     b_d + ((kk * 32) >> 4), P_IDESC, (kb | kk) != 0);
          }
          tc_commit_pair_elect(smem_u32(&empty[s]), 0x3);
        }
        if (!ok) break;
        tc_commit_pair_elect(smem_u32(acc_full), 0x3);
      }
      if (!ok) {
        if (lane == 0) fail();
        tc_commit_pair_elect(smem_u32(drain), 0x1);
        mbar_wait(smem_u32(drain), 0, nullptr);
      }
    }
  } else {
    const int ew = warp - 2;
    const int qd = warp & 3;
    const int half = ew >> 2;
    uint8_t* stage = smem + P_OUT_OFFSET + ew * OUT_WARP_BYTES;
    const uint32_t stage_s = smem_u32(stage);
    const uint32_t leader_acc_empty = mapa_shared(smem_u32(acc_empty), 0);
    const float gsa = p.gs_a ? __ldg(p.gs_a) : 1.f;
    uint32_t amax2 = 0;                  // packed |bf16(D)| max of this warp's rows
    uint32_t i = 0;
    if (lane == 0) prefetch_tmap(&p.tmap_d);
    for (int t = pair_id; t < num_tiles; t += num_pairs, ++i) {
      const int m0 = (t / p.n_tiles) * 256 + 128 * (int)rank, n0 = (t % p.n_tiles) * BN;
      const bool ready = __all_sync(0xffffffffu, mbar_wait(smem_u32(acc_full), i & 1, abort_flag));
      if (!ready) {
        fail();
        break;
      }
      tc_fence_after();
      uint32_t acc[128];
      const uint32_t taddr = tmem + ACC_COL + ((uint32_t)(qd * 32) << 16) + half * 128;
      tmem_ld_32x32b_x64(taddr, acc);
      tmem_ld_32x32b_x64(taddr + 64, acc + 64);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(leader_acc_empty);
      epilogue_rows<SWIGLU>(p, acc, m0, n0, half, qd, lane, stage, stage_s, gsa, amax2);
    }
    if (lane == 0) bulk_wait0();
    if (p.amax_out) {
      float amax = amax_bf16x2_value(amax2);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      if (lane == 0 && amax > 0.f)
        atomicMax(reinterpret_cast<unsigned int*>(p.amax_out), __float_as_uint(amax));
    }
  }

  tc_fence_before();
  __syncthreads();
  // the pair meets before either frees tensor memory or exits: the peer's
  // accumulator is written by the leader's MMAs, its loads count on the
  // leader's barriers
  if (threadIdx.x == 0) {
    mbar_arrive_cluster(mapa_shared(smem_u32(bye), rank ^ 1u));
    if (!mbar_wait(smem_u32(bye), 0, nullptr)) record_error(H3B_ERR_TIMEOUT);
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem, TMEM_COLS);
  }
}

}  // namespace gemm

}  // namespace h3b
