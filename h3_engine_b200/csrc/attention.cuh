// Packed variable-length self-attention on the 5th-generation tensor cores
// (bf16 in, fp32 softmax / accumulation, bf16 out), head_dim 128.
//
// Replaces F.scaled_dot_product_attention over the packed sequence in
// packed_self_attention (h3_inference/kernels/packed_self_attn.py:8-37):
// non-causal softmax(Q K^T * scale) V, restricted to each document of the
// packing (cu_seqlens).  A single document reproduces the reference model,
// which attends over the whole packed sequence.
//
// One CTA = one 128-row query tile of one head of one document:
//   warp 0      TMA producer: Q tile once, then K and V tiles (128 rows x 128)
//               into two separate 2-stage rings, read straight from the packed
//               QKV activation (q|k|v blocks of one [T, row_stride] buffer).
//   warp 1      TMEM allocator + single-thread MMA issuer:
//                 S_j = Q K_j^T   (tcgen05.mma kind::f16, SS, M=128 N=128 K=16 x8)
//                 O  += P_j V_j   (TS form: P_j read from tensor memory, V_j
//                                  MN-major from shared memory)
//   warps 2-5   softmax + epilogue, one query row per thread: read S_j from
//               TMEM, online softmax in the exp2 domain, write P_j (bf16) back
//               into S_j's columns; O is rescaled in TMEM only when a row max
//               grows by more than 2^8 (the final O / l is exact either way);
//               at the end O / l -> bf16 -> global.
// TMEM: three S buffers (cols 0..383, QK_{j+1} overlaps softmax_j) + O (384..511).
// Every wait is bounded (2 s); on expiry the CTA records H3B_ERR_TIMEOUT and
// unwinds.
#pragma once

#include "common.cuh"

namespace h3b {
namespace attn {

constexpr int BQ = 128;          // query rows per CTA
constexpr int BK = 128;          // key / value rows per step
constexpr int D = 128;           // head dim
constexpr int TILE_BYTES = BQ * D * 2;   // 32 KiB (two 64-column, 128B-swizzled boxes)
constexpr int BOX_BYTES = TILE_BYTES / 2;
constexpr int Q_OFF = 0;
constexpr int K_OFF = TILE_BYTES;                  // 2 stages
constexpr int V_OFF = K_OFF + 2 * TILE_BYTES;      // 2 stages
constexpr int BAR_OFF = V_OFF + 2 * TILE_BYTES;
constexpr int SMEM_BYTES = BAR_OFF + 256 + 1024;
constexpr int THREADS = 192;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t O_COL = 384;
constexpr int MAX_DOCS = 64;
// kind::f16: D fp32 (bit 4), A = B = bf16 (bits 7, 10), N>>3 at 17, M>>4 at 24
constexpr uint32_t IDESC_QK = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BK >> 3) << 17) |
                              ((uint32_t)(BQ >> 4) << 24);
// P V: B = V is MN-major (head dim contiguous): bit 16
constexpr uint32_t IDESC_PV = IDESC_QK | (1u << 16);
constexpr float kRescaleLog2 = 8.0f;

static_assert(SMEM_BYTES <= 232448, "shared memory budget");

struct Args {
  CUtensorMap tmap_q;      // bf16 [q_rows, q_stride], box 64 x 128, 128B swizzle
  CUtensorMap tmap_kv;     // bf16 [kv_rows, kv_stride], same box
  __nv_bfloat16* out;      // [q_rows, ldo]; head h at columns h*D
  long long ldo;
  int q_off, k_off, v_off; // element offsets of the q / k / v head blocks in their rows
  int H;
  float scale_log2;        // softmax scale * log2(e)
  int ndocs;
  int doc_start[MAX_DOCS]; // first key row of the document (kv buffer rows)
  int doc_len[MAX_DOCS];   // keys in the document
  int q_start[MAX_DOCS];   // first local query row of the document (q buffer rows)
  int q_len[MAX_DOCS];     // local queries in the document
  int item_end[MAX_DOCS];  // cumulative CTA counts (q_tiles * H) per document
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(THREADS, 1) k_fmha(const __grid_constant__ Args p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint64_t* q_full = bars;           // 1
  uint64_t* k_full = bars + 1;       // 2
  uint64_t* k_empty = bars + 3;      // 2
  uint64_t* v_full = bars + 5;       // 2
  uint64_t* v_empty = bars + 7;      // 2
  uint64_t* s_full = bars + 9;       // 3
  uint64_t* p_full = bars + 12;      // 3
  uint64_t* pv_done = bars + 15;     // 3
  uint64_t* drain = bars + 18;       // 1
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 19);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // work item -> (document, query tile, head); query tiles vary fastest so
  // neighbouring CTAs share K / V of one head in L2
  int doc = 0;
  while (doc + 1 < p.ndocs && (int)blockIdx.x >= p.item_end[doc]) ++doc;
  const int item = (int)blockIdx.x - (doc > 0 ? p.item_end[doc - 1] : 0);
  const int len = p.doc_len[doc];
  const int q_len = p.q_len[doc];
  const int q_tiles = (q_len + BQ - 1) / BQ;
  const int head = item / q_tiles;
  const int qt = item - head * q_tiles;
  const int row0 = p.doc_start[doc];
  const int q_row = p.q_start[doc] + qt * BQ;   // local row in the q / out buffers
  const int n_kv = (len + BK - 1) / BK;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(q_full), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&k_full[i]), 1);
      mbar_init(smem_u32(&k_empty[i]), 1);
      mbar_init(smem_u32(&v_full[i]), 1);
      mbar_init(smem_u32(&v_empty[i]), 1);
    }
    for (int i = 0; i < 3; ++i) {
      mbar_init(smem_u32(&s_full[i]), 1);
      mbar_init(smem_u32(&p_full[i]), 4);
      mbar_init(smem_u32(&pv_done[i]), 1);
    }
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

  auto fail = [&]() {
    if (!*abort_flag) {
      record_error(H3B_ERR_TIMEOUT);
      *abort_flag = 1;
    }
  };

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&p.tmap_q);
      prefetch_tmap(&p.tmap_kv);
      const int qx = p.q_off + head * D, kx = p.k_off + head * D, vx = p.v_off + head * D;
      uint32_t fb = smem_u32(q_full);
      mbar_expect_tx(fb, TILE_BYTES);
      tma_load_2d(smem_u32(smem + Q_OFF), &p.tmap_q, qx, q_row, fb);
      tma_load_2d(smem_u32(smem + Q_OFF + BOX_BYTES), &p.tmap_q, qx + 64, q_row, fb);
      // issue order: K_0, then {K_{j+1}, V_j}: K runs one tile ahead of V
      int nk = 0, nv = 0;   // tiles issued
      bool ok = true;
      auto load_k = [&](int j) -> bool {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(smem_u32(&k_empty[s]), ((j >> 1) - 1) & 1, abort_flag)) return false;
        const uint32_t b = smem_u32(&k_full[s]);
        mbar_expect_tx(b, TILE_BYTES);
        uint8_t* dst = smem + K_OFF + s * TILE_BYTES;
        tma_load_2d(smem_u32(dst), &p.tmap_kv, kx, row0 + j * BK, b);
        tma_load_2d(smem_u32(dst + BOX_BYTES), &p.tmap_kv, kx + 64, row0 + j * BK, b);
        ++nk;
        return true;
      };
      auto load_v = [&](int j) -> bool {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(smem_u32(&v_empty[s]), ((j >> 1) - 1) & 1, abort_flag)) return false;
        const uint32_t b = smem_u32(&v_full[s]);
        mbar_expect_tx(b, TILE_BYTES);
        uint8_t* dst = smem + V_OFF + s * TILE_BYTES;
        tma_load_2d(smem_u32(dst), &p.tmap_kv, vx, row0 + j * BK, b);
        tma_load_2d(smem_u32(dst + BOX_BYTES), &p.tmap_kv, vx + 64, row0 + j * BK, b);
        ++nv;
        return true;
      };
      ok = load_k(0);
      for (int j = 0; j < n_kv && ok; ++j) {
        if (j + 1 < n_kv) ok = load_k(j + 1);
        if (ok) ok = load_v(j);
      }
      if (!ok) {
        fail();
        // let every copy in flight land before the CTA can exit
        mbar_wait(smem_u32(q_full), 0, nullptr);
        for (int j = nk > 2 ? nk - 2 : 0; j < nk; ++j)
          mbar_wait(smem_u32(&k_full[j & 1]), (j >> 1) & 1, nullptr);
        for (int j = nv > 2 ? nv - 2 : 0; j < nv; ++j)
          mbar_wait(smem_u32(&v_full[j & 1]), (j >> 1) & 1, nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t q_s = smem_u32(smem + Q_OFF);
      auto issue_qk = [&](int j) {
        const uint32_t k_s = smem_u32(smem + K_OFF + (j & 1) * TILE_BYTES);
        const uint32_t d = tmem + (uint32_t)(j % 3) * 128;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * BOX_BYTES + (kk & 3) * 32;   // 16 head dims
          tc_mma_bf16_ss(d, desc_kmajor_sw128(q_s + off), desc_kmajor_sw128(k_s + off), IDESC_QK,
                         kk != 0);
        }
        tc_commit(smem_u32(&s_full[j % 3]));
        tc_commit(smem_u32(&k_empty[j & 1]));
      };
      bool ok = mbar_wait(smem_u32(q_full), 0, abort_flag) &&
                mbar_wait(smem_u32(&k_full[0]), 0, abort_flag);
      if (ok) {
        tc_fence_after();
        issue_qk(0);
      }
      for (int j = 0; j < n_kv && ok; ++j) {
        if (j + 1 < n_kv) {
          const int jn = j + 1;
          // S buffer jn % 3 last held P_{jn-3}: its P V must be done
          if (jn >= 3 && !mbar_wait(smem_u32(&pv_done[jn % 3]), ((jn - 3) / 3) & 1, abort_flag)) {
            ok = false;
            break;
          }
          if (!mbar_wait(smem_u32(&k_full[jn & 1]), (jn >> 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_qk(jn);
        }
        if (!mbar_wait(smem_u32(&p_full[j % 3]), (j / 3) & 1, abort_flag) ||
            !mbar_wait(smem_u32(&v_full[j & 1]), (j >> 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t p_t = tmem + (uint32_t)(j % 3) * 128;
        const uint32_t v_s = smem_u32(smem + V_OFF + (j & 1) * TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          // 16 keys: P columns kk*8.. (bf16 pairs), V rows kk*16.. (MN-major:
          // 64-dim chunks LBO = 16 KiB apart, 8-row groups SBO = 1 KiB apart)
          tc_mma_bf16_ts(tmem + O_COL, p_t + kk * 8, smem_desc(v_s + kk * 2048, BOX_BYTES, 1024, 2),
                         IDESC_PV, (j | kk) != 0);
        }
        tc_commit(smem_u32(&v_empty[j & 1]));
        tc_commit(smem_u32(&pv_done[j % 3]));
      }
      if (!ok) {
        fail();
        tc_commit(smem_u32(drain));
        mbar_wait(smem_u32(drain), 0, nullptr);
      }
    }
  } else {
    // softmax: thread = query row (TMEM lane quadrant warp % 4)
    const int qd = warp & 3;
    const int r = qd * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(qd * 32) << 16;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&s_full[j % 3]), (j / 3) & 1, abort_flag));
      if (!ok) break;
      tc_fence_after();
      const uint32_t s_t = tmem + lane_addr + (uint32_t)(j % 3) * 128;
      uint32_t sv[128];
      tmem_ld_32x32b_x64(s_t, sv);
      tmem_ld_32x32b_x64(s_t + 64, sv + 64);
      tmem_ld_wait();
      const int valid = min(BK, len - j * BK);   // keys of this tile inside the document
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < BK; ++c) {
        const float t = c < valid ? __uint_as_float(sv[c]) * p.scale_log2 : -INFINITY;
        sv[c] = __float_as_uint(t);
        mx = fmaxf(mx, t);
      }
      const float m_new = fmaxf(m_used, mx);
      if (__any_sync(0xffffffffu, m_new > m_used + kRescaleLog2)) {
        const float alpha = ex2(m_used - m_new);   // 0 on the first tile (m_used = -inf)
        if (j > 0) {
          // O must be final for P_{j-1} before it is rescaled
          ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&pv_done[(j - 1) % 3]),
                                                  ((j - 1) / 3) & 1, abort_flag));
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            uint32_t ov[32];
            tmem_ld_32x32b_x32(tmem + lane_addr + O_COL + h * 32, ov);
            tmem_ld_wait();
#pragma unroll
            for (int c = 0; c < 32; ++c) ov[c] = __float_as_uint(__uint_as_float(ov[c]) * alpha);
            tmem_st_32x32b_x32(tmem + lane_addr + O_COL + h * 32, ov);
          }
          tmem_st_wait();
        }
        l *= alpha;
        m_used = m_new;
      }
      float sum = 0.f;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float a = ex2(__uint_as_float(sv[h * 64 + 2 * c]) - m_used);
          const float b = ex2(__uint_as_float(sv[h * 64 + 2 * c + 1]) - m_used);
          sum += a + b;
          pk[c] = pack_bf16x2(a, b);
        }
        tmem_st_32x32b_x32(s_t + h * 32, pk);   // P_j over the first 64 columns of S_j
      }
      l += sum;
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&p_full[j % 3]));
    }
    if (ok && n_kv > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&pv_done[(n_kv - 1) % 3]),
                                              ((n_kv - 1) / 3) & 1, abort_flag));
    }
    if (!ok) {
      fail();
    } else if (n_kv > 0) {
      tc_fence_after();
      const float inv_l = 1.0f / l;
      const bool row_ok = qt * BQ + r < q_len;
      __nv_bfloat16* op = p.out + (size_t)(q_row + r) * p.ldo + (size_t)head * D;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t ov[64];
        tmem_ld_32x32b_x64(tmem + lane_addr + O_COL + h * 64, ov);
        tmem_ld_wait();
        if (row_ok) {
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(ov[8 * c + 0]) * inv_l, __uint_as_float(ov[8 * c + 1]) * inv_l);
            w.y = pack_bf16x2(__uint_as_float(ov[8 * c + 2]) * inv_l, __uint_as_float(ov[8 * c + 3]) * inv_l);
            w.z = pack_bf16x2(__uint_as_float(ov[8 * c + 4]) * inv_l, __uint_as_float(ov[8 * c + 5]) * inv_l);
            w.w = pack_bf16x2(__uint_as_float(ov[8 * c + 6]) * inv_l, __uint_as_float(ov[8 * c + 7]) * inv_l);
            *reinterpret_cast<uint4*>(op + h * 64 + c * 8) = w;
          }
        }
      }
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

}  // namespace attn
}  // namespace h3b
