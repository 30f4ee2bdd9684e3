// Packed variable-length self-attention on the 5th-generation tensor cores
// (bf16 in, fp32 softmax / accumulation, bf16 out), head_dim 128.
//
// Replaces F.scaled_dot_product_attention over the packed sequence in
// packed_self_attention (h3_inference/kernels/packed_self_attn.py:8-37):
// non-causal softmax(Q K^T * scale) V, restricted to each document of the
// packing (cu_seqlens).  A single document reproduces the reference model,
// which attends over the whole packed sequence.
//
// One CTA = two 128-row query tiles (A, B) of one head of one document; K/V
// tiles are loaded once for both:
//   warp 8      TMA producer: Q_A, Q_B and K(0) once, then V(j) with K(j+1)
//               into 2-stage rings, read straight from the q / kv activations,
//               with L2 prefetches a few tiles ahead.
//   warp 9      TMEM allocator + MMA issuer (the whole warp runs the issue
//               loop, one elected lane issues each op).  One in-order MMA
//               stream, staggered so the tensor core works on one tile while
//               the other tile's softmax runs:
//                 QK_A(0) QK_B(0) | PV_A(j) QK_A(j+1) PV_B(j) QK_B(j+1) | ...
//               S = Q K^T: tcgen05.mma kind::f16, SS, M=128 N=128 K=16 x8;
//               O += P V: TS form, P read from tensor memory, V MN-major,
//               issued in two halves: keys [0, 64) as soon as softmax has
//               stored their P (p_half), the rest on p_full, so the first
//               half runs under the second half's exponentials.
//               P_X(j) lives in the columns of S_X; QK_X(j+1) overwrites them
//               only after PV_X(j), in issue order.
//   warps 0-3   softmax of tile A, warps 4-7 of tile B (one query row per
//               thread): the row of S is read from TMEM into registers once,
//               its max taken, exponentiated (5/8 on the MUFU ex2 unit, 3/8 by
//               an FMA polynomial), summed and written back as P (bf16); O is
//               rescaled in TMEM only when a row max grows by more than 2^8
//               (the final O / l is exact either way); at the end
//               O / l -> bf16 -> global.
// TMEM: S_A [0,128), S_B [128,256), O_A [256,384), O_B [384,512).
// Every wait is bounded (2 s); on expiry the CTA records H3B_ERR_TIMEOUT and
// unwinds.
#pragma once

#include "common.cuh"

namespace h3b {
namespace attn {

constexpr int BQ = 128;          // query rows per tile (two tiles per CTA)
constexpr int BK = 128;          // key / value rows per step
constexpr int D = 128;           // head dim
constexpr int TILE_BYTES = BQ * D * 2;   // 32 KiB (two 64-column, 128B-swizzled boxes)
constexpr int BOX_BYTES = TILE_BYTES / 2;
constexpr int Q_OFF = 0;                           // Q_A, Q_B
constexpr int K_OFF = 2 * TILE_BYTES;              // 2 stages
constexpr int V_OFF = K_OFF + 2 * TILE_BYTES;      // 2 stages
constexpr int BAR_OFF = V_OFF + 2 * TILE_BYTES;
constexpr int SMEM_BYTES = BAR_OFF + 256 + 1024;
constexpr int THREADS = 384;       // three warpgroups: softmax A, softmax B, producer + MMA
// Register split (setmaxnreg): the kernel launches at kLaunchRegs per thread
// (three warps per SM sub-partition); the producer/MMA warpgroup gives back
// down to kCtrlRegs so the two softmax warpgroups can hold a whole 128-key row
// of S: 128 * kCtrlRegs + 256 * kSoftmaxRegs == THREADS * kLaunchRegs.
constexpr int kLaunchRegs = 168;
constexpr int kCtrlRegs = 72;
constexpr int kSoftmaxRegs = 216;
static_assert(128 * kCtrlRegs + 256 * kSoftmaxRegs <= THREADS * kLaunchRegs, "register split");
constexpr uint32_t TMEM_COLS = 512;
__host__ __device__ constexpr uint32_t s_col(int t) { return (uint32_t)t * 128u; }
__host__ __device__ constexpr uint32_t o_col(int t) { return 256u + (uint32_t)t * 128u; }
constexpr int MAX_DOCS = 64;
// kind::f16: D fp32 (bit 4), A = B = bf16 (bits 7, 10), N>>3 at 17, M>>4 at 24
constexpr uint32_t IDESC_QK = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BK >> 3) << 17) |
                              ((uint32_t)(BQ >> 4) << 24);
// P V: B = V is MN-major (head dim contiguous): bit 16
constexpr uint32_t IDESC_PV = IDESC_QK | (1u << 16);
constexpr float kRescaleLog2 = 8.0f;
constexpr int kPrefetchTiles = 4;     // K / V tiles warmed in L2 ahead of the loads

static_assert(SMEM_BYTES <= 232448, "shared memory budget");

struct Args {
  CUtensorMap tmap_q;      // bf16 [q_rows, q_stride], box 64 x 128, 128B swizzle
  CUtensorMap tmap_kv;     // keys: bf16 [kv_rows, k_stride], same box
  CUtensorMap tmap_v;      // values: bf16 [kv_rows, v_stride] (often the keys' map)
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
  int item_end[MAX_DOCS];  // cumulative CTA counts (query-tile pairs * H) per document
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for two lanes on the FMA pipe: x = n + f with n = round(x) (adding
// 1.5 * 2^23 rounds to an integer in the low mantissa bits), f in [-0.5, 0.5];
// 2^f by a cubic fitted here by relative-error-weighted least squares on
// Chebyshev nodes (max relative error 1.2e-4, below the bf16 rounding P
// receives); 2^n added into the exponent field.  x is clamped to >= -120 so the
// result stays a normal number; callers never pass masked keys here.
__device__ __forceinline__ float2 ex2_poly2(float2 x) {
  x.x = fmaxf(x.x, -120.0f);
  x.y = fmaxf(x.y, -120.0f);
  const float2 magic = make_float2(12582912.0f, 12582912.0f);
  const float2 t = add2(x, magic);
  const float2 f = sub2(x, sub2(t, magic));
  float2 q = fma2(f, make_float2(0.05459282547235489f, 0.05459282547235489f),
                  make_float2(0.24221783876419067f, 0.24221783876419067f));
  q = fma2(f, q, make_float2(0.6933686137199402f, 0.6933686137199402f));
  q = fma2(f, q, make_float2(1.0f, 1.0f));
  return make_float2(__int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23)));
}

// Key pairs (of each 8) whose exponentials go to the FMA polynomial; the rest
// use the MUFU ex2 unit (16 results per clock per SM).
constexpr uint32_t kPolyPairs = 0x52u;   // pairs 1, 4, 6

// P = 2^(S * scale_log2 - m) for NC keys of one row held in registers, packed
// to bf16 pairs and stored over NC / 2 columns of the row's S in tensor
// memory from s_addr; returns the sum (two lanes).  Once the first 64 keys'
// P is stored the warp arrives on half_bar.  MIXED splits the
// exponentials between MUFU and the polynomial; a partial last tile of a
// document uses MUFU only, where a masked key (S = -inf) gives exactly 0.
template <int NC, bool MIXED>
__device__ __forceinline__ float2 softmax_exp_store(uint32_t (&sv)[NC], float scale_log2, float m,
                                                    uint32_t s_addr, uint32_t half_bar) {
  const float2 sc = make_float2(scale_log2, scale_log2);
  const float2 nm = make_float2(-m, -m);
  float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll
  for (int h = 0; h < NC / 64; ++h) {
    uint32_t pk[32];
#pragma unroll
    for (int c = 0; c < 32; ++c) {
      const int k = h * 64 + 2 * c;
      const float2 x = fma2(make_float2(__uint_as_float(sv[k]), __uint_as_float(sv[k + 1])), sc, nm);
      float2 e;
      if (MIXED && ((kPolyPairs >> (c & 7)) & 1u)) {
        e = ex2_poly2(x);
      } else {
        e = make_float2(ex2(x.x), ex2(x.y));
      }
      if (c & 1) acc1 = add2(acc1, e);
      else acc0 = add2(acc0, e);
      pk[c] = pack_bf16x2(e.x, e.y);
    }
    tmem_st_32x32b_x32(s_addr + h * 32, pk);
    if (h == 0) {
      // the first 64 keys of P are in TMEM: PV on them can start
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if ((threadIdx.x & 31) == 0) mbar_arrive(half_bar);
    }
  }
  return add2(acc0, acc1);
}

__global__ void __launch_bounds__(THREADS, 1) k_fmha(const __grid_constant__ Args p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  // q_full: Q_A, Q_B and K(0).  kv_full[j % 2]: V(j) and K(j + 1), loaded
  // together.  kv_empty[j % 2]: released by the commit after QK_B(j + 1),
  // which follows PV_B(j) (frees V stage j % 2 and K stage (j + 1) % 2; the
  // prologue's release of K(0) counts as j = -1).  pv_done: the last PV of a
  // tile (the next QK commit already implies every earlier PV, tcgen05 ops of
  // one thread completing in issue order).
  uint64_t* q_full = bars;           // 1
  uint64_t* kv_full = bars + 1;      // 2
  uint64_t* kv_empty = bars + 3;     // 2
  uint64_t* s_full = bars + 5;       // 2 (tile A, B)
  uint64_t* p_full = bars + 7;       // 2
  uint64_t* pv_done = bars + 9;      // 2
  uint64_t* drain = bars + 11;       // 1
  uint64_t* p_half = bars + 12;      // 2: P of keys [0, 64) stored
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // work item -> (document, query-tile pair, head); pairs vary fastest so
  // neighbouring CTAs share K / V of one head in L2
  int doc = 0;
  while (doc + 1 < p.ndocs && (int)blockIdx.x >= p.item_end[doc]) ++doc;
  const int item = (int)blockIdx.x - (doc > 0 ? p.item_end[doc - 1] : 0);
  const int len = p.doc_len[doc];
  const int q_len = p.q_len[doc];
  const int pairs = (q_len + 2 * BQ - 1) / (2 * BQ);
  const int head = item / pairs;
  const int qp = item - head * pairs;
  const int row0 = p.doc_start[doc];
  const int q_row = p.q_start[doc] + qp * 2 * BQ;   // local row of tile A
  const int n_kv = (len + BK - 1) / BK;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(q_full), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&kv_full[i]), 1);
      mbar_init(smem_u32(&kv_empty[i]), 1);
      mbar_init(smem_u32(&s_full[i]), 1);
      mbar_init(smem_u32(&p_full[i]), 4);
      mbar_init(smem_u32(&p_half[i]), 4);
      mbar_init(smem_u32(&pv_done[i]), 1);
    }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
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

  // Each warpgroup changes its register limit inside its own branch and leaves
  // through its own copy of the teardown barrier, so no code runs under two
  // limits.
  if (warp >= 8) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kCtrlRegs));
   if (warp == 8) {
    if (lane == 0) {
      prefetch_tmap(&p.tmap_q);
      prefetch_tmap(&p.tmap_kv);
      prefetch_tmap(&p.tmap_v);
      const int qx = p.q_off + head * D, kx = p.k_off + head * D, vx = p.v_off + head * D;
      uint32_t fb = smem_u32(q_full);
      mbar_expect_tx(fb, 3 * TILE_BYTES);
      for (int t = 0; t < 2; ++t) {
        uint8_t* dst = smem + Q_OFF + t * TILE_BYTES;
        tma_load_2d(smem_u32(dst), &p.tmap_q, qx, q_row + t * BQ, fb);
        tma_load_2d(smem_u32(dst + BOX_BYTES), &p.tmap_q, qx + 64, q_row + t * BQ, fb);
      }
      tma_load_2d(smem_u32(smem + K_OFF), &p.tmap_kv, kx, row0, fb);
      tma_load_2d(smem_u32(smem + K_OFF + BOX_BYTES), &p.tmap_kv, kx + 64, row0, fb);
      // K / V tiles are first touched by all CTAs of a head at about the same
      // time; L2 prefetches kPrefetchTiles ahead hide the DRAM latency that
      // the two-stage shared-memory ring cannot.
      auto prefetch = [&](int j) {
        if (j < n_kv) {
          tma_prefetch_2d(&p.tmap_kv, kx, row0 + j * BK);
          tma_prefetch_2d(&p.tmap_kv, kx + 64, row0 + j * BK);
          tma_prefetch_2d(&p.tmap_v, vx, row0 + j * BK);
          tma_prefetch_2d(&p.tmap_v, vx + 64, row0 + j * BK);
        }
      };
      for (int j = 1; j < kPrefetchTiles; ++j) prefetch(j);
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < n_kv; ++j) {
        prefetch(j + kPrefetchTiles);
        if (j >= 1) {
          // release r = j - 2 frees K stage (j + 1) % 2 and V stage j % 2
          const int r = j - 2;
          const int st = r & 1;
          const int completion = st ? (r + 1) >> 1 : r >> 1;
          if (!mbar_wait(smem_u32(&kv_empty[st]), completion & 1, abort_flag)) {
            ok = false;
            break;
          }
        }
        const bool more = j + 1 < n_kv;
        const uint32_t b = smem_u32(&kv_full[j & 1]);
        mbar_expect_tx(b, more ? 2 * TILE_BYTES : TILE_BYTES);
        uint8_t* vdst = smem + V_OFF + (j & 1) * TILE_BYTES;
        tma_load_2d(smem_u32(vdst), &p.tmap_v, vx, row0 + j * BK, b);
        tma_load_2d(smem_u32(vdst + BOX_BYTES), &p.tmap_v, vx + 64, row0 + j * BK, b);
        if (more) {
          uint8_t* kdst = smem + K_OFF + ((j + 1) & 1) * TILE_BYTES;
          tma_load_2d(smem_u32(kdst), &p.tmap_kv, kx, row0 + (j + 1) * BK, b);
          tma_load_2d(smem_u32(kdst + BOX_BYTES), &p.tmap_kv, kx + 64, row0 + (j + 1) * BK, b);
        }
        ++issued;
      }
      if (!ok) {
        // no copy may still be landing when the CTA exits
        fail();
        mbar_wait(smem_u32(q_full), 0, nullptr);
        for (int j = issued > 2 ? issued - 2 : 0; j < issued; ++j)
          mbar_wait(smem_u32(&kv_full[j & 1]), (j >> 1) & 1, nullptr);
      }
    }
  } else if (warp == 9) {
      // The whole warp runs the issue loop on warp-uniform values; each
      // tcgen05 op is issued by one elected lane.
      auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
        return __all_sync(0xffffffffu, mbar_wait(smem_u32(bar), parity, abort_flag));
      };
      // descriptors advance by adding (byte offset >> 4) to the start-address
      // field (shared-memory addresses stay below 256 KiB: no carry out)
      auto issue_qk = [&](int t, int j) {
        const uint64_t qd = desc_kmajor_sw128(smem_u32(smem + Q_OFF + t * TILE_BYTES));
        const uint64_t kd = desc_kmajor_sw128(smem_u32(smem + K_OFF + (j & 1) * TILE_BYTES));
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = ((kk >> 2) * BOX_BYTES + (kk & 3) * 32) >> 4;   // 16 head dims
          tc_mma_bf16_ss_elect(tmem + s_col(t), qd + off, kd + off, IDESC_QK, kk != 0);
        }
        tc_commit_elect(smem_u32(&s_full[t]));
      };
      auto issue_pv = [&](int t, int j, int half) {
        // 16 keys per MMA: P columns kk*8.. (bf16 pairs), V rows kk*16..
        // (MN-major: 64-dim chunks LBO = 16 KiB apart, 8-row groups SBO = 1 KiB)
        const uint64_t vd = smem_desc(smem_u32(smem + V_OFF + (j & 1) * TILE_BYTES), BOX_BYTES, 1024, 2);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int kk = half * 4 + i;
          tc_mma_bf16_ts_elect(tmem + o_col(t), tmem + s_col(t) + kk * 8, vd + kk * (2048 >> 4),
                               IDESC_PV, (j | kk) != 0);
        }
        if (half == 1 && j + 1 == n_kv) tc_commit_elect(smem_u32(&pv_done[t]));
      };
      // PV of tile t in two halves: keys [0, 64) once softmax has stored
      // them, the rest once the whole P is in TMEM
      auto pv_tile = [&](int t, int j) -> bool {
        if (!wait(&p_half[t], j & 1)) return false;
        tc_fence_after();
        issue_pv(t, j, 0);
        if (!wait(&p_full[t], j & 1)) return false;
        tc_fence_after();
        issue_pv(t, j, 1);
        return true;
      };
      bool ok = wait(q_full, 0);
      if (ok) {
        tc_fence_after();
        issue_qk(0, 0);
        issue_qk(1, 0);
        tc_commit_elect(smem_u32(&kv_empty[1]));        // release of K(0)
      }
      for (int j = 0; j < n_kv && ok; ++j) {
        const bool more = j + 1 < n_kv;
        if (!wait(&kv_full[j & 1], (j >> 1) & 1) || !pv_tile(0, j)) {
          ok = false;
          break;
        }
        if (more) issue_qk(0, j + 1);
        if (!pv_tile(1, j)) {
          ok = false;
          break;
        }
        if (more) issue_qk(1, j + 1);
        tc_commit_elect(smem_u32(&kv_empty[j & 1]));
      }
      if (!ok) {
        if (lane == 0) fail();
        tc_commit_elect(smem_u32(drain));
        mbar_wait(smem_u32(drain), 0, nullptr);
      }
   }
    tc_fence_before();
    named_barrier_sync(1, THREADS);
    if (warp == 9) {
      __syncwarp();
      tc_fence_after();
      tmem_dealloc(tmem, TMEM_COLS);
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftmaxRegs));
    // softmax of tile t: thread = query row (TMEM lane quadrant warp % 4)
    const int t = warp >> 2;
    const int qd = warp & 3;
    const int r = qd * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(qd * 32) << 16;
    const uint32_t s_t = tmem + lane_addr + s_col(t);
    const uint32_t o_t = tmem + lane_addr + o_col(t);
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&s_full[t]), j & 1, abort_flag));
      if (!ok) break;
      tc_fence_after();
      const int valid = min(BK, len - j * BK);   // keys of this tile inside the document
      uint32_t sv[128];
      tmem_ld_32x32b_x64(s_t, sv);
      tmem_ld_32x32b_x64(s_t + 64, sv + 64);
      tmem_ld_wait();
      const bool partial = valid < BK;             // warp-uniform
      if (partial) {
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (c >= valid) sv[c] = 0xff800000u;     // -inf: masked key
      }
      // row max of the scaled logits (scale > 0 commutes with max)
      float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < 128; c += 8) {
#pragma unroll
        for (int u = 0; u < 4; ++u)
          m4[u] = max3(m4[u], __uint_as_float(sv[c + 2 * u]), __uint_as_float(sv[c + 2 * u + 1]));
      }
      const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * p.scale_log2;
      const float m_new = fmaxf(m_used, mx);
      const bool rescale = __any_sync(0xffffffffu, m_new > m_used + kRescaleLog2);
      float alpha = 1.f;
      if (rescale) {
        alpha = ex2(m_used - m_new);               // 0 on the first tile (m_used = -inf)
        m_used = m_new;
      }
      if (rescale && j > 0) {
        // O is final for P(j-1): QK(j), whose completion s_full signalled, was
        // issued after PV(j-1); PV(j) waits for p_half, whose arrival follows
        // these stores
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          uint32_t ov[32];
          tmem_ld_32x32b_x32(o_t + h * 32, ov);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 32; ++c) ov[c] = __float_as_uint(__uint_as_float(ov[c]) * alpha);
          tmem_st_32x32b_x32(o_t + h * 32, ov);
        }
      }
      // P written over the S columns already read
      const uint32_t hb = smem_u32(&p_half[t]);
      const float2 s2 = partial ? softmax_exp_store<128, false>(sv, p.scale_log2, m_used, s_t, hb)
                                : softmax_exp_store<128, true>(sv, p.scale_log2, m_used, s_t, hb);
      l = l * alpha + (s2.x + s2.y);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&p_full[t]));
    }
    if (ok && n_kv > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&pv_done[t]), 0, abort_flag));
    }
    if (!ok) {
      fail();
    } else if (n_kv > 0) {
      tc_fence_after();
      const float inv_l = 1.0f / l;
      const int lr = qp * 2 * BQ + t * BQ + r;      // row within the document's local queries
      const bool row_ok = lr < q_len;
      __nv_bfloat16* op = p.out + (size_t)(q_row + t * BQ + r) * p.ldo + (size_t)head * D;
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        uint32_t ov[32];
        tmem_ld_32x32b_x32(o_t + h * 32, ov);
        tmem_ld_wait();
        if (row_ok) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(ov[8 * c + 0]) * inv_l, __uint_as_float(ov[8 * c + 1]) * inv_l);
            w.y = pack_bf16x2(__uint_as_float(ov[8 * c + 2]) * inv_l, __uint_as_float(ov[8 * c + 3]) * inv_l);
            w.z = pack_bf16x2(__uint_as_float(ov[8 * c + 4]) * inv_l, __uint_as_float(ov[8 * c + 5]) * inv_l);
            w.w = pack_bf16x2(__uint_as_float(ov[8 * c + 6]) * inv_l, __uint_as_float(ov[8 * c + 7]) * inv_l);
            *reinterpret_cast<uint4*>(op + h * 32 + c * 8) = w;
          }
        }
      }
    }
    tc_fence_before();
    named_barrier_sync(1, THREADS);
  }
}

}  // namespace attn
}  // namespace h3b
