// C-ABI entry points of libh3b.so (declared in include/h3b.h).
//
// All kernels live in this one translation unit so they share the device
// error word.  The host functions validate shapes / alignment, build TMA
// descriptors, launch on the caller's stream and never synchronize (except
// h3b_device_error, which is documented to).
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "quant.cuh"
#include "gemm_nvfp4.cuh"
#include "norm.cuh"
#include "rope.cuh"
#include "attention.cuh"
#include "elementwise.cuh"
#include "peer.cuh"

namespace h3b {

static std::atomic<long long> g_launches{0};

static inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev < 64 && cached[dev]) return cached[dev];
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev < 64) cached[dev] = n;
  return n;
}

static int check_sm100() {
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return H3B_ERR_CUDA;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return H3B_ERR_CUDA;
  return major == 10 ? H3B_OK : H3B_ERR_UNSUPPORTED;
}

static inline int launched(cudaError_t e) {
  if (e != cudaSuccess) return H3B_ERR_CUDA;
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return H3B_OK;
}

// ------------------------------------------------------------------ TMA descriptors
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D u8 tensor [rows, cols_bytes] (row pitch = pitch bytes), box box_cols x box_rows,
// 128-byte swizzle.
static int make_tmap_u8_sw128(CUtensorMap* map, const void* base, uint64_t rows,
                              uint64_t cols_bytes, uint64_t pitch, uint32_t box_cols,
                              uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return H3B_ERR_UNSUPPORTED;
  cuuint64_t dims[2] = {cols_bytes, rows};
  cuuint64_t strides[1] = {pitch};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? H3B_OK : H3B_ERR_INVALID_ARG;
}

// 2-D bf16 tensor [rows, cols] (row pitch = pitch_elems), box box_cols x box_rows,
// 128-byte swizzle (box_cols * 2 must be 128).
static int make_tmap_bf16_sw128(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                                uint64_t pitch_elems, uint32_t box_cols, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return H3B_ERR_UNSUPPORTED;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {pitch_elems * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? H3B_OK : H3B_ERR_INVALID_ARG;
}

// 2-D tensor of 8-byte elements [rows, cols] (row pitch = cols * 8 bytes),
// box box_cols x box_rows, no swizzle: the blocked scale atoms of one k-block
// (4 x 512 B) of one or two 128-row blocks, as TMA-loadable boxes.
static int make_tmap_u64(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                         uint32_t box_cols, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return H3B_ERR_UNSUPPORTED;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 8};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? H3B_OK : H3B_ERR_INVALID_ARG;
}

}  // namespace h3b

using namespace h3b;

extern "C" {

int h3b_version(void) { return 1; }

const char* h3b_status_string(int s) {
  switch (s) {
    case H3B_OK: return "ok";
    case H3B_ERR_INVALID_ARG: return "invalid argument (shape, size or enum out of range)";
    case H3B_ERR_ALIGNMENT: return "misaligned pointer or leading dimension";
    case H3B_ERR_CUDA: return "CUDA runtime error";
    case H3B_ERR_UNSUPPORTED: return "unsupported device or feature (needs sm_100)";
    case H3B_ERR_TIMEOUT: return "device-side bounded wait expired";
    case H3B_ERR_DEVICE: return "device-side failure recorded";
    default: return "unknown status";
  }
}

long long h3b_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int h3b_device_error(int* code_out, int clear) {
  if (!code_out) return H3B_ERR_INVALID_ARG;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return H3B_ERR_CUDA;
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(int));
  if (e != cudaSuccess) return H3B_ERR_CUDA;
  if (clear && v) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(int));
    if (e != cudaSuccess) return H3B_ERR_CUDA;
  }
  *code_out = v;
  return H3B_OK;
}

// ------------------------------------------------------------------ quantize
int h3b_amax_bf16(const void* x, int64_t rows, int64_t cols, int64_t ldx, float* amax_out,
                  void* stream) {
  if (!amax_out || rows < 0 || cols < 0 || ldx < cols) return H3B_ERR_INVALID_ARG;
  if (cols % 8 || ldx % 8) return H3B_ERR_INVALID_ARG;
  if (!aligned16(x) || (reinterpret_cast<uintptr_t>(amax_out) & 3u)) return H3B_ERR_ALIGNMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(amax_out, 0, sizeof(float), st);
  if (e != cudaSuccess) return H3B_ERR_CUDA;
  const int64_t total = rows * (cols / 8);
  if (total == 0) return H3B_OK;
  int64_t blocks = (total + kAmaxThreads * 4 - 1) / (kAmaxThreads * 4);
  const int64_t cap = (int64_t)num_sms() * 8;
  if (blocks > cap) blocks = cap;
  k_amax_bf16<<<(unsigned)blocks, kAmaxThreads, 0, st>>>(
      static_cast<const __nv_bfloat16*>(x), rows, cols, ldx, amax_out);
  return launched(cudaGetLastError());
}

int h3b_nvfp4_quantize(const void* x, int64_t M, int64_t K, int64_t ldx, const float* amax,
                       float gs_in, float* gs_out, void* q, void* sf, int sf_layout, int64_t Mpad,
                       void* stream) {
  if (M < 0 || K <= 0 || K % 64 || ldx < K || ldx % 8 || Mpad < M) return H3B_ERR_INVALID_ARG;
  if (sf_layout != H3B_SF_ROWMAJOR && sf_layout != H3B_SF_SWIZZLED) return H3B_ERR_INVALID_ARG;
  if (sf_layout == H3B_SF_SWIZZLED && Mpad % 128) return H3B_ERR_INVALID_ARG;
  if (!amax && !(gs_in > 0.f)) return H3B_ERR_INVALID_ARG;
  if (!q || !sf || (M > 0 && !x)) return H3B_ERR_INVALID_ARG;
  if ((M > 0 && !aligned16(x)) || (reinterpret_cast<uintptr_t>(q) & 3u)) return H3B_ERR_ALIGNMENT;
  if (Mpad == 0) return H3B_OK;
  constexpr int64_t rows_per_block = kQuantThreads / 32;      // one warp per row
  int64_t blocks = (Mpad + rows_per_block - 1) / rows_per_block;
  const int64_t cap = (int64_t)num_sms() * 8;
  if (blocks > cap) blocks = cap;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto xp = static_cast<const __nv_bfloat16*>(x);
  auto qp = static_cast<uint8_t*>(q);
  auto sp = static_cast<uint8_t*>(sf);
  // loads in flight per lane: 6 or 7 where a row is a whole number of such
  // steps (32 lanes x 8 values each), else 4
  const int64_t hpr = K / 8;
  const int unroll = hpr % (32 * 6) == 0 ? 6 : hpr % (32 * 7) == 0 ? 7 : 4;
  auto launch = [&](auto kernel) {
    kernel<<<(unsigned)blocks, kQuantThreads, 0, st>>>(xp, M, K, ldx, amax, gs_in, gs_out, qp,
                                                       sp, Mpad);
  };
  if (sf_layout == H3B_SF_SWIZZLED) {
    if (unroll == 6) launch(k_nvfp4_quantize<H3B_SF_SWIZZLED, 6>);
    else if (unroll == 7) launch(k_nvfp4_quantize<H3B_SF_SWIZZLED, 7>);
    else launch(k_nvfp4_quantize<H3B_SF_SWIZZLED, 4>);
  } else {
    if (unroll == 6) launch(k_nvfp4_quantize<H3B_SF_ROWMAJOR, 6>);
    else if (unroll == 7) launch(k_nvfp4_quantize<H3B_SF_ROWMAJOR, 7>);
    else launch(k_nvfp4_quantize<H3B_SF_ROWMAJOR, 4>);
  }
  return launched(cudaGetLastError());
}

int h3b_nvfp4_dequantize(const void* q, const void* sf, int sf_layout, int64_t sf_rows,
                         const float* gs, int64_t M, int64_t K, void* out, void* stream) {
  if (M < 0 || K <= 0 || K % 64 || sf_rows < M) return H3B_ERR_INVALID_ARG;
  if (sf_layout != H3B_SF_ROWMAJOR && sf_layout != H3B_SF_SWIZZLED) return H3B_ERR_INVALID_ARG;
  if (sf_layout == H3B_SF_SWIZZLED && sf_rows % 128) return H3B_ERR_INVALID_ARG;
  if (M == 0) return H3B_OK;
  if (!q || !sf || !out) return H3B_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(q) & 3u) || !aligned16(out)) return H3B_ERR_ALIGNMENT;
  if (K / 8 > (int64_t)INT32_MAX) return H3B_ERR_INVALID_ARG;
  int64_t blocks = (M + 7) / 8;                       // one warp per row, 8 per CTA
  const int64_t cap = (int64_t)num_sms() * 8;
  if (blocks > cap) blocks = cap;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto qp = static_cast<const uint8_t*>(q);
  auto sp = static_cast<const uint8_t*>(sf);
  auto op = static_cast<__nv_bfloat16*>(out);
  if (sf_layout == H3B_SF_SWIZZLED)
    k_nvfp4_dequantize<H3B_SF_SWIZZLED><<<(unsigned)blocks, 256, 0, st>>>(qp, sp, gs, M, K, op);
  else
    k_nvfp4_dequantize<H3B_SF_ROWMAJOR><<<(unsigned)blocks, 256, 0, st>>>(qp, sp, gs, M, K, op);
  return launched(cudaGetLastError());
}

// ------------------------------------------------------------------ GEMM
int h3b_nvfp4_gemm(const void* A, const void* sfA, const float* gsA, int64_t M, int64_t a_rows,
                   const void* B, const void* sfB, const float* gsB, int64_t gsb_seg, int64_t N,
                   int64_t K, const void* bias, const void* residual, int64_t ldr,
                   const void* gate, const int32_t* gate_idx, int act, void* D, int64_t ldd,
                   float* amax_out, void* stream) {
  if (M < 0 || N <= 0 || K <= 0) return H3B_ERR_INVALID_ARG;
  if (gate_idx && !gate) return H3B_ERR_INVALID_ARG;
  if (gsb_seg < 0 || (gsb_seg && (gsb_seg % 128 || N % gsb_seg))) return H3B_ERR_INVALID_ARG;
  if (K % gemm::KB_ELEMS || N % 128 || a_rows % 128 || a_rows < M) return H3B_ERR_INVALID_ARG;
  if (act != H3B_ACT_NONE && act != H3B_ACT_GELU_TANH && act != H3B_ACT_SWIGLU)
    return H3B_ERR_INVALID_ARG;
  const bool swiglu = act == H3B_ACT_SWIGLU;
  if (swiglu && (N % gemm::BN || bias || residual || gate || gsb_seg)) return H3B_ERR_INVALID_ARG;
  const int64_t n_out = swiglu ? N / 2 : N;          // columns of D
  if (ldd < n_out || ldd % 8) return H3B_ERR_INVALID_ARG;
  if (residual && (ldr < N || ldr % 8)) return H3B_ERR_INVALID_ARG;
  if (M > (int64_t)INT32_MAX - 256 || N > (int64_t)INT32_MAX || K > (int64_t)INT32_MAX)
    return H3B_ERR_INVALID_ARG;
  if (M == 0) return H3B_OK;
  if (!A || !sfA || !B || !sfB || !D) return H3B_ERR_INVALID_ARG;
  if (!aligned16(A) || !aligned16(B) || !aligned16(sfA) || !aligned16(sfB) || !aligned16(D) ||
      (bias && !aligned16(bias)) || (residual && !aligned16(residual)) ||
      (gate && !aligned16(gate)))
    return H3B_ERR_ALIGNMENT;
  int st0 = check_sm100();
  if (st0 != H3B_OK) return st0;

  static std::once_flag attr_once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(attr_once, [] {
    attr_err = cudaFuncSetAttribute(gemm::k_gemm_nvfp4<false>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    gemm::SMEM_BYTES);
    if (attr_err == cudaSuccess)
      attr_err = cudaFuncSetAttribute(gemm::k_gemm_nvfp4<true>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      gemm::SMEM_BYTES);
  });
  if (attr_err != cudaSuccess) return H3B_ERR_CUDA;

  gemm::Args args;
  memset(&args, 0, sizeof(args));
  int rc = make_tmap_u8_sw128(&args.tmap_a, A, (uint64_t)a_rows, (uint64_t)(K / 2),
                              (uint64_t)(K / 2), gemm::KB_BYTES, gemm::BM);
  if (rc != H3B_OK) return rc;
  rc = make_tmap_u8_sw128(&args.tmap_b, B, (uint64_t)N, (uint64_t)(K / 2), (uint64_t)(K / 2),
                          gemm::KB_BYTES, gemm::BN);
  if (rc != H3B_OK) return rc;
  rc = make_tmap_bf16_sw128(&args.tmap_d, D, (uint64_t)M, (uint64_t)n_out, (uint64_t)ldd,
                            gemm::OUT_CHUNK_COLS, 32);
  if (rc != H3B_OK) return rc;
  args.sfa = static_cast<const uint8_t*>(sfA);
  args.sfb = static_cast<const uint8_t*>(sfB);
  args.gs_a = gsA;
  args.gs_b = gsB;
  args.bias = static_cast<const __nv_bfloat16*>(bias);
  args.residual = static_cast<const __nv_bfloat16*>(residual);
  args.gate = static_cast<const __nv_bfloat16*>(gate);
  args.gate_idx = gate_idx;
  args.amax_out = amax_out;
  args.ldr = residual ? ldr : 0;
  args.M = (int)M;
  args.N = (int)N;
  args.K = (int)K;
  args.sf_atoms_k = (int)(K / 64);
  args.act = act;
  args.gsb_seg = (int)gsb_seg;
  args.n_tiles = (int)((N + gemm::BN - 1) / gemm::BN);
  const int64_t num_tiles = (int64_t)args.n_tiles * ((M + gemm::BM - 1) / gemm::BM);
  if (num_tiles > INT32_MAX) return H3B_ERR_INVALID_ARG;
  args.num_tiles = (int)num_tiles;
  // CTA pairs (one 256 x 256 tile per pair) for the long-K projections (the
  // FFN down-projections, K = 12288: 13-16 % faster than single CTAs, which
  // pay a full B tile of shared-memory traffic per SM per k-block); at
  // K = 3072 both forms run at the same speed and the single-CTA kernel is
  // kept.  N must fill whole 256-column tiles and M span more than one
  // 128-row block.  Both forms give the same bits.
  if (N % 256 == 0 && M > gemm::BM && K >= 8192 && num_sms() >= 2) {
    static std::once_flag pair_once;
    static cudaError_t pair_err = cudaSuccess;
    std::call_once(pair_once, [] {
      pair_err = cudaFuncSetAttribute(gemm::k_gemm_nvfp4_pair<false>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      gemm::P_SMEM_BYTES);
      if (pair_err == cudaSuccess)
        pair_err = cudaFuncSetAttribute(gemm::k_gemm_nvfp4_pair<true>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        gemm::P_SMEM_BYTES);
    });
    if (pair_err != cudaSuccess) return H3B_ERR_CUDA;
    gemm::PairArgs pa;
    memset(&pa, 0, sizeof(pa));
    pa.base = args;
    rc = make_tmap_u8_sw128(&pa.base.tmap_b, B, (uint64_t)N, (uint64_t)(K / 2), (uint64_t)(K / 2),
                            gemm::KB_BYTES, 128);
    if (rc != H3B_OK) return rc;
    rc = make_tmap_u64(&pa.tmap_sfa, sfA, (uint64_t)(a_rows / 128), (uint64_t)K, 256, 1);
    if (rc != H3B_OK) return rc;
    rc = make_tmap_u64(&pa.tmap_sfb, sfB, (uint64_t)(N / 128), (uint64_t)K, 256, 2);
    if (rc != H3B_OK) return rc;
    pa.m_tiles = (int)((M + 255) / 256);
    const int64_t pair_tiles = (int64_t)pa.m_tiles * args.n_tiles;
    const int pairs = (int)std::min<int64_t>(pair_tiles, num_sms() / 2);
    if (swiglu)
      gemm::k_gemm_nvfp4_pair<true><<<2 * pairs, gemm::THREADS, gemm::P_SMEM_BYTES,
                                      static_cast<cudaStream_t>(stream)>>>(pa);
    else
      gemm::k_gemm_nvfp4_pair<false><<<2 * pairs, gemm::THREADS, gemm::P_SMEM_BYTES,
                                       static_cast<cudaStream_t>(stream)>>>(pa);
    return launched(cudaGetLastError());
  }
  const int grid = (int)std::min<int64_t>(num_tiles, num_sms());
  if (swiglu)
    gemm::k_gemm_nvfp4<true><<<grid, gemm::THREADS, gemm::SMEM_BYTES,
                               static_cast<cudaStream_t>(stream)>>>(args);
  else
    gemm::k_gemm_nvfp4<false><<<grid, gemm::THREADS, gemm::SMEM_BYTES,
                                static_cast<cudaStream_t>(stream)>>>(args);
  return launched(cudaGetLastError());
}

// ------------------------------------------------------------------ RMSNorm -> NVFP4
static int norm_args(NormArgs& a, const void* x, int64_t M, int64_t K, int64_t ldx,
                     const void* gamma, float eps, const void* shift, const void* scale,
                     const int32_t* mod_idx) {
  if (M < 0 || K <= 0 || K % 256 || ldx < K || ldx % 8) return H3B_ERR_INVALID_ARG;
  if (!gamma || (M > 0 && !x) || ((shift == nullptr) != (scale == nullptr))) return H3B_ERR_INVALID_ARG;
  if ((M > 0 && !aligned16(x)) || !aligned16(gamma) || (shift && !aligned16(shift)) ||
      (scale && !aligned16(scale)))
    return H3B_ERR_ALIGNMENT;
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.gamma = static_cast<const __nv_bfloat16*>(gamma);
  a.shift = static_cast<const __nv_bfloat16*>(shift);
  a.scale = static_cast<const __nv_bfloat16*>(scale);
  a.mod_idx = mod_idx;
  a.ldx = ldx;
  a.M = M;
  a.K = K;
  a.eps = eps;
  return H3B_OK;
}

int h3b_rmsnorm_stats(const void* x, int64_t M, int64_t K, int64_t ldx, const void* gamma,
                      float eps, const void* shift, const void* scale, const int32_t* mod_idx,
                      float* rstd_out, float* amax_out, void* stream) {
  NormArgs a;
  int rc = norm_args(a, x, M, K, ldx, gamma, eps, shift, scale, mod_idx);
  if (rc != H3B_OK) return rc;
  if (!amax_out || (M > 0 && !rstd_out)) return H3B_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(amax_out, 0, sizeof(float), st) != cudaSuccess) return H3B_ERR_CUDA;
  if (M == 0) return H3B_OK;
  const unsigned blocks = (unsigned)((M + kNormWarps - 1) / kNormWarps);
  if (K <= kNormCacheChunks * 256)
    k_rmsnorm_stats<kNormCacheChunks><<<blocks, kNormWarps * 32, 0, st>>>(a, rstd_out, amax_out);
  else
    k_rmsnorm_stats<0><<<blocks, kNormWarps * 32, 0, st>>>(a, rstd_out, amax_out);
  return launched(cudaGetLastError());
}

int h3b_rmsnorm_quantize(const void* x, int64_t M, int64_t K, int64_t ldx, const void* gamma,
                         const void* shift, const void* scale, const int32_t* mod_idx,
                         const float* rstd, const float* amax, float* gs_out, void* q, void* sf,
                         int64_t Mpad, void* y_out, void* stream) {
  NormArgs a;
  int rc = norm_args(a, x, M, K, ldx, gamma, 0.f, shift, scale, mod_idx);
  if (rc != H3B_OK) return rc;
  if (!amax || !q || !sf || (M > 0 && !rstd) || Mpad < M || Mpad % 128) return H3B_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(q) & 3u) || (y_out && !aligned16(y_out))) return H3B_ERR_ALIGNMENT;
  if (Mpad == 0) return H3B_OK;
  const unsigned blocks = (unsigned)((Mpad + kNormWarps - 1) / kNormWarps);
  k_rmsnorm_quant<<<blocks, kNormWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(
      a, rstd, amax, gs_out, static_cast<uint8_t*>(q), static_cast<uint8_t*>(sf), Mpad,
      static_cast<__nv_bfloat16*>(y_out));
  return launched(cudaGetLastError());
}

// ------------------------------------------------------------------ qk-norm + RoPE
}  // extern "C"

namespace h3b {
// Shared by the in-place and the out-of-place entry points: q / k are read at
// (stride, off), the results written to qo / ko at (o_stride, o_off).
static int qk_norm_rope_launch(const void* q, int64_t q_stride, int64_t q_off, const void* k,
                               int64_t k_stride, int64_t k_off, void* qo, int64_t qo_stride,
                               int64_t qo_off, void* ko, int64_t ko_stride, int64_t ko_off,
                               int64_t T, int H, int D, const void* wq, const void* wk, float eps,
                               const float* cos, const float* sin, int R, int64_t cs_stride,
                               void* stream) {
  if (T < 0 || H <= 0 || (D != 64 && D != 128)) return H3B_ERR_INVALID_ARG;
  if (cos != nullptr) {
    // the partner of a lane's 8 columns is a whole lane away: R/2 % 8 == 0;
    // rows of the tables are read as float4: 16-byte aligned
    if (!sin || R <= 0 || R > D || (R / 2) % 8 || cs_stride < R || cs_stride % 4)
      return H3B_ERR_INVALID_ARG;
    if (!aligned16(cos) || !aligned16(sin)) return H3B_ERR_ALIGNMENT;
  } else {
    R = 0;
  }
  const int64_t hd = (int64_t)H * D;
  // a NULL q (or k) skips those heads: its strides and offsets are not used
  if (q && (q_off < 0 || qo_off < 0 || q_off + hd > q_stride || qo_off + hd > qo_stride))
    return H3B_ERR_INVALID_ARG;
  if (k && (k_off < 0 || ko_off < 0 || k_off + hd > k_stride || ko_off + hd > ko_stride))
    return H3B_ERR_INVALID_ARG;
  if ((q && (q_stride | q_off | qo_stride | qo_off) % 8) ||
      (k && (k_stride | k_off | ko_stride | ko_off) % 8))
    return H3B_ERR_ALIGNMENT;
  if (T == 0) return H3B_OK;
  if (!q && !k) return H3B_ERR_INVALID_ARG;            // NULL q or k: those heads are skipped
  if ((q && !qo) || (k && !ko)) return H3B_ERR_INVALID_ARG;
  if ((q && (!aligned16(q) || !aligned16(qo))) || (k && (!aligned16(k) || !aligned16(ko))))
    return H3B_ERR_ALIGNMENT;
  RopeArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k = static_cast<const __nv_bfloat16*>(k);
  a.qo = static_cast<__nv_bfloat16*>(qo);
  a.ko = static_cast<__nv_bfloat16*>(ko);
  a.T = T;
  a.q_stride = q_stride;
  a.k_stride = k_stride;
  a.q_off = q_off;
  a.k_off = k_off;
  a.qo_stride = qo_stride;
  a.ko_stride = ko_stride;
  a.qo_off = qo_off;
  a.ko_off = ko_off;
  a.H = H;
  a.hq = q ? H : 0;
  a.hk = k ? H : 0;
  a.R = R;
  a.wq = static_cast<const __nv_bfloat16*>(wq);
  a.wk = static_cast<const __nv_bfloat16*>(wk);
  a.cos = cos;
  a.sin = sin;
  a.cs_stride = cs_stride;
  a.eps = eps;
  int64_t blocks = (T + kRopeWarps - 1) / kRopeWarps;     // one warp per row
  const int64_t cap = (int64_t)num_sms() * 8;
  if (blocks > cap) blocks = cap;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (R == D) {
    // full-width rotary: each lane holds a column block and its rotate-half
    // partner; head vectors per warp instruction 32 / (D / 16); 3 or 4 of
    // them in flight per lane (4 unless only 3 divides the row's head vectors)
    const int steps = (a.hq + a.hk) / (512 / D);
    const bool three = steps % 4 != 0 && steps % 3 == 0;
    if (D == 128) {
      if (three) k_qk_norm_rope_full<128, 3><<<(unsigned)blocks, kRopeWarps * 32, 0, st>>>(a);
      else k_qk_norm_rope_full<128, 4><<<(unsigned)blocks, kRopeWarps * 32, 0, st>>>(a);
    } else {
      if (three) k_qk_norm_rope_full<64, 3><<<(unsigned)blocks, kRopeWarps * 32, 0, st>>>(a);
      else k_qk_norm_rope_full<64, 4><<<(unsigned)blocks, kRopeWarps * 32, 0, st>>>(a);
    }
    return launched(cudaGetLastError());
  }
  // head vectors of a row per warp instruction: 32 lanes / (D / 8 lanes each)
  const int steps = (a.hq + a.hk) / (256 / D);
  const bool seven = steps % 6 != 0 && steps % 7 == 0;
  if (D == 128) {
    if (seven) k_qk_norm_rope<128, 7><<<(unsigned)blocks, kRopeWarps * 32, 0, st>>>(a);
    else k_qk_norm_rope<128, 6><<<(unsigned)blocks, kRopeWarps * 32, 0, st>>>(a);
  } else {
    if (seven) k_qk_norm_rope<64, 7><<<(unsigned)blocks, kRopeWarps * 32, 0, st>>>(a);
    else k_qk_norm_rope<64, 6><<<(unsigned)blocks, kRopeWarps * 32, 0, st>>>(a);
  }
  return launched(cudaGetLastError());
}
}  // namespace h3b

extern "C" {

int h3b_qk_norm_rope(void* q, int64_t q_stride, int64_t q_off, void* k, int64_t k_stride,
                     int64_t k_off, int64_t T, int H, int D, const void* wq, const void* wk,
                     float eps, const float* cos, const float* sin, int R, int64_t cs_stride,
                     void* stream) {
  return qk_norm_rope_launch(q, q_stride, q_off, k, k_stride, k_off, q, q_stride, q_off, k,
                             k_stride, k_off, T, H, D, wq, wk, eps, cos, sin, R, cs_stride,
                             stream);
}

int h3b_qk_norm_rope_out(const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                         void* q_out, int64_t qo_stride, void* k_out, int64_t ko_stride,
                         int64_t T, int H, int D, const void* wq, const void* wk, float eps,
                         const float* cos, const float* sin, int R, int64_t cs_stride,
                         void* stream) {
  return qk_norm_rope_launch(q, q_stride, 0, k, k_stride, 0, q_out, qo_stride, 0, k_out,
                             ko_stride, 0, T, H, D, wq, wk, eps, cos, sin, R, cs_stride, stream);
}

// ------------------------------------------------------------------ gathered gate / modulation
}  // extern "C"

namespace h3b {
static int gather_elementwise_launch(bool gate, const void* a, int64_t lda, const void* b,
                                     int64_t ldb, const void* t0, const void* t1,
                                     const int32_t* idx, int64_t n_idx, int64_t rows,
                                     int64_t cols, void* out, int64_t ldo, void* stream) {
  if (rows < 0 || cols <= 0 || cols % 8 || lda < cols || ldo < cols || n_idx < 0)
    return H3B_ERR_INVALID_ARG;
  if (gate && ldb < cols) return H3B_ERR_INVALID_ARG;
  if (idx && n_idx == 0) return H3B_ERR_INVALID_ARG;
  if ((lda | ldo | (gate ? ldb : 0)) % 8) return H3B_ERR_ALIGNMENT;
  if (rows == 0) return H3B_OK;
  if (!a || !t0 || !out || (gate && !b) || (!gate && !t1)) return H3B_ERR_INVALID_ARG;
  if (!aligned16(a) || !aligned16(t0) || !aligned16(out) || (gate && !aligned16(b)) ||
      (!gate && !aligned16(t1)))
    return H3B_ERR_ALIGNMENT;
  EwArgs p;
  p.a = static_cast<const __nv_bfloat16*>(a);
  p.b = static_cast<const __nv_bfloat16*>(b);
  p.t0 = static_cast<const __nv_bfloat16*>(t0);
  p.t1 = static_cast<const __nv_bfloat16*>(t1);
  p.idx = idx;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.rows = rows;
  p.cols = cols;
  p.lda = lda;
  p.ldb = gate ? ldb : 0;
  p.ldo = ldo;
  p.n_idx = n_idx;
  int64_t blocks = (rows + 7) / 8;                      // one warp per row, 8 per CTA
  const int64_t cap = (int64_t)num_sms() * 8;
  if (blocks > cap) blocks = cap;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (gate) k_gather_elementwise<true><<<(unsigned)blocks, 256, 0, st>>>(p);
  else k_gather_elementwise<false><<<(unsigned)blocks, 256, 0, st>>>(p);
  return launched(cudaGetLastError());
}
}  // namespace h3b

extern "C" {

int h3b_gate_residual(const void* residual, int64_t ldr, const void* y, int64_t ldy,
                      const void* gate, const int32_t* idx, int64_t n_idx, int64_t rows,
                      int64_t cols, void* out, int64_t ldo, void* stream) {
  return gather_elementwise_launch(true, residual, ldr, y, ldy, gate, nullptr, idx, n_idx, rows,
                                   cols, out, ldo, stream);
}

int h3b_ada_modulate(const void* x, int64_t ldx, const void* scale, const void* shift,
                     const int32_t* idx, int64_t n_idx, int64_t rows, int64_t cols, void* out,
                     int64_t ldo, void* stream) {
  return gather_elementwise_launch(false, x, ldx, nullptr, 0, scale, shift, idx, n_idx, rows,
                                   cols, out, ldo, stream);
}

// ------------------------------------------------------------------ packed varlen attention
static int tmap_bf16_rows(CUtensorMap* tm, const void* base, int64_t rows, int64_t stride) {
  auto fn = encode_fn();
  if (!fn) return H3B_ERR_UNSUPPORTED;
  cuuint64_t dims[2] = {(cuuint64_t)stride, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)stride * 2};
  cuuint32_t box[2] = {64, attn::BK};
  cuuint32_t estr[2] = {1, 1};
  return fn(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? H3B_OK
             : H3B_ERR_INVALID_ARG;
}

}  // extern "C"

namespace h3b {
// Shared by both attention entry points: queries from q_buf (q_rows local
// rows starting at global row q_row0), keys from k_buf and values from v_buf
// (kv_rows rows each, the whole sequence).
static int attention_launch(const void* q_buf, int64_t q_rows, int64_t q_stride, int64_t q_off,
                            int64_t q_row0, const void* k_buf, int64_t k_stride, int64_t k_off,
                            const void* v_buf, int64_t v_stride, int64_t v_off, int64_t kv_rows,
                            int H, int D, const int32_t* cu_seqlens_host, int ndocs, float scale,
                            void* out, int64_t ldo, void* stream) {
  if (q_rows < 0 || kv_rows < 0 || q_row0 < 0 || q_row0 + q_rows > kv_rows) return H3B_ERR_INVALID_ARG;
  if (H <= 0 || D != attn::D || ndocs <= 0 || ndocs > attn::MAX_DOCS || !cu_seqlens_host)
    return H3B_ERR_INVALID_ARG;
  if (!(scale > 0.f)) return H3B_ERR_INVALID_ARG;
  if (cu_seqlens_host[0] != 0 || cu_seqlens_host[ndocs] != kv_rows) return H3B_ERR_INVALID_ARG;
  for (int i = 0; i < ndocs; ++i)
    if (cu_seqlens_host[i + 1] < cu_seqlens_host[i]) return H3B_ERR_INVALID_ARG;
  const int64_t hd = (int64_t)H * D;
  if (q_off < 0 || k_off < 0 || v_off < 0 || q_off + hd > q_stride || k_off + hd > k_stride ||
      v_off + hd > v_stride || ldo < hd)
    return H3B_ERR_INVALID_ARG;
  if ((q_stride | k_stride | v_stride | q_off | k_off | v_off | ldo) % 8) return H3B_ERR_ALIGNMENT;
  if (kv_rows > (int64_t)INT32_MAX - 256 || q_stride > (int64_t)INT32_MAX ||
      k_stride > (int64_t)INT32_MAX || v_stride > (int64_t)INT32_MAX)
    return H3B_ERR_INVALID_ARG;
  if (q_rows == 0) return H3B_OK;
  if (!q_buf || !k_buf || !v_buf || !out) return H3B_ERR_INVALID_ARG;
  if (!aligned16(q_buf) || !aligned16(k_buf) || !aligned16(v_buf) || !aligned16(out))
    return H3B_ERR_ALIGNMENT;
  int rc = check_sm100();
  if (rc != H3B_OK) return rc;

  static std::once_flag attr_once;
  static cudaError_t attr_err = cudaSuccess;
  static int attr_regs = 0;
  std::call_once(attr_once, [] {
    attr_err = cudaFuncSetAttribute(attn::k_fmha, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    attn::SMEM_BYTES);
    cudaFuncAttributes fa;
    if (attr_err == cudaSuccess) attr_err = cudaFuncGetAttributes(&fa, attn::k_fmha);
    if (attr_err == cudaSuccess) attr_regs = fa.numRegs;
  });
  if (attr_err != cudaSuccess) return H3B_ERR_CUDA;
  // the kernel's setmaxnreg split assumes this launch register count
  if (attr_regs != attn::kLaunchRegs) return H3B_ERR_UNSUPPORTED;

  attn::Args args;
  memset(&args, 0, sizeof(args));
  rc = tmap_bf16_rows(&args.tmap_q, q_buf, q_rows, q_stride);
  if (rc != H3B_OK) return rc;
  rc = tmap_bf16_rows(&args.tmap_kv, k_buf, kv_rows, k_stride);
  if (rc != H3B_OK) return rc;
  if (v_buf == k_buf && v_stride == k_stride) {
    args.tmap_v = args.tmap_kv;
  } else {
    rc = tmap_bf16_rows(&args.tmap_v, v_buf, kv_rows, v_stride);
    if (rc != H3B_OK) return rc;
  }
  args.out = static_cast<__nv_bfloat16*>(out);
  args.ldo = ldo;
  args.q_off = (int)q_off;
  args.k_off = (int)k_off;
  args.v_off = (int)v_off;
  args.H = H;
  args.scale_log2 = scale * 1.4426950408889634f;
  // documents that own local queries; longest key ranges first (most work per CTA)
  int order[attn::MAX_DOCS];
  int n = 0;
  for (int i = 0; i < ndocs; ++i) {
    const int64_t a = std::max<int64_t>(cu_seqlens_host[i], q_row0);
    const int64_t b = std::min<int64_t>(cu_seqlens_host[i + 1], q_row0 + q_rows);
    if (b > a) order[n++] = i;
  }
  std::sort(order, order + n, [&](int a, int b) {
    return cu_seqlens_host[a + 1] - cu_seqlens_host[a] > cu_seqlens_host[b + 1] - cu_seqlens_host[b];
  });
  int64_t items = 0;
  for (int i = 0; i < n; ++i) {
    const int d = order[i];
    const int64_t qa = std::max<int64_t>(cu_seqlens_host[d], q_row0);
    const int64_t qb = std::min<int64_t>(cu_seqlens_host[d + 1], q_row0 + q_rows);
    args.doc_start[i] = cu_seqlens_host[d];
    args.doc_len[i] = cu_seqlens_host[d + 1] - cu_seqlens_host[d];
    args.q_start[i] = (int)(qa - q_row0);
    args.q_len[i] = (int)(qb - qa);
    items += (int64_t)((args.q_len[i] + 2 * attn::BQ - 1) / (2 * attn::BQ)) * H;
    if (items > INT32_MAX) return H3B_ERR_INVALID_ARG;
    args.item_end[i] = (int)items;
  }
  args.ndocs = n;
  if (items == 0) return H3B_OK;
  attn::k_fmha<<<(unsigned)items, attn::THREADS, attn::SMEM_BYTES,
                 static_cast<cudaStream_t>(stream)>>>(args);
  return launched(cudaGetLastError());
}
}  // namespace h3b

extern "C" {

int h3b_attention_varlen(const void* q_buf, int64_t q_rows, int64_t q_stride, int64_t q_off,
                         int64_t q_row0, const void* kv_buf, int64_t kv_rows, int64_t kv_stride,
                         int64_t k_off, int64_t v_off, int H, int D,
                         const int32_t* cu_seqlens_host, int ndocs, float scale, void* out,
                         int64_t ldo, void* stream) {
  return attention_launch(q_buf, q_rows, q_stride, q_off, q_row0, kv_buf, kv_stride, k_off,
                          kv_buf, kv_stride, v_off, kv_rows, H, D, cu_seqlens_host, ndocs, scale,
                          out, ldo, stream);
}

int h3b_attention_qkv(const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                      const void* v, int64_t v_stride, int64_t rows, int H, int D,
                      const int32_t* cu_seqlens_host, int ndocs, float scale, void* out,
                      int64_t ldo, void* stream) {
  return attention_launch(q, rows, q_stride, 0, 0, k, k_stride, 0, v, v_stride, 0, rows, H, D,
                          cu_seqlens_host, ndocs, scale, out, ldo, stream);
}

// ------------------------------------------------------------------ RMSNorm -> NVFP4, no allocation
// Some callers of this library cannot allocate device memory while they run:
// inference servers that hand every kernel a fixed, pre-planned memory pool,
// plugin hosts whose execute callback must not touch the allocator, and code
// that runs while another allocator owns the device.  Such callers cannot
// provide the per-row rstd / amax scratch that h3b_rmsnorm_stats and
// h3b_rmsnorm_quantize pass between them.  h3b_rmsnorm_quantize_noalloc runs
// the same two kernels with that scratch in a fixed array compiled into the
// library: every GPU that loads libh3b.so holds it (kNoAllocRows * 4 + 256
// bytes) until the process exits.  All calls on a device share the array, so
// calls that overlap on the GPU (different streams, no ordering between
// them) race; calls on one stream, or otherwise ordered, are safe.
constexpr int64_t kNoAllocRows = 131072;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocRows + 64];

namespace h3b {
constexpr int kNoAllocMaxDevices = 64;
static float* g_noalloc_ptr[kNoAllocMaxDevices];
static CUcontext g_noalloc_ctx[kNoAllocMaxDevices];
static std::mutex g_noalloc_mu;

// The driver's current context, through the runtime's driver entry point
// (the library links only cudart).
static int current_context(CUcontext* ctx) {
  using Fn = CUresult (*)(CUcontext*);
  static Fn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<Fn>(p);
  });
  if (!fn || fn(ctx) != CUDA_SUCCESS) return H3B_ERR_CUDA;
  return H3B_OK;
}

// Device address of g_noalloc_scratch on the current device.  In host code the
// symbol itself is only a host-side stand-in, so the address is looked up with
// cudaGetSymbolAddress (with the device current) and cached per device,
// together with the context it belongs to: after a device reset the runtime
// creates a new context and loads the module again, so a context change
// triggers a fresh lookup instead of reusing a stale address.
static int noalloc_scratch(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return H3B_ERR_CUDA;
  if (dev < 0 || dev >= kNoAllocMaxDevices) return H3B_ERR_UNSUPPORTED;
  // NULL before the runtime has made this device's primary context current
  CUcontext ctx = nullptr;
  int rc = current_context(&ctx);
  if (rc != H3B_OK) return rc;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr || ctx == nullptr || g_noalloc_ctx[dev] != ctx) {
    void* p = nullptr;
    // the lookup itself initialises the primary context when needed
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr)
      return H3B_ERR_CUDA;
    rc = current_context(&ctx);
    if (rc != H3B_OK) return rc;
    g_noalloc_ptr[dev] = static_cast<float*>(p);
    g_noalloc_ctx[dev] = ctx;
  }
  *out = g_noalloc_ptr[dev];
  return H3B_OK;
}
}  // namespace h3b

int h3b_selftest_bounded_wait(int64_t limit_us, void* stream) {
  if (limit_us < 1 || limit_us > 1000000) return H3B_ERR_INVALID_ARG;
  int rc = check_sm100();
  if (rc != H3B_OK) return rc;
  k_selftest_bounded_wait<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      (uint64_t)limit_us * 1000ull);
  return launched(cudaGetLastError());
}

// ------------------------------------------------------------------ peer amax exchange
static_assert(sizeof(cudaIpcMemHandle_t) == H3B_PEER_HANDLE_BYTES, "IPC handle size");

int h3b_peer_buffer_create(int64_t bytes, void** dev_ptr, void* ipc_handle) {
  if (!dev_ptr || !ipc_handle || bytes <= 0 || bytes > (int64_t)(1 << 20))
    return H3B_ERR_INVALID_ARG;
  void* p = nullptr;
  if (cudaMalloc(&p, (size_t)bytes) != cudaSuccess) return H3B_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, (size_t)bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
      cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return H3B_ERR_CUDA;
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *dev_ptr = p;
  return H3B_OK;
}

int h3b_peer_buffer_open(const void* ipc_handle, void** dev_ptr) {
  if (!ipc_handle || !dev_ptr) return H3B_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return H3B_ERR_CUDA;
  *dev_ptr = p;
  return H3B_OK;
}

int h3b_peer_buffer_close(void* dev_ptr) {
  if (!dev_ptr) return H3B_ERR_INVALID_ARG;
  return cudaIpcCloseMemHandle(dev_ptr) == cudaSuccess ? H3B_OK : H3B_ERR_CUDA;
}

int h3b_peer_buffer_destroy(void* dev_ptr) {
  if (!dev_ptr) return H3B_ERR_INVALID_ARG;
  return cudaFree(dev_ptr) == cudaSuccess ? H3B_OK : H3B_ERR_CUDA;
}

int h3b_amax_exchange(float* amax, const void* slot_table, int rank, int world, int64_t epoch,
                      int64_t limit_us, void* stream) {
  if (!amax || !slot_table || world < 1 || world > peer::kMaxRanks || rank < 0 || rank >= world)
    return H3B_ERR_INVALID_ARG;
  if (epoch < 1 || epoch > (int64_t)0xFFFFFFFFll || limit_us < 1 || limit_us > 60000000)
    return H3B_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(amax) & 3u) || (reinterpret_cast<uintptr_t>(slot_table) & 7u))
    return H3B_ERR_ALIGNMENT;
  int rc = check_sm100();
  if (rc != H3B_OK) return rc;
  peer::k_amax_exchange<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      amax, static_cast<const unsigned long long* const*>(slot_table), rank, world,
      (uint32_t)epoch, (uint64_t)limit_us * 1000ull);
  return launched(cudaGetLastError());
}

int h3b_rmsnorm_quantize_noalloc(const void* x, int64_t M, int64_t K, int64_t ldx,
                                 const void* gamma, float eps, const void* shift,
                                 const void* scale, const int32_t* mod_idx, float* gs_out,
                                 void* q, void* sf, int64_t Mpad, void* stream) {
  if (M > kNoAllocRows) return H3B_ERR_INVALID_ARG;   // beyond the fixed scratch
  NormArgs a;
  int rc = norm_args(a, x, M, K, ldx, gamma, eps, shift, scale, mod_idx);
  if (rc != H3B_OK) return rc;
  if (!q || !sf || Mpad < M || Mpad % 128) return H3B_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(q) & 3u) return H3B_ERR_ALIGNMENT;
  if (Mpad == 0) return H3B_OK;
  rc = check_sm100();
  if (rc != H3B_OK) return rc;
  float* scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc != H3B_OK) return rc;
  float* rstd = scratch;                    // [kNoAllocRows]
  float* amax = scratch + kNoAllocRows;     // 1 float, 256-byte aligned
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the array keeps the previous call's contents: amax must start at zero
  if (cudaMemsetAsync(amax, 0, sizeof(float), st) != cudaSuccess) return H3B_ERR_CUDA;
  const unsigned stat_blocks = (unsigned)((M + kNormWarps - 1) / kNormWarps);
  if (M > 0) {
    if (K <= kNormCacheChunks * 256)
      k_rmsnorm_stats<kNormCacheChunks><<<stat_blocks, kNormWarps * 32, 0, st>>>(a, rstd, amax);
    else
      k_rmsnorm_stats<0><<<stat_blocks, kNormWarps * 32, 0, st>>>(a, rstd, amax);
    rc = launched(cudaGetLastError());
    if (rc != H3B_OK) return rc;
  }
  const unsigned q_blocks = (unsigned)((Mpad + kNormWarps - 1) / kNormWarps);
  k_rmsnorm_quant<<<q_blocks, kNormWarps * 32, 0, st>>>(
      a, rstd, amax, gs_out, static_cast<uint8_t*>(q), static_cast<uint8_t*>(sf), Mpad, nullptr);
  return launched(cudaGetLastError());
}

}  // extern "C"
