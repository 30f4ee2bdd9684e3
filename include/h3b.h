/*
 * h3b -- C ABI of the B200 (sm_100a) NVFP4 hot path of the h3-engine DiT.
 *
 * Every pointer argument is a DEVICE pointer unless stated otherwise; `stream`
 * is a cudaStream_t passed as void*.  Calls are asynchronous on `stream`,
 * allocate no device memory, do not synchronize the host, and return an
 * h3b_status.  Shapes are validated on the host before any launch; a kernel
 * that detects a fault at run time (a bounded wait that ran out) records it
 * in a per-device error word, read with h3b_device_error().
 *
 * Reference interfaces these entry points replace are cited per function as
 * h3_inference/<file>:<line> (shauray8/h3-engine).
 */
#ifndef H3B_H_
#define H3B_H_

#include <stdint.h>

#if defined(__GNUC__)
#define H3B_API __attribute__((visibility("default")))
#else
#define H3B_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  H3B_OK = 0,
  H3B_ERR_INVALID_ARG = 1,   /* a shape, size or enum value is out of range        */
  H3B_ERR_ALIGNMENT = 2,     /* a pointer or leading dimension is misaligned       */
  H3B_ERR_CUDA = 3,          /* a CUDA runtime call failed                         */
  H3B_ERR_UNSUPPORTED = 4,   /* device is not sm_100 or a feature is unavailable   */
  H3B_ERR_TIMEOUT = 5,       /* device side: a bounded wait expired               */
  H3B_ERR_DEVICE = 6         /* device side: other recorded failure               */
} h3b_status;

/* Scale-factor layouts. */
enum { H3B_SF_ROWMAJOR = 0,  /* e4m3 [rows, K/16], row-major                                   */
       H3B_SF_SWIZZLED = 1   /* 128x4 tiles of 512 B: (r,c) at ((r/128)*(C/4)+c/4)*512
                                + (r%32)*16 + ((r%128)/32)*4 + c%4 (C = K/16)                   */
};

/* GEMM epilogue activations. */
enum { H3B_ACT_NONE = 0, H3B_ACT_GELU_TANH = 1, H3B_ACT_SWIGLU = 2 };

/* ------------------------------------------------------------------ library */
H3B_API int h3b_version(void);
H3B_API const char* h3b_status_string(int status);
/* Number of kernels this library has launched in this process (all devices). */
H3B_API long long h3b_launch_count(void);
/* Reads (and with clear != 0 resets) the current device's error word.
   Synchronizes the device.  *code_out = 0 when no kernel recorded a fault. */
H3B_API int h3b_device_error(int* code_out, int clear);

/* ------------------------------------------------------------------ quantize
 * amax_out[0] = max |x| over a [rows, cols] bf16 matrix with row stride ldx
 * (elements).  Replaces the global-amax half of the maiku quantizer behind
 * h3_inference/nvfp4.py:20-23 (the three-level recipe's fp32 global scale).
 * amax_out is overwritten (zeroed on `stream`, then reduced into).            */
H3B_API int h3b_amax_bf16(const void* x, int64_t rows, int64_t cols, int64_t ldx, float* amax_out,
                  void* stream);

/* NVFP4 quantize/pack.  Replaces _quantize / _quantize_padded + _swizzle
 * (h3_inference/nvfp4.py:20-46):
 *   x      bf16 [M, K], row stride ldx (elements), K % 64 == 0
 *   amax   device fp32 scalar (from h3b_amax_bf16 or a fused producer); the
 *          global scale is gs = amax / 2688 (gs = 1 when amax == 0).  When
 *          amax is NULL, gs_in is used instead (pass 1.0 for the two-level
 *          scheme of the reference).
 *   gs_out device fp32 scalar receiving gs (may be NULL)
 *   q      u8 [Mpad, K/2]: E2M1 codes, low nibble = even K index
 *   sf     e4m3 scales, layout H3B_SF_ROWMAJOR [Mpad, K/16] or
 *          H3B_SF_SWIZZLED (Mpad % 128 == 0)
 *   Mpad   >= M; rows M..Mpad-1 get zero codes and zero scales.              */
H3B_API int h3b_nvfp4_quantize(const void* x, int64_t M, int64_t K, int64_t ldx, const float* amax,
                       float gs_in, float* gs_out, void* q, void* sf, int sf_layout, int64_t Mpad,
                       void* stream);

/* NVFP4 unpack: out bf16 [M, K] = bf16((LUT[code] * s) * gs).  The CPU decode
 * this mirrors is h3_inference/render.py:178-183 (plus the global scale).
 * sf is laid out as sf_layout over `sf_rows` rows (>= M).                    */
H3B_API int h3b_nvfp4_dequantize(const void* q, const void* sf, int sf_layout, int64_t sf_rows,
                         const float* gs, int64_t M, int64_t K, void* out, void* stream);

/* ------------------------------------------------------------------ GEMM
 * D[M, N] (bf16, row stride ldd) = epilogue( alpha * (A * sfA) x (B * sfB)^T )
 * with alpha = gsA * gsB (device fp32; NULL means 1).  gsB holds one value
 * per `gsb_seg` output columns (gsb_seg % 128 == 0, N % gsb_seg == 0), or a
 * single value when gsb_seg == 0 -- this lets weights that were quantized
 * separately (to_q, to_k, to_v) run as one N-concatenated GEMM.  Replaces
 * QuantizedActivation.mm / torch._scaled_mm (h3_inference/nvfp4.py:112-115)
 * and, through the epilogue, the bias/GELU/residual work around it
 * (h3_inference/kernels/ffn_qkvo_gemms.py:10-54).
 *   A    u8 [a_rows, K/2] packed E2M1, a_rows % 128 == 0, a_rows >= M
 *   sfA  swizzled e4m3 scales of A (a_rows rows)
 *   B    u8 [N, K/2] packed E2M1 (the weight, K-major), N % 128 == 0
 *   sfB  swizzled e4m3 scales of B
 *   K    % 256 == 0
 *   epilogue, in order: v = acc*alpha; v += bias[n] (bf16, optional);
 *   v = act(v); v *= gate[gate_idx[m], n] (bf16 [rows, N], optional; NULL
 *   gate_idx means row 0 -- the adaLN-zero gate of gate_residual,
 *   h3_inference/kernels/elementwise_norm_rope.py:150-163; every gate_idx[m]
 *   must be >= 0 and below the gate table's row count, it is not checked);
 *   v += residual[m, n] (bf16, row stride ldr, optional);
 *   D = bf16(v); amax_out (optional) is atomically max-reduced with |D|
 *   (the caller zeroes it first).
 * act == H3B_ACT_SWIGLU: the fused up-projection of a SwiGLU feed-forward
 *   (h3_inference/kernels/ffn_qkvo_gemms.py:31-35, transformer/ops.py:62-73:
 *   value, gate = proj(x).chunk(2); value * silu(gate)).  B holds the 2F rows
 *   [value | gate] interleaved in 64-row blocks -- per 256 rows: value
 *   f..f+63, gate f..f+63, value f+64..f+127, gate f+64..f+127 (f = 128 t) --
 *   and D is [M, N/2]: D = bf16(bf16(v) * bf16(silu(bf16(g)))), the rounding
 *   of the reference's bf16 ops.  N % 256 == 0; bias, gate and residual must
 *   be NULL.                                                                 */
H3B_API int h3b_nvfp4_gemm(const void* A, const void* sfA, const float* gsA, int64_t M, int64_t a_rows,
                   const void* B, const void* sfB, const float* gsB, int64_t gsb_seg, int64_t N,
                   int64_t K, const void* bias, const void* residual, int64_t ldr,
                   const void* gate, const int32_t* gate_idx, int act, void* D, int64_t ldd,
                   float* amax_out, void* stream);

/* ------------------------------------------------------------------ RMSNorm -> NVFP4
 * The norm that feeds the QKV and FFN-up GEMMs, fused with the activation
 * quantization.  Replaces rms_norm / norm_modulate / ada_modulate
 * (h3_inference/kernels/elementwise_norm_rope.py:19-23,42-52,69-102) and the
 * QuantizedActivation quantization of their output (h3_inference/nvfp4.py:92-110):
 *   y[m, k] = bf16( x*rstd*gamma[k] * (1 + scale[idx[m], k]) + shift[idx[m], k] )
 *   rstd[m] = 1 / sqrt(mean_k x[m,k]^2 + eps)
 * (modulation optional: shift/scale NULL; idx NULL means table row 0).
 * Every idx[m] must be >= 0 and below the number of rows of the shift / scale
 * tables: the kernels index the tables with it unchecked (the same holds
 * for gate_idx and the gate table of h3b_nvfp4_gemm).
 * K % 256 == 0.  Pass 1 writes rstd [M] and amax_out = max|y| (zeroed on
 * `stream` first); pass 2 recomputes y and writes E2M1 codes [Mpad, K/2] and
 * swizzled scales with gs = amax / 2688 (Mpad % 128 == 0), plus y itself
 * when y_out is non-NULL.                                                   */
H3B_API int h3b_rmsnorm_stats(const void* x, int64_t M, int64_t K, int64_t ldx, const void* gamma,
                              float eps, const void* shift, const void* scale,
                              const int32_t* mod_idx, float* rstd_out, float* amax_out,
                              void* stream);
H3B_API int h3b_rmsnorm_quantize(const void* x, int64_t M, int64_t K, int64_t ldx,
                                 const void* gamma, const void* shift, const void* scale,
                                 const int32_t* mod_idx, const float* rstd, const float* amax,
                                 float* gs_out, void* q, void* sf, int64_t Mpad, void* y_out,
                                 void* stream);

/* ------------------------------------------------------------------ qk-norm + RoPE
 * In place on the query and key heads of the projected activations (bf16):
 * query head h of token t at q[t*q_stride + q_off + h*D], key head h at
 * k[t*k_stride + k_off + h*D] (q and k may be the same packed QKV buffer).
 * Per head vector: RMSNorm over D with weight wq / wk (NULL: no norm), then
 * rotate-half RoPE over the first R dims with the (T, R) fp32 cos/sin tables
 * (row stride cs_stride; NULL cos: no RoPE), dims >= R pass through.
 * Replaces qk_norm + apply_rotary_emb / norm_rope
 * (h3_inference/kernels/elementwise_norm_rope.py:19-40,104-148).
 * D in {64, 128}; R <= D, (R/2) % 8 == 0; q/k strides and offsets
 * multiples of 8; cos/sin 16-byte aligned with cs_stride % 4 == 0.  q or k
 * may be NULL (only the other heads are processed), not both.             */
H3B_API int h3b_qk_norm_rope(void* q, int64_t q_stride, int64_t q_off, void* k, int64_t k_stride,
                             int64_t k_off, int64_t T, int H, int D, const void* wq,
                             const void* wk, float eps, const float* cos, const float* sin, int R,
                             int64_t cs_stride, void* stream);

/* The same, out of place: query heads read from q (head h at column h*D of
 * row t, row stride q_stride) and written to q_out (row stride qo_stride),
 * key heads from k to k_out likewise; q or k may be NULL (with its output),
 * not both.  The function form of the row shims norm_rope / apply_rotary_emb
 * (h3_inference/kernels/elementwise_norm_rope.py:25-40,133-148), whose
 * inputs stay untouched.  Limits as above.                                */
H3B_API int h3b_qk_norm_rope_out(const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                                 void* q_out, int64_t qo_stride, void* k_out, int64_t ko_stride,
                                 int64_t T, int H, int D, const void* wq, const void* wk, float eps,
                                 const float* cos, const float* sin, int R, int64_t cs_stride,
                                 void* stream);

/* ------------------------------------------------------------------ gathered adaLN ops
 * Per-row table gathers of the reference block, bf16 [rows, cols] (row
 * strides in elements, cols % 8 == 0, 16-byte aligned rows), the table row
 * of row r being idx[r % n_idx] (idx NULL: row 0), with torch's bf16 rounding
 * after every op (bit-identical to the reference's stock expressions):
 *   h3b_gate_residual: out = residual + gate[idx] * y
 *     (gate_residual, h3_inference/kernels/elementwise_norm_rope.py:150-163)
 *   h3b_ada_modulate:  out = x * (1 + scale[idx]) + shift[idx]
 *     (ada_modulate, h3_inference/kernels/elementwise_norm_rope.py:90-102)
 * Tables are bf16 [n_rows, cols]; every idx value must be >= 0 and below
 * n_rows (not checked).  out may alias residual / x (same strides).        */
H3B_API int h3b_gate_residual(const void* residual, int64_t ldr, const void* y, int64_t ldy,
                              const void* gate, const int32_t* idx, int64_t n_idx, int64_t rows,
                              int64_t cols, void* out, int64_t ldo, void* stream);
H3B_API int h3b_ada_modulate(const void* x, int64_t ldx, const void* scale, const void* shift,
                             const int32_t* idx, int64_t n_idx, int64_t rows, int64_t cols,
                             void* out, int64_t ldo, void* stream);

/* ------------------------------------------------------------------ packed varlen attention
 * out[i, h*D + d] = softmax_j(q_i . k_j * scale) v_j for every local query row
 * i, over the keys j of the document that contains its global row q_row0 + i
 * (non-causal), bf16 in/out, fp32 softmax and accumulation.
 *   q head h: q_buf[i, q_off + h*D .. +D)       (q_rows rows, row stride q_stride)
 *   k / v head h: kv_buf[j, {k,v}_off + h*D ..) (kv_rows rows = the full sequence)
 * With q_buf == kv_buf, q_row0 = 0 and q_rows = kv_rows this is plain packed
 * attention over one QKV activation; with a token-sharded sequence q_buf is
 * the local shard and kv_buf the gathered keys / values.
 * cu_seqlens_host: HOST array of ndocs+1 global document boundaries, [0] = 0,
 * [ndocs] = kv_rows, non-decreasing (the launch shape depends on it);
 * ndocs <= 64; D == 128; strides / offsets multiples of 8.
 * Replaces F.scaled_dot_product_attention in packed_self_attention
 * (h3_inference/kernels/packed_self_attn.py:8-37); cu_seqlens = {0, T}
 * reproduces the reference's single-document attention.                    */
H3B_API int h3b_attention_varlen(const void* q_buf, int64_t q_rows, int64_t q_stride, int64_t q_off,
                                 int64_t q_row0, const void* kv_buf, int64_t kv_rows,
                                 int64_t kv_stride, int64_t k_off, int64_t v_off, int H, int D,
                                 const int32_t* cu_seqlens_host, int ndocs, float scale,
                                 void* out, int64_t ldo, void* stream);

/* The same attention over three separate bf16 activations [rows, *]: head h
 * of q, k and v at column h*D of their rows (row strides q_stride, k_stride,
 * v_stride), every row a query and a key; the shape of
 * packed_self_attention's (B, T, H, D) query / key / value tensors
 * (h3_inference/kernels/packed_self_attn.py:8-37), which need not share a
 * buffer.  Limits as above.                                                 */
H3B_API int h3b_attention_qkv(const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                              const void* v, int64_t v_stride, int64_t rows, int H, int D,
                              const int32_t* cu_seqlens_host, int ndocs, float scale, void* out,
                              int64_t ldo, void* stream);

/* ------------------------------------------------------------------ no-allocation variant
 * No counterpart in the reference.  The same RMSNorm(+modulation) -> NVFP4
 * result as h3b_rmsnorm_stats followed by h3b_rmsnorm_quantize (y_out not
 * available), for callers that cannot allocate device memory while they run
 * -- servers that give kernels a fixed pre-planned memory pool, plugin hosts
 * whose execute path must not call the allocator -- and so cannot provide the
 * rstd / amax scratch the two-call form needs.  The scratch is a fixed array
 * inside libh3b.so (every GPU that loads the library keeps it, about 512 KiB,
 * until the process exits); the call itself allocates nothing.
 *   M <= 131072 rows, else H3B_ERR_INVALID_ARG; other limits as above.
 *   The first call on a device looks up the array's device address (once per
 *   device and context, with that device current; a device reset makes the
 *   next call look it up again); make that first call before any stream
 *   capture.
 *   All calls on a device share the array: calls that overlap on the GPU
 *   race.  Order them (one stream, or events) if more than one can be in
 *   flight.                                                                  */
H3B_API int h3b_rmsnorm_quantize_noalloc(const void* x, int64_t M, int64_t K, int64_t ldx,
                                         const void* gamma, float eps, const void* shift,
                                         const void* scale, const int32_t* mod_idx,
                                         float* gs_out, void* q, void* sf, int64_t Mpad,
                                         void* stream);

/* Self-test of the failure path every kernel above shares (no reference
 * counterpart): one CTA waits, with the kernels' bounded mbarrier wait but a
 * bound of limit_us microseconds, on a barrier that nothing arrives on; when
 * the bound expires it records H3B_ERR_TIMEOUT in the device error word and
 * returns, as the GEMM and attention kernels do when a pipeline stage never
 * completes.  The context stays usable; read and clear the word with
 * h3b_device_error.  1 <= limit_us <= 1000000, else H3B_ERR_INVALID_ARG.    */
H3B_API int h3b_selftest_bounded_wait(int64_t limit_us, void* stream);

/* ------------------------------------------------------------------ peer amax exchange
 * The max of a per-rank fp32 amax over the ranks of a sharded run, through
 * peer memory (replaces the NCCL max all-reduce before every NVFP4
 * activation quantization of a token-/CFG-sharded run, which keeps one
 * global scale per activation as QuantizedActivation computes it over the
 * whole tensor, h3_inference/nvfp4.py:92-110).
 *
 * Set-up, once per run on every rank (not on the hot path):
 *   h3b_peer_buffer_create  cudaMalloc'd, zeroed slot array of `bytes`
 *                           (2 * world * 8 bytes) on the current device and
 *                           its CUDA IPC handle (H3B_PEER_HANDLE_BYTES bytes)
 *   h3b_peer_buffer_open    maps another rank's array from its handle
 *   h3b_peer_buffer_close / h3b_peer_buffer_destroy  undo the two
 * Exchange number `epoch` (1, 2, 3, ... in the same order on every rank):
 *   h3b_amax_exchange       *amax = max over ranks of each rank's *amax;
 *                           slot_table: device array of `world` pointers,
 *                           entry r = rank r's array as mapped here (entry
 *                           `rank` = this rank's own).  One warp; peer stores
 *                           and polling loads, no multicast.  The wait for the
 *                           other ranks is bounded by limit_us (1 ..
 *                           60000000): on expiry the kernel records
 *                           H3B_ERR_TIMEOUT, leaves *amax local and returns.
 * world <= 32.                                                             */
#define H3B_PEER_HANDLE_BYTES 64
H3B_API int h3b_peer_buffer_create(int64_t bytes, void** dev_ptr, void* ipc_handle);
H3B_API int h3b_peer_buffer_open(const void* ipc_handle, void** dev_ptr);
H3B_API int h3b_peer_buffer_close(void* dev_ptr);
H3B_API int h3b_peer_buffer_destroy(void* dev_ptr);
H3B_API int h3b_amax_exchange(float* amax, const void* slot_table, int rank, int world,
                              int64_t epoch, int64_t limit_us, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* H3B_H_ */
