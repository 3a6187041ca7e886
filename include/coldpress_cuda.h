/*
 * coldpress_cuda.h -- C ABI of libcoldpress_cuda.so, the B200 (sm_100a) encoder hot path of
 * coldpress: k-quant fit + pack, committed-grid decode, FP64 error-feedback factorisation, the
 * ordered error-feedback column sweep and X^T X Hessian accumulation.
 *
 * Conventions
 *   - Every array argument is a DEVICE pointer (cudaMalloc / torch CUDA memory), row-major,
 *     16-byte aligned.  `stream` is a cudaStream_t passed as void* (NULL = legacy stream).
 *   - Calls only enqueue work; they return before it finishes.  The return value is a
 *     CP_* status (0 = ok); CP_ERR_CUDA carries the CUDA message in cp_last_error().
 *   - Types are GGML type ids: Q8_0 = 8, Q2_K = 10, Q3_K = 11, Q4_K = 12, Q5_K = 13, Q6_K = 14.
 *   - Weights are float32 [nrow, n] with n a multiple of 256 (32 for Q8_0); imatrix vectors
 *     are float32 [n] and apply to every row; packed rows are n/256 * cp_block_bytes(type).
 *   - Output bytes are identical to the reference numpy codec (coldpress/kquant.py) for the
 *     same float32 inputs; inputs containing NaN or Inf are outside that guarantee.
 *
 * Line references are to the reference package (coldpress/...), whose Python functions
 * these entry points replace when coldpress runs with device="cuda".
 */
#ifndef COLDPRESS_CUDA_H
#define COLDPRESS_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CP_OK 0
#define CP_ERR_TYPE 1      /* unsupported GGML type (ef.py:127,176 raise ValueError) */
#define CP_ERR_SHAPE 2     /* n not a multiple of the block size (kquant.py:351 assert) */
#define CP_ERR_NOT_PD 3    /* factorisation hit a non-positive pivot (ef.py:74 LinAlgError) */
#define CP_ERR_CUDA 4      /* a CUDA launch or call failed; see cp_last_error() */
#define CP_ERR_ARG 5       /* null pointer or out-of-range argument */
#define CP_ERR_WORKSPACE 6 /* workspace smaller than the matching *_workspace_bytes() */
#define CP_ERR_TIMEOUT 7   /* a kernel's bounded wait ran out (cp_xtx_status) */

/* Library version (major*10000 + minor*100 + patch) and the last error message of the
 * calling thread. */
int cp_version(void);
const char* cp_last_error(void);

/* Per-kernel-class device timing for benchmarks.  While enabled, every launch made by this
 * thread through the calls below is bracketed by CUDA events on its stream.
 * cp_profile_collect waits for them and returns, per class (0 k-quant fit, 1 error-feedback
 * sweep, 2 factorisation, 3 other), the summed milliseconds and the number of calls, then
 * clears the record.  Either output pointer may be NULL (host arrays of 4). */
void cp_profile_enable(int on);
/* Kernels launched by this library since it was loaded (all threads). */
int64_t cp_launch_count(void);
int cp_profile_collect(double* ms, int64_t* launches);

/* Bytes of one packed block of `ggml_type` (kquant.py:21 BYTES_PER_SB; 34 for Q8_0), or 0. */
int cp_block_bytes(int ggml_type);

/* kquant.py:732 QUANTIZE[type](x, qw): fit and pack every superblock.  qw == NULL selects
 * the reference (no imatrix) path.  out: [nrow, n/256 * cp_block_bytes(type)] bytes. */
int cp_kquant_encode(int ggml_type, const float* x, int64_t nrow, int64_t n, const float* qw,
                     uint8_t* out, void* stream);

/* kquant.py:734 DEQUANTIZE[type](raw, n): out float32 [nrow, n]. */
int cp_kquant_decode(int ggml_type, const uint8_t* raw, int64_t nrow, int64_t n, float* out,
                     void* stream);

/* ef.py:87-127 _grid_params: per (row, sub-block) step dl and offset ml of committed bytes,
 * float32 [nrow, n/16] (Q2_K, Q3_K, Q6_K) or [nrow, n/32] (Q4_K, Q5_K).  ml may be NULL; it
 * is written as 0 for the types without a min (Q3_K, Q6_K). */
int cp_grid_params(int ggml_type, const uint8_t* raw, int64_t nrow, int64_t n, float* dl, float* ml,
                   void* stream);

/* Signed integer codes held by committed bytes (ef.py's L: Q2_K 0..3, Q3_K -4..3, Q4_K 0..15,
 * Q5_K 0..31, Q6_K -32..31) as int8 [nrow, n]. */
int cp_kquant_codes(int ggml_type, const uint8_t* raw, int64_t nrow, int64_t n, int8_t* codes,
                    void* stream);

/* ef.py:130-176 _repack: write int8 codes [nrow, n] into committed bytes, scales unchanged. */
int cp_kquant_repack(int ggml_type, uint8_t* raw, const int8_t* codes, int64_t nrow, int64_t n,
                     void* stream);

/* ef.py:298-301 encode_gguf statistics: *out (device float64) = sum over the tensor of
 * (DEQUANTIZE(raw) - x)^2 * w[column], with w == NULL meaning 1 (the reference's weights are
 * qw or ones).  Accumulated in float64 (the reference sums in float32; this is a diagnostic). */
int cp_weighted_err(int ggml_type, const uint8_t* raw, const float* x, const float* w, int64_t nrow, int64_t n,
                    double* out, void* stream);

/* perm/objective.py:22-28 (x[idx] row sample, then x[:, perm]): out float32 [nrow_out, n_out]
 * with out[i][j] = x[row(i) * ld + col(j)], row(i) = rows[i] and col(j) = cols[j] (int64 device
 * arrays), or i and j where rows / cols is NULL.  Indices are not range-checked. */
int cp_gather_f32(const float* x, int64_t ld, const int64_t* rows, int64_t nrow_out, const int64_t* cols,
                  int64_t n_out, float* out, void* stream);

/* perm/objective.py:32-33 and 42-49: out float64 [n] with out[c] = sum over r < nrow of
 * (x[r * ld + c] - y[r * ld + c])^2 (y == NULL: x^2), accumulated in float64 in a fixed order
 * (repeated calls give identical bits; the reference's own summation order differs, so the
 * last bits of float64 may too). */
int cp_col_sqdiff(const float* x, const float* y, int64_t nrow, int64_t n, int64_t ld, double* out, void* stream);

/* hessians.py:225-245 load_hessian arithmetic: H (float64 [d, d]) = float64(h16) * hscale with
 * the exact float32 diagonal diag32 (may be NULL) written over it; h16 holds float16 bits. */
int cp_hessian_decode(const uint16_t* h16, const float* diag32, double hscale, int64_t d, double* H, void* stream);

/* ef.py:46-84 cholesky_inv_upper with ef.py:187-189 folded in: for the act-order permutation
 * `order` (int32 [n]), U_out = float32(chol(inv(H[order][:,order] + diag_shift*I)).T), upper
 * triangular [n, n].  diag_shift is the reference's damp*mean(diag(H[order][:,order])) + 1e-8.
 * H: float64 [n, n] symmetric, n a multiple of 64.  *status_dev (device int32) is set to 0,
 * or to CP_ERR_NOT_PD when a pivot is not positive; callers escalate damp and retry as
 * ef.py:67-76 does.  workspace >= cp_factor_workspace_bytes(n). */
size_t cp_factor_workspace_bytes(int64_t n);
int cp_factor_u(const double* H, int64_t n, const int32_t* order, double diag_shift, float* U_out,
                void* workspace, size_t workspace_bytes, int32_t* status_dev, void* stream);
/* Same factor left in float64 (ef.py:46-84 returns float64; ef_encode casts it). */
int cp_factor_u_f64(const double* H, int64_t n, const int32_t* order, double diag_shift, double* U_out,
                    void* workspace, size_t workspace_bytes, int32_t* status_dev, void* stream);

/* Device layout of U for the sweep: U row-major float32 [n][n] followed by its diagonal,
 * cp_ef_u_bytes(n) bytes (U and u_prepared 16-byte aligned).  Built once per factor (q/k/v
 * and gate/up share theirs).  u_prepared may equal U (the factor written straight into the
 * start of a cp_ef_u_bytes(n) buffer): then only the diagonal is appended. */
size_t cp_ef_u_bytes(int64_t n);
int cp_ef_prepare_u(const float* U, int64_t n, float* u_prepared, void* stream);

/* ef.py:179-218 ef_encode given the prepared factor of H[order][:, order] and the act-order
 * permutation `order` (int32 [n]): n_iter rounds of {commit grid with QUANTIZE(w_cur, qw);
 * ordered column sweep; repack}.  out: packed bytes as cp_kquant_encode.  first_fit_out
 * (optional, may be NULL) receives the first round's committed bytes, which equal
 * QUANTIZE(x, qw), encode_gguf's stock baseline (ef.py:298).
 * workspace >= cp_ef_workspace_bytes(type, nrow, n). */
size_t cp_ef_workspace_bytes(int ggml_type, int64_t nrow, int64_t n);
int cp_ef_encode(int ggml_type, const float* x, int64_t nrow, int64_t n, const int32_t* order,
                 const float* u_prepared, const float* qw, int n_iter, uint8_t* out, uint8_t* first_fit_out,
                 void* workspace, size_t workspace_bytes, void* stream);

/* One error-feedback pass (ef.py:197-216) against a committed grid (dl, ml from
 * cp_grid_params): codes int8 [nrow, n] in storage order; w_out (optional) receives the
 * compensated weights un-permuted (ef.py:215-216), the next round's fit input.
 * workspace >= cp_ef_sweep_workspace_bytes(nrow, n). */
size_t cp_ef_sweep_workspace_bytes(int64_t nrow, int64_t n);
int cp_ef_sweep(int ggml_type, const float* x, int64_t nrow, int64_t n, const int32_t* order,
                const float* u_prepared, const float* dl, const float* ml, int8_t* codes, float* w_out,
                void* workspace, size_t workspace_bytes, void* stream);

/* cp_ef_sweep for callers that cannot allocate device memory.  No counterpart in the
 * reference: it exists for hosts whose device memory is owned by another allocator (a
 * framework's caching allocator, a serving runtime that reserves the whole GPU up front) or
 * that reach this library through an FFI with no way to allocate or pass a scratch buffer.
 * The sweep's per-row errors go to a fixed array of CP_NOALLOC_SCRATCH_BYTES inside the
 * library, held on every GPU that loads it until the process exits; this call itself
 * allocates nothing.  Shapes with ceil(nrow/128)*128 * n * 4 > CP_NOALLOC_SCRATCH_BYTES are
 * rejected with CP_ERR_WORKSPACE.  The first call on a device looks the array's address up
 * (make that call before any stream capture) and keeps it for the life of the process, so
 * the call must not be used on a device after cudaDeviceReset (or any other teardown of its
 * primary context) in the same process.  All calls share the array: calls that overlap on
 * the GPU (other streams, other threads) race and must be serialised. */
#define CP_NOALLOC_SCRATCH_BYTES ((size_t)16 << 20)
int cp_ef_sweep_noalloc(int ggml_type, const float* x, int64_t nrow, int64_t n, const int32_t* order,
                        const float* u_prepared, const float* dl, const float* ml, int8_t* codes, float* w_out,
                        void* stream);

/* ---------------------------------------------------------------- grouped calls
 * The same operations over many tensors in as few launches as possible (one per ~256 jobs),
 * so a whole model fills the GPU even where single tensors are small.  Job arrays live in
 * host memory and may be discarded when the call returns. */

typedef struct {
  const float* x;   /* [nrow, n] */
  const float* qw;  /* [n] imatrix means, or NULL for the reference path */
  uint8_t* out;     /* [nrow, n/256 * cp_block_bytes(type)] */
  int64_t nrow, n;
} cp_fit_job;
/* kquant.py:732 QUANTIZE for every job (all of one k-quant type). */
int cp_kquant_encode_batch(int ggml_type, const cp_fit_job* jobs, int count, void* stream);

typedef struct {
  int ggml_type;
  const uint8_t* raw;   /* committed bytes (grid params, weighted error) */
  uint8_t* raw_out;     /* bytes to re-pack (repack) */
  const int8_t* codes;  /* [nrow, n] (repack) */
  const float* x;       /* [nrow, n] (weighted error) */
  const float* w;       /* [n] or NULL (weighted error) */
  float* dl;            /* grid params outputs, as cp_grid_params */
  float* ml;
  double* err;          /* weighted error: the call ADDS this tensor's sum to *err */
  int64_t nrow, n;
  int64_t grid_pitch;   /* grid params: 0 writes dl, ml as [nrow, n/sbw]; > 0 column-major,
                           element (row, sub-block s) at s * grid_pitch + row (the layout a
                           cp_sweep_job with pitch = grid_pitch reads) */
} cp_block_job;
int cp_grid_params_batch(const cp_block_job* jobs, int count, void* stream);   /* ef.py:87-127 */
int cp_kquant_repack_batch(const cp_block_job* jobs, int count, void* stream); /* ef.py:130-176; codes 16-byte aligned */
int cp_weighted_err_batch(const cp_block_job* jobs, int count, void* stream);  /* ef.py:298-301 */

typedef struct {
  int ggml_type;
  const float* x;
  int64_t nrow, n;
  const int32_t* order;
  const float* u_prepared;
  const float* dl;
  const float* ml;      /* NULL for Q3_K / Q6_K */
  int8_t* codes;
  float* w_out;         /* optional */
  void* workspace;      /* cp_ef_sweep_workspace_bytes(nrow, n) bytes, one per job */
  int64_t pitch;        /* 0: x, codes, w_out row-major [nrow, n] and dl, ml [nrow, n/sbw].
                           >= cp_ef_sweep_rows(nrow): all five column-major, element (row, col)
                           at col * pitch + row; the sweep's one-lane-per-row accesses then
                           coalesce (cp_transpose_batch converts) */
} cp_sweep_job;
/* ef.py:197-216 for every job in one launch (a CTA per 128 rows of any job). */
/* Rows a tensor's sweep CTAs cover: nrow rounded up to 128, the smallest column-major pitch. */
int64_t cp_ef_sweep_rows(int64_t nrow);

/* Grouped transposes (layout conversions around the column-major sweep): dst[c * dst_ld + r]
 * = src[r * src_ld + c] for r < rows, c < cols; elements of elem_bytes = 1 or 4. */
typedef struct {
  const void* src;
  void* dst;
  int64_t rows, cols, src_ld, dst_ld;
  int32_t elem_bytes;
} cp_transpose_job;
int cp_transpose_batch(const cp_transpose_job* jobs, int count, void* stream);

/* Copy `bytes` from pinned host memory (cudaHostAlloc / page-locked, hence mapped) to device
 * memory with a kernel that reads the host buffer over the bus.  Stream-ordered like
 * cudaMemcpyAsync, but it does not wait behind copy-engine transfers queued earlier on other
 * streams (the factorisation's act orders use it so that they are not held up by a bulk
 * weight upload).  CP_ERR_ARG if src_host is not pinned. */
int cp_fetch_host(void* dst, const void* src_host, int64_t bytes, void* stream);
int cp_ef_sweep_batch(const cp_sweep_job* jobs, int count, void* stream);

typedef struct {
  const double* H;       /* [n, n] */
  int64_t n;             /* multiple of 64 */
  const int32_t* order;  /* act-order permutation [n] */
  double diag_shift;     /* damp * mean(diag(H[order][:,order])) + 1e-8 */
  float* U_out;          /* [n, n] float32 upper factor */
  void* workspace;       /* cp_factor_workspace_bytes(n) bytes, one per job */
  int32_t* status_dev;   /* device int32: 0, or CP_ERR_NOT_PD */
} cp_factor_job;
/* ef.py:46-84 for every job: jobs of the same n advance through each factorisation step in
 * one launch (up to 64 per launch). */
int cp_factor_u_batch(const cp_factor_job* jobs, int count, void* stream);

/* Activation element types of cp_xtx_*. */
#define CP_XTX_BF16 0
#define CP_XTX_F32 1

/* Device workspace that cp_xtx_accumulate needs for x of `dtype` [T, d] on the current
 * device: a status word, one partial tile per work item (a 256 x 256 tile over a token
 * range) and, for float32 input, the hi/lo bf16 copies of x.  Zero-fill it once when it is
 * allocated. */
size_t cp_xtx_workspace_bytes(int dtype, int64_t T, int64_t d);

/* hessians.py:137-152 hook arithmetic (`x.float(); acc += x.T @ x`): H += x^T x for x
 * [T, d] row-major (bf16, or float32 split exactly into hi + lo bf16 with a 2^-17 relative
 * remainder), H float32 [d, d] row-major, d a multiple of 8, accumulated in float32 on the
 * tensor cores.  H stays exactly symmetric and repeated calls give identical bits.  One
 * workspace serves one stream at a time. */
int cp_xtx_accumulate(int dtype, const void* x, int64_t T, int64_t d, float* H, void* workspace,
                      size_t ws_bytes, void* stream);

/* Failure-path testing of the bounded waits (no counterpart in the reference): arms the
 * calling thread's NEXT cp_xtx_accumulate so that its loader issues no loads for the 64-token
 * step `skip_step` (of every tile) and every wait in that call gives up after wait_ns nanoseconds
 * (1 us .. 2 s).  The waits on the unfilled stage then run out, the kernel stops, drains the
 * loads it did issue, frees its tensor memory and sets the status word, so cp_xtx_status
 * returns CP_ERR_TIMEOUT and the device stays usable.  Nothing else changes; one call only. */
int cp_xtx_inject_stall(int skip_step, int64_t wait_ns);

/* Synchronises `stream`, reads and clears the workspace status word: CP_OK, or
 * CP_ERR_TIMEOUT when a wait inside an earlier cp_xtx_accumulate ran out (its H is then
 * incomplete). */
int cp_xtx_status(void* workspace, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* COLDPRESS_CUDA_H */
