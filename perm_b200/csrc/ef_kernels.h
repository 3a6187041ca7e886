// Internal launcher declarations for the error-feedback path (sweep, U layout, factorisation).
#pragma once
#include <atomic>
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace cpk {
// Streaming multiprocessors of the current device, looked up once per device index (148 on
// B200; 148 is also the answer when the lookup fails).  Safe to call from several threads.
inline int device_sm_count() {
  constexpr int kMaxDevices = 64;
  static std::atomic<int> cache[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  int v = cache[dev].load(std::memory_order_relaxed);
  if (v > 0) return v;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
  cache[dev].store(v, std::memory_order_relaxed);
  return v;
}
// Rows per sweep CTA = 32 * kSweepWarps.
constexpr int kSweepWarps = 4;
// One tensor of a grouped error-feedback sweep launch (CTAs [tile0, tile0 + sweep_ctas(nrow))).
struct SweepDesc {
  const float* x;
  const int* order;
  const float* u;     // prepared U: row-major float32 [n][n], then the diagonal
  const float* dl;
  const float* ml;    // null for types without a min
  float* work;        // errors, [32-row tile][n][32]
  int8_t* codes;
  float* wout;        // null in the last round
  int nrow, n, sbw, lo, hi, tile0;
  // 0: x, codes, wout row-major [nrow][n] and dl, ml [nrow][n/sbw].  > 0: all five
  // column-major with this many elements from one column to the next (rows contiguous, so the
  // sweep's lane-per-row accesses coalesce); pitch >= the rows the tensor's CTAs cover.
  int pitch;
};
constexpr int kSweepBatchMax = 320;  // 96-byte descriptors: the table travels as a kernel parameter
struct SweepBatch {
  int count;
  SweepDesc d[kSweepBatchMax];
};
bool sweep_desc(int type, const float* x, int64_t nrow, int64_t n, const int* order, const float* u_prep,
                const float* dl, const float* ml, void* work, int8_t* codes, float* wcur, SweepDesc* d);
// Rows a tensor's sweep CTAs cover (nrow rounded up to 32 * kSweepWarps): the smallest pitch.
int64_t sweep_rows_padded(int64_t nrow);
int sweep_ctas(int64_t nrow);
// CTAs of the column-split form with `split` (2 or 4) warps per 32 rows, each applying the
// errors to 1/split of every 64-column block: for launches too small to fill the GPU.
int sweep_split_ctas(int64_t nrow, int split);
// split: 1 for the ordinary form (sweep_ctas CTAs), 2 or 4 for the column-split form.
int launch_ef_sweep_batch(const SweepBatch& b, int total_ctas, int split, cudaStream_t stream);
// Sweep with its working rows in a fixed per-device array (no caller workspace).
constexpr size_t kNoAllocScratchBytes = (size_t)16 << 20;
int launch_ef_sweep_noalloc(int type, const float* x, int64_t nrow, int64_t n, const int* order, const float* u_prep,
                            const float* dl, const float* ml, int8_t* codes, float* wcur, cudaStream_t stream);
size_t ef_sweep_workspace_bytes(int64_t nrow, int64_t n);
size_t ef_u_prepared_bytes(int64_t n);
int launch_prepare_u(const float* U, int64_t n, float* out, cudaStream_t stream);
int launch_ef_sweep(int type, const float* x, int64_t nrow, int64_t n, const int* order, const float* u_prep,
                    const float* dl, const float* ml, void* work, int8_t* codes, float* wcur, cudaStream_t stream);
size_t factor_workspace_bytes(int64_t n);
// Same-size factorisations advanced step by step together (grid y / z index the item).
constexpr int kFactorBatchMax = 64;
struct FactorBatch {
  int count, n, out_f64;
  const double* H[kFactorBatchMax];
  const int* order[kFactorBatchMax];
  double* P[kFactorBatchMax];     // workspace of factor_workspace_bytes(n) each
  void* U[kFactorBatchMax];
  int* status[kFactorBatchMax];
  double shift[kFactorBatchMax];
};
int launch_factor_batch(const FactorBatch& fb, cudaStream_t stream);
int launch_factor_u(const double* H, int64_t n, const int* order, double shift, void* U, bool out_f64,
                    void* work, int* status, cudaStream_t stream);
}  // namespace cpk
