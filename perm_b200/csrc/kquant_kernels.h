// Internal launcher declarations shared by the CUDA translation units and the C ABI.
#pragma once
#include <atomic>
#include <cstdint>
#include <cuda_runtime.h>

namespace cpk {
// Number of kernels this library has launched (all threads); read through cp_launch_count().
inline std::atomic<int64_t> g_launches{0};
inline void note_launch(int64_t k = 1) { g_launches.fetch_add(k, std::memory_order_relaxed); }

// One tensor of a grouped fit launch: superblocks [0, nsb) of x, CTAs [cta0, cta0 + ctas).
struct FitDesc {
  const float* x;
  const float* qw;
  uint8_t* out;
  int64_t nsb, nsb_row, cta0;
};
constexpr int kFitBatchMax = 256;  // 48-byte descriptors: the table travels as a kernel parameter
struct FitBatch {
  int count;
  FitDesc d[kFitBatchMax];
};
int64_t quantize_batch_ctas(int type, int64_t nsb);
int launch_quantize_batch(int type, bool imat, const FitBatch& b, int64_t total_ctas, cudaStream_t stream);
int launch_quantize(int type, const float* x, int64_t nrow, int64_t n, const float* qw, uint8_t* out,
                    cudaStream_t stream);
int launch_dequantize(int type, const uint8_t* raw, int64_t nrow, int64_t n, float* out, cudaStream_t stream);
int launch_grid_params(int type, const uint8_t* raw, int64_t nrow, int64_t n, float* dl, float* ml,
                       cudaStream_t stream);
int launch_codes(int type, const uint8_t* raw, int64_t nrow, int64_t n, int8_t* codes, cudaStream_t stream);
int launch_repack(int type, uint8_t* raw, const int8_t* codes, int64_t nrow, int64_t n, cudaStream_t stream);
int launch_hessian_decode(const uint16_t* h16, const float* diag32, double hscale, int64_t d, double* H,
                          cudaStream_t stream);
int launch_weighted_err(int type, const uint8_t* raw, const float* x, const float* w, int64_t nrow, int64_t n,
                        double* out, cudaStream_t stream);
// One tensor of a grouped per-superblock launch (grid params, repack or weighted error).
struct SbDesc {
  const uint8_t* raw;   // committed bytes (read)
  uint8_t* raw_w;       // repack target
  const int8_t* codes;
  const float* x;
  const float* w;
  float* dl;
  float* ml;
  double* err;
  int64_t nsb, nsb_row, sb0;
  int64_t gpitch;       // grid output: 0 row-major [nrow][n/sbw], else column-major with this pitch
  int type;
};
constexpr int kSbBatchMax = 300;  // 104-byte descriptors in the kernel parameters (32 KB limit)
struct SbBatch {
  int count;
  SbDesc d[kSbBatchMax];
};
// op 0: grid params, 1: repack codes (one CTA per superblock), 2: weighted squared error
// added to *err (one CTA per 16 superblocks; sb0 counts CTAs)
int launch_sb_batch(int op, const SbBatch& b, int64_t total_sb, cudaStream_t stream);
// (sub-block width, code lo, code hi, has-min) of a k-quant type; false for other types.
bool grid_spec(int type, int* sbw, int* lo, int* hi, bool* has_min);
}  // namespace cpk
