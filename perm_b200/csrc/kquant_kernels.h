// Internal launcher declarations shared by the CUDA translation units and the C ABI.
#pragma once
#include <atomic>
#include <cstdint>
#include <cuda_runtime.h>

namespace cpk {
// Number of kernels this library has launched (all threads); read through cp_launch_count().
inline std::atomic<int64_t> g_launches{0};
inline void note_launch(int64_t k = 1) { g_launches.fetch_add(k, std::memory_order_relaxed); }

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
// (sub-block width, code lo, code hi, has-min) of a k-quant type; false for other types.
bool grid_spec(int type, int* sbw, int* lo, int* hi, bool* has_min);
}  // namespace cpk
