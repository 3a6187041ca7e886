// Internal launcher declarations for the grouped transposes.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace cpk {
// One transpose of a grouped launch: dst[c * dst_ld + r] = src[r * src_ld + c], CTAs
// [tile0, tile0 + transpose_tiles(rows, cols, elem_bytes)) over square tiles of
// transpose_tile_dim(elem_bytes) (tiles_c tiles per row of tiles).
struct TrDesc {
  const void* src;
  void* dst;
  int64_t rows, cols, src_ld, dst_ld, tile0, tiles_c;
};
constexpr int kTrBatchMax = 256;   // 64-byte descriptors in the kernel parameters
struct TrBatch {
  int count;
  TrDesc d[kTrBatchMax];
};
int transpose_tile_dim(int elem_bytes);
int64_t transpose_tiles(int64_t rows, int64_t cols, int elem_bytes);
int launch_transpose_batch(const TrBatch& b, int elem_bytes, int64_t total_tiles, cudaStream_t stream);
// bytes from mapped (pinned) host memory to device memory, read by a kernel
int launch_fetch_host(void* dst, const void* src_mapped, int64_t bytes, cudaStream_t stream);
// out [nrow_out, n_out] = src[row(i) * ld + col(j)] (int64 index lists, NULL = identity)
int launch_gather_f32(const float* src, int64_t ld, const int64_t* rows, int64_t nrow_out, const int64_t* cols,
                      int64_t n_out, float* out, cudaStream_t stream);
// acc[c] = sum_r (x[r * ld + c] - y[r * ld + c])^2, y NULL meaning 0 (float64, fixed order)
int launch_col_sqdiff(const float* x, const float* y, int64_t nrow, int64_t n, int64_t ld, double* acc,
                      cudaStream_t stream);
}  // namespace cpk
