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
}  // namespace cpk
