// Grouped transposes: layout conversions around the column-major EF sweep.  The sweep runs
// one lane per row, so it wants its per-element arrays (weights, codes, compensated weights)
// column-major: a warp's access to one column of 32 rows is then one contiguous segment
// instead of 32 row-strided sectors.  These kernels move tensors between the row-major
// storage order and that layout with 32 x 32 tiles staged in shared memory, so both the reads
// and the writes are coalesced.
#include <cuda_runtime.h>
#include <cstdint>
#include "layout_kernels.h"
#include "kquant_kernels.h"

namespace cpk {

// dst[c * dst_ld + r] = src[r * src_ld + c] over one 32 x 32 tile per CTA (256 threads).
template <typename E>
__global__ void __launch_bounds__(256) transpose_batch_kernel(const __grid_constant__ TrBatch b) {
  __shared__ E tile[32][33];
  int lo = 0, hi = b.count - 1;
  const int64_t cta = blockIdx.x;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (b.d[mid].tile0 <= cta) lo = mid;
    else hi = mid - 1;
  }
  const TrDesc& t = b.d[lo];
  const int64_t k = cta - t.tile0;
  const int64_t r0 = (k / t.tiles_c) * 32, c0 = (k % t.tiles_c) * 32;
  const E* __restrict__ src = static_cast<const E*>(t.src);
  E* __restrict__ dst = static_cast<E*>(t.dst);
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int64_t r = r0 + ty + 8 * i, c = c0 + tx;
    if (r < t.rows && c < t.cols) tile[ty + 8 * i][tx] = src[r * t.src_ld + c];
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int64_t c = c0 + ty + 8 * i, r = r0 + tx;
    if (r < t.rows && c < t.cols) dst[c * t.dst_ld + r] = tile[tx][ty + 8 * i];
  }
}

int64_t transpose_tiles(int64_t rows, int64_t cols) { return ((rows + 31) / 32) * ((cols + 31) / 32); }

int launch_transpose_batch(const TrBatch& b, int elem_bytes, int64_t total_tiles, cudaStream_t stream) {
  if (b.count == 0 || total_tiles == 0) return 0;
  if (total_tiles > INT32_MAX) return 2;
  if (elem_bytes == 4) transpose_batch_kernel<float><<<(unsigned)total_tiles, 256, 0, stream>>>(b);
  else if (elem_bytes == 1) transpose_batch_kernel<uint8_t><<<(unsigned)total_tiles, 256, 0, stream>>>(b);
  else return 2;
  note_launch();
  return 0;
}

}  // namespace cpk
