// Grouped transposes: layout conversions around the column-major EF sweep.  The sweep runs
// one lane per row, so it wants its per-element arrays (weights, codes, compensated weights)
// column-major: a warp's access to one column of 32 rows is then one contiguous segment
// instead of 32 row-strided sectors.  These kernels move tensors between the row-major
// storage order and that layout with tiles staged in shared memory (64 x 64 floats, 128 x 128
// bytes), so both the reads and the writes are coalesced.
#include <cuda_runtime.h>
#include <cstdint>
#include "layout_kernels.h"
#include "kquant_kernels.h"

namespace cpk {

__device__ __forceinline__ const TrDesc& tr_desc(const TrBatch& b, int64_t cta) {
  int lo = 0, hi = b.count - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (b.d[mid].tile0 <= cta) lo = mid;
    else hi = mid - 1;
  }
  return b.d[lo];
}

// float32: dst[c * dst_ld + r] = src[r * src_ld + c] over one 64 x 64 tile per CTA (256
// threads, 16 elements each); warps read and write 128-byte row segments.
__global__ void __launch_bounds__(256) transpose_f32_kernel(const __grid_constant__ TrBatch b) {
  __shared__ float tile[64][65];
  const int64_t cta = blockIdx.x;
  const TrDesc& t = tr_desc(b, cta);
  const int64_t k = cta - t.tile0;
  const int64_t r0 = (k / t.tiles_c) * 64, c0 = (k % t.tiles_c) * 64;
  const float* __restrict__ src = static_cast<const float*>(t.src);
  float* __restrict__ dst = static_cast<float*>(t.dst);
  const int tx = threadIdx.x & 63, ty = threadIdx.x >> 6;
  float v[16];
#pragma unroll
  for (int i = 0; i < 16; i++) {
    const int64_t r = r0 + ty + 4 * i, c = c0 + tx;
    v[i] = (r < t.rows && c < t.cols) ? src[r * t.src_ld + c] : 0.0f;
  }
#pragma unroll
  for (int i = 0; i < 16; i++) tile[ty + 4 * i][tx] = v[i];
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 16; i++) {
    const int64_t c = c0 + ty + 4 * i, r = r0 + tx;
    if (r < t.rows && c < t.cols) dst[c * t.dst_ld + r] = tile[tx][ty + 4 * i];
  }
}

// bytes: one 128 x 128 tile per CTA; full tiles move 4-byte words both ways (a warp reads or
// writes one 128-byte row segment), edge tiles go byte by byte.
__global__ void __launch_bounds__(256) transpose_u8_kernel(const __grid_constant__ TrBatch b) {
  __shared__ uint8_t tile[128][132];
  const int64_t cta = blockIdx.x;
  const TrDesc& t = tr_desc(b, cta);
  const int64_t k = cta - t.tile0;
  const int64_t r0 = (k / t.tiles_c) * 128, c0 = (k % t.tiles_c) * 128;
  const uint8_t* __restrict__ src = static_cast<const uint8_t*>(t.src);
  uint8_t* __restrict__ dst = static_cast<uint8_t*>(t.dst);
  const int tid = threadIdx.x;
  const bool full = r0 + 128 <= t.rows && c0 + 128 <= t.cols && ((t.src_ld | t.dst_ld) & 3) == 0 &&
                    ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 3) == 0;
  if (full) {
#pragma unroll 4
    for (int w = tid; w < 128 * 32; w += 256) {
      const int r = w >> 5, wc = w & 31;
      const uint32_t v = *reinterpret_cast<const uint32_t*>(src + (r0 + r) * t.src_ld + c0 + 4 * wc);
      *reinterpret_cast<uint32_t*>(&tile[r][4 * wc]) = v;
    }
    __syncthreads();
#pragma unroll 4
    for (int w = tid; w < 128 * 32; w += 256) {
      const int c = w >> 5, wr = w & 31;
      const uint32_t v = (uint32_t)tile[4 * wr][c] | ((uint32_t)tile[4 * wr + 1][c] << 8) |
                         ((uint32_t)tile[4 * wr + 2][c] << 16) | ((uint32_t)tile[4 * wr + 3][c] << 24);
      *reinterpret_cast<uint32_t*>(dst + (c0 + c) * t.dst_ld + r0 + 4 * wr) = v;
    }
  } else {
    for (int e = tid; e < 128 * 128; e += 256) {
      const int r = e >> 7, c = e & 127;
      if (r0 + r < t.rows && c0 + c < t.cols) tile[r][c] = src[(r0 + r) * t.src_ld + c0 + c];
    }
    __syncthreads();
    for (int e = tid; e < 128 * 128; e += 256) {
      const int c = e >> 7, r = e & 127;
      if (r0 + r < t.rows && c0 + c < t.cols) dst[(c0 + c) * t.dst_ld + r0 + r] = tile[r][c];
    }
  }
}

// Copy from pinned host memory read directly by the kernel over the bus (mapped memory):
// unlike a copy-engine transfer, it does not queue behind large transfers issued earlier on
// other streams.  16-byte words when both ends are aligned, bytes otherwise.
__global__ void __launch_bounds__(256) fetch_host_kernel(void* __restrict__ dst, const void* __restrict__ src,
                                                         int64_t bytes) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool vec = ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) == 0;
  int64_t done = 0;
  if (vec) {
    const int64_t n16 = bytes >> 4;
    const uint4* s4 = static_cast<const uint4*>(src);
    uint4* d4 = static_cast<uint4*>(dst);
    for (int64_t i = t0; i < n16; i += stride) d4[i] = s4[i];
    done = n16 << 4;
  }
  const uint8_t* s1 = static_cast<const uint8_t*>(src);
  uint8_t* d1 = static_cast<uint8_t*>(dst);
  for (int64_t i = done + t0; i < bytes; i += stride) d1[i] = s1[i];
}

int launch_fetch_host(void* dst, const void* src_mapped, int64_t bytes, cudaStream_t stream) {
  if (bytes <= 0) return 0;
  int64_t blocks = ((bytes >> 4) + 255) / 256;
  if (blocks < 1) blocks = 1;
  if (blocks > 1184) blocks = 1184;
  fetch_host_kernel<<<(unsigned)blocks, 256, 0, stream>>>(dst, src_mapped, bytes);
  note_launch();
  return 0;
}

int transpose_tile_dim(int elem_bytes) { return elem_bytes == 1 ? 128 : 64; }

int64_t transpose_tiles(int64_t rows, int64_t cols, int elem_bytes) {
  const int T = transpose_tile_dim(elem_bytes);
  return ((rows + T - 1) / T) * ((cols + T - 1) / T);
}

int launch_transpose_batch(const TrBatch& b, int elem_bytes, int64_t total_tiles, cudaStream_t stream) {
  if (b.count == 0 || total_tiles == 0) return 0;
  if (total_tiles > INT32_MAX) return 2;
  if (elem_bytes == 4) transpose_f32_kernel<<<(unsigned)total_tiles, 256, 0, stream>>>(b);
  else if (elem_bytes == 1) transpose_u8_kernel<<<(unsigned)total_tiles, 256, 0, stream>>>(b);
  else return 2;
  note_launch();
  return 0;
}

// out[i * n_out + j] = src[row(i) * ld + col(j)] with row(i) = rows ? rows[i] : i and col(j)
// likewise: the row sample and column permutation of the PERM objective in one pass.  Each
// thread writes 4 consecutive outputs of one row (coalesced stores; the reads follow the
// permutation within a row that stays in L1/L2).  Rows stride over gridDim.y.
__global__ void __launch_bounds__(256) gather_f32_kernel(const float* __restrict__ src, int64_t ld,
                                                         const int64_t* __restrict__ rows, int64_t nrow_out,
                                                         const int64_t* __restrict__ cols, int64_t n_out,
                                                         float* __restrict__ out) {
  const int64_t j0 = ((int64_t)blockIdx.x * 256 + threadIdx.x) * 4;
  if (j0 >= n_out) return;
  int64_t c[4];
#pragma unroll
  for (int u = 0; u < 4; u++) c[u] = (j0 + u < n_out) ? (cols ? cols[j0 + u] : j0 + u) : 0;
  for (int64_t i = blockIdx.y; i < nrow_out; i += gridDim.y) {
    const float* __restrict__ s = src + (rows ? rows[i] : i) * ld;
    float* __restrict__ o = out + i * n_out;
#pragma unroll
    for (int u = 0; u < 4; u++)
      if (j0 + u < n_out) o[j0 + u] = s[c[u]];
  }
}

// acc[c] = sum over rows of (x[r * ld + c] - y[r * ld + c])^2 in float64 (y == NULL: x^2).  A
// CTA owns 32 columns: warp w sums rows w, w + 8, ... (lane = column, so each row read is one
// 128-byte segment) in two alternating accumulators, then the eight warp partials are added
// in warp order, so the result does not depend on scheduling.
__global__ void __launch_bounds__(256) col_sqdiff_kernel(const float* __restrict__ x, const float* __restrict__ y,
                                                         int64_t nrow, int64_t n, int64_t ld,
                                                         double* __restrict__ acc) {
  __shared__ double part[8][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t c = (int64_t)blockIdx.x * 32 + lane;
  double s0 = 0.0, s1 = 0.0;
  if (c < n) {
    int64_t r = warp;
    for (; r + 8 < nrow; r += 16) {
      double a = x[r * ld + c], b = x[(r + 8) * ld + c];
      if (y) {
        a -= (double)y[r * ld + c];
        b -= (double)y[(r + 8) * ld + c];
      }
      s0 += a * a;
      s1 += b * b;
    }
    if (r < nrow) {
      double a = x[r * ld + c];
      if (y) a -= (double)y[r * ld + c];
      s0 += a * a;
    }
  }
  part[warp][lane] = s0 + s1;
  __syncthreads();
  if (warp == 0 && c < n) {
    double t = 0.0;
#pragma unroll
    for (int w = 0; w < 8; w++) t += part[w][lane];
    acc[c] = t;
  }
}

int launch_gather_f32(const float* src, int64_t ld, const int64_t* rows, int64_t nrow_out, const int64_t* cols,
                      int64_t n_out, float* out, cudaStream_t stream) {
  if (nrow_out <= 0 || n_out <= 0) return 0;
  const int64_t bx = (n_out + 1023) / 1024;
  if (bx > INT32_MAX) return 2;
  const int64_t by = nrow_out < 8192 ? nrow_out : 8192;
  gather_f32_kernel<<<dim3((unsigned)bx, (unsigned)by), 256, 0, stream>>>(src, ld, rows, nrow_out, cols, n_out, out);
  note_launch();
  return 0;
}

int launch_col_sqdiff(const float* x, const float* y, int64_t nrow, int64_t n, int64_t ld, double* acc,
                      cudaStream_t stream) {
  if (n <= 0) return 0;
  const int64_t bx = (n + 31) / 32;
  if (bx > INT32_MAX) return 2;
  col_sqdiff_kernel<<<(unsigned)bx, 256, 0, stream>>>(x, y, nrow, n, ld, acc);
  note_launch();
  return 0;
}

}  // namespace cpk
