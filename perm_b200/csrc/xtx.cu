// H += X^T X for bf16 activations X [T, d] (coldpress/hessians.py:455-470 hook arithmetic).
// First version: CUDA-core float32 accumulation over lower 64x64 tiles, mirrored to the
// upper triangle.  Products of bf16 values are exact in float32, so this differs from the
// reference's float32 matmul only in summation order.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include "xtx_kernels.h"
#include "kquant_kernels.h"

namespace cpk {

__global__ void __launch_bounds__(256) xtx_simt_kernel(const __nv_bfloat16* __restrict__ X, int64_t T, int d,
                                                       float* __restrict__ H) {
  __shared__ float sa[32][64 + 4];
  __shared__ float sb[32][64 + 4];
  int idx = blockIdx.x, ti = 0;
  while (idx > ti) { idx -= ti + 1; ti++; }
  const int tj = idx;
  const int i0 = ti * 64, j0 = tj * 64;
  const int t = threadIdx.x, tr = t / 16, tc = t % 16;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < T; k0 += 32) {
    for (int e = t; e < 32 * 64; e += 256) {
      const int r = e / 64, c = e % 64;
      const bool ok = k0 + r < T;
      sa[r][c] = ok ? __bfloat162float(X[(k0 + r) * d + i0 + c]) : 0.0f;
      sb[r][c] = ok ? __bfloat162float(X[(k0 + r) * d + j0 + c]) : 0.0f;
    }
    __syncthreads();
#pragma unroll 8
    for (int r = 0; r < 32; r++) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; i++) a[i] = sa[r][tr + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; j++) b[j] = sb[r][tc + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int r = i0 + tr + 16 * i, c = j0 + tc + 16 * j;
      H[(size_t)r * d + c] += acc[i][j];
      if (ti != tj) H[(size_t)c * d + r] += acc[i][j];
    }
}

int launch_xtx(const uint16_t* x, int64_t T, int64_t d, float* H, cudaStream_t stream) {
  const int tiles = (int)(d / 64);
  xtx_simt_kernel<<<tiles * (tiles + 1) / 2, 256, 0, stream>>>((const __nv_bfloat16*)x, T, (int)d, H);
  note_launch();
  return 0;
}

}  // namespace cpk
