// FP64 factorization for error feedback: U = chol(inv(Hd)).T, the upper-triangular factor of
// coldpress/ef.py:46-84 (cholesky_inv_upper) cast to float32, computed on the GPU as
//     P  = J * Hd[order][:, order] * J          (act-order permutation, then reversal J)
//     P  = L L^T                                (blocked right-looking Cholesky, nb = 64)
//     U  = J * L^{-1} * J                       (blocked triangular inverse, then reversal)
// Because Hd = (J L J)(J L J)^T with J L J upper, (J L^{-1} J) is the unique upper factor
// with U^T U = inv(Hd): the same matrix as the reference's inv-then-cholesky route, in one
// Cholesky plus one triangular inverse.  Every step stays in float64 so the float32 cast
// matches the reference's cast.  A non-positive pivot sets a status word (no trap); the host
// then escalates the damping exactly like the reference does.
#include <cuda_runtime.h>
#include <cstdint>
#include "ef_kernels.h"
#include "kquant_kernels.h"

namespace cpk {

constexpr int NB = 64;

// P[i][j] = H[order[n-1-i]][order[n-1-j]] (+ shift on the diagonal).  Only the lower
// triangle is consumed; the strict upper triangle is written as zero.
__global__ void permute_reverse_kernel(const double* __restrict__ H, int n, const int* __restrict__ order,
                                       double shift, double* __restrict__ P) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x, i = blockIdx.y;
  if (j >= n) return;
  double v = 0.0;
  if (j <= i) {
    v = H[(size_t)order[n - 1 - i] * n + order[n - 1 - j]];
    if (i == j) v += shift;
  }
  P[(size_t)i * n + j] = v;
}

// Diagonal block at (k, k): Cholesky factor L11 of the (already updated) block, then its
// inverse, written in place of the block.  One warp; lane l owns rows l and l + 32 and the
// block lives in shared memory.  Nothing after this step needs L11 itself: the panel below is
// solved with inv(L11) and the diagonal blocks of L^-1 are exactly these inverses.
// A non-positive (or NaN) pivot sets *status and leaves the rest of the factorisation idle.
__global__ void __launch_bounds__(32) potrf_inv_diag_kernel(double* __restrict__ A, int n, int k,
                                                            int* __restrict__ status) {
  __shared__ double a[NB][NB + 1];
  const int l = threadIdx.x;
  if (*status) return;
  for (int i = l; i < NB * NB; i += 32) {
    const int r = i / NB, c = i % NB;
    a[r][c] = (c <= r) ? A[(size_t)(k + r) * n + k + c] : 0.0;
  }
  __syncwarp();
  const int rows[2] = {l, l + 32};
  for (int j = 0; j < NB; j++) {
    const double d = a[j][j];
    if (!(d > 0.0)) {  // uniform: every lane read the same pivot
      if (l == 0) *status = 1;
      return;
    }
    const double s = sqrt(d);
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 2; q++) {
      const int r = rows[q];
      if (r == j) a[r][j] = s;
      else if (r > j) a[r][j] /= s;
    }
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 2; q++) {
      const int r = rows[q];
      if (r > j) {
        const double v = a[r][j];
        for (int c = j + 1; c <= r; c++) a[r][c] = fma(-v, a[c][j], a[r][c]);
      }
    }
    __syncwarp();
  }
  // in-place inverse of the lower-triangular block, columns right to left (LAPACK dtrti2)
  for (int j = NB - 1; j >= 0; j--) {
    const double inv_jj = 1.0 / a[j][j];
    double acc[2] = {0.0, 0.0};
#pragma unroll
    for (int q = 0; q < 2; q++) {
      const int i = rows[q];
      if (i > j) {
        double t = 0.0;
        for (int kk = j + 1; kk <= i; kk++) t = fma(a[i][kk], a[kk][j], t);
        acc[q] = t;
      }
    }
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 2; q++) {
      const int i = rows[q];
      if (i > j) a[i][j] = -inv_jj * acc[q];
      else if (i == j) a[i][j] = inv_jj;
    }
    __syncwarp();
  }
  for (int i = l; i < NB * NB; i += 32) {
    const int r = i / NB, c = i % NB;
    A[(size_t)(k + r) * n + k + c] = (c <= r) ? a[r][c] : 0.0;
  }
}

// Tile GEMM: C[64x64 tile] = alpha * sum_l A[i][l] * Bop[l][j] (+ beta * C), FP64 on CUDA
// cores, 256 threads with a 4x4 register tile each, K streamed in chunks of 16 through
// shared memory.  B_TRANS: Bop[l][j] = B[j][l] (A*B^T), else Bop[l][j] = B[l][j].
template <bool B_TRANS>
__device__ __forceinline__ void tile_gemm(const double* __restrict__ A, int lda, const double* __restrict__ B,
                                          int ldb, int m_lim, int n_lim, int k_len, double (&acc)[4][4]) {
  __shared__ double sa[16][64 + 1];
  __shared__ double sb[16][64 + 1];
  const int t = threadIdx.x, tr = t / 16, tc = t % 16;
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) acc[i][j] = 0.0;
  for (int l0 = 0; l0 < k_len; l0 += 16) {
    for (int i = t; i < 16 * 64; i += 256) {
      const int r = i / 16, l = i % 16;  // A row r, column l0+l
      sa[l][r] = (r < m_lim && l0 + l < k_len) ? A[(size_t)r * lda + l0 + l] : 0.0;
    }
    if (B_TRANS) {
      for (int i = t; i < 16 * 64; i += 256) {
        const int c = i / 16, l = i % 16;
        sb[l][c] = (c < n_lim && l0 + l < k_len) ? B[(size_t)c * ldb + l0 + l] : 0.0;
      }
    } else {
      for (int i = t; i < 16 * 64; i += 256) {
        const int l = i / 64, c = i % 64;
        sb[l][c] = (c < n_lim && l0 + l < k_len) ? B[(size_t)(l0 + l) * ldb + c] : 0.0;
      }
    }
    __syncthreads();
#pragma unroll
    for (int l = 0; l < 16; l++) {
      double av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; i++) av[i] = sa[l][tr + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; j++) bv[j] = sb[l][tc + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = fma(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
}

// Panel below the diagonal block: A21 := A21 * inv(L11)^T, inv(L11) read from the diagonal.
__global__ void __launch_bounds__(256) trsm_panel_kernel(double* __restrict__ A, int n, int k, const int* status) {
  if (*status) return;
  const int r0 = k + NB + blockIdx.x * 64;
  const int m = min(64, n - r0);
  const int nb = min(NB, n - k);
  double acc[4][4];
  // out[r][c] = sum_l A21[r][l] * inv(L11)[c][l]
  tile_gemm<true>(A + (size_t)r0 * n + k, n, A + (size_t)k * n + k, n, m, nb, nb, acc);
  const int t = threadIdx.x, tr = t / 16, tc = t % 16;
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int r = tr + 16 * i, c = tc + 16 * j;
      if (r < m && c < nb) A[(size_t)(r0 + r) * n + k + c] = acc[i][j];
    }
}

// Trailing update A22 -= A21 A21^T on lower 64x64 tiles.
__global__ void __launch_bounds__(256) syrk_kernel(double* __restrict__ A, int n, int k, const int* status) {
  if (*status) return;
  // blockIdx.x enumerates lower tiles (ti >= tj) of the trailing matrix
  int idx = blockIdx.x, ti = 0;
  while (idx > ti) { idx -= ti + 1; ti++; }
  const int tj = idx;
  const int base = k + NB;
  const int r0 = base + ti * 64, c0 = base + tj * 64;
  const int m = min(64, n - r0), nn = min(64, n - c0);
  double acc[4][4];
  tile_gemm<true>(A + (size_t)r0 * n + k, n, A + (size_t)c0 * n + k, n, m, nn, NB, acc);
  const int t = threadIdx.x, tr = t / 16, tc = t % 16;
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int r = tr + 16 * i, c = tc + 16 * j;
      if (r < m && c < nn && r0 + r >= c0 + c) A[(size_t)(r0 + r) * n + c0 + c] -= acc[i][j];
    }
}

// Triangular inverse, step for diagonal block j (blocks to its lower right already inverted):
//   T   = -Linv22 * L21          (rows below, into scratch)
__global__ void __launch_bounds__(256) trmm_kernel(const double* __restrict__ A, int n, int j,
                                                   double* __restrict__ T, const int* status) {
  if (*status) return;
  const int base = j + NB;
  const int r0 = base + blockIdx.x * 64;
  const int m = min(64, n - r0);
  // rows r0.. of Linv22 have nonzeros only in columns base .. r0+m-1
  const int k_len = r0 + m - base;
  double acc[4][4];
  tile_gemm<false>(A + (size_t)r0 * n + base, n, A + (size_t)base * n + j, n, m, NB, k_len, acc);
  const int t = threadIdx.x, tr = t / 16, tc = t % 16;
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const int r = tr + 16 * i, cc = tc + 16 * c;
      if (r < m) T[(size_t)(r0 - base + r) * NB + cc] = -acc[i][c];
    }
}

//   L21 := T * inv(L11)   (inv(L11) already sits on the diagonal)
__global__ void __launch_bounds__(256) trinv_apply_kernel(double* __restrict__ A, int n, int j,
                                                          const double* __restrict__ T, const int* status) {
  if (*status) return;
  const int base = j + NB;
  const int r0 = base + blockIdx.x * 64;
  const int m = min(64, n - r0);
  double acc[4][4];
  tile_gemm<false>(T + (size_t)(r0 - base) * NB, NB, A + (size_t)j * n + j, n, m, NB, NB, acc);
  const int t = threadIdx.x, tr = t / 16, tc = t % 16;
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const int r = tr + 16 * i, cc = tc + 16 * c;
      if (r < m) A[(size_t)(r0 + r) * n + j + cc] = acc[i][c];
    }
}

// U[i][j] = Linv[n-1-i][n-1-j] for j >= i, else 0 (cast to OutT).
template <typename OutT>
__global__ void unreverse_cast_kernel(const double* __restrict__ Linv, int n, OutT* __restrict__ U) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x, i = blockIdx.y;
  if (j >= n) return;
  U[(size_t)i * n + j] = (j >= i) ? (OutT)Linv[(size_t)(n - 1 - i) * n + (n - 1 - j)] : (OutT)0;
}

size_t factor_workspace_bytes(int64_t n) {
  // P (n x n f64) + T (n x nb)
  return ((size_t)n * n + (size_t)n * NB) * sizeof(double);
}

int launch_factor_u(const double* H, int64_t n64, const int* order, double shift, void* U, bool out_f64,
                    void* work, int* status, cudaStream_t stream) {
  if (n64 <= 0 || n64 % NB) return 2;
  const int n = (int)n64;
  double* P = (double*)work;
  double* T = P + (size_t)n * n;
  cudaMemsetAsync(status, 0, sizeof(int), stream);
  {
    dim3 g((unsigned)((n + 255) / 256), (unsigned)n);
    permute_reverse_kernel<<<g, 256, 0, stream>>>(H, n, order, shift, P);
    note_launch();
  }
  for (int k = 0; k < n; k += NB) {
    potrf_inv_diag_kernel<<<1, 32, 0, stream>>>(P, n, k, status);
    note_launch();
    const int rem = n - k - NB;
    if (rem > 0) {
      const int tiles = (rem + 63) / 64;
      trsm_panel_kernel<<<tiles, 256, 0, stream>>>(P, n, k, status);
      note_launch();
      syrk_kernel<<<tiles * (tiles + 1) / 2, 256, 0, stream>>>(P, n, k, status);
      note_launch();
    }
  }
  // blocked inverse of L, bottom-right to top-left (LAPACK dtrtri, lower); the diagonal
  // blocks were inverted by the factorisation
  for (int j = n - 2 * NB; j >= 0; j -= NB) {
    const int rem = n - j - NB;
    const int tiles = (rem + 63) / 64;
    trmm_kernel<<<tiles, 256, 0, stream>>>(P, n, j, T, status);
    note_launch();
    trinv_apply_kernel<<<tiles, 256, 0, stream>>>(P, n, j, T, status);
    note_launch();
  }
  {
    dim3 g((unsigned)((n + 255) / 256), (unsigned)n);
    if (out_f64) unreverse_cast_kernel<double><<<g, 256, 0, stream>>>(P, n, (double*)U);
    else unreverse_cast_kernel<float><<<g, 256, 0, stream>>>(P, n, (float*)U);
    note_launch();
  }
  return 0;
}

}  // namespace cpk
