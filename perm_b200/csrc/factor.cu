// FP64 factorization for error feedback: U = chol(inv(Hd)).T, the upper-triangular factor of
// coldpress/ef.py:46-84 (cholesky_inv_upper) cast to float32, computed on the GPU as
//     P  = J * Hd[order][:, order] * J          (act-order permutation, then reversal J)
//     P  = L L^T                                (blocked left-looking Cholesky, nb = 64)
//     U  = J * L^{-1} * J                       (row-blocked triangular inverse, reversed)
// The inverse runs as a second chain on a helper stream, one block row behind the
// Cholesky: block row j of L^{-1} needs only block row j of L, the diagonal inverses and the
// earlier rows of L^{-1}, so the two dependent chains overlap instead of following each other.
// Because Hd = (J L J)(J L J)^T with J L J upper, (J L^{-1} J) is the unique upper factor
// with U^T U = inv(Hd): the same matrix as the reference's inv-then-cholesky route, in one
// Cholesky plus one triangular inverse.  Every step stays in float64 so the float32 cast
// matches the reference's cast.  A non-positive pivot sets a status word (no trap); the host
// then escalates the damping exactly like the reference does.
#include <cuda_runtime.h>
#include <cstdint>
#include <map>
#include <utility>
#include "ef_kernels.h"
#include "kquant_kernels.h"

namespace cpk {

constexpr int NB = 64;
constexpr int kSplitMax = 16;

// K splitting of the long products: chunks of about 256 (a multiple of 16), at most 16.
__host__ __device__ inline int ksplit(int K) {
  if (K <= 384) return 1;
  const int s = (K + 255) / 256;
  return s > kSplitMax ? kSplitMax : s;
}
__host__ __device__ inline int kchunk(int K, int S) { return ((K + S - 1) / S + 15) / 16 * 16; }

// Split count of one batched launch: split K only while the tiles of all items leave the
// GPU short of one wave (3 resident 128-thread tile CTAs per SM), then as little as fills it.
// Every extra split costs a partial-tile write and a reduction pass.
static int ksplit_batch(int K, int tiles, int count) {
  const int sms = device_sm_count();
  const int smax = ksplit(K);
  const long long base = (long long)tiles * count, slots = 3LL * sms;
  if (smax <= 1 || base >= slots) return 1;
  const int s = (int)((slots + base - 1) / base);
  return s < smax ? s : smax;
}
// Workspace of one item: P (n x n), T (n x 64: a 64 x 64 scratch tile per block column),
// D (n x 64: the transposed inverse of each 64 x 64 diagonal block of L), then the split-K
// partial tiles (kSplitMax x n x 64).
__device__ __forceinline__ double* t_base(double* P, int n) { return P + (size_t)n * n; }
__device__ __forceinline__ double* d_base(double* P, int n) { return P + (size_t)n * n + (size_t)n * NB; }
__device__ __forceinline__ double* part_base(double* P, int n) { return P + (size_t)n * n + 2 * (size_t)n * NB; }

// P[i][j] = H[order[n-1-i]][order[n-1-j]] (+ shift on the diagonal).  Only the lower
// triangle is consumed; the strict upper triangle is written as zero.  blockIdx.z: item.
__global__ void permute_reverse_kernel(const __grid_constant__ FactorBatch fb) {
  const int n = fb.n;
  const int j = blockIdx.x * blockDim.x + threadIdx.x, i = blockIdx.y, b = blockIdx.z;
  if (j >= n) return;
  const int* order = fb.order[b];
  double v = 0.0;
  if (j <= i) {
    v = fb.H[b][(size_t)order[n - 1 - i] * n + order[n - 1 - j]];
    if (i == j) v += fb.shift[b];
  }
  fb.P[b][(size_t)i * n + j] = v;
}

// Row-staged form of permute_reverse_kernel: the CTA reads its source row of H once, with
// coalesced loads, into shared memory and gathers the permuted columns from there (the direct
// form's scattered 8-byte reads move four times the bytes through L2).  blockIdx.x: row i of
// P, blockIdx.y: item.  Used while a row (n doubles) fits in shared memory.
constexpr int kPermRowSmemMax = 227 * 1024;
__global__ void __launch_bounds__(256) permute_reverse_rows_kernel(const __grid_constant__ FactorBatch fb) {
  extern __shared__ double hrow[];
  const int n = fb.n, i = blockIdx.x, b = blockIdx.y;
  const int* __restrict__ order = fb.order[b];
  const double* __restrict__ src = fb.H[b] + (size_t)order[n - 1 - i] * n;
  for (int c = threadIdx.x; c < n; c += 256) hrow[c] = src[c];
  __syncthreads();
  double* __restrict__ dst = fb.P[b] + (size_t)i * n;
  const double sh = fb.shift[b];
  for (int j = threadIdx.x; j < n; j += 256) {
    double v = 0.0;
    if (j <= i) {
      v = hrow[order[n - 1 - j]];
      if (i == j) v += sh;
    }
    dst[j] = v;
  }
}

// Diagonal block at (k, k): Cholesky factor L11 of the (already updated) 64 x 64 block, then
// its inverse, written in place of the block.  Nothing after this step needs L11 itself: the
// panel below is solved with inv(L11) and the diagonal blocks of L^-1 are exactly these
// inverses.  256 threads, blocked by 16:
//   for each 16-column panel p: warp 0 factors the 16 x 16 diagonal block column by column
//   (warp-synchronous; sqrt and rsqrt of the pivot side by side, no divisions) and inverts
//   it (lane j forms column j); then all threads solve the rows below with that inverse
//   (X = A * inv(Lpp)^T) and update the trailing triangle (A22 -= X X^T);
//   inv(L11) block by block: X_ii = inv(L_ii), then for the block diagonals d = 1, 2, 3
//   X_ij = -X_ii * sum_{k=j}^{i-1} L_ik X_kj (i = j + d).
// About 30 block barriers instead of two per column.  A non-positive (or NaN) pivot sets
// *status and leaves the rest of the factorisation idle.
constexpr int kPotrfSmemBytes = (2 * 64 * 65 + 64) * (int)sizeof(double);
__global__ void __launch_bounds__(256) potrf_inv_diag_kernel(const __grid_constant__ FactorBatch fb, int k) {
  extern __shared__ __align__(16) double psm[];
  double(*a)[65] = reinterpret_cast<double(*)[65]>(psm);            // the block, then L
  double(*x)[65] = reinterpret_cast<double(*)[65]>(psm + 64 * 65);  // inv(L), lower
  double* isq = psm + 2 * 64 * 65;                                   // 1 / L[c][c]
  __shared__ int bad;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int n = fb.n;
  double* __restrict__ A = fb.P[blockIdx.x];
  int* status = fb.status[blockIdx.x];
  if (*status) return;
  if (t == 0) bad = 0;
  for (int i = t; i < 64 * 64; i += 256) {
    const int r = i >> 6, c = i & 63;
    a[r][c] = (c <= r) ? A[(size_t)(k + r) * n + k + c] : 0.0;
  }
  __syncthreads();
  for (int p = 0; p < 4; p++) {
    const int c0 = 16 * p;
    if (warp == 0) {
      // the 16 x 16 diagonal block in registers: lane r (and r + 16) holds row r; the pivot and
      // column c's values come by shuffle, so a column step has no shared-memory round trip
      const int r = lane & 15;
      double lr[16];
#pragma unroll
      for (int k = 0; k < 16; k++) lr[k] = a[c0 + r][c0 + k];  // zero above the diagonal
      bool okp = true;
#pragma unroll
      for (int c = 0; c < 16; c++) {
        const double d = __shfl_sync(0xffffffffu, lr[c], c);
        okp = okp && (d > 0.0);  // uniform: every lane got the same pivot
        if (!okp) continue;      // (no break: the loop must unroll to keep lr in registers)
        const double sq = sqrt(d), is = rsqrt(d);
        if (r == c) {
          lr[c] = sq;
          if (lane == c) isq[c0 + c] = is;
        } else if (r > c) {
          lr[c] *= is;
        }
#pragma unroll
        for (int k = c + 1; k < 16; k++) {
          const double lkc = __shfl_sync(0xffffffffu, lr[c], k);
          if (r >= k) lr[k] = fma(-lr[c], lkc, lr[k]);
        }
      }
      if (!okp) {
        if (lane == 0) bad = 1;
      } else if (lane < 16) {
#pragma unroll
        for (int k = 0; k < 16; k++) a[c0 + r][c0 + k] = lr[k];
      }
      __syncwarp();  // the factor and lane 0's bad flag
      if (!bad && lane < 16) {  // inverse of the 16 x 16 factor into x's diagonal block
        const int j = lane;
        double col[16];
#pragma unroll
        for (int i = 0; i < 16; i++) {
          double s = 0.0;
#pragma unroll
          for (int kk = 0; kk < i; kk++) s = fma(a[c0 + i][c0 + kk], col[kk], s);
          col[i] = (i < j) ? 0.0 : (i == j ? isq[c0 + i] : -isq[c0 + i] * s);
        }
#pragma unroll
        for (int i = 0; i < 16; i++) x[c0 + i][c0 + j] = col[i];
      }
    }
    __syncthreads();
    if (bad) {
      if (t == 0) *status = 1;
      return;
    }
    const int m = 48 - c0;  // rows below the panel
    if (m == 0) break;
    {  // X = A[rows][panel] * inv(Lpp)^T, at most 3 elements a thread
      double v[3];
#pragma unroll
      for (int u = 0; u < 3; u++) {
        const int e = t + 256 * u;
        v[u] = 0.0;
        if (e < m * 16) {
          const int r = c0 + 16 + (e >> 4), c = e & 15;
          double s = 0.0;
          for (int kk = 0; kk <= c; kk++) s = fma(a[r][c0 + kk], x[c0 + c][c0 + kk], s);
          v[u] = s;
        }
      }
      __syncthreads();
#pragma unroll
      for (int u = 0; u < 3; u++) {
        const int e = t + 256 * u;
        if (e < m * 16) a[c0 + 16 + (e >> 4)][c0 + (e & 15)] = v[u];
      }
    }
    __syncthreads();
    for (int e = t; e < m * m; e += 256) {  // trailing triangle: A22 -= X X^T
      const int r = c0 + 16 + e / m, s = c0 + 16 + e % m;
      if (s > r) continue;
      double acc = a[r][s];
#pragma unroll
      for (int kk = 0; kk < 16; kk++) acc -= a[r][c0 + kk] * a[s][c0 + kk];
      a[r][s] = acc;
    }
    __syncthreads();
  }
  // off-diagonal blocks of inv(L): T = sum_k L_ik X_kj into block (i, j), then X_ij = -X_ii T
  for (int d = 1; d < 4; d++) {
    const int pairs = 4 - d;
    double v[3];
#pragma unroll
    for (int u = 0; u < 3; u++) {
      const int e = t + 256 * u;
      v[u] = 0.0;
      if (e < pairs * 256) {
        const int jb = e >> 8, ib = jb + d, r = (e >> 4) & 15, c = e & 15;
        double s = 0.0;
        for (int kk = 16 * jb; kk < 16 * ib; kk++) s = fma(a[16 * ib + r][kk], x[kk][16 * jb + c], s);
        v[u] = s;
      }
    }
#pragma unroll
    for (int u = 0; u < 3; u++) {
      const int e = t + 256 * u;
      if (e < pairs * 256) {
        const int jb = e >> 8, ib = jb + d, r = (e >> 4) & 15, c = e & 15;
        x[16 * ib + r][16 * jb + c] = v[u];
      }
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < 3; u++) {
      const int e = t + 256 * u;
      v[u] = 0.0;
      if (e < pairs * 256) {
        const int jb = e >> 8, ib = jb + d, r = (e >> 4) & 15, c = e & 15;
        double s = 0.0;
        for (int q = 0; q <= r; q++) s = fma(x[16 * ib + r][16 * ib + q], x[16 * ib + q][16 * jb + c], s);
        v[u] = -s;
      }
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < 3; u++) {
      const int e = t + 256 * u;
      if (e < pairs * 256) {
        const int jb = e >> 8, ib = jb + d, r = (e >> 4) & 15, c = e & 15;
        x[16 * ib + r][16 * jb + c] = v[u];
      }
    }
    __syncthreads();
  }
  for (int i = t; i < 64 * 64; i += 256) {
    const int r = i >> 6, c = i & 63;
    A[(size_t)(k + r) * n + k + c] = (c <= r) ? x[r][c] : 0.0;
  }
  // the inverse chain reads this block transposed: D_k[c][r] = inv(L_kk)[r][c] (zero for r < c)
  double* __restrict__ Dk = d_base(A, n) + (size_t)k * 64;
  for (int i = t; i < 64 * 64; i += 256) {
    const int c = i >> 6, r = i & 63;
    Dk[i] = (r >= c) ? x[r][c] : 0.0;
  }
  // U's diagonal block: U[n-1-(k+r)][n-1-(k+c)] = inv(L_kk)[r][c] for c <= r
  for (int i = t; i < 64 * 64; i += 256) {
    const int r = i >> 6, c = i & 63;
    if (c > r) continue;
    const size_t u = (size_t)(n - 1 - (k + r)) * n + (size_t)(n - 1 - (k + c));
    if (fb.out_f64) static_cast<double*>(fb.U[blockIdx.x])[u] = x[r][c];
    else static_cast<float*>(fb.U[blockIdx.x])[u] = (float)x[r][c];
  }
}

__device__ __forceinline__ void cp_async16_zfill(void* smem, const void* gmem, bool ok) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
  const int src_bytes = ok ? 16 : 0;  // 0: nothing is read, the 16 bytes are zero-filled
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(sa), "l"(gmem), "r"(src_bytes) : "memory");
}

// 64 x 64 FP64 tile product on the FP64 tensor path: acc = sum_l A[i][l] * Bop[l][j] over
// l < k_len, with mma.sync m16n8k16 (f64).  kFT = 128 threads: warp w owns the 32 x 32
// quarter (rows 32 (w >> 1), columns 32 (w & 1)) as 2 x 4 fragments; with g = lane >> 2 and
// q = lane & 3, acc[mf][nf][v] is element
//   row 32 (w >> 1) + 16 mf + g + 8 (v >> 1),  column 32 (w & 1) + 8 nf + 2 q + (v & 1)
// (tile_for_each).  K streams in chunks of 16 through a two-stage zero-filling cp.async
// pipeline.  Shared-memory pitches (20 doubles for rows of A and of B stored [N][K], 68 for
// B stored [K][N]) keep the fragment loads free of bank conflicts.
// B_NK: B is stored [N][K] (Bop = B^T, the A*B^T form); otherwise B is [K][N].
// Rows >= m_lim of A and columns >= n_lim of Bop read as zero.
constexpr int kFT = 128;
constexpr int kAP = 20;
constexpr int kBP = 68;

__device__ __forceinline__ void mma_f64(double (&d)[4], const double (&a)[8], const double (&b)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f64.f64.f64.f64 {%0, %1, %2, %3}, {%4, %5, %6, %7, %8, %9, %10, %11}, "
      "{%12, %13, %14, %15}, {%0, %1, %2, %3};"
      : "+d"(d[0]), "+d"(d[1]), "+d"(d[2]), "+d"(d[3])
      : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(a[4]), "d"(a[5]), "d"(a[6]), "d"(a[7]), "d"(b[0]),
        "d"(b[1]), "d"(b[2]), "d"(b[3]));
}

template <bool B_NK>
__device__ __forceinline__ void tile64(const double* __restrict__ A, int lda, const double* __restrict__ B, int ldb,
                                       int m_lim, int n_lim, int k_len, double (&acc)[2][4][4],
                                       bool accumulate = false) {
  __shared__ __align__(16) double sa[2][64 * kAP];
  __shared__ __align__(16) double sb[2][B_NK ? 64 * kAP : 16 * kBP];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5, g = lane >> 2, q = lane & 3;
  const int wm = 32 * (warp >> 1), wn = 32 * (warp & 1);
  if (!accumulate) {
#pragma unroll
    for (int i = 0; i < 2; i++)
#pragma unroll
      for (int j = 0; j < 4; j++)
#pragma unroll
        for (int v = 0; v < 4; v++) acc[i][j][v] = 0.0;
  }
  auto load = [&](int l0, int buf) {
#pragma unroll
    for (int k = 0; k < 512 / kFT; k++) {  // A chunk: 64 rows x 16 doubles = 512 x 16 bytes
      const int i = t + kFT * k, r = i >> 3, kk = (i & 7) * 2;
      const bool ok = r < m_lim && l0 + kk < k_len;
      cp_async16_zfill(&sa[buf][r * kAP + kk], ok ? (const void*)(A + (size_t)r * lda + l0 + kk) : (const void*)A, ok);
    }
    if (B_NK) {
#pragma unroll
      for (int k = 0; k < 512 / kFT; k++) {
        const int i = t + kFT * k, c = i >> 3, kk = (i & 7) * 2;
        const bool ok = c < n_lim && l0 + kk < k_len;
        cp_async16_zfill(&sb[buf][c * kAP + kk], ok ? (const void*)(B + (size_t)c * ldb + l0 + kk) : (const void*)B,
                         ok);
      }
    } else {
#pragma unroll
      for (int k = 0; k < 512 / kFT; k++) {  // row kk of the chunk holds Bop[kk][0..63]
        const int i = t + kFT * k, kk = i >> 5, c = (i & 31) * 2;
        const bool ok = c < n_lim && l0 + kk < k_len;
        cp_async16_zfill(&sb[buf][kk * kBP + c], ok ? (const void*)(B + (size_t)(l0 + kk) * ldb + c) : (const void*)B,
                         ok);
      }
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  };
  if (k_len <= 0) return;
  load(0, 0);
  int buf = 0;
  for (int l0 = 0; l0 < k_len; l0 += 16, buf ^= 1) {
    if (l0 + 16 < k_len) {
      load(l0 + 16, buf ^ 1);
      asm volatile("cp.async.wait_group 1;\n" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    }
    __syncthreads();
    double a[2][8], bf[4][4];
#pragma unroll
    for (int mf = 0; mf < 2; mf++)
#pragma unroll
      for (int r = 0; r < 8; r++) a[mf][r] = sa[buf][(wm + 16 * mf + g + 8 * (r & 1)) * kAP + q + 4 * (r >> 1)];
#pragma unroll
    for (int nf = 0; nf < 4; nf++)
#pragma unroll
      for (int v = 0; v < 4; v++)
        bf[nf][v] = B_NK ? sb[buf][(wn + 8 * nf + g) * kAP + q + 4 * v] : sb[buf][(q + 4 * v) * kBP + wn + 8 * nf + g];
#pragma unroll
    for (int mf = 0; mf < 2; mf++)
#pragma unroll
      for (int nf = 0; nf < 4; nf++) mma_f64(acc[mf][nf], a[mf], bf[nf]);
    __syncthreads();
  }
}

// Calls f(row, column, value) for every element of the 64 x 64 tile this thread holds.
template <typename F>
__device__ __forceinline__ void tile_for_each(const double (&acc)[2][4][4], F f) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, q = lane & 3;
#pragma unroll
  for (int mf = 0; mf < 2; mf++)
#pragma unroll
    for (int nf = 0; nf < 4; nf++)
#pragma unroll
      for (int v = 0; v < 4; v++)
        f(32 * (warp >> 1) + 16 * mf + g + 8 * (v >> 1), 32 * (warp & 1) + 8 * nf + 2 * q + (v & 1), acc[mf][nf][v]);
}

// Left-looking Cholesky step j, before the diagonal factorisation:
//   A[j:n, j:j+64] -= L[j:n, 0:j] * L[j:j+64, 0:j]^T        (one 64-row tile per CTA)
// With S > 1 the K range is split over blockIdx.y and each CTA writes its partial product;
// chol_reduce_kernel then subtracts the partials from the block column in order.
__global__ void __launch_bounds__(kFT) chol_update_kernel(const __grid_constant__ FactorBatch fb, int j, int S) {
  const int n = fb.n;
  double* __restrict__ A = fb.P[blockIdx.z];
  if (*fb.status[blockIdx.z]) return;
  const int r0 = j + blockIdx.x * 64;
  const int q = blockIdx.y, chunk = kchunk(j, S);
  const int k0 = q * chunk, k1 = min(j, k0 + chunk);
  double acc[2][4][4];
  tile64<true>(A + (size_t)r0 * n + k0, n, A + (size_t)j * n + k0, n, n - r0, 64, k1 - k0, acc);
  double* part = part_base(A, n) + (size_t)q * n * NB;
  tile_for_each(acc, [&](int r, int c, double v) {
    const int rr = r0 + r;
    if (rr >= n) return;
    if (S == 1) {
      if (rr >= j + c) A[(size_t)rr * n + j + c] -= v;
    } else {
      part[(size_t)rr * NB + c] = v;
    }
  });
}

// Split-K reduction of a Cholesky step's update: A[r][j+c] -= part_0 - ... - part_{S-1}, in
// that order, for every row r >= j of the block column (rows of the diagonal tile only on or
// below the diagonal).  256 threads, one 64-row tile per CTA, 16 elements a thread.
__global__ void __launch_bounds__(256) chol_reduce_kernel(const __grid_constant__ FactorBatch fb, int j, int S) {
  const int n = fb.n;
  double* __restrict__ A = fb.P[blockIdx.y];
  if (*fb.status[blockIdx.y]) return;
  const double* part = part_base(A, n);
  const int r0 = j + blockIdx.x * 64;
  for (int i = threadIdx.x; i < 64 * 64; i += 256) {
    const int rr = r0 + i / 64, c = i % 64;
    if (rr >= n || rr < j + c) continue;
    double v = A[(size_t)rr * n + j + c];
    for (int q = 0; q < S; q++) v -= part[((size_t)q * n + rr) * NB + c];
    A[(size_t)rr * n + j + c] = v;
  }
}

// Panel below the diagonal block: A[j+64:n, j:j+64] := A * inv(L_jj)^T (inverse on the diagonal).
__global__ void __launch_bounds__(kFT) trsm_panel_kernel(const __grid_constant__ FactorBatch fb, int j) {
  const int n = fb.n;
  double* __restrict__ A = fb.P[blockIdx.y];
  if (*fb.status[blockIdx.y]) return;
  const int r0 = j + 64 + blockIdx.x * 64;
  double acc[2][4][4];
  tile64<true>(A + (size_t)r0 * n + j, n, A + (size_t)j * n + j, n, n - r0, 64, 64, acc);
  __syncthreads();  // every CTA reads only its own rows of the panel, so in-place is safe
  tile_for_each(acc, [&](int r, int c, double v) {
    const int rr = r0 + r;
    if (rr < n) A[(size_t)rr * n + j + c] = v;
  });
}

// Triangular inverse, block row j (a chain on the helper stream, started once the Cholesky
// chain has inverted the diagonal block j):
//   Linv[jb, c] = -inv(L_jj) * (L[jb, c] inv(L_cc) + sum_{c < k < j} L[jb, k] Linv[k, c])
// for every 64-column tile c < j, where jb is block row j.  Block row j of L is final (the
// Cholesky chain no longer touches it), the diagonal inverses come transposed from D, and the
// off-diagonal blocks of Linv are kept transposed in the strict upper triangle of P, which
// the Cholesky chain never reads.  Each result also goes straight to U (reversed, cast).
// Tile c reduces over j - 64c columns, so a CTA takes tiles c and nt - 1 - c together: every
// CTA then does the same work (j + 192 columns of products) and a launch has no long tail.
// T holds each tile's intermediate product.
__device__ __forceinline__ void trinv_row_tile(const FactorBatch& fb, double* __restrict__ P, int n, int j, int c0,
                                               int item) {
  double* __restrict__ S = t_base(P, n) + (size_t)c0 * 64;   // S[c][r] = product[r][c]
  double acc[2][4][4];
  tile64<true>(P + (size_t)j * n + c0, n, d_base(P, n) + (size_t)c0 * 64, 64, 64, 64, 64, acc, false);
  if (j - c0 - 64 > 0)
    tile64<true>(P + (size_t)j * n + c0 + 64, n, P + (size_t)c0 * n + c0 + 64, n, 64, 64, j - c0 - 64, acc, true);
  tile_for_each(acc, [&](int r, int c, double v) { S[(size_t)c * 64 + r] = v; });
  __threadfence_block();
  __syncthreads();
  tile64<true>(P + (size_t)j * n + j, n, S, 64, 64, 64, 64, acc, false);
  tile_for_each(acc, [&](int r, int c, double v) {
    P[(size_t)(c0 + c) * n + j + r] = -v;
    const size_t u = (size_t)(n - 1 - (j + r)) * n + (size_t)(n - 1 - (c0 + c));
    if (fb.out_f64) static_cast<double*>(fb.U[item])[u] = -v;
    else static_cast<float*>(fb.U[item])[u] = (float)(-v);
  });
}

__global__ void __launch_bounds__(kFT) trinv_row_kernel(const __grid_constant__ FactorBatch fb, int j) {
  const int n = fb.n, item = blockIdx.y;
  double* __restrict__ P = fb.P[item];
  if (*fb.status[item]) return;
  const int nt = j / 64, ca = blockIdx.x, cb = nt - 1 - blockIdx.x;
  trinv_row_tile(fb, P, n, j, ca * 64, item);
  if (cb > ca) {
    __syncthreads();   // the first tile's last shared-memory reads are done
    trinv_row_tile(fb, P, n, j, cb * 64, item);
  }
}

size_t factor_workspace_bytes(int64_t n) {
  // P (n x n f64) + T and D (n x nb each) + split-K partial tiles (kSplitMax x n x nb)
  return ((size_t)n * n + 2 * (size_t)n * NB + (size_t)kSplitMax * n * NB) * sizeof(double);
}

namespace {
// The inverse chain's stream: one per (host thread, device, caller stream), created on first
// use with the caller stream's priority, plus the events that fork it from the caller, hand
// it each inverted diagonal block and join it back.
struct InvHelper {
  cudaStream_t s = nullptr;
  cudaEvent_t fork = nullptr, step = nullptr, join = nullptr;
};
int inv_helper(cudaStream_t caller, InvHelper** out) {
  static thread_local std::map<std::pair<int, cudaStream_t>, InvHelper> helpers;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 1;
  InvHelper& h = helpers[std::make_pair(dev, caller)];
  if (!h.s) {
    int prio = 0;
    if (cudaStreamGetPriority(caller, &prio) != cudaSuccess) prio = 0;
    if (cudaStreamCreateWithPriority(&h.s, cudaStreamNonBlocking, prio) != cudaSuccess ||
        cudaEventCreateWithFlags(&h.fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&h.step, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&h.join, cudaEventDisableTiming) != cudaSuccess)
      return 1;
  }
  *out = &h;
  return 0;
}
}  // namespace

int launch_factor_batch(const FactorBatch& fb, cudaStream_t stream) {
  const int n = fb.n, cnt = fb.count;
  if (cnt <= 0) return 0;
  if (n <= 0 || n % NB) return 2;
  {  // the diagonal-block and row-staged permute kernels use more than the 48 KB default (per device)
    static std::atomic<unsigned long long> opted{0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1;
    if (!(opted.load() & (1ULL << dev))) {
      if (cudaFuncSetAttribute(potrf_inv_diag_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kPotrfSmemBytes) != cudaSuccess ||
          cudaFuncSetAttribute(permute_reverse_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kPermRowSmemMax) != cudaSuccess)
        return 1;
      opted.fetch_or(1ULL << dev);
    }
  }
  InvHelper* hp = nullptr;
  if (inv_helper(stream, &hp)) return 1;
  const size_t ubytes = (size_t)n * n * (fb.out_f64 ? sizeof(double) : sizeof(float));
  for (int b = 0; b < cnt; b++) {
    cudaMemsetAsync(fb.status[b], 0, sizeof(int), stream);
    cudaMemsetAsync(fb.U[b], 0, ubytes, stream);   // U's strict lower triangle stays zero
  }
  if ((size_t)n * sizeof(double) <= (size_t)kPermRowSmemMax) {
    permute_reverse_rows_kernel<<<dim3((unsigned)n, (unsigned)cnt), 256, (size_t)n * sizeof(double), stream>>>(fb);
    note_launch();
  } else {
    dim3 g((unsigned)((n + 255) / 256), (unsigned)n, (unsigned)cnt);
    permute_reverse_kernel<<<g, 256, 0, stream>>>(fb);
    note_launch();
  }
  cudaEventRecord(hp->fork, stream);
  cudaStreamWaitEvent(hp->s, hp->fork, 0);
  for (int j = 0; j < n; j += NB) {
    const int S = j > 0 ? ksplit_batch(j, (n - j) / 64, cnt) : 1;
    if (j > 0) {
      chol_update_kernel<<<dim3((unsigned)((n - j) / 64), (unsigned)S, (unsigned)cnt), kFT, 0, stream>>>(fb, j, S);
      note_launch();
      if (S > 1) {
        chol_reduce_kernel<<<dim3((unsigned)((n - j) / 64), (unsigned)cnt), 256, 0, stream>>>(fb, j, S);
        note_launch();
      }
    }
    potrf_inv_diag_kernel<<<(unsigned)cnt, 256, kPotrfSmemBytes, stream>>>(fb, j);
    note_launch();
    if (j > 0) {   // block row j of the inverse, on the helper stream
      cudaEventRecord(hp->step, stream);
      cudaStreamWaitEvent(hp->s, hp->step, 0);
      trinv_row_kernel<<<dim3((unsigned)((j / 64 + 1) / 2), (unsigned)cnt), kFT, 0, hp->s>>>(fb, j);
      note_launch();
    }
    if (n - j - NB > 0) {
      trsm_panel_kernel<<<dim3((unsigned)((n - j - NB) / 64), (unsigned)cnt), kFT, 0, stream>>>(fb, j);
      note_launch();
    }
  }
  cudaEventRecord(hp->join, hp->s);
  cudaStreamWaitEvent(stream, hp->join, 0);
  return 0;
}

int launch_factor_u(const double* H, int64_t n64, const int* order, double shift, void* U, bool out_f64,
                    void* work, int* status, cudaStream_t stream) {
  if (n64 <= 0 || n64 % NB) return 2;
  FactorBatch fb;
  fb.count = 1;
  fb.n = (int)n64;
  fb.out_f64 = out_f64 ? 1 : 0;
  fb.H[0] = H;
  fb.order[0] = order;
  fb.P[0] = (double*)work;
  fb.U[0] = U;
  fb.status[0] = status;
  fb.shift[0] = shift;
  return launch_factor_batch(fb, stream);
}

}  // namespace cpk
