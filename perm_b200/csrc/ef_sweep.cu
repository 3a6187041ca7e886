// GPTQ-style error-feedback column sweep (coldpress/ef.py:197-216) for sm_100a.
//
// Reference semantics, per row r and act-order column jj ascending:
//   q  = clip(nearest_int((w[jj] + ml) / dl), lo, hi)     (q = 0, e = 0 where dl == 0)
//   e  = (w[jj] - (dl*q - ml)) / U[jj][jj]
//   w[k] = fl(w[k] - fl(e * U[jj][k]))   for every k > jj, in ascending jj order
// Rows are independent, so a CTA owns a tile of 32 rows and runs the whole sweep for them
// with no inter-CTA synchronisation.  Columns are processed in blocks of 32:
//   panel    (warp 0, lane = row): the 32 sequential quantize/error steps of the block with
//            its in-block updates, in registers;
//   trailing (8 warps): every later column gets the block's 32 updates in jj order, two
//            columns at a time with packed f32x2 arithmetic that rounds the product and the
//            difference separately (see upd2), so each element sees exactly the
//            reference's rounding sequence.
// The working rows live in a global workspace laid out [tile][column pair][32 rows][2]
// (coalesced float2 per lane); U is read from a column-pair-interleaved transpose
// UT2[pair][jj][2] so one 16-byte broadcast load feeds two jj steps of a column pair.
#include <cuda_runtime.h>
#include "kq_common.cuh"
#include "kquant_kernels.h"
#include "ef_kernels.h"

namespace cpk {

// Two updates w = fl(w - fl(e*u)) on a column pair.  The product is formed by a packed FMA
// whose addend is -0.0 supplied at run time (fl(e*u + -0) == fl(e*u) for every input, signed
// zeros included); a literal -0.0 or a packed multiply would let ptxas contract the product
// and the subtraction into one fused op, which rounds once and breaks parity.
__device__ __forceinline__ void upd2(float& wx, float& wy, float ex, float ey, float ux, float uy, float nz) {
  asm("{\n\t.reg .b64 w, e, u, p, z;\n\t"
      "mov.b64 w, {%0, %1};\n\t"
      "mov.b64 e, {%2, %3};\n\t"
      "mov.b64 u, {%4, %5};\n\t"
      "mov.b64 z, {%6, %6};\n\t"
      "fma.rn.f32x2 p, e, u, z;\n\t"
      "sub.rn.f32x2 w, w, p;\n\t"
      "mov.b64 {%0, %1}, w;\n\t}"
      : "+f"(wx), "+f"(wy)
      : "f"(ex), "f"(ey), "f"(ux), "f"(uy), "f"(nz));
}

// UT2[kp][jj][p] = U[jj][2kp+p] for jj <= 2kp+p, else 0; diagU[jj] = U[jj][jj].
__global__ void build_ut2_kernel(const float* __restrict__ U, int n, float* __restrict__ UT2,
                                 float* __restrict__ diagU) {
  __shared__ float t[32][33];
  const int k0 = blockIdx.x * 32, j0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 256 threads: ty 0..7
  for (int r = ty; r < 32; r += 8) {
    const int jj = j0 + r, k = k0 + tx;
    t[r][tx] = (jj <= k) ? U[(size_t)jj * n + k] : 0.0f;
    if (jj == k) diagU[jj] = U[(size_t)jj * n + k];
  }
  __syncthreads();
  // output: for column pair kp = (k0/2) + c (c 0..15), jj = j0 + r: 64 floats per kp row segment
  for (int i = threadIdx.x; i < 16 * 64; i += 256) {
    const int c = i >> 6, rem = i & 63, r = rem >> 1, p = rem & 1;
    const int kp = (k0 >> 1) + c;
    UT2[((size_t)kp * n + j0 + r) * 2 + p] = t[r][2 * c + p];
  }
}

template <bool HAS_MIN>
__global__ void __launch_bounds__(256, 2)
ef_sweep_kernel(const float* __restrict__ x, int nrow, int n, const int* __restrict__ order,
                const float* __restrict__ UT2, const float* __restrict__ diagU,
                const float* __restrict__ dl, const float* __restrict__ ml, int sbw, int lo, int hi,
                float2* __restrict__ work, int8_t* __restrict__ codes, float* __restrict__ wcur, float nz) {
  __shared__ float s_u[32][33];
  __shared__ __align__(16) float2 s_e[32][32];
  __shared__ int s_ord[32];
  const int tile = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int row = tile * 32 + lane;
  const bool rv = row < nrow;
  const int npair = n >> 1;
  const int nsub = n / sbw;
  float2* W = work + (size_t)tile * npair * 32;
  const float* xr = x + (size_t)row * n;

  // wp = x[:, order]
  for (int kp = warp; kp < npair; kp += 8) {
    float2 v = make_float2(0.0f, 0.0f);
    if (rv) {
      v.x = __ldg(xr + __ldg(order + 2 * kp));
      v.y = __ldg(xr + __ldg(order + 2 * kp + 1));
    }
    W[kp * 32 + lane] = v;
  }
  __syncthreads();

  for (int j0 = 0; j0 < n; j0 += 32) {
    for (int i = threadIdx.x; i < 32 * 32; i += 256) {  // s_u[a][b] = U[j0+a][j0+b]
      const int a = i & 31, b = i >> 5;
      s_u[a][b] = __ldg(UT2 + ((size_t)((j0 + b) >> 1) * n + j0 + a) * 2 + (b & 1));
    }
    if (threadIdx.x < 32) s_ord[threadIdx.x] = __ldg(order + j0 + threadIdx.x);
    __syncthreads();

    if (warp == 0) {
      float w[32];
#pragma unroll
      for (int a = 0; a < 16; a++) {
        const float2 t = W[((j0 >> 1) + a) * 32 + lane];
        w[2 * a] = t.x;
        w[2 * a + 1] = t.y;
      }
      const float* dlr = dl + (size_t)row * nsub;
      const float* mlr = HAS_MIN ? ml + (size_t)row * nsub : nullptr;
#pragma unroll
      for (int a = 0; a < 32; a++) {
        const int j = s_ord[a];
        const int s = j / sbw;
        const float dlv = rv ? __ldg(dlr + s) : 0.0f;
        const float mlv = (HAS_MIN && rv) ? __ldg(mlr + s) : 0.0f;
        int q = 0;
        float e = 0.0f;
        if (dlv != 0.0f) {
          q = clampi(nint((w[a] + mlv) / dlv), lo, hi);
          const float recon = dlv * (float)q - mlv;
          e = (w[a] - recon) / __ldg(diagU + j0 + a);
        }
        if (rv) {
          codes[(size_t)row * n + j] = (int8_t)q;
          if (wcur) wcur[(size_t)row * n + j] = w[a];
        }
        s_e[a][lane] = make_float2(e, e);
#pragma unroll
        for (int b = a + 1; b < 32; b++) w[b] = w[b] - e * s_u[a][b];
      }
    }
    __syncthreads();

    const int kp0 = (j0 + 32) >> 1;
    if (kp0 < npair) {
      float2 ee[32];
#pragma unroll
      for (int a = 0; a < 32; a++) ee[a] = s_e[a][lane];
      for (int kp = kp0 + warp; kp < npair; kp += 8) {
        float2 wv = W[kp * 32 + lane];
        const float4* up = reinterpret_cast<const float4*>(UT2 + ((size_t)kp * n + j0) * 2);
#pragma unroll
        for (int a4 = 0; a4 < 16; a4++) {
          const float4 u = __ldg(up + a4);
          upd2(wv.x, wv.y, ee[2 * a4].x, ee[2 * a4].y, u.x, u.y, nz);
          upd2(wv.x, wv.y, ee[2 * a4 + 1].x, ee[2 * a4 + 1].y, u.z, u.w, nz);
        }
        W[kp * 32 + lane] = wv;
      }
    }
    __syncthreads();
  }
}

size_t ef_sweep_workspace_bytes(int64_t nrow, int64_t n) {
  const int64_t ntiles = (nrow + 31) / 32;
  return (size_t)ntiles * (size_t)n * 32 * sizeof(float);
}

size_t ef_ut2_bytes(int64_t n) { return (size_t)n * (size_t)n * sizeof(float) + (size_t)n * sizeof(float); }

int launch_build_ut2(const float* U, int64_t n, float* UT2, float* diagU, cudaStream_t stream) {
  if (n % 32) return 2;
  dim3 grid((unsigned)(n / 32), (unsigned)(n / 32));
  build_ut2_kernel<<<grid, 256, 0, stream>>>(U, (int)n, UT2, diagU);
  note_launch();
  return 0;
}

int launch_ef_sweep(int type, const float* x, int64_t nrow, int64_t n, const int* order,
                    const float* UT2, const float* diagU, const float* dl, const float* ml, void* work,
                    int8_t* codes, float* wcur, cudaStream_t stream) {
  int sbw, lo, hi;
  bool has_min;
  if (!grid_spec(type, &sbw, &lo, &hi, &has_min)) return 1;
  if (n % 256 || nrow <= 0) return 2;
  const unsigned ntiles = (unsigned)((nrow + 31) / 32);
  if (has_min)
    ef_sweep_kernel<true><<<ntiles, 256, 0, stream>>>(x, (int)nrow, (int)n, order, UT2, diagU, dl, ml, sbw, lo,
                                                     hi, (float2*)work, codes, wcur, -0.0f);
  else
    ef_sweep_kernel<false><<<ntiles, 256, 0, stream>>>(x, (int)nrow, (int)n, order, UT2, diagU, dl, nullptr,
                                                      sbw, lo, hi, (float2*)work, codes, wcur, -0.0f);
  note_launch();
  return 0;
}

}  // namespace cpk
