// GPTQ-style error-feedback column sweep (coldpress/ef.py:197-216) for sm_100a.
//
// Reference semantics, per row r and act-order column jj ascending:
//   q  = clip(nearest_int((w[jj] + ml) / dl), lo, hi)     (q = 0, e = 0 where dl == 0)
//   e  = (w[jj] - (dl*q - ml)) / U[jj][jj]
//   w[k] = fl(w[k] - fl(e * U[jj][k]))   for every k > jj, in ascending jj order
// Rows are independent.  A CTA of kSweepWarps = 4 warps owns 128 rows (lane = row) and walks the
// columns in act order in blocks of 64, left-looking:
//   1. the row's 64 working values of the block are gathered from x into registers;
//   2. the errors of every earlier column are applied in ascending jj: per jj, each thread
//      updates its 64 values with e_jj * U[jj][block] (32 independent packed pairs, see
//      upd2), U rows and the stored errors streamed through a shared-memory cp.async ring
//      that the four warps share;
//   3. the block's panel: the 64 dependent quantize/error steps, each followed by its
//      in-block updates, in registers (four sub-panels of 16 in a run-time loop); the
//      errors go to the workspace for later blocks.
// Every element therefore receives exactly the reference's updates, in the reference's
// order, each rounded as the reference rounds it.  Per row, the workspace holds the n
// errors (written once, read once per later block), instead of a working copy of the row
// that a right-looking sweep would rewrite after every block.
#include <cuda_runtime.h>
#include <algorithm>
#include <mutex>
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

// The same two updates as upd2, written with the packed FMA intrinsic: p = RN(e*u) with the
// -0 addend, then w = RN(p * -1 + w), which is RN(w - p) exactly (p * -1 only flips a sign;
// signed zeros come out as in w - p).  Both factors that would let ptxas fuse the pair, the
// -0 addend and the -1, are run-time values (built from the nz kernel argument), so each
// step rounds on its own.  Unlike the inline-assembly form, the scheduler sees the two FFMA2
// and interleaves the 32 independent pairs of a column: 3-4 % faster in the ordinary sweep
// (the column-split forms, which hold fewer pairs per warp, keep upd2).
__device__ __forceinline__ void upd2f(float& wx, float& wy, float e, float ux, float uy, float nz) {
  const float m1 = __int_as_float(__float_as_int(nz) | 0x3f800000);   // -1.0f from nz = -0.0f
  const float2 p = __ffma2_rn(make_float2(e, e), make_float2(ux, uy), make_float2(nz, nz));
  const float2 r = __ffma2_rn(p, make_float2(m1, m1), make_float2(wx, wy));
  wx = r.x;
  wy = r.y;
}

// Prepared U for the sweep: U row-major (float32 [n][n]) followed by its diagonal.
__global__ void prepare_u_kernel(const float* __restrict__ U, int n, float* __restrict__ out) {
  const size_t n4 = (size_t)n * n / 4;
  const float4* src = reinterpret_cast<const float4*>(U);
  float4* dst = reinterpret_cast<float4*>(out);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = src[i];
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    out[(size_t)n * n + i] = U[(size_t)i * n + i];
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

constexpr int kSwB = 64;      // columns per block
constexpr int kSwJS = 8;      // earlier columns (jj) per ring stage
constexpr int kSwST = 4;      // ring stages
constexpr int kSwThreads = 32 * kSweepWarps;

struct SweepSmem {
  __align__(16) float ud[kSwB][kSwB];                // ud[a][b] = U[j0+a][j0+b], the block's diagonal block
  float dg[kSwB];                                    // U[j0+a][j0+a]
  int ord[kSwB];                                     // order[j0+a]
  __align__(16) float ru[kSwST][kSwJS][kSwB];        // ring: U[jj][j0 .. j0+63]
  union __align__(16) {
    float re[kSwST][kSweepWarps][kSwJS][32];         // ring: errors e_jj of each warp's rows
    struct {                                         // column-split form (sweep_rows_split)
      float re[kSwST][2][kSwJS][32];                 // ring: errors e_jj of the CTA's row tiles
      float xb[2 * 32 * 32];                         // errors handed between a tile's warps
    } cs;
  };
};

// One CTA = kSweepWarps x 32 rows of one tensor.
__device__ __forceinline__ void sweep_rows(const SweepDesc& t, int cta, float nz, SweepSmem& sm) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = t.n, nrow = t.nrow;
  const int tile32 = cta * kSweepWarps + warp;
  const int row = tile32 * 32 + lane;
  const bool rv = row < nrow;
  const int sbw = t.sbw, lo = t.lo, hi = t.hi, nsub = n / sbw;
  const float* __restrict__ U = t.u;
  const float* __restrict__ diagU = t.u + (size_t)n * n;
  float* __restrict__ E = t.work;                              // [tile32][n][32]
  const float* __restrict__ Ecta = t.work + (size_t)cta * kSweepWarps * n * 32;
  float* __restrict__ Erow = E + (size_t)tile32 * n * 32 + lane;
  // element (row, column) of x, codes and wout sits at row * rs + column * cs (grid arrays:
  // row * rsg + sub-block * cs); the column-major layout makes each warp access one 128-byte
  // (or 32-byte for codes) segment
  const int64_t cs = t.pitch ? t.pitch : 1, rs = t.pitch ? 1 : n, rsg = t.pitch ? 1 : nsub;
  const float* __restrict__ xr = t.x + (size_t)(rv ? row : 0) * rs;
  const float* __restrict__ dlr = t.dl + (size_t)(rv ? row : 0) * rsg;
  const float* __restrict__ mlr = t.ml ? t.ml + (size_t)(rv ? row : 0) * rsg : nullptr;
  int8_t* __restrict__ codes = t.codes + (size_t)row * rs;
  float* __restrict__ wout = t.wout ? t.wout + (size_t)row * rs : nullptr;

  for (int j0 = 0; j0 < n; j0 += kSwB) {
    __syncthreads();  // the previous block's readers of the shared buffers are done
    const int nst = j0 / kSwJS;
    // stage s = U rows jj in [s*JS, s*JS + JS) of this block's columns + the CTA's errors
    // of those jj (16 + 8 * kSweepWarps = 48 chunks of 16 bytes per jj)
    auto issue = [&](int s) {
      if (s < nst) {
        const int st = s % kSwST, jj0 = s * kSwJS;
        for (int c = tid; c < kSwJS * (16 + 8 * kSweepWarps); c += kSwThreads) {
          if (c < kSwJS * 16) {
            const int k = c >> 4, c4 = c & 15;
            cp_async16(&sm.ru[st][k][4 * c4], U + (size_t)(jj0 + k) * n + j0 + 4 * c4);
          } else {
            const int c2 = c - kSwJS * 16, w = c2 / (kSwJS * 8), rem = c2 % (kSwJS * 8);
            const int k = rem >> 3, l4 = rem & 7;
            cp_async16(&sm.re[st][w][k][4 * l4], Ecta + ((size_t)w * n + jj0 + k) * 32 + 4 * l4);
          }
        }
      }
      cp_async_commit();
    };
#pragma unroll
    for (int s = 0; s < kSwST - 1; s++) issue(s);
    for (int i = tid; i < kSwB * kSwB / 4; i += kSwThreads) {
      const int a = i >> 4, c4 = i & 15;
      reinterpret_cast<float4*>(sm.ud[a])[c4] =
          __ldg(reinterpret_cast<const float4*>(U + (size_t)(j0 + a) * n + j0) + c4);
    }
    if (tid < kSwB) {
      sm.ord[tid] = __ldg(t.order + j0 + tid);
      sm.dg[tid] = __ldg(diagU + j0 + tid);
    }
    __syncthreads();

    // 1. the block's working values, w = x[row, order[j0 + c]]
    float w[kSwB];
#pragma unroll
    for (int c = 0; c < kSwB; c++) w[c] = rv ? __ldg(xr + sm.ord[c] * cs) : 0.0f;

    // 2. errors of every earlier column, ascending jj
    for (int s = 0; s < nst; s++) {
      cp_async_wait<kSwST - 2>();
      __syncthreads();  // stage s landed for everyone; everyone is done with stage s - 1
      issue(s + kSwST - 1);
      const int st = s % kSwST;
#pragma unroll
      for (int k = 0; k < kSwJS; k++) {
        const float e = sm.re[st][warp][k][lane];
        const float4* u4 = reinterpret_cast<const float4*>(sm.ru[st][k]);
#pragma unroll
        for (int c4 = 0; c4 < kSwB / 4; c4++) {
          const float4 u = u4[c4];
          upd2f(w[4 * c4], w[4 * c4 + 1], e, u.x, u.y, nz);
          upd2f(w[4 * c4 + 2], w[4 * c4 + 3], e, u.z, u.w, nz);
        }
      }
    }
    cp_async_wait<0>();

    // 3. panel: the block's 64 dependent quantize/error steps, as four sub-panels of 16
    // (a run-time loop).  Sub-panel p quantizes w[0..15] in order, each step followed by its
    // updates of the later columns of the sub-panel; then the 16 errors update the block's
    // remaining 16-column groups (ascending jj, packed); then w shifts down by 16 registers so
    // the next sub-panel again finds its columns in w[0..15].  Register indices stay
    // compile-time and no update is computed that the reference does not make.  The grid
    // values are loaded at the start of each sub-panel: keeping the next sub-panel's in
    // registers costs the fourth resident CTA per SM, which hides more latency than the
    // prefetch does.
#pragma unroll 1
    for (int p = 0; p < kSwB / 16; p++) {
      const int a0 = 16 * p;
      float es[16];
      float cd[16], cm[16];
#pragma unroll
      for (int i = 0; i < 16; i++) {
        const int sidx = sm.ord[a0 + i] / sbw;
        cd[i] = rv ? __ldg(dlr + sidx * cs) : 0.0f;
        cm[i] = (rv && mlr) ? __ldg(mlr + sidx * cs) : 0.0f;
      }
#pragma unroll
      for (int i = 0; i < 16; i++) {
        const int a = a0 + i, j = sm.ord[a];
        const float dlv = cd[i], mlv = cm[i], wa = w[i];
        int q = 0;
        float e = 0.0f;
        if (dlv != 0.0f) {
          q = clampi(nint((wa + mlv) / dlv), lo, hi);
          const float recon = dlv * (float)q - mlv;
          e = (wa - recon) / sm.dg[a];
        }
        if (rv) {
          codes[j * cs] = (int8_t)q;
          if (wout) wout[j * cs] = wa;
        }
        Erow[(size_t)(j0 + a) * 32] = e;
        es[i] = e;
#pragma unroll
        for (int b = i + 1; b < 16; b++) w[b] = w[b] - e * sm.ud[a][a0 + b];
      }
      // later 16-column groups g of the block (columns a0 + 16 g .. +15 are w[16 g ..])
#pragma unroll
      for (int g = 1; g < 4; g++) {
        if (p + g < kSwB / 16) {
#pragma unroll
          for (int i = 0; i < 16; i++) {
            const float2* u2 = reinterpret_cast<const float2*>(&sm.ud[a0 + i][a0 + 16 * g]);
#pragma unroll
            for (int c2 = 0; c2 < 8; c2++) {
              const float2 u = u2[c2];
              upd2f(w[16 * g + 2 * c2], w[16 * g + 2 * c2 + 1], es[i], u.x, u.y, nz);
            }
          }
        }
      }
#pragma unroll
      for (int c = 0; c < kSwB - 16; c++) w[c] = w[c + 16];
    }
  }
}

// Column-split form, for launches too small to fill the GPU (their time is the serial work of
// their longest rows): S = 2 or 4 warps share each 32-row tile (lane = row), warp h keeping
// block columns CW*h .. CW*h + CW - 1 (CW = 64 / S) of every 64-column block in registers, so
// each warp applies the earlier columns' errors to 1/S of the row.  The panel goes warp by
// warp: warp q quantizes its columns and leaves their errors in shared memory; after a
// barrier the warps after it apply them, in ascending order, to their own columns.  Every
// element still receives exactly the reference's updates in the reference's order, each
// rounded as the reference rounds it.
template <int S>
__device__ __forceinline__ void sweep_rows_split(const SweepDesc& t, int cta, float nz, SweepSmem& sm) {
  constexpr int G = kSweepWarps / S;  // row tiles per CTA
  constexpr int CW = kSwB / S;        // block columns per warp
  constexpr int NSP = CW / 16;        // 16-column sub-panels per warp
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int grp = warp / S, h = warp % S, cb = CW * h;
  const int n = t.n, nrow = t.nrow;
  const int tile32 = cta * G + grp;
  const int row = tile32 * 32 + lane;
  const bool rv = row < nrow;
  const int sbw = t.sbw, lo = t.lo, hi = t.hi, nsub = n / sbw;
  const float* __restrict__ U = t.u;
  const float* __restrict__ diagU = t.u + (size_t)n * n;
  float* __restrict__ E = t.work;                              // [tile32][n][32]
  const float* __restrict__ Ecta = t.work + (size_t)cta * G * n * 32;
  float* __restrict__ Erow = E + (size_t)tile32 * n * 32 + lane;
  const int64_t cs = t.pitch ? t.pitch : 1, rs = t.pitch ? 1 : n, rsg = t.pitch ? 1 : nsub;
  const float* __restrict__ xr = t.x + (size_t)(rv ? row : 0) * rs;
  const float* __restrict__ dlr = t.dl + (size_t)(rv ? row : 0) * rsg;
  const float* __restrict__ mlr = t.ml ? t.ml + (size_t)(rv ? row : 0) * rsg : nullptr;
  int8_t* __restrict__ codes = t.codes + (size_t)row * rs;
  float* __restrict__ wout = t.wout ? t.wout + (size_t)row * rs : nullptr;
  // errors handed between the warps of a tile: block columns 0 .. 64 - CW - 1
  float* __restrict__ xb = sm.cs.xb + (size_t)grp * (kSwB - CW) * 32 + lane;

  for (int j0 = 0; j0 < n; j0 += kSwB) {
    __syncthreads();  // the previous block's readers of the shared buffers are done
    const int nst = j0 / kSwJS;
    // stage s = U rows jj in [s*JS, s*JS + JS) of this block's columns + the errors of those
    // jj for the CTA's G row tiles (16 + 8 G chunks of 16 bytes per jj)
    auto issue = [&](int s) {
      if (s < nst) {
        const int st = s % kSwST, jj0 = s * kSwJS;
        for (int c = tid; c < kSwJS * (16 + 8 * G); c += kSwThreads) {
          if (c < kSwJS * 16) {
            const int k = c >> 4, c4 = c & 15;
            cp_async16(&sm.ru[st][k][4 * c4], U + (size_t)(jj0 + k) * n + j0 + 4 * c4);
          } else {
            const int c2 = c - kSwJS * 16, w = c2 / (kSwJS * 8), rem = c2 % (kSwJS * 8);
            const int k = rem >> 3, l4 = rem & 7;
            cp_async16(&sm.cs.re[st][w][k][4 * l4], Ecta + ((size_t)w * n + jj0 + k) * 32 + 4 * l4);
          }
        }
      }
      cp_async_commit();
    };
#pragma unroll
    for (int s = 0; s < kSwST - 1; s++) issue(s);
    for (int i = tid; i < kSwB * kSwB / 4; i += kSwThreads) {
      const int a = i >> 4, c4 = i & 15;
      reinterpret_cast<float4*>(sm.ud[a])[c4] =
          __ldg(reinterpret_cast<const float4*>(U + (size_t)(j0 + a) * n + j0) + c4);
    }
    if (tid < kSwB) {
      sm.ord[tid] = __ldg(t.order + j0 + tid);
      sm.dg[tid] = __ldg(diagU + j0 + tid);
    }
    __syncthreads();

    // 1. this warp's columns of the block, w = x[row, order[j0 + cb + c]]
    float w[CW];
#pragma unroll
    for (int c = 0; c < CW; c++) w[c] = rv ? __ldg(xr + sm.ord[cb + c] * cs) : 0.0f;

    // 2. errors of every earlier column, ascending jj, on this warp's columns
    for (int s = 0; s < nst; s++) {
      cp_async_wait<kSwST - 2>();
      __syncthreads();  // stage s landed for everyone; everyone is done with stage s - 1
      issue(s + kSwST - 1);
      const int st = s % kSwST;
#pragma unroll
      for (int k = 0; k < kSwJS; k++) {
        const float e = sm.cs.re[st][grp][k][lane];
        const float4* u4 = reinterpret_cast<const float4*>(&sm.ru[st][k][cb]);
#pragma unroll
        for (int c4 = 0; c4 < CW / 4; c4++) {
          const float4 u = u4[c4];
          upd2(w[4 * c4], w[4 * c4 + 1], e, e, u.x, u.y, nz);
          upd2(w[4 * c4 + 2], w[4 * c4 + 3], e, e, u.z, u.w, nz);
        }
      }
    }
    cp_async_wait<0>();

    // 3. panel of this warp's columns: NSP sub-panels of 16 (as in sweep_rows, the later
    // sub-panel of the warp updated after the first); the errors go to xb for later warps
    auto panel = [&]() {
#pragma unroll 1
      for (int p = 0; p < NSP; p++) {
        const int a0 = cb + 16 * p;
        float es[16];
        float cd[16], cm[16];
#pragma unroll
        for (int i = 0; i < 16; i++) {
          const int sidx = sm.ord[a0 + i] / sbw;
          cd[i] = rv ? __ldg(dlr + sidx * cs) : 0.0f;
          cm[i] = (rv && mlr) ? __ldg(mlr + sidx * cs) : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < 16; i++) {
          const int a = a0 + i, j = sm.ord[a];
          const float dlv = cd[i], mlv = cm[i], wa = w[i];
          int q = 0;
          float e = 0.0f;
          if (dlv != 0.0f) {
            q = clampi(nint((wa + mlv) / dlv), lo, hi);
            const float recon = dlv * (float)q - mlv;
            e = (wa - recon) / sm.dg[a];
          }
          if (rv) {
            codes[j * cs] = (int8_t)q;
            if (wout) wout[j * cs] = wa;
          }
          Erow[(size_t)(j0 + a) * 32] = e;
          if (h < S - 1) xb[a * 32] = e;
          es[i] = e;
#pragma unroll
          for (int b = i + 1; b < 16; b++) w[b] = w[b] - e * sm.ud[a][a0 + b];
        }
        if (NSP == 2 && p == 0) {  // the warp's second 16 columns (w[16..31])
#pragma unroll
          for (int i = 0; i < 16; i++) {
            const float2* u2 = reinterpret_cast<const float2*>(&sm.ud[a0 + i][a0 + 16]);
#pragma unroll
            for (int c2 = 0; c2 < 8; c2++) {
              const float2 u = u2[c2];
              upd2(w[(16 + 2 * c2) % CW], w[(16 + 2 * c2 + 1) % CW], es[i], es[i], u.x, u.y, nz);
            }
          }
#pragma unroll
          for (int c = 0; c < CW - 16; c++) w[c] = w[c + 16];
        }
      }
    };
#pragma unroll
    for (int q = 0; q < S; q++) {
      if (h == q) panel();
      __syncthreads();  // warp q's errors are in xb
      if (h > q) {      // ... applied, ascending, to this warp's columns
#pragma unroll 4
        for (int i = 0; i < CW; i++) {
          const float e = xb[(CW * q + i) * 32];
          const float2* u2 = reinterpret_cast<const float2*>(&sm.ud[CW * q + i][cb]);
#pragma unroll
          for (int c2 = 0; c2 < CW / 2; c2++) {
            const float2 u = u2[c2];
            upd2(w[2 * c2], w[2 * c2 + 1], e, e, u.x, u.y, nz);
          }
        }
      }
    }
  }
}

__device__ __forceinline__ int sweep_desc_of(const SweepBatch& b, int cta) {
  int lo = 0, hi = b.count - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (b.d[mid].tile0 <= cta) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__global__ void __launch_bounds__(kSwThreads, 4) ef_sweep_batch_kernel(const __grid_constant__ SweepBatch b, float nz) {
  __shared__ SweepSmem sm;
  const int k = sweep_desc_of(b, blockIdx.x);
  sweep_rows(b.d[k], blockIdx.x - b.d[k].tile0, nz, sm);
}

// The column-split forms as kernels of their own, so that no form's register allocation
// constrains another's.
template <int S>
__global__ void __launch_bounds__(kSwThreads, 4) ef_sweep_split_batch_kernel(const __grid_constant__ SweepBatch b,
                                                                             float nz) {
  __shared__ SweepSmem sm;
  const int k = sweep_desc_of(b, blockIdx.x);
  sweep_rows_split<S>(b.d[k], blockIdx.x - b.d[k].tile0, nz, sm);
}

size_t ef_sweep_workspace_bytes(int64_t nrow, int64_t n) {
  const int64_t rows = (nrow + 32 * kSweepWarps - 1) / (32 * kSweepWarps) * (32 * kSweepWarps);
  return (size_t)rows * (size_t)n * sizeof(float);
}

size_t ef_u_prepared_bytes(int64_t n) { return (size_t)n * (size_t)n * sizeof(float) + (size_t)n * sizeof(float); }

// The factor already sits at the start of the prepared buffer (U == out): append the diagonal.
__global__ void prepare_u_diag_kernel(float* out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[(size_t)n * n + i] = out[(size_t)i * n + i];
}

int launch_prepare_u(const float* U, int64_t n, float* out, cudaStream_t stream) {
  if (n % 32) return 2;
  if (U == out) {
    prepare_u_diag_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(out, (int)n);
    note_launch();
    return 0;
  }
  const size_t n4 = (size_t)n * n / 4;
  const int grid = (int)std::min<size_t>((n4 + 255) / 256, (size_t)148 * 8);
  prepare_u_kernel<<<grid, 256, 0, stream>>>(U, (int)n, out);
  note_launch();
  return 0;
}

int64_t sweep_rows_padded(int64_t nrow) {
  return (nrow + 32 * kSweepWarps - 1) / (32 * kSweepWarps) * (32 * kSweepWarps);
}

int sweep_ctas(int64_t nrow) { return (int)((nrow + 32 * kSweepWarps - 1) / (32 * kSweepWarps)); }

int sweep_split_ctas(int64_t nrow, int split) {
  const int rows = 32 * (kSweepWarps / split);
  return (int)((nrow + rows - 1) / rows);
}

int launch_ef_sweep_batch(const SweepBatch& b, int total_ctas, int split, cudaStream_t stream) {
  if (b.count == 0 || total_ctas == 0) return 0;
  if (split == 4) ef_sweep_split_batch_kernel<4><<<total_ctas, kSwThreads, 0, stream>>>(b, -0.0f);
  else if (split == 2) ef_sweep_split_batch_kernel<2><<<total_ctas, kSwThreads, 0, stream>>>(b, -0.0f);
  else if (split == 1) ef_sweep_batch_kernel<<<total_ctas, kSwThreads, 0, stream>>>(b, -0.0f);
  else return 2;
  note_launch();
  return 0;
}

bool sweep_desc(int type, const float* x, int64_t nrow, int64_t n, const int* order, const float* u_prep,
                const float* dl, const float* ml, void* work, int8_t* codes, float* wcur, SweepDesc* d) {
  int sbw, lo, hi;
  bool has_min;
  if (!grid_spec(type, &sbw, &lo, &hi, &has_min)) return false;
  d->x = x;
  d->order = order;
  d->u = u_prep;
  d->dl = dl;
  d->ml = has_min ? ml : nullptr;
  d->work = (float*)work;
  d->codes = codes;
  d->wout = wcur;
  d->pitch = 0;
  d->nrow = (int)nrow;
  d->n = (int)n;
  d->sbw = sbw;
  d->lo = lo;
  d->hi = hi;
  d->tile0 = 0;
  return true;
}

int launch_ef_sweep(int type, const float* x, int64_t nrow, int64_t n, const int* order, const float* u_prep,
                    const float* dl, const float* ml, void* work, int8_t* codes, float* wcur, cudaStream_t stream) {
  if (n % 256 || nrow <= 0) return 2;
  SweepBatch b;
  b.count = 1;
  if (!sweep_desc(type, x, nrow, n, order, u_prep, dl, ml, work, codes, wcur, &b.d[0])) return 1;
  return launch_ef_sweep_batch(b, sweep_ctas(nrow), 1, stream);
}

// ---------------------------------------------------------------------------- no-allocation sweep
// For callers that cannot allocate device memory, the sweep can run with its working rows in
// this fixed array instead of a caller workspace.  It is a file-scope device variable, so every
// GPU that loads the library reserves it until the process exits.  Host code must not use the
// name g_noalloc_scratch as an address: on the host it is only a stand-in for the symbol, so
// the device address is looked up once per device with cudaGetSymbolAddress.  All calls share
// the array (the last call's contents stay in it), so calls that overlap on the GPU race.
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

namespace {
constexpr int kMaxNoAllocDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxNoAllocDevices] = {};
}  // namespace

// Device address of the scratch array on the current device; looked up on the first call per
// device (which must therefore not happen during a stream capture) and kept until the process
// exits: a device reset would leave the cached address stale, which the header rules out.
static int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 4;
  if (dev < 0 || dev >= kMaxNoAllocDevices) return 5;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return 4;
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return 0;
}

int launch_ef_sweep_noalloc(int type, const float* x, int64_t nrow, int64_t n, const int* order, const float* u_prep,
                            const float* dl, const float* ml, int8_t* codes, float* wcur, cudaStream_t stream) {
  if (ef_sweep_workspace_bytes(nrow, n) > kNoAllocScratchBytes) return 6;
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  // The sweep writes every error before reading it, so the array's previous contents need
  // no clearing.
  return launch_ef_sweep(type, x, nrow, n, order, u_prep, dl, ml, scratch, codes, wcur, stream);
}

}  // namespace cpk
