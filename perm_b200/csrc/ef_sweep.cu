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

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// Sweep of one 32-row tile of one tensor.  WARPS warps per CTA: warp 0 runs the panels,
// all WARPS warps share the trailing updates (WARPS = 1: one warp does everything and keeps
// the block's errors in registers, many such CTAs per SM hide each other's panel latency;
// WARPS = 8: for launches with few tiles).  Each warp streams the column pairs it updates
// (the U segment and the 32 working rows, 512 bytes a pair) through a 4-stage cp.async ring
// in shared memory, so global latency overlaps the update chains.
template <int WARPS>
__device__ __forceinline__ void sweep_tile(const SweepDesc& t, int tile, float nz) {
  constexpr int ST = 4;
  __shared__ float s_u[32][33];
  __shared__ __align__(16) float2 s_e[WARPS == 1 ? 1 : 32][32];
  __shared__ int s_ord[32];
  __shared__ __align__(16) float4 s_ring[WARPS][ST][32];
  constexpr int NT = 32 * WARPS;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n = t.n, nrow = t.nrow;
  const int row = tile * 32 + lane;
  const bool rv = row < nrow;
  const int npair = n >> 1;
  const int sbw = t.sbw, lo = t.lo, hi = t.hi;
  const int nsub = n / sbw;
  const int* __restrict__ order = t.order;
  const float* __restrict__ UT2 = t.ut2;
  const float* __restrict__ diagU = t.ut2 + (size_t)n * n;
  float2* W = t.work + (size_t)tile * npair * 32;
  const float* xr = t.x + (size_t)row * n;

  // wp = x[:, order]
  for (int kp = warp; kp < npair; kp += WARPS) {
    float2 v = make_float2(0.0f, 0.0f);
    if (rv) {
      v.x = __ldg(xr + __ldg(order + 2 * kp));
      v.y = __ldg(xr + __ldg(order + 2 * kp + 1));
    }
    W[kp * 32 + lane] = v;
  }
  __syncthreads();

  float2 ee[32];
  for (int j0 = 0; j0 < n; j0 += 32) {
    for (int i = threadIdx.x; i < 32 * 32; i += NT) {  // s_u[a][b] = U[j0+a][j0+b]
      const int a = i & 31, b = i >> 5;
      s_u[a][b] = __ldg(UT2 + ((size_t)((j0 + b) >> 1) * n + j0 + a) * 2 + (b & 1));
    }
    if (threadIdx.x < 32) s_ord[threadIdx.x] = __ldg(order + j0 + threadIdx.x);
    __syncthreads();

    if (warp == 0) {
      float w[32], dlv[32], mlv[32];
#pragma unroll
      for (int a = 0; a < 16; a++) {
        const float2 v = W[((j0 >> 1) + a) * 32 + lane];
        w[2 * a] = v.x;
        w[2 * a + 1] = v.y;
      }
      const float* dlr = t.dl + (size_t)row * nsub;
      const float* mlr = t.ml ? t.ml + (size_t)row * nsub : nullptr;
#pragma unroll
      for (int a = 0; a < 32; a++) {  // independent loads, issued ahead of the dependent chain
        const int sidx = s_ord[a] / sbw;
        dlv[a] = rv ? __ldg(dlr + sidx) : 0.0f;
        mlv[a] = (rv && mlr) ? __ldg(mlr + sidx) : 0.0f;
      }
#pragma unroll
      for (int a = 0; a < 32; a++) {
        const int j = s_ord[a];
        int q = 0;
        float e = 0.0f;
        if (dlv[a] != 0.0f) {
          q = clampi(nint((w[a] + mlv[a]) / dlv[a]), lo, hi);
          const float recon = dlv[a] * (float)q - mlv[a];
          e = (w[a] - recon) / __ldg(diagU + j0 + a);
        }
        if (rv) {
          t.codes[(size_t)row * n + j] = (int8_t)q;
          if (t.wout) t.wout[(size_t)row * n + j] = w[a];
        }
        if constexpr (WARPS == 1) ee[a] = make_float2(e, e);
        else s_e[a][lane] = make_float2(e, e);
#pragma unroll
        for (int b = a + 1; b < 32; b++) w[b] = w[b] - e * s_u[a][b];
      }
    }
    if constexpr (WARPS > 1) __syncthreads();

    const int kp0 = (j0 + 32) >> 1;
    const int first = kp0 + warp;
    const int count = first < npair ? (npair - first + WARPS - 1) / WARPS : 0;
    if (count > 0) {
      if constexpr (WARPS > 1) {
#pragma unroll
        for (int a = 0; a < 32; a++) ee[a] = s_e[a][lane];
      }
      // lanes 0-15 fetch the pair's 64 U values, lanes 16-31 its 32 working-row float2s
      auto issue = [&](int i) {
        if (i < count) {
          const int kp = first + i * WARPS;
          const float4* src = lane < 16
              ? reinterpret_cast<const float4*>(UT2 + ((size_t)kp * n + j0) * 2) + lane
              : reinterpret_cast<const float4*>(W + (size_t)kp * 32) + (lane - 16);
          cp_async16(&s_ring[warp][i % ST][lane], src);
        }
        cp_async_commit();
      };
#pragma unroll
      for (int i = 0; i < ST - 1; i++) issue(i);
      for (int i = 0; i < count; i++) {
        issue(i + ST - 1);
        cp_async_wait<ST - 1>();
        __syncwarp();
        const float4* U4 = &s_ring[warp][i % ST][0];
        float2 wv = reinterpret_cast<const float2*>(&s_ring[warp][i % ST][16])[lane];
#pragma unroll
        for (int a4 = 0; a4 < 16; a4++) {
          const float4 u = U4[a4];
          upd2(wv.x, wv.y, ee[2 * a4].x, ee[2 * a4].y, u.x, u.y, nz);
          upd2(wv.x, wv.y, ee[2 * a4 + 1].x, ee[2 * a4 + 1].y, u.z, u.w, nz);
        }
        W[(size_t)(first + i * WARPS) * 32 + lane] = wv;
        __syncwarp();
      }
      cp_async_wait<0>();
    }
    __syncthreads();
  }
}

template <int WARPS>
__global__ void __launch_bounds__(32 * WARPS, WARPS == 1 ? 16 : 2)
ef_sweep_batch_kernel(const __grid_constant__ SweepBatch b, float nz) {
  int lo = 0, hi = b.count - 1;
  const int cta = blockIdx.x;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (b.d[mid].tile0 <= cta) lo = mid;
    else hi = mid - 1;
  }
  sweep_tile<WARPS>(b.d[lo], cta - b.d[lo].tile0, nz);
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

int launch_ef_sweep_batch(const SweepBatch& b, int total_tiles, int warps, cudaStream_t stream) {
  if (b.count == 0 || total_tiles == 0) return 0;
  if (warps == 1) ef_sweep_batch_kernel<1><<<total_tiles, 32, 0, stream>>>(b, -0.0f);
  else ef_sweep_batch_kernel<8><<<total_tiles, 256, 0, stream>>>(b, -0.0f);
  note_launch();
  return 0;
}

bool sweep_desc(int type, const float* x, int64_t nrow, int64_t n, const int* order, const float* ut2,
                const float* dl, const float* ml, void* work, int8_t* codes, float* wcur, SweepDesc* d) {
  int sbw, lo, hi;
  bool has_min;
  if (!grid_spec(type, &sbw, &lo, &hi, &has_min)) return false;
  d->x = x;
  d->order = order;
  d->ut2 = ut2;
  d->dl = dl;
  d->ml = has_min ? ml : nullptr;
  d->work = (float2*)work;
  d->codes = codes;
  d->wout = wcur;
  d->nrow = (int)nrow;
  d->n = (int)n;
  d->sbw = sbw;
  d->lo = lo;
  d->hi = hi;
  d->tile0 = 0;
  return true;
}

int launch_ef_sweep(int type, const float* x, int64_t nrow, int64_t n, const int* order,
                    const float* UT2, const float* diagU, const float* dl, const float* ml, void* work,
                    int8_t* codes, float* wcur, cudaStream_t stream) {
  (void)diagU;
  if (n % 256 || nrow <= 0) return 2;
  SweepBatch b;
  b.count = 1;
  if (!sweep_desc(type, x, nrow, n, order, UT2, dl, ml, work, codes, wcur, &b.d[0])) return 1;
  const int tiles = (int)((nrow + 31) / 32);
  return launch_ef_sweep_batch(b, tiles, tiles >= 2 * 16 * 148 ? 1 : 8, stream);
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
// device (which must therefore not happen during a stream capture).
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

int launch_ef_sweep_noalloc(int type, const float* x, int64_t nrow, int64_t n, const int* order, const float* UT2,
                            const float* dl, const float* ml, int8_t* codes, float* wcur, cudaStream_t stream) {
  if (ef_sweep_workspace_bytes(nrow, n) > kNoAllocScratchBytes) return 6;
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  // The sweep writes every working element of its tiles before reading it, so the array's
  // previous contents need no clearing.
  return launch_ef_sweep(type, x, nrow, n, order, UT2, UT2 + (size_t)n * n, dl, ml, scratch, codes, wcur, stream);
}

}  // namespace cpk
