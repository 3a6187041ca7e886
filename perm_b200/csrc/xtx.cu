// H += X^T X for a batch of activations X [T, d] (coldpress/hessians.py:137-152 hook
// arithmetic: `x.float(); acc += x.T @ x`).
//
// Tensor-core kernel for sm_100a: TMA loads of X tiles (128-byte swizzle) into a 4-stage
// shared-memory ring, tcgen05.mma (kind::f16, bf16 x bf16 -> f32) issued by one thread with
// the accumulator in TMEM, tcgen05.ld epilogue.  Both operands come from the same X; along
// the GEMM's reduction dimension (tokens) they are MN-major, so no transpose is staged.
//
// Accumulation chains.  The tensor core's f32 accumulation does not round to nearest, so its
// error grows with the number of MMAs chained into one accumulator.  The MMA thread therefore
// restarts the accumulation every 8 steps of 64 tokens (32 MMAs), alternating between two
// TMEM accumulators, and the epilogue warps add each finished chunk into f32 registers with
// ordinary round-to-nearest adds while the next chunk runs.  The error then stays at the
// level of a float32 matmul for any number of tokens.
//
// Work units.  H is symmetric, so only tiles on or below the diagonal are computed: a CTA
// owns a 128 x 256 tile (rows i in 128-block ti, columns j in 128-blocks 2p and 2p+1 with
// 2p <= ti) over one token split.  Its epilogue adds the 128 x 128 sub-blocks with tj < ti
// to H[i, j] and to H[j, i]; a diagonal sub-block adds its lower triangle twice the same way
// (the strict upper part comes from the mirror), so H stays exactly symmetric; sub-blocks
// above the diagonal are dropped.
//
// Write-out.  After the last chunk the tile is staged row-major in the (now idle) TMA ring in
// shared memory, so that both H[i, j] and the mirror H[j, i] are updated with coalesced
// 128-byte row segments, loads batched ahead of stores.
//
// Token splits.  When there are too few tiles to fill the SMs, tokens are cut into S splits
// of whole 64-token steps.  Each split CTA writes its f32 partial tile to the workspace; a
// second kernel (eight CTAs per tile) sums the S partials in split order 0..S-1 and adds the
// sum to H the same way.  Repeated runs give identical bits and no CTA waits for another.
//
// float32 activations.  The reference casts activations to float32 before the product and
// small teachers run in float32.  For those inputs X is first split into two bf16 arrays,
// hi = bf16(x) and lo = bf16(x - hi), and the kernel accumulates
// hi^T hi + hi^T lo + lo^T hi + lo^T lo as four token "phases" into the same TMEM
// accumulator.  That is exactly (hi + lo)^T (hi + lo) with f32 accumulation; hi + lo is
// within 2^-17 relative of x, so the result carries float32-level accuracy.
//
// Every mbarrier wait is bounded (about one second of global time).  A wait that runs out
// sets the workspace status word, makes the CTA's other roles stop, drains the TMA loads it
// issued, frees its TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <atomic>
#include <mutex>
#include "xtx_kernels.h"
#include "kquant_kernels.h"

namespace cpk {
namespace {

constexpr int kBM = 128;             // tile rows (i), UMMA M
constexpr int kBN = 256;             // tile columns (j), UMMA N
constexpr int kBK = 64;              // tokens per pipeline stage
constexpr int kStages = 4;
constexpr int kBoxBytes = kBK * 128;                 // one 64-column x 64-token box: 8 KB
constexpr int kABytes = kBM / 64 * kBoxBytes;        // 16 KB
constexpr int kBBytes = kBN / 64 * kBoxBytes;        // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;       // 48 KB
constexpr int kEpiWarps = 8;                         // two per TMEM lane quarter
constexpr int kThreads = 64 + 32 * kEpiWarps;        // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
constexpr int kChunkSteps = 8;                       // 64-token steps per TMEM accumulation chain
constexpr uint32_t kTmemCols = 2 * kBN;              // two accumulators (double buffer)
constexpr int kPartialFloats = kBM * kBN;            // 128 KB per (tile, split) partial
constexpr unsigned long long kWaitNs = 1000000000ull;   // default bound of every mbarrier wait
constexpr size_t kSmemBytes = 1024 + (size_t)kStages * kStageBytes + 256;

// UMMA instruction descriptor: f32 accumulate (bits 4-5 = 1), A and B bf16 (bits 7-9, 10-12
// = 1), both MN-major (bits 15, 16), N >> 3 at bits 17-22, M >> 4 at bits 24-28.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | (1u << 16) |
                            ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);

struct XtxParams {
  float* H;
  int d, nt, tiles, splits, phases;
  int ki;            // 64-token steps per phase
  int steps_per_split;
  float* partial;    // [splits][tiles][2][4][128][32] when splits > 1
  int* status;       // sticky error word
  unsigned long long wait_ns;   // bound of every mbarrier wait
  int skip_step;     // failure-path tests only: the producer issues no loads for this 64-token
                     // step (its stage is never filled, so the waits on it run out); -1 = none
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t a, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t a, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t a) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(a) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t a, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(a), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with the given parity.  False when it ran out (limit_ns of
// global time) or another role of this CTA gave up (abort word nonzero).
__device__ __forceinline__ bool mbar_wait(uint32_t a, uint32_t parity, volatile int* abort,
                                          unsigned long long limit_ns) {
  if (mbar_try(a, parity)) return true;
  const unsigned long long t0 = gtime();
  for (uint32_t n = 1; n < (1u << 30); n++) {
    if (mbar_try(a, parity)) return true;
    if ((n & 255) == 0 && (*abort || gtime() - t0 > limit_ns)) return false;
  }
  return false;
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(mbar)
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, 128-byte swizzle, MN-major: rows of 64 bf16 (128 B) at a
// 128 B pitch, 8-row groups SBO bytes apart, 64-column atoms LBO bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) | (2ull << 61);
}
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accum)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar) : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int e = 0; e < 32; e++) v[e] = __uint_as_float(r[e]);
}

// Named barrier 1 over the epilogue warps; epi_all is true on all of them when v holds on
// each of them.
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, %0;" ::"n"(32 * kEpiWarps) : "memory"); }
__device__ __forceinline__ bool epi_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(32 * kEpiWarps)
      : "memory");
  return r != 0;
}

// Tile index -> (ti, p): row block ti holds tiles p = 0 .. ti/2.
__device__ __forceinline__ void tile_coords(int tile, int& ti, int& p) {
  int t = tile, r = 0;
  while (t >= r / 2 + 1) {
    t -= r / 2 + 1;
    r++;
  }
  ti = r;
  p = t;
}

// Adds a staged 128 x 256 tile (shared memory, row pitch `pitch` floats, columns 0-127 =
// sub-block 2tp, 128-255 = sub-block 2tp+1) to H[i, j] and to the mirror H[j, i].  Sub-blocks
// above the diagonal or past d are skipped; a diagonal sub-block adds j <= i directly and
// j < i mirrored, so H stays exactly symmetric.  kEpiWarps warps cooperate; every warp-wide
// access is a 128-byte row segment, and each group of 8 loads is issued before its stores.
__device__ __forceinline__ void add_tile_to_h(float* __restrict__ H, int d, int ti, int tp, int nt,
                                              const float* tile_s, int pitch, int warp_id, int lane) {
  const int i0 = ti * kBM;
#pragma unroll 1
  for (int hh = 0; hh < 2; hh++) {
    const int tj = 2 * tp + hh;
    if (tj > ti || tj >= nt) continue;
    const bool diag = tj == ti;
    const int j0 = tj * kBM;
    // direct: 128 rows x 4 column chunks = 512 row segments, 64 per warp, 8 loads in flight
#pragma unroll 1
    for (int base_seg = warp_id; base_seg < kBM * 4; base_seg += 8 * kEpiWarps) {
      float h[8];
#pragma unroll
      for (int k = 0; k < 8; k++) {
        const int seg = base_seg + k * kEpiWarps, r = seg >> 2, j = j0 + (seg & 3) * 32 + lane, i = i0 + r;
        h[k] = (i < d && j < d && (!diag || j <= i)) ? H[(size_t)i * d + j] : 0.0f;
      }
#pragma unroll
      for (int k = 0; k < 8; k++) {
        const int seg = base_seg + k * kEpiWarps, r = seg >> 2, c = (seg & 3) * 32 + lane, j = j0 + c, i = i0 + r;
        if (i < d && j < d && (!diag || j <= i)) H[(size_t)i * d + j] = h[k] + tile_s[r * pitch + hh * 128 + c];
      }
    }
    // mirror: 128 columns x 4 row groups of 32, lanes over rows
#pragma unroll 1
    for (int base_seg = warp_id; base_seg < kBM * 4; base_seg += 8 * kEpiWarps) {
      float h[8];
#pragma unroll
      for (int k = 0; k < 8; k++) {
        const int seg = base_seg + k * kEpiWarps, c = seg >> 2, r = (seg & 3) * 32 + lane, j = j0 + c, i = i0 + r;
        h[k] = (i < d && j < d && (!diag || j < i)) ? H[(size_t)j * d + i] : 0.0f;
      }
#pragma unroll
      for (int k = 0; k < 8; k++) {
        const int seg = base_seg + k * kEpiWarps, c = seg >> 2, r = (seg & 3) * 32 + lane, j = j0 + c, i = i0 + r;
        if (i < d && j < d && (!diag || j < i)) H[(size_t)j * d + i] = h[k] + tile_s[r * pitch + hh * 128 + c];
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    xtx_tc_kernel(const __grid_constant__ CUtensorMap map_hi, const __grid_constant__ CUtensorMap map_lo,
                  const XtxParams prm) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // barriers: full[kStages], empty[kStages], acc_full[2], acc_empty[2], mma_done
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + kStages * kStageBytes);
  volatile int* misc = reinterpret_cast<volatile int*>(bars + 2 * kStages + 5);  // [0] tmem, [1] abort
  const uint32_t ring_s = smem_u32(base);
  const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * kStages;
  const uint32_t accf0 = full0 + 16 * kStages, acce0 = accf0 + 16, done_bar = acce0 + 16;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int split = blockIdx.x / prm.tiles, tile = blockIdx.x % prm.tiles;
  int ti, tp;
  tile_coords(tile, ti, tp);
  // A (rows of block ti) is a slice of B (blocks 2tp, 2tp+1) on tiles that reach the diagonal,
  // in the phases whose A and B come from the same array (hi.hi and lo.lo)
  const bool a_in_b = (ti >> 1) == tp;
  const int total = prm.phases * prm.ki;
  const int g0 = split * prm.steps_per_split;
  const int g1 = min(total, g0 + prm.steps_per_split);
  const int nchunks = (g1 - g0 + kChunkSteps - 1) / kChunkSteps;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; s++) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(accf0 + 8 * b, 1);
      mbar_init(acce0 + 8 * b, kEpiWarps);
    }
    mbar_init(done_bar, 1);
    misc[1] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_hi)) : "memory");
    if (prm.phases > 1) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_lo)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32((const void*)&misc[0])),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = (uint32_t)misc[0];
  volatile int* abort = &misc[1];
  float m_out[4][32];   // epilogue warps: this thread's row of its sub-block, round-to-nearest sums
#pragma unroll
  for (int cc = 0; cc < 4; cc++)
#pragma unroll
    for (int e = 0; e < 32; e++) m_out[cc][e] = 0.0f;

  if (warp == 0) {
    // ---- TMA producer
    if (lane == 0) {
      int last_round[kStages];
      for (int s = 0; s < kStages; s++) last_round[s] = -1;
      for (int g = g0, it = 0; g < g1; g++, it++) {
        const int st = it % kStages, round = it / kStages;
        if (round > 0 && !mbar_wait(empty0 + 8 * st, (round - 1) & 1, abort, prm.wait_ns)) {
          *abort = 1;
          atomicOr(prm.status, 1);
          break;
        }
        if (g == prm.skip_step) continue;   // failure-path test: this stage stays empty
        const int phase = g / prm.ki, t0 = (g % prm.ki) * kBK;
        const CUtensorMap* ma = phase < 2 ? &map_hi : &map_lo;
        const CUtensorMap* mb = (phase & 1) ? &map_lo : &map_hi;
        const uint32_t fb = full0 + 8 * st, sa = ring_s + st * kStageBytes, sb = sa + kABytes;
        const bool share = a_in_b && ma == mb;
        mbar_expect_tx(fb, share ? kBBytes : kStageBytes);
        if (!share) {
#pragma unroll
          for (int c = 0; c < kBM / 64; c++) tma_load_2d(sa + c * kBoxBytes, ma, ti * kBM + 64 * c, t0, fb);
        }
#pragma unroll
        for (int c = 0; c < kBN / 64; c++) tma_load_2d(sb + c * kBoxBytes, mb, tp * kBN + 64 * c, t0, fb);
        last_round[st] = round;
      }
      // every load this thread issued lands before the CTA exits
      for (int s = 0; s < kStages; s++)
        if (last_round[s] >= 0 && !mbar_wait(full0 + 8 * s, last_round[s] & 1, abort, prm.wait_ns)) {
          int zero = 0;
          mbar_wait(full0 + 8 * s, last_round[s] & 1, &zero, prm.wait_ns);
        }
    }
  } else if (warp == 1) {
    // ---- MMA issuer: chunk c accumulates kChunkSteps steps into TMEM buffer c & 1
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int c = 0; c < nchunks && ok; c++) {
        const int b = c & 1;
        if (c >= 2 && !mbar_wait(acce0 + 8 * b, ((c >> 1) - 1) & 1, abort, prm.wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + b * kBN;
        const int ge = min(g1, g0 + (c + 1) * kChunkSteps);
        for (int g = g0 + c * kChunkSteps, k = 0; g < ge; g++, it++, k++) {
          const int st = it % kStages, round = it / kStages;
          if (!mbar_wait(full0 + 8 * st, round & 1, abort, prm.wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int phase = g / prm.ki;
          const bool share = a_in_b && (phase == 0 || phase == 3);   // A and B from the same map
          const uint32_t sb = ring_s + st * kStageBytes + kABytes;
          const uint32_t sa = share ? sb + (ti & 1) * 2 * kBoxBytes : sb - kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; kk++) {
            const uint64_t ad = sw128_desc(sa + kk * 2048, kBoxBytes, 1024);
            const uint64_t bd = sw128_desc(sb + kk * 2048, kBoxBytes, 1024);
            umma_bf16(acc, ad, bd, (k | kk) != 0);
          }
          umma_commit(empty0 + 8 * st);
        }
        if (ok) umma_commit(accf0 + 8 * b);
      }
      if (!ok) {
        *abort = 1;
        atomicOr(prm.status, 1);
      }
      // all MMAs issued above complete before TMEM is freed
      umma_commit(done_bar);
      int zero = 0;
      mbar_wait(done_bar, 0, &zero, prm.wait_ns);
    }
  } else {
    // ---- epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 (tile rows) and the 128
    // columns of sub-block hh; each chunk is drained into round-to-nearest f32 registers
    const int ew = warp - 2, q = warp & 3, hh = ew >> 2, tj = 2 * tp + hh;
    const bool live = tj <= ti && tj < prm.nt;
    const uint32_t trow = tmem + ((uint32_t)(32 * q) << 16) + hh * 128;
    float(&m)[4][32] = m_out;
    bool ok = true;
    for (int c = 0; c < nchunks; c++) {
      const int b = c & 1;
      const bool got = mbar_wait(accf0 + 8 * b, (c >> 1) & 1, abort, prm.wait_ns);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (live) {
#pragma unroll
        for (int cc = 0; cc < 4; cc++) {
          float v[32];
          tmem_ld32(trow + b * kBN + cc * 32, v);
#pragma unroll
          for (int e = 0; e < 32; e++) m[cc][e] += v[e];
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce0 + 8 * b);
    }
    if (!ok) {
      *abort = 1;
      atomicOr(prm.status, 1);
    }
  }
  // The producer has drained its loads and every MMA has completed: the ring is free and
  // the TMEM accumulators can go.
  __syncwarp();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
  if (warp < 2) return;
  // ---- write-out through shared memory: tile[r][c], row pitch kBN + 1 floats
  float* tile_s = reinterpret_cast<float*>(base);
  const int et = threadIdx.x - 64, ew = et / 32;
  const bool go = epi_all(!*abort);
  if (!go) return;
  {
    const int q = warp & 3, hh = ew >> 2, r = 32 * q + lane;
#pragma unroll
    for (int cc = 0; cc < 4; cc++)
#pragma unroll
      for (int e = 0; e < 32; e++) tile_s[r * (kBN + 1) + hh * 128 + cc * 32 + e] = m_out[cc][e];
  }
  epi_sync();
  if (prm.splits > 1) {
    // partial (split, tile) as row-major [128][256]: one warp per row
    float* dst = prm.partial + ((size_t)split * prm.tiles + tile) * kPartialFloats;
    for (int r = ew; r < kBM; r += kEpiWarps)
#pragma unroll
      for (int c = lane; c < kBN; c += 32) dst[r * kBN + c] = tile_s[r * (kBN + 1) + c];
    return;
  }
  add_tile_to_h(prm.H, prm.d, ti, tp, prm.nt, tile_s, kBN + 1, ew, lane);
}

// Token-split reduction.  One CTA per (tile, sub-block hh, 32-row group): it sums that
// 32 x 128 slice of the partials of splits 0 .. S-1 in that order (partials are row-major
// [128][256]), stages the sum in shared memory and adds it to H[i, j] and to the mirror
// H[j, i] with 128-byte row segments, loads batched ahead of stores.
__global__ void __launch_bounds__(256) xtx_reduce_kernel(const float* __restrict__ partial, int splits, int tiles,
                                                         float* __restrict__ H, int d, int nt) {
  __shared__ float sv[32][129];
  const int tile = blockIdx.x >> 3, hh = (blockIdx.x >> 2) & 1, rg = blockIdx.x & 3;
  int ti, tp;
  tile_coords(tile, ti, tp);
  const int tj = 2 * tp + hh;
  if (tj > ti || tj >= nt) return;
  const int t = threadIdx.x, warp = t / 32, lane = t % 32;
  const int i0 = ti * kBM + rg * 32, j0 = tj * kBM;
  const bool diag = tj == ti;
  // slice = 32 rows x 32 float4; thread t takes float4 t + 256 k: row (t + 256 k) / 32, column lane
  float4 acc[4];
#pragma unroll 1
  for (int s = 0; s < splits; s++) {
    const float4* src = reinterpret_cast<const float4*>(partial + ((size_t)s * tiles + tile) * kPartialFloats +
                                                        (size_t)(rg * 32) * kBN + hh * 128);
    float4 w[4];
#pragma unroll
    for (int k = 0; k < 4; k++) w[k] = __ldcg(src + (size_t)(warp + 8 * k) * (kBN / 4) + lane);
#pragma unroll
    for (int k = 0; k < 4; k++) {
      if (s == 0) {
        acc[k] = w[k];
      } else {
        acc[k].x += w[k].x;
        acc[k].y += w[k].y;
        acc[k].z += w[k].z;
        acc[k].w += w[k].w;
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 4; k++) {
    float* row = &sv[warp + 8 * k][4 * lane];
    row[0] = acc[k].x;
    row[1] = acc[k].y;
    row[2] = acc[k].z;
    row[3] = acc[k].w;
  }
  __syncthreads();
  // direct: 32 rows x 4 column chunks; warp w takes segments w, w + 8, ... (16 each)
  {
    float h[16];
#pragma unroll
    for (int k = 0; k < 16; k++) {
      const int seg = warp + 8 * k, r = seg >> 2, i = i0 + r, j = j0 + (seg & 3) * 32 + lane;
      h[k] = (i < d && j < d && (!diag || j <= i)) ? H[(size_t)i * d + j] : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < 16; k++) {
      const int seg = warp + 8 * k, r = seg >> 2, c = (seg & 3) * 32 + lane, i = i0 + r, j = j0 + c;
      if (i < d && j < d && (!diag || j <= i)) H[(size_t)i * d + j] = h[k] + sv[r][c];
    }
  }
  // mirror: 128 columns j, lanes over the 32 rows i; warp w takes columns w, w + 8, ...
  {
    const int i = i0 + lane;
    float h[16];
#pragma unroll
    for (int k = 0; k < 16; k++) {
      const int j = j0 + warp + 8 * k;
      h[k] = (i < d && j < d && (!diag || j < i)) ? H[(size_t)j * d + i] : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < 16; k++) {
      const int c = warp + 8 * k, j = j0 + c;
      if (i < d && j < d && (!diag || j < i)) H[(size_t)j * d + i] = h[k] + sv[lane][c];
    }
  }
  (void)tiles;
}

// float32 activations -> hi = bf16(x), lo = bf16(x - hi), four elements per thread.
__global__ void __launch_bounds__(256) xtx_split_kernel(const float4* __restrict__ x, size_t n4,
                                                        uint2* __restrict__ hi, uint2* __restrict__ lo) {
  for (size_t k = blockIdx.x * (size_t)blockDim.x + threadIdx.x; k < n4; k += (size_t)gridDim.x * blockDim.x) {
    const float4 v = x[k];
    const __nv_bfloat162 h01 = __floats2bfloat162_rn(v.x, v.y), h23 = __floats2bfloat162_rn(v.z, v.w);
    const float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
    const __nv_bfloat162 l01 = __floats2bfloat162_rn(v.x - f01.x, v.y - f01.y);
    const __nv_bfloat162 l23 = __floats2bfloat162_rn(v.z - f23.x, v.w - f23.y);
    hi[k] = make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h23));
    lo[k] = make_uint2(*reinterpret_cast<const uint32_t*>(&l01), *reinterpret_cast<const uint32_t*>(&l23));
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int make_map(CUtensorMap* m, const void* x, int64_t T, int64_t d) {
  auto fn = encode_fn();
  if (!fn) return 2;
  const cuuint64_t dims[2] = {(cuuint64_t)d, (cuuint64_t)T};
  const cuuint64_t strides[1] = {(cuuint64_t)d * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)kBK};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : 3;
}

}  // namespace

XtxPlan xtx_plan(int64_t T, int64_t d, int f32_input, int num_sms) {
  XtxPlan p{};
  p.nt = (int)((d + kBM - 1) / kBM);
  p.tiles = 0;
  for (int ti = 0; ti < p.nt; ti++) p.tiles += ti / 2 + 1;
  p.phases = f32_input ? 4 : 1;
  p.ki = (int)((T + kBK - 1) / kBK);
  const int total = p.phases * p.ki;
  // cost model (microseconds): waves x steps per split at ~0.42 us per 64-token step of a
  // 128 x 256 tile, plus, with splits, the partial tiles' traffic (written and read once,
  // ~6 TB/s) and the reduction launch
  int best_s = 1;
  double best = 1e300;
  const int smax = total < 2 ? 1 : (total / 2 < 32 ? total / 2 : 32);
  for (int s = 1; s <= smax; s++) {
    const int per = (total + s - 1) / s;
    const int s_eff = (total + per - 1) / per;
    if (s_eff != s) continue;
    const double waves = (double)((p.tiles * (int64_t)s + num_sms - 1) / num_sms);
    double cost = waves * per * 0.42;
    if (s > 1) cost += (double)p.tiles * s * 2.0 * kPartialFloats * 4 / 6e6 + 4.0;
    if (cost < best - 1e-9) {
      best = cost;
      best_s = s;
    }
  }
  p.splits = best_s;
  p.steps_per_split = (total + best_s - 1) / best_s;
  // workspace: [status 256 B][partials][hi][lo]
  p.off_partial = 256;
  p.off_hi = p.off_partial + (p.splits > 1 ? (size_t)p.splits * p.tiles * kPartialFloats * 4 : 0);
  const size_t half = f32_input ? (((size_t)T * d * 2 + 255) / 256) * 256 : 0;
  p.off_lo = p.off_hi + half;
  p.ws_bytes = p.off_lo + half;
  return p;
}

int launch_xtx(const void* x, int f32_input, int64_t T, int64_t d, float* H, void* ws, const XtxPlan& p,
               cudaStream_t stream, int skip_step, unsigned long long wait_ns) {
  {  // the kernel's dynamic shared memory exceeds the 48 KB default: opt in once per device
    static std::atomic<unsigned long long> opted{0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1;
    if (!(opted.load() & (1ULL << dev))) {
      if (cudaFuncSetAttribute(xtx_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes) !=
          cudaSuccess)
        return 1;
      opted.fetch_or(1ULL << dev);
    }
  }
  uint8_t* w = static_cast<uint8_t*>(ws);
  const void* hi = x;
  const void* lo = x;
  if (f32_input) {
    hi = w + p.off_hi;
    lo = w + p.off_lo;
    const size_t n4 = (size_t)T * d / 4;
    const int grid = (int)std::min<size_t>((n4 + 255) / 256, (size_t)148 * 16);
    xtx_split_kernel<<<grid, 256, 0, stream>>>(static_cast<const float4*>(x), n4, (uint2*)(w + p.off_hi),
                                               (uint2*)(w + p.off_lo));
    note_launch();
  }
  CUtensorMap mh, ml;
  if (int rc = make_map(&mh, hi, T, d)) return rc;
  if (int rc = make_map(&ml, lo, T, d)) return rc;
  XtxParams prm;
  prm.H = H;
  prm.d = (int)d;
  prm.nt = p.nt;
  prm.tiles = p.tiles;
  prm.splits = p.splits;
  prm.phases = p.phases;
  prm.ki = p.ki;
  prm.steps_per_split = p.steps_per_split;
  prm.partial = reinterpret_cast<float*>(w + p.off_partial);
  prm.status = reinterpret_cast<int*>(w);
  prm.wait_ns = wait_ns ? wait_ns : kWaitNs;
  prm.skip_step = skip_step;
  xtx_tc_kernel<<<p.tiles * p.splits, kThreads, kSmemBytes, stream>>>(mh, ml, prm);
  note_launch();
  if (p.splits > 1) {
    xtx_reduce_kernel<<<p.tiles * 8, 256, 0, stream>>>(reinterpret_cast<const float*>(w + p.off_partial), p.splits,
                                                       p.tiles, H, (int)d, p.nt);
    note_launch();
  }
  return 0;
}

}  // namespace cpk
