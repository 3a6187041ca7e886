// H += X^T X for a batch of activations X [T, d] (coldpress/hessians.py:137-152 hook
// arithmetic: `x.float(); acc += x.T @ x`).
//
// Tensor-core kernel for sm_100a on SM pairs: a cluster of two CTAs (one per SM) computes a
// 256 x 256 tile of H with tcgen05.mma.cta_group::2 (kind::f16, bf16 x bf16 -> f32, M = 256,
// N = 256).  Each CTA loads, by TMA (128-byte swizzle, no multicast), its own half of the
// operands into its own shared memory: the 128 rows of A it accumulates and 128 of the 256
// columns of B.  The MMA, issued by one thread of the even CTA, reads both CTAs' halves, so
// each SM fetches 32 KB per 64-token step where a one-SM 128 x 256 tile fetches 48 KB.  Both
// operands come from the same X; along the reduction dimension (tokens) they are MN-major,
// so no transpose is staged.
//
// Pipeline.  Each CTA's producer waits for its own "empty" barrier of a stage, and both CTAs'
// loads complete on the even CTA's "full" barrier of that stage (the cta_group::2 form of the
// TMA load), which the even CTA's producer arms with the bytes of both halves.  The MMA thread
// waits for that barrier, issues four MMAs and commits the stage back to the empty barriers of
// both CTAs.  Every wait is CTA-scoped: the cross-SM signals are the TMA completions and the
// tcgen05 commits themselves.
//
// Accumulation chains.  The tensor core's f32 accumulation does not round to nearest, so its
// error grows with the number of MMAs chained into one accumulator.  The MMA thread therefore
// restarts the accumulation every 8 steps of 64 tokens (32 MMAs), alternating between two
// TMEM accumulators, and the epilogue warps of each CTA add each finished chunk of their 128
// rows into f32 registers with ordinary round-to-nearest adds while the next chunk runs.  The
// error then stays at the level of a float32 matmul for any number of tokens.
//
// Work.  H is symmetric, so only the 256 x 256 tiles on or below the diagonal are computed
// ("pairs" of 128 x 256 halves, one per CTA).  The kernel is persistent, one cluster per SM
// pair, and takes work items round-robin (cluster c: items c, c + G, ...), so the clusters
// that run at the same time work on the same token range and share X through L2.  A regular
// item is one pair tile over one token split; the regular items that would leave part of a
// last round idle are each cut into sub-items, so that round spreads over all SM pairs.  Each
// item's sum is written from registers as a partial tile into its own workspace slot while the
// MMAs of the next item run; a second kernel sums each tile's slots in token order and adds
// the sum to H[i, j] and to the mirror H[j, i] (a diagonal sub-block adds j <= i directly and
// j < i mirrored, so H stays exactly symmetric).  The schedule depends only on T, d and the
// number of SM pairs, so repeated runs give identical bits.
//
// float32 activations.  The reference casts activations to float32 before the product and
// small teachers run in float32.  For those inputs X is first split into two bf16 arrays,
// hi = bf16(x) and lo = bf16(x - hi), and the kernel accumulates
// hi^T hi + hi^T lo + lo^T hi + lo^T lo as four token "phases" into the same TMEM
// accumulator.  That is exactly (hi + lo)^T (hi + lo) with f32 accumulation; hi + lo is
// within 2^-17 relative of x, so the result carries float32-level accuracy.
//
// Every mbarrier wait is bounded (about one second of global time).  A wait that runs out
// sets the workspace status word and the abort words of both CTAs of the pair, which makes
// their other roles stop.  The even CTA's producer then waits (bounded) for the full barriers
// it armed, the odd CTA's producer for the empty barriers of the stages it loaded (committed
// once the MMAs that read them complete, else the bound passes), the MMA thread for its MMAs,
// and both CTAs free their TMEM after a cluster barrier.
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

constexpr int kBM = 128;             // rows of H per CTA (TMEM lanes)
constexpr int kBN = 256;             // tile columns, UMMA N
constexpr int kBK = 64;              // tokens per pipeline stage
constexpr int kStages = 6;
constexpr int kBoxBytes = kBK * 128;                 // one 64-column x 64-token box: 8 KB
constexpr int kHalfBytes = 2 * kBoxBytes;            // 128 columns of X: this CTA's A or B half
constexpr int kStageBytes = 2 * kHalfBytes;          // 32 KB
constexpr int kEpiWarps = 8;                         // two per TMEM lane quarter
constexpr int kThreads = 64 + 32 * kEpiWarps;        // warp 0 TMA, warp 1 MMA (even CTA), warps 2-9 epilogue
constexpr int kChunkSteps = 8;                       // 64-token steps per TMEM accumulation chain
constexpr uint32_t kTmemCols = 2 * kBN;              // two accumulators (double buffer)
constexpr int kSubFloats = kBM * 32;                 // one 32-column group of a CTA's rows
constexpr int kSlotFloats = 2 * 2 * 4 * kSubFloats;  // partial [CTA][sub-block][32-column group][row][32]: 256 KB
constexpr unsigned long long kWaitNs = 1000000000ull;   // default bound of every mbarrier wait
constexpr size_t kSmemBytes = 1024 + (size_t)kStages * kStageBytes + 512;

// UMMA instruction descriptor: f32 accumulate (bits 4-5 = 1), A and B bf16 (bits 7-9, 10-12
// = 1), both MN-major (bits 15, 16), N >> 3 at bits 17-22, M >> 4 at bits 24-28 (M = 256 over
// the CTA pair).
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | (1u << 16) |
                            ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)((2 * kBM) >> 4) << 24);

struct XtxParams {
  float* partial;    // [items][kSlotFloats]
  int* status;       // sticky error word
  unsigned long long wait_ns;   // bound of every mbarrier wait
  int nt;            // 128-blocks of d
  int pairs, splits, per;   // token splits of per steps: regular item i = (split i / pairs, pair i % pairs)
  int full_items;    // regular items run in whole rounds (a multiple of clusters)
  int rem_q, sub_per;   // each later regular item is cut into rem_q sub-items of sub_per steps
  int items;         // full_items + (pairs * splits - full_items) * rem_q
  int clusters;      // CTA pairs of the persistent launch; cluster c takes items c, c + clusters, ...
  int total;         // 64-token steps per pair tile (phases * ki)
  int ki;            // 64-token steps per phase
  int skip_step;     // failure-path tests only: no loads are issued for this 64-token step of
                     // any pair tile, so the waits on its stage run out; -1 = none
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
// Address in the shared::cluster window of the same variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t peer_addr(uint32_t a, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
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
// Arrive on a barrier of the other CTA of the pair (a = shared::cluster address).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t a) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(a) : "memory");
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
// global time) or a role of this CTA pair gave up (abort word nonzero).
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
// Load into this CTA's shared memory, completing on a barrier of either CTA of the pair.
__device__ __forceinline__ void tma_load_pair(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
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
// One M = 256 MMA over the CTA pair: the descriptors' shared-memory offsets address the same
// layout in both CTAs (A rows 0-127 and B columns 0-127 in the even CTA, the rest in the odd).
__device__ __forceinline__ void umma_pair_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accum)
      : "memory");
}
// Arrive on the barrier at shared::cluster address `mbar` once the MMAs issued so far complete.
__device__ __forceinline__ void umma_commit_pair(uint32_t mbar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar) : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int e = 0; e < 16; e++) v[e] = __uint_as_float(r[e]);
}

// Pair index p -> (TI, TJ), TJ <= TI: row block TI holds pairs TJ = 0 .. TI.
__device__ __forceinline__ void pair_coords(int p, int& ti2, int& tj2) {
  int r = 0;
  while ((r + 1) * (r + 2) / 2 <= p) r++;
  ti2 = r;
  tj2 = p - r * (r + 1) / 2;
}

// Item i of a launch -> pair tile p and its steps [gb, ge).  Regular items are (split i / pairs,
// pair i % pairs); the regular items past full_items, which would leave part of a last round
// idle, are cut into rem_q sub-items each, so the last round spreads over all clusters.
struct Seg {
  int p, gb, ge;
};
__device__ __forceinline__ void item_coords(int i, const XtxParams& prm, Seg& sg) {
  int base = i, sub = -1;
  if (i >= prm.full_items) {
    base = prm.full_items + (i - prm.full_items) / prm.rem_q;
    sub = (i - prm.full_items) % prm.rem_q;
  }
  const int k = base / prm.pairs;
  sg.p = base - k * prm.pairs;
  sg.gb = k * prm.per;
  sg.ge = min(prm.total, sg.gb + prm.per);
  if (sub >= 0) {   // a sub-item may be empty (gb >= ge): it then contributes a zero partial
    const int gb = sg.gb + sub * prm.sub_per;
    sg.ge = min(sg.ge, gb + prm.sub_per);
    sg.gb = gb;
  }
}

// A role that gives up stops both CTAs of the pair and records the failure.
__device__ __forceinline__ void fail_pair(volatile int* abort, uint32_t peer_abort, int* status) {
  *abort = 1;
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(peer_abort), "r"(1) : "memory");
  atomicOr(status, 1);
}

__global__ void __launch_bounds__(kThreads, 1)
    xtx_pair_kernel(const __grid_constant__ CUtensorMap map_hi, const __grid_constant__ CUtensorMap map_lo,
                    const XtxParams prm) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // barriers: full[kStages], empty[kStages], acc_full[2], acc_empty[2], mma_done
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + kStages * kStageBytes);
  volatile int* misc = reinterpret_cast<volatile int*>(bars + 2 * kStages + 5);  // [0] tmem, [1] abort
  const uint32_t ring_s = smem_u32(base);
  const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * kStages;
  const uint32_t accf0 = empty0 + 8 * kStages, acce0 = accf0 + 16, done_bar = acce0 + 16;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int c = (int)cluster_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; s++) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(accf0 + 8 * b, 1);
      mbar_init(acce0 + 8 * b, 2 * kEpiWarps);
    }
    mbar_init(done_bar, 1);
    misc[1] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_hi)) : "memory");
    if (prm.total > prm.ki) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_lo)) : "memory");
  }
  if (warp == 1) {
    // both CTAs' warp 1 allocate together: the same columns in both SMs' TMEM
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32((const void*)&misc[0])),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();   // both CTAs' barriers are initialised and their TMEM allocated
  tc_fence_after();
  const uint32_t tmem = (uint32_t)misc[0];
  volatile int* abort = &misc[1];
  const uint32_t peer_abort = peer_addr(smem_u32((const void*)&misc[1]), rank ^ 1u);

  if (warp == 0) {
    // ---- TMA producer (both CTAs): this CTA's A rows and B columns into its own ring; the
    // loads of both CTAs complete on the even CTA's full barrier, which the even CTA arms
    // with both halves' bytes
    if (lane == 0) {
      const uint32_t lead_full0 = peer_addr(full0, 0);
      int last_round[kStages];
      for (int s = 0; s < kStages; s++) last_round[s] = -1;
      Seg sg;
      int it = 0;
      bool ok = true;
      for (int item = c; ok && item < prm.items; item += prm.clusters) {
        item_coords(item, prm, sg);
        int tI, tJ;
        pair_coords(sg.p, tI, tJ);
        for (int g = sg.gb; g < sg.ge; g++, it++) {
          const int st = it % kStages, round = it / kStages;
          if (round > 0 && !mbar_wait(empty0 + 8 * st, (round - 1) & 1, abort, prm.wait_ns)) {
            fail_pair(abort, peer_abort, prm.status);
            ok = false;
            break;
          }
          if (g == prm.skip_step) continue;   // failure-path test: this stage stays empty
          const int phase = g / prm.ki, t0 = (g - phase * prm.ki) * kBK;
          const CUtensorMap* ma = phase < 2 ? &map_hi : &map_lo;
          const CUtensorMap* mb = (phase & 1) ? &map_lo : &map_hi;
          const uint32_t fb = lead_full0 + 8 * st, sa = ring_s + st * kStageBytes, sb = sa + kHalfBytes;
          const bool share = tI == tJ && ma == mb;
          if (leader) mbar_expect_tx(full0 + 8 * st, 2 * (share ? kHalfBytes : kStageBytes));
          if (!share) {
#pragma unroll
            for (int k = 0; k < 2; k++) tma_load_pair(sa + k * kBoxBytes, ma, (2 * tI + (int)rank) * kBM + 64 * k, t0, fb);
          }
#pragma unroll
          for (int k = 0; k < 2; k++) tma_load_pair(sb + k * kBoxBytes, mb, tJ * kBN + (int)rank * 128 + 64 * k, t0, fb);
#pragma unroll
          for (int k = 0; k < kStages; k++)
            if (k == st) last_round[k] = round;
        }
      }
      // every load issued lands before the CTA exits: the even CTA waits for its full
      // barriers, the odd CTA for the MMAs that consumed its loads (or for the wait bound)
#pragma unroll
      for (int st = 0; st < kStages; st++) {
        if (last_round[st] < 0) continue;
        const uint32_t bar = leader ? full0 + 8 * st : empty0 + 8 * st;
        if (!mbar_wait(bar, last_round[st] & 1, abort, prm.wait_ns)) {
          int zero = 0;
          mbar_wait(bar, last_round[st] & 1, &zero, prm.wait_ns);
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer (even CTA): chunk cg accumulates up to kChunkSteps steps into TMEM
    // buffer cg & 1 of both SMs
    if (lane == 0 && leader) {
      const uint32_t peer_empty0 = peer_addr(empty0, 1), peer_accf0 = peer_addr(accf0, 1);
      Seg sg;
      int it = 0, cg = 0;
      bool ok = true;
      for (int item = c; ok && item < prm.items; item += prm.clusters) {
        item_coords(item, prm, sg);
        int tI, tJ;
        pair_coords(sg.p, tI, tJ);
        for (int g0 = sg.gb; g0 < sg.ge && ok; g0 += kChunkSteps, cg++) {
          const int b = cg & 1;
          if (cg >= 2 && !mbar_wait(acce0 + 8 * b, ((cg >> 1) - 1) & 1, abort, prm.wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t acc = tmem + b * kBN;
          const int ge = min(sg.ge, g0 + kChunkSteps);
          for (int g = g0, k = 0; g < ge; g++, it++, k++) {
            const int st = it % kStages, round = it / kStages;
            if (!mbar_wait(full0 + 8 * st, round & 1, abort, prm.wait_ns)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const int phase = g / prm.ki;
            const bool share = tI == tJ && (phase == 0 || phase == 3);   // A and B from the same map
            const uint32_t sb = ring_s + st * kStageBytes + kHalfBytes;
            const uint32_t sa = share ? sb : sb - kHalfBytes;
#pragma unroll
            for (int kk = 0; kk < kBK / 16; kk++) {
              const uint64_t ad = sw128_desc(sa + kk * 2048, kBoxBytes, 1024);
              const uint64_t bd = sw128_desc(sb + kk * 2048, kBoxBytes, 1024);
              umma_pair_bf16(acc, ad, bd, (k | kk) != 0);
            }
            umma_commit_pair(empty0 + 8 * st);
            umma_commit_pair(peer_empty0 + 8 * st);
          }
          if (ok) {
            umma_commit_pair(accf0 + 8 * b);
            umma_commit_pair(peer_accf0 + 8 * b);
          }
        }
      }
      if (!ok) fail_pair(abort, peer_abort, prm.status);
      // all MMAs issued above complete before TMEM is freed and before the odd CTA, whose
      // shared memory they read, may exit
      umma_commit_pair(done_bar);
      int zero = 0;
      mbar_wait(done_bar, 0, &zero, prm.wait_ns);
    }
  } else {
    // ---- epilogue (both CTAs): warp w reads TMEM lanes 32 (w % 4) .. +31 (this CTA's rows
    // of the tile) and the 128 columns of sub-block hh; each chunk is drained into
    // round-to-nearest f32 registers, and each finished segment goes out as a partial tile
    const int ew = warp - 2, q = warp & 3, hh = ew >> 2;
    const uint32_t trow = tmem + ((uint32_t)(32 * q) << 16) + hh * 128;
    const uint32_t lead_acce0 = peer_addr(acce0, 0);
    float m[4][32];
    Seg sg;
    int cg = 0;
    bool ok = true;
    for (int item = c; ok && item < prm.items; item += prm.clusters) {
      item_coords(item, prm, sg);
      int tI, tJ;
      pair_coords(sg.p, tI, tJ);
      const int ti = 2 * tI + (int)rank, tj = 2 * tJ + hh;
      const bool live = ti < prm.nt && tj < prm.nt && tj <= ti;
#pragma unroll
      for (int cc = 0; cc < 4; cc++)
#pragma unroll
        for (int e = 0; e < 32; e++) m[cc][e] = 0.0f;
      for (int g0 = sg.gb; g0 < sg.ge; g0 += kChunkSteps, cg++) {
        const int b = cg & 1;
        const bool got = mbar_wait(accf0 + 8 * b, (cg >> 1) & 1, abort, prm.wait_ns);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (live) {
#pragma unroll
          for (int cc = 0; cc < 4; cc++)
#pragma unroll
            for (int hf = 0; hf < 2; hf++) {
              float v[16];
              tmem_ld16(trow + b * kBN + cc * 32 + hf * 16, v);
#pragma unroll
              for (int e = 0; e < 16; e++) m[cc][hf * 16 + e] += v[e];
            }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (leader)
            mbar_arrive(acce0 + 8 * b);
          else
            mbar_arrive_remote(lead_acce0 + 8 * b);
        }
      }
      if (!ok) break;
      if (live) {
        // this item's sum goes to its partial slot; the reduction adds the splits to H
        float* dst = prm.partial + (size_t)item * kSlotFloats + (size_t)((rank * 2 + hh) * 4) * kSubFloats +
                     (32 * q + lane) * 32;
#pragma unroll
        for (int cc = 0; cc < 4; cc++)
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            __stcg(reinterpret_cast<float4*>(dst + cc * kSubFloats + e),
                   make_float4(m[cc][e], m[cc][e + 1], m[cc][e + 2], m[cc][e + 3]));
      }
    }
    if (!ok) fail_pair(abort, peer_abort, prm.status);
  }
  // Every role is done: the producers have drained their loads and the MMA thread has seen
  // its MMAs complete.  After the cluster barrier neither CTA touches the other's memory.
  __syncwarp();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// Token-split reduction.  One CTA per (pair, CTA half v, sub-block hh, 32-row group rg): it
// sums that 32 x 128 slice of the pair's split partials in split order 0 .. S-1, stages the sum
// in shared memory and adds it to H[i, j] and to the mirror H[j, i] with 128-byte row segments,
// loads batched ahead of stores.
__global__ void __launch_bounds__(256) xtx_reduce_kernel(const float* __restrict__ partial, int pairs, int splits,
                                                         int full_items, int rem_q, float* __restrict__ H, int d,
                                                         int nt) {
  __shared__ float sv[32][129];
  const int p = blockIdx.x >> 4, v = (blockIdx.x >> 3) & 1, hh = (blockIdx.x >> 2) & 1, rg = blockIdx.x & 3;
  int tI, tJ;
  pair_coords(p, tI, tJ);
  const int ti = 2 * tI + v, tj = 2 * tJ + hh;
  if (ti >= nt || tj >= nt || tj > ti) return;
  const int t = threadIdx.x, warp = t / 32, lane = t % 32;
  const int r = t >> 3, f4 = t & 7;
  const int i0 = ti * kBM + rg * 32, j0 = tj * kBM;
  const bool diag = tj == ti;
  float4 acc[4];
#pragma unroll
  for (int cc = 0; cc < 4; cc++) acc[cc] = make_float4(0.f, 0.f, 0.f, 0.f);
  // this pair's slots in token order: regular item k * pairs + p, or its rem_q sub-items
#pragma unroll 1
  for (int k = 0; k < splits; k++) {
    const int i0 = k * pairs + p;
    const int n = i0 < full_items ? 1 : rem_q;
    const int s0 = i0 < full_items ? i0 : full_items + (i0 - full_items) * rem_q;
#pragma unroll 1
    for (int u = 0; u < n; u++) {
      const float* src = partial + (size_t)(s0 + u) * kSlotFloats + (size_t)((v * 2 + hh) * 4) * kSubFloats +
                         (rg * 32 + r) * 32 + 4 * f4;
      float4 w[4];
#pragma unroll
      for (int cc = 0; cc < 4; cc++) w[cc] = __ldcg(reinterpret_cast<const float4*>(src + cc * kSubFloats));
#pragma unroll
      for (int cc = 0; cc < 4; cc++) {
        acc[cc].x += w[cc].x;
        acc[cc].y += w[cc].y;
        acc[cc].z += w[cc].z;
        acc[cc].w += w[cc].w;
      }
    }
  }
#pragma unroll
  for (int cc = 0; cc < 4; cc++) {
    float* row = &sv[r][cc * 32 + 4 * f4];
    row[0] = acc[cc].x;
    row[1] = acc[cc].y;
    row[2] = acc[cc].z;
    row[3] = acc[cc].w;
  }
  __syncthreads();
  // direct: 32 rows x 4 column chunks; warp w takes segments w, w + 8, ... (16 each)
  {
    float h[16];
#pragma unroll
    for (int k = 0; k < 16; k++) {
      const int seg = warp + 8 * k, rr = seg >> 2, i = i0 + rr, j = j0 + (seg & 3) * 32 + lane;
      h[k] = (i < d && j < d && (!diag || j <= i)) ? H[(size_t)i * d + j] : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < 16; k++) {
      const int seg = warp + 8 * k, rr = seg >> 2, cl = (seg & 3) * 32 + lane, i = i0 + rr, j = j0 + cl;
      if (i < d && j < d && (!diag || j <= i)) H[(size_t)i * d + j] = h[k] + sv[rr][cl];
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
      const int cl = warp + 8 * k, j = j0 + cl;
      if (i < d && j < d && (!diag || j < i)) H[(size_t)j * d + i] = h[k] + sv[lane][cl];
    }
  }
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
// Opts the pair kernel into its shared memory once per device; false on failure.
bool opt_in() {
  static std::atomic<unsigned long long> opted{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  if (opted.load() & (1ULL << dev)) return true;
  if (cudaFuncSetAttribute(xtx_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes) !=
      cudaSuccess)
    return false;
  opted.fetch_or(1ULL << dev);
  return true;
}

// SM pairs that can hold a cluster of the pair kernel at once on the current device (cached
// per device; half the SM count when the occupancy query is unavailable).
int pair_capacity(int num_sms) {
  static std::atomic<int> cap[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return num_sms / 2 > 0 ? num_sms / 2 : 1;
  int n = cap[dev].load();
  if (n > 0) return n;
  n = 0;
  if (opt_in()) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = kSmemBytes;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, xtx_pair_kernel, &cfg) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
  }
  if (n <= 0) n = num_sms / 2 > 0 ? num_sms / 2 : 1;
  cap[dev].store(n);
  return n;
}

}  // namespace

XtxPlan xtx_plan(int64_t T, int64_t d, int f32_input, int num_sms) {
  XtxPlan p{};
  p.nt = (int)((d + kBM - 1) / kBM);
  const int nT = (int)((d + kBN - 1) / kBN);
  p.pairs = nT * (nT + 1) / 2;
  p.phases = f32_input ? 4 : 1;
  p.ki = (int)((T + kBK - 1) / kBK);
  p.total = p.phases * p.ki;
  const int cap = pair_capacity(num_sms);
  // cost model (microseconds): whole rounds of regular items (one per cluster) at ~0.42 us per
  // 64-token step of a 256 x 256 pair tile, one last round of sub-items, and the partial
  // tiles' traffic (written and read once, ~6 TB/s)
  int best_s = 1, best_q = 1;
  double best = 1e300;
  const int smax = p.total < 2 ? 1 : (p.total / 2 < 64 ? p.total / 2 : 64);
  for (int s = 1; s <= smax; s++) {
    const int per = (p.total + s - 1) / s;
    if ((p.total + per - 1) / per != s) continue;
    const int items0 = p.pairs * s, full = items0 / cap * cap, rem = items0 - full;
    const int qmax = rem > 0 ? std::max(1, std::min(cap / rem, per)) : 1;
    for (int q = 1; q <= qmax; q++) {
      const int sub = (per + q - 1) / q, slots = full + rem * q;
      const double cost = (double)(full / cap) * per * 0.42 + (rem > 0 ? sub * 0.42 : 0.0) +
                          (double)slots * 2.0 * kSlotFloats * 4 / 6e6;
      if (cost < best - 1e-9) {
        best = cost;
        best_s = s;
        best_q = q;
      }
    }
  }
  p.splits = p.total > 0 ? best_s : 0;
  p.per = p.splits > 0 ? (p.total + best_s - 1) / best_s : 0;
  {
    const int items0 = p.pairs * p.splits;
    p.full_items = items0 / cap * cap;
    p.rem_q = best_q;
    p.sub_per = (p.per + p.rem_q - 1) / p.rem_q;
    p.items = p.full_items + (items0 - p.full_items) * p.rem_q;
  }
  p.clusters = p.items < cap ? p.items : cap;
  // workspace: [status 256 B][partials][hi][lo]
  p.off_partial = 256;
  p.off_hi = p.off_partial + (size_t)p.items * kSlotFloats * 4;
  const size_t half = f32_input ? (((size_t)T * d * 2 + 255) / 256) * 256 : 0;
  p.off_lo = p.off_hi + half;
  p.ws_bytes = p.off_lo + half;
  return p;
}

int launch_xtx(const void* x, int f32_input, int64_t T, int64_t d, float* H, void* ws, const XtxPlan& p,
               cudaStream_t stream, int skip_step, unsigned long long wait_ns) {
  if (p.items == 0) return 0;
  if (!opt_in()) return 1;
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
  prm.partial = reinterpret_cast<float*>(w + p.off_partial);
  prm.status = reinterpret_cast<int*>(w);
  prm.wait_ns = wait_ns ? wait_ns : kWaitNs;
  prm.nt = p.nt;
  prm.pairs = p.pairs;
  prm.splits = p.splits;
  prm.per = p.per;
  prm.full_items = p.full_items;
  prm.rem_q = p.rem_q;
  prm.sub_per = p.sub_per;
  prm.items = p.items;
  prm.clusters = p.clusters;
  prm.total = p.total;
  prm.ki = p.ki;
  prm.skip_step = skip_step;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * (unsigned)p.clusters, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, xtx_pair_kernel, mh, ml, prm) != cudaSuccess) return 1;
  note_launch();
  xtx_reduce_kernel<<<p.pairs * 16, 256, 0, stream>>>(reinterpret_cast<const float*>(w + p.off_partial), p.pairs,
                                                     p.splits, p.full_items, p.rem_q, H, (int)d, p.nt);
  note_launch();
  return 0;
}

}  // namespace cpk
