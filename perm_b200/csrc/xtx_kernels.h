// Internal launcher declarations for X^T X accumulation.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace cpk {

// Launch shape and workspace layout of one X^T X call (all offsets in bytes).
struct XtxPlan {
  int nt;               // 128-wide blocks of d
  int pairs;            // 256 x 256 tiles on or below the diagonal (one CTA pair each)
  int phases;           // 1 (bf16 input) or 4 (float32 input split into hi/lo bf16)
  int ki;               // 64-token steps per phase
  int total;            // 64-token steps per pair tile (phases * ki)
  int splits;           // token splits
  int per;              // 64-token steps per split
  int full_items;       // regular (split, pair) items run in whole rounds
  int rem_q, sub_per;   // the remaining regular items are cut into rem_q sub-items of sub_per steps
  int items;            // full_items + remaining regular items * rem_q
  int clusters;         // CTA pairs of the persistent launch
  size_t off_partial, off_hi, off_lo, ws_bytes;
};

XtxPlan xtx_plan(int64_t T, int64_t d, int f32_input, int num_sms);
// skip_step >= 0 (failure-path tests only): no loads are issued for that 64-token step, so
// the waits on it run out after wait_ns (0: the default bound of about one second).
int launch_xtx(const void* x, int f32_input, int64_t T, int64_t d, float* H, void* ws, const XtxPlan& p,
               cudaStream_t stream, int skip_step = -1, unsigned long long wait_ns = 0);

}  // namespace cpk
