// Internal launcher declarations for X^T X accumulation.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace cpk {

// Launch shape and workspace layout of one X^T X call (all offsets in bytes).
struct XtxPlan {
  int nt;               // 128-wide blocks of d
  int tiles;            // 128 x 256 tiles on or below the diagonal
  int phases;           // 1 (bf16 input) or 4 (float32 input split into hi/lo bf16)
  int ki;               // 64-token steps per phase
  int splits;           // token splits
  int steps_per_split;
  size_t off_partial, off_hi, off_lo, ws_bytes;
};

XtxPlan xtx_plan(int64_t T, int64_t d, int f32_input, int num_sms);
// skip_step >= 0 (failure-path tests only): no loads are issued for that 64-token step, so
// the waits on it run out after wait_ns (0: the default bound of about one second).
int launch_xtx(const void* x, int f32_input, int64_t T, int64_t d, float* H, void* ws, const XtxPlan& p,
               cudaStream_t stream, int skip_step = -1, unsigned long long wait_ns = 0);

}  // namespace cpk
