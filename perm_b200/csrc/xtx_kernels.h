// Internal launcher declarations for X^T X accumulation.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace cpk {
int launch_xtx(const uint16_t* x_bf16, int64_t T, int64_t d, float* H, cudaStream_t stream);
}  // namespace cpk
