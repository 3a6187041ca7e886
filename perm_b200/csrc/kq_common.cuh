// Device helpers that reproduce coldpress's numpy float32 semantics bit for bit
// (coldpress/kquant.py).  Every translation unit that includes this header is compiled with
// -fmad=false, so each `a * b + c` rounds twice exactly like numpy's elementwise ufuncs.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

namespace cpk {

constexpr int kQK = 256;
constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23, kquant.py:28
constexpr float kGroupEps = 1e-15f;    // kquant.py:18

// GGML type ids (ggml.h enum ggml_type) used on the C ABI.
enum TypeId : int { kQ8_0 = 8, kQ2_K = 10, kQ3_K = 11, kQ4_K = 12, kQ5_K = 13, kQ6_K = 14 };

__host__ __device__ constexpr int block_bytes(int t) {
  return t == kQ2_K ? 84 : t == kQ3_K ? 110 : t == kQ4_K ? 144 : t == kQ5_K ? 176
       : t == kQ6_K ? 210 : t == kQ8_0 ? 34 : 0;
}

// nearest_int (kquant.py:25-28): magic add, low 23 bits, re-centre.  A NaN sum is treated
// as the x86 default NaN (payload 0x400000), which is what numpy produces on the host.
__device__ __forceinline__ int32_t nint(float x) {
  float y = __fadd_rn(x, kMagic);
  int32_t r = (__float_as_int(y) & 0x007FFFFF) - 0x00400000;
  return (y != y) ? 0 : r;
}

// clip(nearest_int(v), lo, hi) returned as float.  Works on the bit pattern of v + magic:
// (bits & 0x7FFFFF) | 0x4B000000 is the float 2^23 + low23, clamped in that domain, and
// subtracting the magic gives low23 - 2^22 exactly.  Matches the integer path for every
// non-NaN v, including the wrap-around of |v| >= 2^22.
__device__ __forceinline__ float nint_clip_f(float v, int lo, int hi) {
  float y = __fadd_rn(v, kMagic);
  int b = (__float_as_int(y) & 0x007FFFFF) | 0x4B000000;
  b = max(b, 0x4B400000 + lo);
  b = min(b, 0x4B400000 + hi);
  return __fsub_rn(__int_as_float(b), kMagic);
}

__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

// np.maximum.reduce / np.minimum.reduce step over <= 16 elements: later equal value wins.
__device__ __forceinline__ float np_max_step(float acc, float v) { return (acc > v || acc != acc) ? acc : v; }
__device__ __forceinline__ float np_min_step(float acc, float v) { return (acc < v || acc != acc) ? acc : v; }
// np.minimum(a, b) elementwise.
__device__ __forceinline__ float np_minimum(float a, float b) { return (a < b || a != a) ? a : b; }

// numpy pairwise sum of a contiguous row of N (8, 16 or 32) float32 values fed in index
// order: 8 accumulators, r[j] += a[8k + j], then ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)),
// then the reduction's +0 identity.
struct Pw8 {
  float r[8];
  template <int I> __device__ __forceinline__ void add(float v) {
    if (I < 8) r[I] = v; else r[I & 7] = r[I & 7] + v;
  }
  __device__ __forceinline__ void addi(int i, float v) {  // i must be a compile-time constant after unrolling
    if (i < 8) r[i] = v; else r[i & 7] = r[i & 7] + v;
  }
  __device__ __forceinline__ float total() const {
    float res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
    return 0.0f + res;
  }
  __device__ __forceinline__ float tree() const {  // without the +0 identity
    return ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
  }
};

template <int N>
__device__ __forceinline__ float np_sum(const float (&a)[N]) {
  Pw8 p;
#pragma unroll
  for (int i = 0; i < N; i++) p.addi(i, a[i]);
  return p.total();
}

__device__ __forceinline__ uint16_t f16bits(float f) { return __half_as_ushort(__float2half_rn(f)); }
__device__ __forceinline__ float f16tof32(uint16_t h) { return __half2float(__ushort_as_half(h)); }

}  // namespace cpk
