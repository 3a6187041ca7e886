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

// ---------------------------------------------------------------- packed float32 pairs
// Two float32 values in one 64-bit register pair (the even element in the low half), operated
// on by the sm_100 f32x2 instructions: one issue slot for two results.  Sums and differences
// are add/sub.rn.f32x2.  Products are fma.rn.f32x2 with a -0.0 addend that arrives at run
// time (a kernel argument): fl(a * b + -0) == fl(a * b) for every input, signed zeros
// included, and ptxas cannot fuse such a product with a following add, as it may a packed
// multiply.  Each pair operation therefore rounds exactly like the scalar float32 operation
// (and numpy's elementwise ufunc) it stands for.
typedef unsigned long long f32x2;

__device__ __forceinline__ f32x2 pk2(float lo, float hi) {
  f32x2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void upk2(f32x2 v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ f32x2 add2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f32x2 sub2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// fl(a * b) per half; nz2 holds -0.0 in both halves.
__device__ __forceinline__ f32x2 mul2(f32x2 a, f32x2 b, f32x2 nz2) {
  f32x2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(nz2));
  return r;
}
// |v| on both halves (the sign bits cleared, as fabsf does).
__device__ __forceinline__ f32x2 abs2(f32x2 v) { return v & 0x7FFFFFFF7FFFFFFFull; }

// nint_clip_f on both halves: the magic add and subtract as pair operations, the clamp on
// the bit patterns of each half.
__device__ __forceinline__ f32x2 nint_clip2(f32x2 v, int lo, int hi, f32x2 magic2) {
  float a, b;
  upk2(add2(v, magic2), a, b);
  int ia = (__float_as_int(a) & 0x007FFFFF) | 0x4B000000;
  int ib = (__float_as_int(b) & 0x007FFFFF) | 0x4B000000;
  ia = min(max(ia, 0x4B400000 + lo), 0x4B400000 + hi);
  ib = min(max(ib, 0x4B400000 + lo), 0x4B400000 + hi);
  return sub2(pk2(__int_as_float(ia), __int_as_float(ib)), magic2);
}

// Pw8 over pairs: pair k carries elements 2k and 2k + 1, which land in accumulators
// 2(k & 3) and 2(k & 3) + 1, so accumulator pair k & 3 receives them in the scalar order.
struct Pw8x2 {
  f32x2 r[4];
  __device__ __forceinline__ void addk(int k, f32x2 v) {  // k a compile-time constant after unrolling
    if (k < 4) r[k] = v; else r[k & 3] = add2(r[k & 3], v);
  }
  __device__ __forceinline__ float total() const {
    float a0, a1, a2, a3, a4, a5, a6, a7;
    upk2(r[0], a0, a1);
    upk2(r[1], a2, a3);
    upk2(r[2], a4, a5);
    upk2(r[3], a6, a7);
    const float res = ((a0 + a1) + (a2 + a3)) + ((a4 + a5) + (a6 + a7));
    return 0.0f + res;
  }
};

}  // namespace cpk
