// k-quant fit + pack kernels (coldpress/kquant.py QUANTIZE, lines 347-718) for sm_100a.
//
// Mapping: one thread per sub-block (16 values for Q2_K/Q3_K/Q6_K, 32 for Q4_K/Q5_K), the
// 16 (or 8) threads of a 256-value superblock sit in one warp segment and exchange
// super-scale data with shuffles; 256-thread CTAs cover 16 (or 32) consecutive
// superblocks, whose packed bytes are staged in shared memory and leave as 16-byte stores.
// All arithmetic follows the numpy reference operation by operation (see kq_common.cuh).
#include <cuda_runtime.h>
#include "kq_common.cuh"
#include "kq_fit.cuh"
#include "kquant_kernels.h"

namespace cpk {

template <int N>
__device__ __forceinline__ void load_vec(const float* __restrict__ p, float (&v)[N]) {
  const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
  for (int i = 0; i < N / 4; i++) {
    float4 t = __ldg(q + i);
    v[4 * i + 0] = t.x;
    v[4 * i + 1] = t.y;
    v[4 * i + 2] = t.z;
    v[4 * i + 3] = t.w;
  }
}

// Copy `nbytes` of staged output from shared to global memory.  Both ends are 16-byte
// aligned when the CTA's chunk is full (CTA chunk sizes are multiples of 16 bytes).
__device__ __forceinline__ void store_chunk(uint8_t* __restrict__ dst, const uint8_t* src, int nbytes) {
  const int nvec = nbytes / 16;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x)
    reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
  for (int i = nvec * 16 + threadIdx.x; i < nbytes; i += blockDim.x) dst[i] = src[i];
}

// 2-bit interleaved code byte (kquant.py:240-249): byte b of the 64-byte qs area.
__device__ __forceinline__ uint8_t qs2_byte(const uint8_t* L, int b, int sub_from_high) {
  const int h = b >> 5, l = b & 31;
  const uint8_t* s = L + h * 128 + l;
  auto c = [&](int k) -> int {
    int v = s[32 * k];
    if (sub_from_high) v = v > 3 ? v - 4 : v;
    return v & 3;
  };
  return (uint8_t)(c(0) | (c(1) << 2) | (c(2) << 4) | (c(3) << 6));
}

// The four 8-bit codes (one per lane of a 4-byte word) in `words`, byte `idx`.
__device__ __forceinline__ int byte_of(const uint32_t (&words)[4], int idx) {
  uint32_t w = words[0];
  w = (idx >> 2) == 1 ? words[1] : w;
  w = (idx >> 2) == 2 ? words[2] : w;
  w = (idx >> 2) == 3 ? words[3] : w;
  return (int)((w >> (8 * (idx & 3))) & 0xFFu);
}

template <int N>
__device__ __forceinline__ void pack_bytes(const uint8_t (&L)[N], uint32_t (&words)[4]) {
#pragma unroll
  for (int k = 0; k < 4; k++) words[k] = 0;
#pragma unroll
  for (int i = 0; i < N; i++) words[i >> 2] |= (uint32_t)L[i] << (8 * (i & 3));
}

// Sum of squares over the superblock (numpy pairwise: two 128 halves, 8 accumulators each)
// for the 16-thread layout.  sq holds the 256 squares of this superblock.
__device__ __forceinline__ float sb_sumsq_16(const float* sq, int sub) {
  const int h = sub >> 3, j = sub & 7;
  float acc = sq[128 * h + j];
#pragma unroll
  for (int k = 1; k < 16; k++) acc = acc + sq[128 * h + j + 8 * k];
  acc = acc + __shfl_xor_sync(0xffffffffu, acc, 1, 16);
  acc = acc + __shfl_xor_sync(0xffffffffu, acc, 2, 16);
  acc = acc + __shfl_xor_sync(0xffffffffu, acc, 4, 16);
  acc = acc + __shfl_xor_sync(0xffffffffu, acc, 8, 16);
  return 0.0f + acc;
}

// Same for the 8-thread layout: thread t owns accumulators 2(t%4), 2(t%4)+1 of half t/4.
__device__ __forceinline__ float sb_sumsq_8(const float* sq, int sub) {
  const int h = sub >> 2, j = 2 * (sub & 3);
  float a = sq[128 * h + j], b = sq[128 * h + j + 1];
#pragma unroll
  for (int k = 1; k < 16; k++) {
    a = a + sq[128 * h + j + 8 * k];
    b = b + sq[128 * h + j + 1 + 8 * k];
  }
  float p = a + b;
  p = p + __shfl_xor_sync(0xffffffffu, p, 1, 8);
  p = p + __shfl_xor_sync(0xffffffffu, p, 2, 8);
  p = p + __shfl_xor_sync(0xffffffffu, p, 4, 8);
  return 0.0f + p;
}

// ---------------------------------------------------------------------------- Q2_K

template <bool IMAT>
__device__ __forceinline__ void q2k_encode_body(const float* __restrict__ x, const float* __restrict__ qw,
                                                int64_t nsb_total, int64_t nsb_row, uint8_t* __restrict__ out,
                                                int64_t blk, float nz) {
  constexpr int BB = 84;
  __shared__ __align__(16) float s_sq[IMAT ? 16 : 1][256];
  __shared__ __align__(16) uint8_t s_L[16][256];
  __shared__ __align__(16) uint8_t s_out[16 * BB];
  const int sbl = threadIdx.x >> 4, sub = threadIdx.x & 15;
  const int64_t sb0 = blk * 16;
  const int64_t sb = sb0 + sbl;
  const bool valid = sb < nsb_total;
  float xv[16];
  if (valid) load_vec<16>(x + sb * 256 + sub * 16, xv);
  else {
#pragma unroll
    for (int i = 0; i < 16; i++) xv[i] = 0.0f;
  }
  float w[16], Lf[16], scale, negmin;
  int sc_i, mn_i;
  uint16_t d16, dmin16;
  if constexpr (IMAT) {
#pragma unroll
    for (int i = 0; i < 16; i++) s_sq[sbl][sub * 16 + i] = xv[i] * xv[i];
    __syncwarp();
    const float sigma2 = sb_sumsq_16(s_sq[sbl], sub) / 256.0f;
    float q[16];
    if (valid) load_vec<16>(qw + (sb % nsb_row) * 256 + sub * 16, q);
    else {
#pragma unroll
      for (int i = 0; i < 16; i++) q[i] = 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 16; i++) w[i] = q[i] * sqrtf(sigma2 + xv[i] * xv[i]);
    const float sw = np_sum(w);
    fit_qkx<16, false, true>(xv, w, 3, -0.9f, 0.05f, 36, scale, negmin, Lf, nz);
    float vs[16], vw[16];
#pragma unroll
    for (int j = 0; j < 16; j++) {
      const float a = __shfl_sync(0xffffffffu, scale, j, 16);
      const float b = __shfl_sync(0xffffffffu, negmin, j, 16);
      vs[j] = (sub == 1) ? b : a;
      vw[j] = __shfl_sync(0xffffffffu, sw, j, 16);
    }
    uint8_t Lq[16];
    float isa, isb;
    bool da, db;
    fit_qp_search_lanes<16>(scale, negmin, sw, 15, isa, da, isb, db);
    const float dd = fit_qp_tail<16>(vs, vw, 15, sub == 1 ? isb : isa, sub == 1 ? db : da, Lq);
    uint32_t words[4];
    pack_bytes(Lq, words);
    uint32_t ws[4], wm[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      ws[k] = __shfl_sync(0xffffffffu, words[k], 0, 16);
      wm[k] = __shfl_sync(0xffffffffu, words[k], 1, 16);
    }
    sc_i = byte_of(ws, sub);
    mn_i = byte_of(wm, sub);
    d16 = f16bits(__shfl_sync(0xffffffffu, dd, 0, 16));
    dmin16 = f16bits(__shfl_sync(0xffffffffu, dd, 1, 16));
  } else {
#pragma unroll
    for (int i = 0; i < 16; i++) w[i] = fabsf(xv[i]);
    fit_qkx<16, true, false>(xv, w, 3, -0.5f, 0.1f, 15, scale, negmin, Lf, nz);
    float max_scale = __shfl_sync(0xffffffffu, scale, 0, 16);
    float max_min = __shfl_sync(0xffffffffu, negmin, 0, 16);
#pragma unroll
    for (int j = 1; j < 16; j++) {
      max_scale = np_max_step(max_scale, __shfl_sync(0xffffffffu, scale, j, 16));
      max_min = np_max_step(max_min, __shfl_sync(0xffffffffu, negmin, j, 16));
    }
    const bool pos = max_scale > 0.0f, posm = max_min > 0.0f;
    const float isc = pos ? 15.0f / max_scale : 0.0f;
    const float iscm = posm ? 15.0f / max_min : 0.0f;
    sc_i = pos ? nint(isc * scale) : 0;
    mn_i = posm ? nint(iscm * negmin) : 0;
    d16 = f16bits(pos ? max_scale / 15.0f : 0.0f);
    dmin16 = f16bits(posm ? max_min / 15.0f : 0.0f);
  }
  // requantize against the rounded grid where dl != 0 (kquant.py:399-405)
  const float dl = f16tof32(d16) * (float)sc_i;
  const float ml = f16tof32(dmin16) * (float)mn_i;
  if (dl != 0.0f) {
#pragma unroll
    for (int i = 0; i < 16; i++) Lf[i] = nint_clip_f((xv[i] + ml) / dl, 0, 3);
  }
  uint8_t* o = s_out + sbl * BB;
#pragma unroll
  for (int i = 0; i < 16; i++) s_L[sbl][sub * 16 + i] = (uint8_t)(int)Lf[i];
  o[sub] = (uint8_t)(((uint8_t)sc_i & 0xF) | (((uint8_t)mn_i & 0xF) << 4));
  if (sub == 0) {
    o[80] = (uint8_t)(d16 & 0xFF);
    o[81] = (uint8_t)(d16 >> 8);
    o[82] = (uint8_t)(dmin16 & 0xFF);
    o[83] = (uint8_t)(dmin16 >> 8);
  }
  __syncwarp();
#pragma unroll
  for (int k = 0; k < 4; k++) o[16 + sub * 4 + k] = qs2_byte(s_L[sbl], sub * 4 + k, 0);
  __syncthreads();
  const int64_t nvalid = min((int64_t)16, nsb_total - sb0);
  store_chunk(out + sb0 * BB, s_out, (int)(nvalid * BB));
}

// ---------------------------------------------------------------------------- Q3_K

template <bool IMAT>
__device__ __forceinline__ void q3k_encode_body(const float* __restrict__ x, const float* __restrict__ qw,
                                                int64_t nsb_total, int64_t nsb_row, uint8_t* __restrict__ out,
                                                int64_t blk, float nz) {
  constexpr int BB = 110;
  __shared__ __align__(16) float s_sq[IMAT ? 16 : 1][256];
  __shared__ __align__(16) uint8_t s_L[16][256];
  __shared__ __align__(16) uint8_t s_Ls[16][16];
  __shared__ __align__(16) uint8_t s_out[16 * BB];
  const int sbl = threadIdx.x >> 4, sub = threadIdx.x & 15;
  const int64_t sb0 = blk * 16;
  const int64_t sb = sb0 + sbl;
  const bool valid = sb < nsb_total;
  float xv[16];
  if (valid) load_vec<16>(x + sb * 256 + sub * 16, xv);
  else {
#pragma unroll
    for (int i = 0; i < 16; i++) xv[i] = 0.0f;
  }
  float Lf[16];
  int my_Ls;
  float d;
  if constexpr (IMAT) {
#pragma unroll
    for (int i = 0; i < 16; i++) s_sq[sbl][sub * 16 + i] = xv[i] * xv[i];
    __syncwarp();
    const float sigma2 = 2.0f * sb_sumsq_16(s_sq[sbl], sub) / 256.0f;
    float q[16], w[16];
    if (valid) load_vec<16>(qw + (sb % nsb_row) * 256 + sub * 16, q);
    else {
#pragma unroll
      for (int i = 0; i < 16; i++) q[i] = 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 16; i++) w[i] = q[i] * sqrtf(sigma2 + xv[i] * xv[i]);
    const float sw = np_sum(w);
    const float scale = fit_qx<16>(xv, w, 4, Lf, nz);
    float vs[16], vw[16], Ls[16];
#pragma unroll
    for (int j = 0; j < 16; j++) {
      vs[j] = __shfl_sync(0xffffffffu, scale, j, 16);
      vw[j] = __shfl_sync(0xffffffffu, sw, j, 16);
    }
    d = fit_qx<16>(vs, vw, 32, Ls, nz);
    my_Ls = (int)select_idx(Ls, sub);
  } else {
    const float scale = fit_q3<16>(xv, 4, Lf);
    float vs[16];
#pragma unroll
    for (int j = 0; j < 16; j++) vs[j] = __shfl_sync(0xffffffffu, scale, j, 16);
    const float max_scale = select_idx(vs, argmax_abs(vs));
    const bool live = max_scale != 0.0f;
    const float isc = live ? -32.0f / max_scale : 0.0f;
    my_Ls = live ? clampi(nint(isc * scale), -32, 31) + 32 : 0;
    d = live ? 1.0f / isc : 0.0f;
    if (!(fabsf(d) <= 3.4028234663852886e38f)) d = 0.0f;
  }
  const uint16_t d16 = f16bits(d);
  // 6-bit scales round-trip unchanged (values 0..63), so the unpacked scale is my_Ls - 32.
  const float ds = f16tof32(d16) * (float)(my_Ls - 32);
  if (ds != 0.0f) {
#pragma unroll
    for (int i = 0; i < 16; i++) Lf[i] = nint_clip_f(xv[i] / ds, -4, 3) + 4.0f;
  }
#pragma unroll
  for (int i = 0; i < 16; i++) s_L[sbl][sub * 16 + i] = (uint8_t)(int)Lf[i];
  s_Ls[sbl][sub] = (uint8_t)my_Ls;
  __syncwarp();
  uint8_t* o = s_out + sbl * BB;
  const uint8_t* L = s_L[sbl];
  // hmask[l] bit j = code of element 32j + l > 3 (kquant.py:474-480)
#pragma unroll
  for (int k = 0; k < 2; k++) {
    const int l = sub * 2 + k;
    uint8_t m = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) m |= (uint8_t)((L[32 * j + l] > 3 ? 1 : 0) << j);
    o[l] = m;
  }
#pragma unroll
  for (int k = 0; k < 4; k++) o[32 + sub * 4 + k] = qs2_byte(L, sub * 4 + k, 1);
  if (sub < 12) {  // _pack_scales_q3 (kquant.py:264-276)
    const uint8_t* Ls = s_Ls[sbl];
    uint8_t b;
    if (sub < 8) b = (uint8_t)((Ls[sub] & 0xF) | ((Ls[sub + 8] & 0xF) << 4));
    else {
      const int c = sub - 8;
      b = 0;
#pragma unroll
      for (int q = 0; q < 4; q++) b |= (uint8_t)((Ls[c + 4 * q] >> 4) << (2 * q));
    }
    o[96 + sub] = b;
  }
  if (sub == 12) {
    o[108] = (uint8_t)(d16 & 0xFF);
    o[109] = (uint8_t)(d16 >> 8);
  }
  __syncthreads();
  const int64_t nvalid = min((int64_t)16, nsb_total - sb0);
  store_chunk(out + sb0 * BB, s_out, (int)(nvalid * BB));
}

// ---------------------------------------------------------------------------- Q6_K

template <bool IMAT>
__device__ __forceinline__ void q6k_encode_body(const float* __restrict__ x, const float* __restrict__ qw,
                                                int64_t nsb_total, int64_t nsb_row, uint8_t* __restrict__ out,
                                                int64_t blk, float nz) {
  constexpr int BB = 210;
  __shared__ __align__(16) uint8_t s_L[16][256];
  __shared__ __align__(16) uint8_t s_out[16 * BB + 16];
  const int sbl = threadIdx.x >> 4, sub = threadIdx.x & 15;
  const int64_t sb0 = blk * 16;
  const int64_t sb = sb0 + sbl;
  const bool valid = sb < nsb_total;
  float xv[16], w[16], Lf[16];
  if (valid) load_vec<16>(x + sb * 256 + sub * 16, xv);
  else {
#pragma unroll
    for (int i = 0; i < 16; i++) xv[i] = 0.0f;
  }
  if constexpr (IMAT) {
    if (valid) load_vec<16>(qw + (sb % nsb_row) * 256 + sub * 16, w);
    else {
#pragma unroll
      for (int i = 0; i < 16; i++) w[i] = 0.0f;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; i++) w[i] = xv[i] * xv[i];
  }
  const float scale = fit_qx<16>(xv, w, 32, Lf, nz);
  float vs[16];
#pragma unroll
  for (int j = 0; j < 16; j++) vs[j] = __shfl_sync(0xffffffffu, scale, j, 16);
  const float max_scale = select_idx(vs, argmax_abs(vs));
  const bool dead = fabsf(max_scale) < kGroupEps;
  const float mxs = dead ? 1.0f : max_scale;
  const float iscale = -128.0f / mxs;
  const float dd = 1.0f / iscale;
  const int8_t sc = (int8_t)min(nint(iscale * scale), 127);
  const uint16_t d16 = f16bits(dead ? 0.0f : dd);
  const float ds = f16tof32(d16) * (float)sc;
  if (ds != 0.0f && !dead) {
#pragma unroll
    for (int i = 0; i < 16; i++) Lf[i] = nint_clip_f(xv[i] / ds, -32, 31) + 32.0f;
  }
#pragma unroll
  for (int i = 0; i < 16; i++) s_L[sbl][sub * 16 + i] = dead ? (uint8_t)0 : (uint8_t)(int)Lf[i];
  __syncwarp();
  uint8_t* o = s_out + sbl * BB;
  const uint8_t* L = s_L[sbl];
  // ql / qh (kquant.py:664-672)
#pragma unroll
  for (int k = 0; k < 8; k++) {
    const int b = sub * 8 + k;  // 0..127
    const int h = b >> 6, r = b & 63;
    const uint8_t* s = L + h * 128 + (r & 31);
    o[b] = (r < 32) ? (uint8_t)((s[0] & 0xF) | ((s[64] & 0xF) << 4))
                    : (uint8_t)((s[32] & 0xF) | ((s[96] & 0xF) << 4));
  }
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const int b = sub * 4 + k;  // 0..63
    const int h = b >> 5, l = b & 31;
    const uint8_t* s = L + h * 128 + l;
    o[128 + b] = (uint8_t)((s[0] >> 4) | ((s[32] >> 4) << 2) | ((s[64] >> 4) << 4) | ((s[96] >> 4) << 6));
  }
  o[192 + sub] = dead ? (uint8_t)0 : (uint8_t)sc;
  if (sub == 0) {
    o[208] = (uint8_t)(d16 & 0xFF);
    o[209] = (uint8_t)(d16 >> 8);
  }
  __syncthreads();
  const int64_t nvalid = min((int64_t)16, nsb_total - sb0);
  store_chunk(out + sb0 * BB, s_out, (int)(nvalid * BB));
}

// ---------------------------------------------------------------------------- Q4_K / Q5_K

template <bool IMAT, bool Q5>
__device__ __forceinline__ void q45k_encode_body(const float* __restrict__ x, const float* __restrict__ qw,
                                                 int64_t nsb_total, int64_t nsb_row, uint8_t* __restrict__ out,
                                                 int64_t blk, float nz) {
  constexpr int BB = Q5 ? 176 : 144;
  constexpr int NMAX = Q5 ? 31 : 15;
  __shared__ __align__(16) float s_sq[IMAT ? 32 : 1][256];
  __shared__ __align__(16) uint8_t s_L[32][256];
  __shared__ __align__(16) uint8_t s_out[32 * BB];
  const int sbl = threadIdx.x >> 3, sub = threadIdx.x & 7;
  const int64_t sb0 = blk * 32;
  const int64_t sb = sb0 + sbl;
  const bool valid = sb < nsb_total;
  float xv[32], w[32], Lf[32], scale, negmin;
  if (valid) load_vec<32>(x + sb * 256 + sub * 32, xv);
  else {
#pragma unroll
    for (int i = 0; i < 32; i++) xv[i] = 0.0f;
  }
  int my_Ls, my_Lm;
  float d, dmin;
  if constexpr (IMAT) {
#pragma unroll
    for (int i = 0; i < 32; i++) s_sq[sbl][sub * 32 + i] = xv[i] * xv[i];
    __syncwarp();
    const float sigma2 = 2.0f * sb_sumsq_8(s_sq[sbl], sub) / 256.0f;
    if (valid) load_vec<32>(qw + (sb % nsb_row) * 256 + sub * 32, w);
    else {
#pragma unroll
      for (int i = 0; i < 32; i++) w[i] = 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 32; i++) w[i] = w[i] * sqrtf(sigma2 + xv[i] * xv[i]);
    const float sw = np_sum(w);
    fit_qkx<32, false, true>(xv, w, NMAX, -0.9f, 0.05f, 36, scale, negmin, Lf, nz);
    float vs[8], vw[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const float a = __shfl_sync(0xffffffffu, scale, j, 8);
      const float b = __shfl_sync(0xffffffffu, negmin, j, 8);
      vs[j] = (sub == 1) ? b : a;
      vw[j] = __shfl_sync(0xffffffffu, sw, j, 8);
    }
    uint8_t Lq[8];
    float isa, isb;
    bool da, db;
    fit_qp_search_lanes<8>(scale, negmin, sw, 63, isa, da, isb, db);
    const float dd = fit_qp_tail<8>(vs, vw, 63, sub == 1 ? isb : isa, sub == 1 ? db : da, Lq);
    uint32_t words[4];
    pack_bytes(Lq, words);
    uint32_t ws[4], wm[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      ws[k] = __shfl_sync(0xffffffffu, words[k], 0, 8);
      wm[k] = __shfl_sync(0xffffffffu, words[k], 1, 8);
    }
    my_Ls = byte_of(ws, sub);
    my_Lm = byte_of(wm, sub);
    if (Q5) {
      my_Ls = min(my_Ls, 63);
      my_Lm = min(my_Lm, 63);
    }
    d = __shfl_sync(0xffffffffu, dd, 0, 8);
    dmin = __shfl_sync(0xffffffffu, dd, 1, 8);
  } else {
    float sq[32];
#pragma unroll
    for (int i = 0; i < 32; i++) sq[i] = xv[i] * xv[i];
    const float av_x = sqrtf(np_sum(sq) / 32.0f);
#pragma unroll
    for (int i = 0; i < 32; i++) w[i] = av_x + fabsf(xv[i]);
    fit_qkx<32, false, false>(xv, w, NMAX, Q5 ? -0.5f : -1.0f, 0.1f, Q5 ? 15 : 20, scale, negmin, Lf, nz);
    float max_scale = __shfl_sync(0xffffffffu, scale, 0, 8);
    float max_min = __shfl_sync(0xffffffffu, negmin, 0, 8);
#pragma unroll
    for (int j = 1; j < 8; j++) {
      max_scale = np_max_step(max_scale, __shfl_sync(0xffffffffu, scale, j, 8));
      max_min = np_max_step(max_min, __shfl_sync(0xffffffffu, negmin, j, 8));
    }
    const float inv_scale = max_scale > 0.0f ? 63.0f / max_scale : 0.0f;
    const float inv_min = max_min > 0.0f ? 63.0f / max_min : 0.0f;
    my_Ls = min((int)(uint8_t)nint(inv_scale * scale), 63);
    my_Lm = min((int)(uint8_t)nint(inv_min * negmin), 63);
    d = max_scale / 63.0f;
    dmin = max_min / 63.0f;
  }
  const uint16_t d16 = f16bits(d), dmin16 = f16bits(dmin);
  // _pack_scales_k4 then get_scale_min_k4 (kquant.py:293-322), on the 8 bytes of this superblock
  uint32_t lsw[4], lmw[4];
  {
    uint32_t a = (uint32_t)(my_Ls & 0xFF) << (8 * (sub & 3));
    uint32_t b = (uint32_t)(my_Lm & 0xFF) << (8 * (sub & 3));
    a |= __shfl_xor_sync(0xffffffffu, a, 1, 8);
    a |= __shfl_xor_sync(0xffffffffu, a, 2, 8);
    b |= __shfl_xor_sync(0xffffffffu, b, 1, 8);
    b |= __shfl_xor_sync(0xffffffffu, b, 2, 8);
    const uint32_t a_lo = __shfl_sync(0xffffffffu, a, 0, 8), a_hi = __shfl_sync(0xffffffffu, a, 4, 8);
    const uint32_t b_lo = __shfl_sync(0xffffffffu, b, 0, 8), b_hi = __shfl_sync(0xffffffffu, b, 4, 8);
    lsw[0] = a_lo; lsw[1] = a_hi; lsw[2] = 0; lsw[3] = 0;
    lmw[0] = b_lo; lmw[1] = b_hi; lmw[2] = 0; lmw[3] = 0;
  }
  uint8_t scp[12];
  {
    uint8_t ls[8], lm[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
      ls[j] = (uint8_t)((lsw[j >> 2] >> (8 * (j & 3))) & 0xFF);
      lm[j] = (uint8_t)((lmw[j >> 2] >> (8 * (j & 3))) & 0xFF);
    }
#pragma unroll
    for (int j = 0; j < 4; j++) {
      scp[j] = ls[j];
      scp[j + 4] = lm[j];
    }
#pragma unroll
    for (int j = 4; j < 8; j++) {
      scp[j + 4] = (uint8_t)((ls[j] & 0xF) | ((lm[j] & 0xF) << 4));
      scp[j - 4] |= (uint8_t)((ls[j] >> 4) << 6);
      scp[j] |= (uint8_t)((lm[j] >> 4) << 6);
    }
  }
  int su, mu;
  {
    // get_scale_min_k4 for sub-block `sub`
    int sa = 0, ma = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      int s_, m_;
      if (j < 4) {
        s_ = scp[j] & 63;
        m_ = scp[j + 4] & 63;
      } else {
        s_ = (scp[j + 4] & 0xF) | ((scp[j - 4] >> 6) << 4);
        m_ = (scp[j + 4] >> 4) | ((scp[j] >> 6) << 4);
      }
      sa = (j == sub) ? s_ : sa;
      ma = (j == sub) ? m_ : ma;
    }
    su = sa;
    mu = ma;
  }
  const float ds = f16tof32(d16) * (float)su;
  const float ms = f16tof32(dmin16) * (float)mu;
  if (ds != 0.0f) {
#pragma unroll
    for (int i = 0; i < 32; i++) Lf[i] = nint_clip_f((xv[i] + ms) / ds, 0, NMAX);
  }
#pragma unroll
  for (int i = 0; i < 32; i++) s_L[sbl][sub * 32 + i] = (uint8_t)(int)Lf[i];
  __syncwarp();
  uint8_t* o = s_out + sbl * BB;
  const uint8_t* L = s_L[sbl];
  if (sub == 0) {
    o[0] = (uint8_t)(d16 & 0xFF);
    o[1] = (uint8_t)(d16 >> 8);
    o[2] = (uint8_t)(dmin16 & 0xFF);
    o[3] = (uint8_t)(dmin16 >> 8);
  }
  if (sub < 6) {
    o[4 + 2 * sub] = scp[2 * sub];
    o[5 + 2 * sub] = scp[2 * sub + 1];
  }
  const int qs_off = Q5 ? 48 : 16;
  // nibbles (kquant.py:325-332): 16 bytes per thread
#pragma unroll
  for (int k = 0; k < 16; k++) {
    const int b = sub * 16 + k;  // 0..127
    const int c = b >> 5, l = b & 31;
    int lo = L[c * 64 + l], hi = L[c * 64 + 32 + l];
    if (Q5) {
      lo = lo > 15 ? lo - 16 : lo;
      hi = hi > 15 ? hi - 16 : hi;
    }
    o[qs_off + b] = (uint8_t)((lo & 0xF) | ((hi & 0xF) << 4));
  }
  if (Q5) {  // qh bit-planes (kquant.py:573-578)
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int l = sub * 4 + k;
      uint8_t m = 0;
#pragma unroll
      for (int c = 0; c < 4; c++) {
        m |= (uint8_t)((L[c * 64 + l] > 15 ? 1 : 0) << (2 * c));
        m |= (uint8_t)((L[c * 64 + 32 + l] > 15 ? 1 : 0) << (2 * c + 1));
      }
      o[16 + l] = m;
    }
  }
  __syncthreads();
  const int64_t nvalid = min((int64_t)32, nsb_total - sb0);
  store_chunk(out + sb0 * BB, s_out, (int)(nvalid * BB));
}

// ---------------------------------------------------------------------------- Q8_0

// One thread per 32-value block; the 34-byte blocks of the CTA are staged in shared memory
// and leave through store_chunk (a thread writing two adjacent bytes of global memory was
// observed to lose one of them on this toolchain, so no kernel here does that).
__global__ void __launch_bounds__(128) q80_encode_kernel(const float* __restrict__ x, int64_t nblk,
                                                         uint8_t* __restrict__ out) {
  __shared__ __align__(16) uint8_t s_out[128 * 34];
  const int64_t b0 = (int64_t)blockIdx.x * 128;
  const int64_t b = b0 + threadIdx.x;
  uint8_t* o = s_out + threadIdx.x * 34;
  if (b < nblk) {
    float xv[32];
    load_vec<32>(x + b * 32, xv);
    float amax = fabsf(xv[0]);
#pragma unroll
    for (int i = 1; i < 32; i++) amax = np_max_step(amax, fabsf(xv[i]));
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    const uint16_t h = f16bits(d);
    o[0] = (uint8_t)(h & 0xFF);
    o[1] = (uint8_t)(h >> 8);
#pragma unroll
    for (int i = 0; i < 32; i++) {
      const float x0 = xv[i] * id;
      const float sg = x0 > 0.0f ? 1.0f : (x0 < 0.0f ? -1.0f : x0);
      const float q = sg * floorf(fabsf(x0) + 0.5f);
      o[2 + i] = (uint8_t)(int8_t)(int32_t)q;
    }
  }
  __syncthreads();
  const int64_t nvalid = min((int64_t)128, nblk - b0);
  store_chunk(out + b0 * 34, s_out, (int)(nvalid * 34));
}

// ---------------------------------------------------------------------------- kernels

// superblocks per 256-thread CTA for each type
template <int TYPE> constexpr int sb_per_cta() { return (TYPE == kQ4_K || TYPE == kQ5_K) ? 32 : 16; }

template <int TYPE, bool IMAT>
__device__ __forceinline__ void encode_body(const float* x, const float* qw, int64_t nsb, int64_t nsb_row, uint8_t* out,
                                            int64_t blk, float nz) {
  if constexpr (TYPE == kQ2_K) q2k_encode_body<IMAT>(x, qw, nsb, nsb_row, out, blk, nz);
  else if constexpr (TYPE == kQ3_K) q3k_encode_body<IMAT>(x, qw, nsb, nsb_row, out, blk, nz);
  else if constexpr (TYPE == kQ4_K) q45k_encode_body<IMAT, false>(x, qw, nsb, nsb_row, out, blk, nz);
  else if constexpr (TYPE == kQ5_K) q45k_encode_body<IMAT, true>(x, qw, nsb, nsb_row, out, blk, nz);
  else q6k_encode_body<IMAT>(x, qw, nsb, nsb_row, out, blk, nz);
}

template <int TYPE, bool IMAT>
__global__ void __launch_bounds__(256) encode_kernel(const float* __restrict__ x, const float* __restrict__ qw,
                                                     int64_t nsb, int64_t nsb_row, uint8_t* __restrict__ out,
                                                     float nz) {
  encode_body<TYPE, IMAT>(x, qw, nsb, nsb_row, out, blockIdx.x, nz);
}

// Grouped launch: every CTA finds its tensor in the descriptor table (sorted by first CTA).
template <int TYPE, bool IMAT>
__global__ void __launch_bounds__(256) encode_batch_kernel(const __grid_constant__ FitBatch b, float nz) {
  int lo = 0, hi = b.count - 1;
  const int64_t cta = blockIdx.x;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (b.d[mid].cta0 <= cta) lo = mid;
    else hi = mid - 1;
  }
  const FitDesc& t = b.d[lo];
  encode_body<TYPE, IMAT>(t.x, t.qw, t.nsb, t.nsb_row, t.out, cta - t.cta0, nz);
}

// ---------------------------------------------------------------------------- launchers

#define CPK_DISPATCH_ENC(type, imat, CALL)                                                  \
  switch (type) {                                                                          \
    case kQ2_K: if (imat) { constexpr int T = kQ2_K; constexpr bool I = true; CALL; }       \
                else { constexpr int T = kQ2_K; constexpr bool I = false; CALL; } break;    \
    case kQ3_K: if (imat) { constexpr int T = kQ3_K; constexpr bool I = true; CALL; }       \
                else { constexpr int T = kQ3_K; constexpr bool I = false; CALL; } break;    \
    case kQ4_K: if (imat) { constexpr int T = kQ4_K; constexpr bool I = true; CALL; }       \
                else { constexpr int T = kQ4_K; constexpr bool I = false; CALL; } break;    \
    case kQ5_K: if (imat) { constexpr int T = kQ5_K; constexpr bool I = true; CALL; }       \
                else { constexpr int T = kQ5_K; constexpr bool I = false; CALL; } break;    \
    case kQ6_K: if (imat) { constexpr int T = kQ6_K; constexpr bool I = true; CALL; }       \
                else { constexpr int T = kQ6_K; constexpr bool I = false; CALL; } break;    \
    default: return 1;                                                                     \
  }

int launch_quantize(int type, const float* x, int64_t nrow, int64_t n, const float* qw, uint8_t* out,
                    cudaStream_t stream) {
  if (type == kQ8_0) {
    const int64_t nblk = nrow * (n / 32);
    if (nblk == 0) return 0;
    q80_encode_kernel<<<(unsigned)((nblk + 127) / 128), 128, 0, stream>>>(x, nblk, out);
    note_launch();
    return 0;
  }
  const int64_t nsb_row = n / 256, total = nrow * nsb_row;
  if (total == 0) return 0;
  const bool im = qw != nullptr;
  CPK_DISPATCH_ENC(type, im, ({
    const unsigned g = (unsigned)((total + sb_per_cta<T>() - 1) / sb_per_cta<T>());
    encode_kernel<T, I><<<g, 256, 0, stream>>>(x, qw, total, nsb_row, out, -0.0f);
  }));
  note_launch();
  return 0;
}

int64_t quantize_batch_ctas(int type, int64_t nsb) {
  const int per = (type == kQ4_K || type == kQ5_K) ? 32 : 16;
  return (nsb + per - 1) / per;
}

int launch_quantize_batch(int type, bool imat, const FitBatch& b, int64_t total_ctas, cudaStream_t stream) {
  if (b.count == 0 || total_ctas == 0) return 0;
  CPK_DISPATCH_ENC(type, imat, (encode_batch_kernel<T, I><<<(unsigned)total_ctas, 256, 0, stream>>>(b, -0.0f)));
  note_launch();
  return 0;
}

}  // namespace cpk
