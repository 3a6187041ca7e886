// Container decoders (coldpress/kquant.py:416-727), committed-grid extraction
// (coldpress/ef.py:87-127) and code re-packing (coldpress/ef.py:130-176).
// One thread per superblock element; bandwidth-bound, each superblock's header is read by
// the 256 threads that decode it (served from L1).
#include <cuda_runtime.h>
#include "kq_common.cuh"
#include "kquant_kernels.h"

namespace cpk {

bool grid_spec(int type, int* sbw, int* lo, int* hi, bool* has_min) {
  switch (type) {
    case kQ2_K: *sbw = 16; *lo = 0; *hi = 3; *has_min = true; return true;
    case kQ3_K: *sbw = 16; *lo = -4; *hi = 3; *has_min = false; return true;
    case kQ4_K: *sbw = 32; *lo = 0; *hi = 15; *has_min = true; return true;
    case kQ5_K: *sbw = 32; *lo = 0; *hi = 31; *has_min = true; return true;
    case kQ6_K: *sbw = 16; *lo = -32; *hi = 31; *has_min = false; return true;
    default: return false;
  }
}

__device__ __forceinline__ uint16_t ld16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

// Signed code (ef.py's L) of element i of superblock b.
template <int T>
__device__ __forceinline__ int code_of(const uint8_t* b, int i) {
  if (T == kQ2_K) {
    const int h = i >> 7, k = (i >> 5) & 3, l = i & 31;
    return (b[16 + h * 32 + l] >> (2 * k)) & 3;
  } else if (T == kQ3_K) {
    const int h = i >> 7, k = (i >> 5) & 3, l = i & 31;
    const int lo = (b[32 + h * 32 + l] >> (2 * k)) & 3;
    const int hb = (b[i & 31] >> (i >> 5)) & 1;
    return lo - (hb ? 0 : 4);
  } else if (T == kQ4_K || T == kQ5_K) {
    const int c = i >> 6, r = i & 63, l = r & 31;
    const int off = (T == kQ5_K) ? 48 : 16;
    int v = (r < 32) ? (b[off + c * 32 + l] & 0xF) : (b[off + c * 32 + l] >> 4);
    if (T == kQ5_K) v += 16 * ((b[16 + l] >> (2 * c + (r >= 32 ? 1 : 0))) & 1);
    return v;
  } else {  // Q6_K
    const int h = i >> 7, r = i & 127, k = r >> 5, l = r & 31;
    const uint8_t* ql = b + h * 64;
    const uint8_t* qh = b + 128 + h * 32;
    int lo4 = (k == 0) ? (ql[l] & 0xF) : (k == 1) ? (ql[32 + l] & 0xF) : (k == 2) ? (ql[l] >> 4) : (ql[32 + l] >> 4);
    return (lo4 | (((qh[l] >> (2 * k)) & 3) << 4)) - 32;
  }
}

// (dl, ml) of sub-block j of superblock b (ml = 0 for types without a min).
template <int T>
__device__ __forceinline__ void grid_of(const uint8_t* b, int j, float& dl, float& ml) {
  if (T == kQ2_K) {
    dl = f16tof32(ld16(b + 80)) * (float)(b[j] & 0xF);
    ml = f16tof32(ld16(b + 82)) * (float)(b[j] >> 4);
  } else if (T == kQ3_K) {
    const int lo = (j < 8) ? (b[96 + j] & 0xF) : (b[96 + j - 8] >> 4);
    const int hi = (b[96 + 8 + (j & 3)] >> (2 * (j >> 2))) & 3;
    dl = f16tof32(ld16(b + 108)) * (float)((lo | (hi << 4)) - 32);
    ml = 0.0f;
  } else if (T == kQ4_K || T == kQ5_K) {
    const uint8_t* sc = b + 4;
    int s, m;
    if (j < 4) {
      s = sc[j] & 63;
      m = sc[j + 4] & 63;
    } else {
      s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
      m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
    dl = f16tof32(ld16(b)) * (float)s;
    ml = f16tof32(ld16(b + 2)) * (float)m;
  } else {
    dl = f16tof32(ld16(b + 208)) * (float)(int8_t)b[192 + j];
    ml = 0.0f;
  }
}

template <int T>
__global__ void dequant_kernel(const uint8_t* __restrict__ raw, int64_t nsb, float* __restrict__ out) {
  const int64_t sb = blockIdx.x;
  const int i = threadIdx.x;
  if (sb >= nsb) return;
  constexpr int BB = block_bytes(T);
  constexpr int SW = (T == kQ4_K || T == kQ5_K) ? 32 : 16;
  const uint8_t* b = raw + sb * BB;
  float dl, ml;
  grid_of<T>(b, i / SW, dl, ml);
  const float v = dl * (float)code_of<T>(b, i);
  out[sb * 256 + i] = (T == kQ3_K || T == kQ6_K) ? v : v - ml;
}

__global__ void dequant_q80_kernel(const uint8_t* __restrict__ raw, int64_t nblk, float* __restrict__ out) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= nblk * 32) return;
  const uint8_t* b = raw + (e >> 5) * 34;
  out[e] = f16tof32(ld16(b)) * (float)(int8_t)b[2 + (e & 31)];
}

template <int T>
__global__ void grid_kernel(const uint8_t* __restrict__ raw, int64_t nsub_total, float* __restrict__ dl,
                            float* __restrict__ ml) {
  constexpr int NS = (T == kQ4_K || T == kQ5_K) ? 8 : 16;
  const int64_t s = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= nsub_total) return;
  float a, m;
  grid_of<T>(raw + (s / NS) * block_bytes(T), (int)(s % NS), a, m);
  dl[s] = a;
  if (ml) ml[s] = m;
}

template <int T>
__global__ void codes_kernel(const uint8_t* __restrict__ raw, int64_t nsb, int8_t* __restrict__ codes) {
  const int64_t sb = blockIdx.x;
  if (sb >= nsb) return;
  codes[sb * 256 + threadIdx.x] = (int8_t)code_of<T>(raw + sb * block_bytes(T), threadIdx.x);
}

// Write signed codes into committed bytes; one thread per output code byte.
template <int T>
__global__ void repack_kernel(uint8_t* __restrict__ raw, const int8_t* __restrict__ codes, int64_t nsb) {
  const int64_t sb = blockIdx.x;
  if (sb >= nsb) return;
  constexpr int BB = block_bytes(T);
  __shared__ int8_t c[256];
  c[threadIdx.x] = codes[sb * 256 + threadIdx.x];
  __syncthreads();
  uint8_t* b = raw + sb * BB;
  const int t = threadIdx.x;
  if (T == kQ2_K) {
    if (t < 64) {
      const int h = t >> 5, l = t & 31;
      const int8_t* s = c + h * 128 + l;
      b[16 + t] = (uint8_t)((s[0] & 3) | ((s[32] & 3) << 2) | ((s[64] & 3) << 4) | ((s[96] & 3) << 6));
    }
  } else if (T == kQ3_K) {
    auto L = [&](int i) { return (int)c[i] + 4; };
    if (t < 32) {
      uint8_t m = 0;
      for (int j = 0; j < 8; j++) m |= (uint8_t)((L(32 * j + t) > 3 ? 1 : 0) << j);
      b[t] = m;
    } else if (t < 96) {
      const int q = t - 32, h = q >> 5, l = q & 31;
      uint8_t v = 0;
      for (int k = 0; k < 4; k++) {
        int x = L(h * 128 + 32 * k + l);
        x = x > 3 ? x - 4 : x;
        v |= (uint8_t)((x & 3) << (2 * k));
      }
      b[32 + q] = v;
    }
  } else if (T == kQ4_K || T == kQ5_K) {
    const int off = (T == kQ5_K) ? 48 : 16;
    if (t < 128) {
      const int cc = t >> 5, l = t & 31;
      int lo = c[cc * 64 + l], hi = c[cc * 64 + 32 + l];
      if (T == kQ5_K) {
        lo = lo > 15 ? lo - 16 : lo;
        hi = hi > 15 ? hi - 16 : hi;
      }
      b[off + t] = (uint8_t)((lo & 0xF) | ((hi & 0xF) << 4));
    } else if (T == kQ5_K && t < 160) {
      const int l = t - 128;
      uint8_t m = 0;
      for (int cc = 0; cc < 4; cc++) {
        m |= (uint8_t)((c[cc * 64 + l] > 15 ? 1 : 0) << (2 * cc));
        m |= (uint8_t)((c[cc * 64 + 32 + l] > 15 ? 1 : 0) << (2 * cc + 1));
      }
      b[16 + l] = m;
    }
  } else {  // Q6_K, codes -32..31 -> 0..63
    auto L = [&](int i) { return (int)c[i] + 32; };
    if (t < 128) {
      const int h = t >> 6, r = t & 63, l = r & 31;
      const int base = h * 128 + l;
      b[t] = (r < 32) ? (uint8_t)((L(base) & 0xF) | ((L(base + 64) & 0xF) << 4))
                      : (uint8_t)((L(base + 32) & 0xF) | ((L(base + 96) & 0xF) << 4));
    } else if (t < 192) {
      const int q = t - 128, h = q >> 5, l = q & 31;
      const int base = h * 128 + l;
      b[128 + q] = (uint8_t)((L(base) >> 4) | ((L(base + 32) >> 4) << 2) | ((L(base + 64) >> 4) << 4) |
                             ((L(base + 96) >> 4) << 6));
    }
  }
}

// encode_gguf statistics (ef.py:298-301): sum over the tensor of (dequant(raw) - x)^2 * w[col]
// (w == nullptr means 1), accumulated in float64.  One CTA per superblock group.
template <int T>
__global__ void __launch_bounds__(256) weighted_err_kernel(const uint8_t* __restrict__ raw, const float* __restrict__ x,
                                                           const float* __restrict__ w, int64_t nsb, int64_t nsb_row,
                                                           double* __restrict__ out) {
  constexpr int BB = block_bytes(T);
  constexpr int SW = (T == kQ4_K || T == kQ5_K) ? 32 : 16;
  double acc = 0.0;
  for (int64_t sb = blockIdx.x; sb < nsb; sb += gridDim.x) {
    const uint8_t* b = raw + sb * BB;
    const int i = threadIdx.x;
    float dl, ml;
    grid_of<T>(b, i / SW, dl, ml);
    float v = dl * (float)code_of<T>(b, i);
    if (!(T == kQ3_K || T == kQ6_K)) v = v - ml;
    const float d = v - x[sb * 256 + i];
    const float wt = w ? w[(sb % nsb_row) * 256 + i] : 1.0f;
    acc += (double)(d * d * wt);
  }
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  __shared__ double red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int k = 0; k < 8; k++) s += red[k];
    atomicAdd(out, s);
  }
}

// ---------------------------------------------------------------------------- grouped launches
// One CTA of 256 threads per 16 superblocks of one tensor; CTAs find their tensor in the
// descriptor table.
constexpr int kSbPerCta = 16;

// Grid of superblocks [c*16, c*16 + 16): one thread per (superblock, sub-block), writes
// coalesced across the CTA.
template <int T>
__device__ __forceinline__ void grid_sb(const SbDesc& t, int64_t c) {
  constexpr int NS = (T == kQ4_K || T == kQ5_K) ? 8 : 16;
  const int k = threadIdx.x / NS, j = threadIdx.x % NS;
  const int64_t sb = c * kSbPerCta + k;
  if (k < kSbPerCta && sb < t.nsb) {
    float a, m;
    grid_of<T>(t.raw + sb * block_bytes(T), j, a, m);
    int64_t o = sb * NS + j;
    if (t.gpitch) {   // column-major: (row, sub-block s) at s * gpitch + row
      const int64_t row = sb / t.nsb_row, sub = (sb % t.nsb_row) * NS + j;
      o = sub * t.gpitch + row;
    }
    t.dl[o] = a;
    if (t.ml) t.ml[o] = m;
  }
}

// Codes of superblocks [c*16, c*16 + 16) into their bit fields; scales and super-scales are
// left as committed.  The 16 x 256 codes come in with one 16-byte load per thread.
template <int T>
__device__ __forceinline__ void repack_sb(const SbDesc& t, int64_t c) {
  __shared__ __align__(16) int8_t cs[kSbPerCta][256];
  const int64_t sb0 = c * kSbPerCta;
  const int nsb = (int)min((int64_t)kSbPerCta, t.nsb - sb0);
  {
    const int k = threadIdx.x >> 4, q = threadIdx.x & 15;
    if (k < nsb) reinterpret_cast<uint4*>(cs[k])[q] = reinterpret_cast<const uint4*>(t.codes + (sb0 + k) * 256)[q];
  }
  __syncthreads();
  const int th = threadIdx.x;
  for (int k = 0; k < nsb; k++) {
    const int8_t* cc = cs[k];
    uint8_t* b = t.raw_w + (sb0 + k) * block_bytes(T);
    if (T == kQ2_K) {
      if (th < 64) {
        const int h = th >> 5, l = th & 31;
        const int8_t* s = cc + h * 128 + l;
        b[16 + th] = (uint8_t)((s[0] & 3) | ((s[32] & 3) << 2) | ((s[64] & 3) << 4) | ((s[96] & 3) << 6));
      }
    } else if (T == kQ3_K) {
      if (th < 32) {
        uint8_t m = 0;
        for (int j = 0; j < 8; j++) m |= (uint8_t)((cc[32 * j + th] + 4 > 3 ? 1 : 0) << j);
        b[th] = m;
      } else if (th < 96) {
        const int q = th - 32, h = q >> 5, l = q & 31;
        uint8_t v = 0;
        for (int kk = 0; kk < 4; kk++) {
          int x = cc[h * 128 + 32 * kk + l] + 4;
          x = x > 3 ? x - 4 : x;
          v |= (uint8_t)((x & 3) << (2 * kk));
        }
        b[32 + q] = v;
      }
    } else if (T == kQ4_K || T == kQ5_K) {
      const int off = (T == kQ5_K) ? 48 : 16;
      if (th < 128) {
        const int g = th >> 5, l = th & 31;
        int lo = cc[g * 64 + l], hi = cc[g * 64 + 32 + l];
        if (T == kQ5_K) {
          lo = lo > 15 ? lo - 16 : lo;
          hi = hi > 15 ? hi - 16 : hi;
        }
        b[off + th] = (uint8_t)((lo & 0xF) | ((hi & 0xF) << 4));
      } else if (T == kQ5_K && th < 160) {
        const int l = th - 128;
        uint8_t m = 0;
        for (int g = 0; g < 4; g++) {
          m |= (uint8_t)((cc[g * 64 + l] > 15 ? 1 : 0) << (2 * g));
          m |= (uint8_t)((cc[g * 64 + 32 + l] > 15 ? 1 : 0) << (2 * g + 1));
        }
        b[16 + l] = m;
      }
    } else {
      if (th < 128) {
        const int h = th >> 6, r = th & 63, l = r & 31;
        const int base = h * 128 + l;
        b[th] = (r < 32) ? (uint8_t)(((cc[base] + 32) & 0xF) | (((cc[base + 64] + 32) & 0xF) << 4))
                         : (uint8_t)(((cc[base + 32] + 32) & 0xF) | (((cc[base + 96] + 32) & 0xF) << 4));
      } else if (th < 192) {
        const int q = th - 128, h = q >> 5, l = q & 31;
        const int base = h * 128 + l;
        b[128 + q] = (uint8_t)(((cc[base] + 32) >> 4) | (((cc[base + 32] + 32) >> 4) << 2) |
                               (((cc[base + 64] + 32) >> 4) << 4) | (((cc[base + 96] + 32) >> 4) << 6));
      }
    }
  }
}


// Weighted squared error of superblocks [c*16, c*16 + 16) of one tensor, one atomic per CTA.
// The group's raw bytes and its sub-block (dl, ml) pairs are staged in shared memory once;
// each thread then decodes one element per superblock.
template <int T>
__device__ __forceinline__ void werr_sb(const SbDesc& t, int64_t c) {
  constexpr int SW = (T == kQ4_K || T == kQ5_K) ? 32 : 16;
  constexpr int NS = 256 / SW;
  constexpr int BB = block_bytes(T);
  __shared__ __align__(16) uint8_t sraw[kSbPerCta * 210];
  __shared__ float sdl[kSbPerCta][16], sml[kSbPerCta][16];
  const int i = threadIdx.x;
  const int64_t sb0 = c * kSbPerCta;
  const int nsb = (int)min((int64_t)kSbPerCta, t.nsb - sb0);
  const uint8_t* src = t.raw + sb0 * BB;
  const int nbytes = nsb * BB;
  if (((reinterpret_cast<uintptr_t>(src) | (uintptr_t)nbytes) & 3) == 0) {  // 4-byte words
    const uint32_t* s4 = reinterpret_cast<const uint32_t*>(src);
    for (int k = i; k < nbytes / 4; k += 256) reinterpret_cast<uint32_t*>(sraw)[k] = s4[k];
  } else {
    for (int k = i; k < nbytes; k += 256) sraw[k] = src[k];
  }
  __syncthreads();
  if (i < nsb * NS) {
    const int k = i / NS, j = i % NS;
    float a, m;
    grid_of<T>(sraw + k * BB, j, a, m);
    sdl[k][j] = a;
    sml[k][j] = m;
  }
  __syncthreads();
  double acc = 0.0;
  int64_t wrow = sb0 % t.nsb_row;  // superblock column of the weight row, stepped with wrap
  const float* __restrict__ xs = t.x + sb0 * 256 + i;
  for (int k = 0; k < nsb; k++) {
    float v = sdl[k][i / SW] * (float)code_of<T>(sraw + k * BB, i);
    if (!(T == kQ3_K || T == kQ6_K)) v = v - sml[k][i / SW];
    const float d = v - xs[k * 256];
    const float wt = t.w ? t.w[wrow * 256 + i] : 1.0f;
    acc += (double)(d * d * wt);
    wrow = (wrow + 1 == t.nsb_row) ? 0 : wrow + 1;
  }
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  __shared__ double red[8];
  if ((i & 31) == 0) red[i >> 5] = acc;
  __syncthreads();
  if (i == 0) {
    double s2 = 0.0;
    for (int k = 0; k < 8; k++) s2 += red[k];
    atomicAdd(t.err, s2);
  }
}

template <int OP>
__global__ void __launch_bounds__(256) sb_batch_kernel(const __grid_constant__ SbBatch b) {
  int lo = 0, hi = b.count - 1;
  const int64_t cta = blockIdx.x;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (b.d[mid].sb0 <= cta) lo = mid;
    else hi = mid - 1;
  }
  const SbDesc& t = b.d[lo];
  const int64_t sb = cta - t.sb0;   // index of the CTA's group of 16 superblocks
#define CPK_SB_OP(T)                              \
  if (OP == 0) grid_sb<T>(t, sb);                 \
  else if (OP == 1) repack_sb<T>(t, sb);          \
  else werr_sb<T>(t, sb);
  switch (t.type) {
    case kQ2_K: CPK_SB_OP(kQ2_K) break;
    case kQ3_K: CPK_SB_OP(kQ3_K) break;
    case kQ4_K: CPK_SB_OP(kQ4_K) break;
    case kQ5_K: CPK_SB_OP(kQ5_K) break;
    default: CPK_SB_OP(kQ6_K) break;
  }
#undef CPK_SB_OP
}

int launch_sb_batch(int op, const SbBatch& b, int64_t total_sb, cudaStream_t stream) {
  if (b.count == 0 || total_sb == 0) return 0;
  if (op == 0) sb_batch_kernel<0><<<(unsigned)total_sb, 256, 0, stream>>>(b);
  else if (op == 1) sb_batch_kernel<1><<<(unsigned)total_sb, 256, 0, stream>>>(b);
  else sb_batch_kernel<2><<<(unsigned)total_sb, 256, 0, stream>>>(b);
  note_launch();
  return 0;
}

#define CPK_DISPATCH_K(type, KERNEL_CALL) \
  switch (type) {                         \
    case kQ2_K: { constexpr int T = kQ2_K; KERNEL_CALL; } break; \
    case kQ3_K: { constexpr int T = kQ3_K; KERNEL_CALL; } break; \
    case kQ4_K: { constexpr int T = kQ4_K; KERNEL_CALL; } break; \
    case kQ5_K: { constexpr int T = kQ5_K; KERNEL_CALL; } break; \
    case kQ6_K: { constexpr int T = kQ6_K; KERNEL_CALL; } break; \
    default: return 1;                    \
  }

int launch_dequantize(int type, const uint8_t* raw, int64_t nrow, int64_t n, float* out, cudaStream_t stream) {
  if (type == kQ8_0) {
    const int64_t nblk = nrow * (n / 32);
    if (nblk) {
      dequant_q80_kernel<<<(unsigned)((nblk * 32 + 255) / 256), 256, 0, stream>>>(raw, nblk, out);
      note_launch();
    }
    return 0;
  }
  const int64_t nsb = nrow * (n / 256);
  if (nsb == 0) return 0;
  CPK_DISPATCH_K(type, (dequant_kernel<T><<<(unsigned)nsb, 256, 0, stream>>>(raw, nsb, out)));
  note_launch();
  return 0;
}

int launch_grid_params(int type, const uint8_t* raw, int64_t nrow, int64_t n, float* dl, float* ml,
                       cudaStream_t stream) {
  int sbw, lo, hi;
  bool hm;
  if (!grid_spec(type, &sbw, &lo, &hi, &hm)) return 1;
  const int64_t ns = nrow * (n / sbw);
  if (ns == 0) return 0;
  const unsigned g = (unsigned)((ns + 255) / 256);
  CPK_DISPATCH_K(type, (grid_kernel<T><<<g, 256, 0, stream>>>(raw, ns, dl, ml)));
  note_launch();
  return 0;
}

int launch_codes(int type, const uint8_t* raw, int64_t nrow, int64_t n, int8_t* codes, cudaStream_t stream) {
  const int64_t nsb = nrow * (n / 256);
  if (nsb == 0) return 0;
  CPK_DISPATCH_K(type, (codes_kernel<T><<<(unsigned)nsb, 256, 0, stream>>>(raw, nsb, codes)));
  note_launch();
  return 0;
}

int launch_repack(int type, uint8_t* raw, const int8_t* codes, int64_t nrow, int64_t n, cudaStream_t stream) {
  const int64_t nsb = nrow * (n / 256);
  if (nsb == 0) return 0;
  CPK_DISPATCH_K(type, (repack_kernel<T><<<(unsigned)nsb, 256, 0, stream>>>(raw, codes, nsb)));
  note_launch();
  return 0;
}

// hessians.py:225-245 load_hessian: H = float64(H16) * hscale, then the exact float32
// diagonal written over it (diag32 may be null for the old float32-only layout).
__global__ void hessian_decode_kernel(const uint16_t* __restrict__ h16, const float* __restrict__ diag32, double hscale,
                                      int64_t d, double* __restrict__ H) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= d * d) return;
  const int64_t r = i / d, c = i - r * d;
  double v = (double)__half2float(__ushort_as_half(h16[i])) * hscale;
  if (r == c && diag32) v = (double)diag32[r];
  H[i] = v;
}

int launch_hessian_decode(const uint16_t* h16, const float* diag32, double hscale, int64_t d, double* H,
                          cudaStream_t stream) {
  const int64_t n = d * d;
  if (n == 0) return 0;
  hessian_decode_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(h16, diag32, hscale, d, H);
  note_launch();
  return 0;
}

int launch_weighted_err(int type, const uint8_t* raw, const float* x, const float* w, int64_t nrow, int64_t n,
                        double* out, cudaStream_t stream) {
  const int64_t nsb = nrow * (n / 256);
  if (cudaMemsetAsync(out, 0, sizeof(double), stream) != cudaSuccess) return 3;
  if (nsb == 0) return 0;
  const unsigned g = (unsigned)(nsb < 4096 ? nsb : 4096);
  CPK_DISPATCH_K(type, (weighted_err_kernel<T><<<g, 256, 0, stream>>>(raw, x, w, nsb, n / 256, out)));
  note_launch();
  return 0;
}

}  // namespace cpk
