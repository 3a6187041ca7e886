// Per-thread k-quant block fitters: one thread fits one sub-block held in registers.
// Each function restates one numpy fitter of coldpress/kquant.py with the same operation
// order, so results are bit-identical (translation units are built with -fmad=false).
#pragma once
#include "kq_common.cuh"

namespace cpk {

// make_qkx_quants (kquant.py:42-94): asymmetric (scale, min) search over nstep+1 candidate
// inverse scales, weighted least squares per candidate, accept on lower weighted error.
// Instead of copying the candidate codes on acceptance, the (iscale, min) pair that produced
// them is recorded and the codes are recomputed once at the end (same arithmetic).
// Outputs: scale, -min and the codes as floats (0..nmax).
// The candidate loop runs on packed pairs (f32x2, with nz = -0.0 from a kernel argument) and
// keeps x - min in registers between acceptances; MAD takes |d| by clearing the sign bits.
template <int N, bool MAD, bool QKX3>
__device__ __forceinline__ void fit_qkx(const float (&x)[N], const float (&w)[N], int nmax, float rmin,
                                        float rdelta, int nstep, float& o_scale, float& o_negmin,
                                        float (&Lf)[N], float nz) {
  float mn = x[0], mx = x[0];
#pragma unroll
  for (int i = 1; i < N; i++) {
    mn = np_min_step(mn, x[i]);
    mx = np_max_step(mx, x[i]);
  }
  Pw8 pw, px;
#pragma unroll
  for (int i = 0; i < N; i++) {
    pw.addi(i, w[i]);
    px.addi(i, w[i] * x[i]);
  }
  const float sum_w = pw.total();
  const float sum_x = px.total();
  mn = np_minimum(mn, 0.0f);
  const bool dead = QKX3 ? (mx <= mn) : (mx == mn);
  const float span = dead ? 1.0f : mx - mn;
  const float iscale = (float)nmax / span;
  float scale = 1.0f / iscale;
  // An infinite inverse scale makes numpy's codes all 0 (inf, -inf and the x86 default NaN
  // all clip to the low end); reproduce that explicitly.
  const bool fin0 = iscale <= 3.4028234663852886e38f;
  float best;
  {
    Pw8 pb;
#pragma unroll
    for (int i = 0; i < N; i++) {
      float l = fin0 ? nint_clip_f(iscale * (x[i] - mn), 0, nmax) : 0.0f;
      float d = scale * l + mn - x[i];
      d = MAD ? fabsf(d) : d * d;
      pb.addi(i, w[i] * d);
    }
    best = pb.total();
  }
  float b_isc = iscale, b_mn = mn;
  bool b_fin = fin0;
  {
    static_assert(N % 16 == 0, "pairs fill the 8 accumulators");
    constexpr int P = N / 2;
    const f32x2 nz2 = pk2(nz, nz), magic2 = pk2(kMagic, kMagic);
    f32x2 xp[P], wp[P], xm[P];
#pragma unroll
    for (int k = 0; k < P; k++) {
      xp[k] = pk2(x[2 * k], x[2 * k + 1]);
      wp[k] = pk2(w[2 * k], w[2 * k + 1]);
    }
    {
      const f32x2 mn2 = pk2(mn, mn);
#pragma unroll
      for (int k = 0; k < P; k++) xm[k] = sub2(xp[k], mn2);
    }
#pragma unroll 1
    for (int step = 0; step <= nstep; step++) {
      float span_cur = mx - mn;
      span_cur = span_cur > 0.0f ? span_cur : 1.0f;
      const float isc = (rmin + rdelta * (float)step + (float)nmax) / span_cur;
      const f32x2 isc2 = pk2(isc, isc);
      f32x2 lf[P];
      Pw8x2 sl, sl2, sxl;
#pragma unroll
      for (int k = 0; k < P; k++) {
        lf[k] = nint_clip2(mul2(isc2, xm[k], nz2), 0, nmax, magic2);
        const f32x2 wl = mul2(wp[k], lf[k], nz2);
        sl.addk(k, wl);
        sl2.addk(k, mul2(wl, lf[k], nz2));
        sxl.addk(k, mul2(wl, xp[k], nz2));
      }
      const float sum_l = sl.total(), sum_l2 = sl2.total(), sum_xl = sxl.total();
      const float D = sum_w * sum_l2 - sum_l * sum_l;
      const bool ok = D > 0.0f && isc <= 3.4028234663852886e38f;
      if (ok && !dead) {
        float this_scale = (sum_w * sum_xl - sum_x * sum_l) / D;
        float this_min = (sum_l2 * sum_x - sum_l * sum_xl) / D;
        if (this_min > 0.0f) {
          this_min = 0.0f;
          this_scale = sum_xl / sum_l2;
        }
        const f32x2 ts2 = pk2(this_scale, this_scale), tm2 = pk2(this_min, this_min);
        Pw8x2 pc;
#pragma unroll
        for (int k = 0; k < P; k++) {
          const f32x2 d = sub2(add2(mul2(ts2, lf[k], nz2), tm2), xp[k]);
          pc.addk(k, mul2(wp[k], MAD ? abs2(d) : mul2(d, d, nz2), nz2));
        }
        const float cur = pc.total();
        if (cur < best) {
          best = cur;
          scale = this_scale;
          b_isc = isc;
          b_mn = mn;
          b_fin = true;
          mn = this_min;
          const f32x2 mn2 = pk2(mn, mn);
#pragma unroll
          for (int k = 0; k < P; k++) xm[k] = sub2(xp[k], mn2);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < N; i++)
    Lf[i] = (dead || !b_fin) ? 0.0f : nint_clip_f(b_isc * (x[i] - b_mn), 0, nmax);
  o_scale = dead ? 0.0f : scale;
  o_negmin = -mn;
}

// Index of the first maximum of |x| (np.argmax: first NaN wins).
template <int N>
__device__ __forceinline__ int argmax_abs(const float (&x)[N]) {
  int idx = 0;
  float best = fabsf(x[0]);
  bool nan_seen = best != best;
#pragma unroll
  for (int i = 1; i < N; i++) {
    const float v = fabsf(x[i]);
    const bool take = !nan_seen && ((v != v) || v > best);
    idx = take ? i : idx;
    best = take ? v : best;
    nan_seen = nan_seen || (v != v);
  }
  return idx;
}

template <int N>
__device__ __forceinline__ float select_idx(const float (&x)[N], int idx) {
  float v = x[0];
#pragma unroll
  for (int i = 1; i < N; i++) v = (i == idx) ? x[i] : v;
  return v;
}

// make_qx_quants with rmse_type 1 (kquant.py:97-133): symmetric scale search over 19
// candidates.  w holds the weights (the caller passes x*x when the reference uses qw=None).
// Returns the scale; L receives the codes as floats offset by +nmax.
template <int N>
// The per-candidate sums run on packed pairs (f32x2; nz = -0.0 from a kernel argument).
__device__ __forceinline__ float fit_qx(const float (&x)[N], const float (&w)[N], int nmax, float (&L)[N],
                                       float nz) {
  static_assert(N % 16 == 0, "pairs fill the 8 accumulators");
  constexpr int P = N / 2;
  const int idx = argmax_abs(x);
  const float xm = select_idx(x, idx);
  const float amax = fabsf(xm);
  const bool dead = amax < kGroupEps;
  const float mx = dead ? 1.0f : xm;
  const f32x2 nz2 = pk2(nz, nz), magic2 = pk2(kMagic, kMagic);
  f32x2 xp[P], wp[P], wxp[P];
#pragma unroll
  for (int k = 0; k < P; k++) {
    xp[k] = pk2(x[2 * k], x[2 * k + 1]);
    wp[k] = pk2(w[2 * k], w[2 * k + 1]);
    wxp[k] = mul2(wp[k], xp[k], nz2);  // wx = w * x
  }
  // sum(wx * l) and sum(w * l * l) for the codes l = clip(nearest_int(isc * x), -nmax, nmax - 1)
  auto sums = [&](float isc, float& slx, float& sl2) {
    const f32x2 isc2 = pk2(isc, isc);
    Pw8x2 a, b;
#pragma unroll
    for (int k = 0; k < P; k++) {
      const f32x2 lf = nint_clip2(mul2(isc2, xp[k], nz2), -nmax, nmax - 1, magic2);
      a.addk(k, mul2(wxp[k], lf, nz2));
      b.addk(k, mul2(mul2(wp[k], lf, nz2), lf, nz2));
    }
    slx = a.total();
    sl2 = b.total();
  };
  const float iscale = -(float)nmax / mx;
  float sumlx, suml2;
  sums(iscale, sumlx, suml2);
  float scale = (suml2 != 0.0f) ? sumlx / suml2 : 0.0f;
  float best = scale * sumlx;
  float b_isc = iscale;
#pragma unroll 1
  for (int s = -9; s <= 9; s++) {
    if (s == 0) continue;
    const float isc = -((float)nmax + 0.1f * (float)s) / mx;
    float slx, sl2;
    sums(isc, slx, sl2);
    if (sl2 > 0.0f && slx * slx > best * sl2 && !dead) {
      const float ns = slx / sl2;
      scale = ns;
      best = ns * slx;
      b_isc = isc;
    }
  }
#pragma unroll
  for (int i = 0; i < N; i++)
    L[i] = dead ? (float)nmax : nint_clip_f(b_isc * x[i], -nmax, nmax - 1) + (float)nmax;
  return dead ? 0.0f : scale;
}

// make_q3_quants (kquant.py:136-179), Q3_K reference path: w = x*x, up to 5 sweeps of
// per-element coordinate descent.  Codes returned offset by +nmax.
template <int N>
__device__ __forceinline__ float fit_q3(const float (&x)[N], int nmax, float (&Lout)[N]) {
  const int idx = argmax_abs(x);
  const float xm = select_idx(x, idx);
  const bool dead = fabsf(xm) < kGroupEps;
  const float mx = dead ? 1.0f : xm;
  const float iscale = -(float)nmax / mx;
  float L[N], w[N];
  Pw8 a, b;
#pragma unroll
  for (int i = 0; i < N; i++) {
    L[i] = nint_clip_f(iscale * x[i], -nmax, nmax - 1);
    w[i] = x[i] * x[i];
  }
#pragma unroll
  for (int i = 0; i < N; i++) {
    a.addi(i, w[i] * x[i] * L[i]);
    b.addi(i, w[i] * L[i] * L[i]);
  }
  float sumlx = a.total(), suml2 = b.total();
  bool active = !dead;
#pragma unroll 1
  for (int it = 0; it < 5 && active; it++) {
    bool changed = false;
#pragma unroll
    for (int i = 0; i < N; i++) {
      const float wi = w[i], xi = x[i], Li = L[i];
      const float slx = sumlx - wi * xi * Li;
      const float sl2 = suml2 - wi * Li * Li;
      const float den = (slx == 0.0f) ? 1.0f : slx;
      const float nl = nint_clip_f(xi * sl2 / den, -nmax, nmax - 1);
      const float slx2 = slx + wi * xi * nl;
      const float sl22 = sl2 + wi * nl * nl;
      const bool acc = slx > 0.0f && nl != Li && sl22 > 0.0f && slx2 * slx2 * suml2 > sumlx * sumlx * sl22;
      L[i] = acc ? nl : Li;
      sumlx = acc ? slx2 : sumlx;
      suml2 = acc ? sl22 : suml2;
      changed = changed || acc;
    }
    active = changed;
  }
  float scale = (suml2 > 0.0f) ? sumlx / suml2 : 0.0f;
#pragma unroll
  for (int i = 0; i < N; i++) Lout[i] = (dead ? 0.0f : L[i]) + (float)nmax;
  return dead ? 0.0f : scale;
}

// The rest of make_qp_quants (kquant.py:205-235) once the inverse scale is chosen: codes, then
// up to 5 coordinate-descent sweeps.  Codes are returned as the bytes numpy's astype(uint8)
// gives (values wrap through int32).
template <int N>
__device__ __forceinline__ float fit_qp_tail(const float (&x)[N], const float (&w)[N], int nmax, float iscale,
                                            bool dead, uint8_t (&Lout)[N]) {
  float L[N];
  Pw8 a, b;
#pragma unroll
  for (int i = 0; i < N; i++) L[i] = (float)min(nint(iscale * x[i]), nmax);
#pragma unroll
  for (int i = 0; i < N; i++) {
    a.addi(i, w[i] * x[i] * L[i]);
    b.addi(i, w[i] * L[i] * L[i]);
  }
  float sumlx = a.total(), suml2 = b.total();
  bool active = !dead;
#pragma unroll 1
  for (int it = 0; it < 5 && active; it++) {
    bool changed = false;
#pragma unroll
    for (int i = 0; i < N; i++) {
      const float wi = w[i], xi = x[i], Li = L[i];
      const float slx = sumlx - wi * xi * Li;
      const float sl2 = suml2 - wi * Li * Li;
      const float den = (slx == 0.0f) ? 1.0f : slx;
      const float nl = (float)min(nint(xi * sl2 / den), nmax);
      const float slx2 = slx + wi * xi * nl;
      const float sl22 = sl2 + wi * nl * nl;
      const bool acc = slx > 0.0f && sl2 > 0.0f && nl != Li && slx2 * slx2 * suml2 > sumlx * sumlx * sl22;
      L[i] = acc ? nl : Li;
      sumlx = acc ? slx2 : sumlx;
      suml2 = acc ? sl22 : suml2;
      changed = changed || acc;
    }
    active = changed;
  }
  float d = (suml2 > 0.0f) ? sumlx / suml2 : 0.0f;
#pragma unroll
  for (int i = 0; i < N; i++) Lout[i] = dead ? (uint8_t)0 : (uint8_t)(int32_t)L[i];
  return dead ? 0.0f : d;
}

// make_qp_quants (kquant.py:182-235): non-negative super-scale quantisation with 1 + 8
// candidates and up to 5 coordinate-descent sweeps.  N is 16 or 8.  Codes are returned as
// the bytes numpy's astype(uint8) gives (values wrap through int32).
template <int N>
__device__ __forceinline__ float fit_qp(const float (&x)[N], const float (&w)[N], int nmax, uint8_t (&Lout)[N]) {
  float mx = x[0];
#pragma unroll
  for (int i = 1; i < N; i++) mx = np_max_step(mx, x[i]);
  const bool dead = mx < kGroupEps;
  const float mxs = dead ? 1.0f : mx;
  float iscale = (float)nmax / mxs;
  float best_mse;
  {
    const float scale = 1.0f / iscale;
    Pw8 p;
#pragma unroll
    for (int i = 0; i < N; i++) {
      const float l0 = (float)nint(iscale * x[i]);
      const float d = x[i] - scale * l0;
      p.addi(i, w[i] * d * d);
    }
    best_mse = p.total();
  }
#pragma unroll 1
  for (int s = -4; s <= 4; s++) {
    if (s == 0) continue;
    const float isc = (0.1f * (float)s + (float)nmax) / mxs;
    const float sc = 1.0f / isc;
    Pw8 p;
#pragma unroll
    for (int i = 0; i < N; i++) {
      const float l = (float)min(nint(isc * x[i]), nmax);
      const float d = x[i] - sc * l;
      p.addi(i, w[i] * d * d);
    }
    const float mse = p.total();
    if (mse < best_mse && !dead) {
      best_mse = mse;
      iscale = isc;
    }
  }
  return fit_qp_tail<N>(x, w, nmax, iscale, dead, Lout);
}

// Sum over an N-lane segment (N = 16 or 8) of one value per lane, in numpy's pairwise order
// for N contiguous values with lane j as element j (Pw8: lane j < 8 adds lane j + 8, then
// ((0+1)+(2+3))+((4+5)+(6+7)), then the +0 identity); every lane of the segment gets it.
template <int N>
__device__ __forceinline__ float seg_pw_sum(float v) {
  if (N == 16) v = v + __shfl_down_sync(0xffffffffu, v, 8, 16);
  v = v + __shfl_xor_sync(0xffffffffu, v, 1, N);
  v = v + __shfl_xor_sync(0xffffffffu, v, 2, N);
  v = v + __shfl_xor_sync(0xffffffffu, v, 4, N);
  return __shfl_sync(0xffffffffu, 0.0f + v, 0, N);
}

// Maximum over an N-lane segment with np_max_step's NaN rule.  Equal values give the same
// value in any order except for the sign of a zero maximum, which only ever meets the
// dead-block test (max < 1e-15) and so cannot change a result.
template <int N>
__device__ __forceinline__ float seg_max(float v) {
#pragma unroll
  for (int o = 1; o < N; o <<= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o, N);
    v = (v > u || v != v) ? v : u;
  }
  return v;
}

// make_qp_quants' scale search (kquant.py:182-204) for the two problems an N-lane segment
// carries (the sub-block scales and the sub-block mins), one element per lane: lane j holds
// element j of each (xa, xb) and its weight.  Each candidate's weighted error is reduced
// across the segment in numpy's order, so the choice is the sequential fit's.  Returns each
// problem's chosen inverse scale and dead flag, for fit_qp_tail.
template <int N>
__device__ __forceinline__ void fit_qp_search_lanes(float xa, float xb, float wme, int nmax, float& isc_a,
                                                    bool& dead_a, float& isc_b, bool& dead_b) {
  auto search = [&](float xv, float& isc_out, bool& dead_out) {
    const float mx = seg_max<N>(xv);
    const bool dead = mx < kGroupEps;
    const float mxs = dead ? 1.0f : mx;
    float iscale = (float)nmax / mxs;
    float best;
    {
      const float scale = 1.0f / iscale;
      const float l0 = (float)nint(iscale * xv);
      const float d = xv - scale * l0;
      best = seg_pw_sum<N>(wme * d * d);
    }
#pragma unroll 1
    for (int s = -4; s <= 4; s++) {
      if (s == 0) continue;
      const float isc = (0.1f * (float)s + (float)nmax) / mxs;
      const float sc = 1.0f / isc;
      const float l = (float)min(nint(isc * xv), nmax);
      const float d = xv - sc * l;
      const float mse = seg_pw_sum<N>(wme * d * d);
      if (mse < best && !dead) {
        best = mse;
        iscale = isc;
      }
    }
    isc_out = iscale;
    dead_out = dead;
  };
  search(xa, isc_a, dead_a);
  search(xb, isc_b, dead_b);
}

}  // namespace cpk
