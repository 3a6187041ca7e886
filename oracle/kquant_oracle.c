/*
 * CPU ORACLE -- test infrastructure only, never shipped or called by the product path.
 *
 * Scalar C restatement of coldpress's numpy k-quant codec (coldpress/kquant.py) and of the
 * error-feedback column sweep (coldpress/ef.py:194-216).  It exists so the CUDA kernels can
 * be checked byte-for-byte on the GPU box, where the Python reference is not available.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it.
 *
 * Parity pin: the fixtures under tests/golden were produced by running the reference kquant.py / ef.py
 * (tests/golden/make_golden.py); tests/test_oracle_golden.py checks this file against them.
 *
 * numpy semantics reproduced here (each was probed on the reference's numpy 2.3):
 *   - arr.sum(axis, dtype=float32) over a contiguous row = 0.0f + pairwise(row):
 *     8 accumulators for 8 <= n <= 128, recursive halving (rounded down to a multiple of 8)
 *     above 128; the +0 identity turns an all -0 sum into +0.
 *   - arr.max/min over <= 16 elements: acc = a[0]; acc = (acc OP a[i] || isnan(acc)) ? acc : a[i]
 *     (the later of two equal values wins, which fixes the sign of zero).
 *   - np.minimum(a, b) = (a < b || isnan(a)) ? a : b.
 *   - argmax returns the first maximum (the first NaN if any).
 *   - every elementwise expression is evaluated left to right, one IEEE rounding per
 *     operation, no fused multiply-add (build with -ffp-contract=off).
 *   - float -> uint8 casts wrap through int32; float32 -> float16 is round-to-nearest-even.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define QK 256
#define EPS_GROUP 1e-15f

enum { T_Q8_0 = 8, T_Q2_K = 10, T_Q3_K = 11, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14 };

/* ------------------------------------------------------------------ numpy primitives */

/* kquant.py:25-28 nearest_int: fp32 magic add, keep the low 23 bits, re-centre. */
static inline int32_t o_nint(float x) {
    float y = x + 12582912.0f;
    int32_t i;
    memcpy(&i, &y, 4);
    return (i & 0x007FFFFF) - 0x00400000;
}

static inline int32_t o_clampi(int32_t v, int32_t lo, int32_t hi) {
    return v < lo ? lo : (v > hi ? hi : v);
}

static float o_pairwise(const float *a, int n) {
    if (n < 8) {
        float r = -0.0f;
        for (int i = 0; i < n; i++) r += a[i];
        return r;
    }
    if (n <= 128) {
        float r[8];
        for (int j = 0; j < 8; j++) r[j] = a[j];
        int i;
        for (i = 8; i < n - (n % 8); i += 8)
            for (int j = 0; j < 8; j++) r[j] += a[i + j];
        float res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
        for (; i < n; i++) res += a[i];
        return res;
    }
    int n2 = n / 2;
    n2 -= n2 % 8;
    return o_pairwise(a, n2) + o_pairwise(a + n2, n - n2);
}

/* row.sum(dtype=float32): the add-reduction starts from its +0 identity. */
static inline float o_sum(const float *a, int n) { return 0.0f + o_pairwise(a, n); }

static float o_max(const float *a, int n) {
    float acc = a[0];
    for (int i = 1; i < n; i++) acc = (acc > a[i] || isnan(acc)) ? acc : a[i];
    return acc;
}

static float o_min(const float *a, int n) {
    float acc = a[0];
    for (int i = 1; i < n; i++) acc = (acc < a[i] || isnan(acc)) ? acc : a[i];
    return acc;
}

static inline float o_minimum(float a, float b) { return (a < b || isnan(a)) ? a : b; }

static int o_argmax_abs(const float *x, int n) {
    int idx = 0;
    float best = fabsf(x[0]);
    if (isnan(best)) return 0;
    for (int i = 1; i < n; i++) {
        float v = fabsf(x[i]);
        if (isnan(v)) return i;
        if (v > best) { best = v; idx = i; }
    }
    return idx;
}

static inline uint8_t o_f2u8(float v) { return (uint8_t)(int32_t)v; }

/* IEEE binary32 -> binary16 bits, round to nearest even (numpy astype(float16)). */
static uint16_t o_f16bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    uint32_t sign = (u >> 16) & 0x8000u;
    uint32_t ex = (u >> 23) & 0xFFu;
    uint32_t man = u & 0x7FFFFFu;
    if (ex == 0xFFu) return (uint16_t)(sign | 0x7C00u | (man ? 0x200u | (man >> 13) : 0u));
    int32_t e = (int32_t)ex - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        uint32_t m = man | 0x800000u;
        uint32_t shift = (uint32_t)(14 - e);
        uint32_t h = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

static float o_f16tof32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t ex = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t u;
    if (ex == 0) {
        if (man == 0) {
            u = sign;
        } else {
            int e = -1;
            do { man <<= 1; e++; } while (!(man & 0x400u));
            man &= 0x3FFu;
            u = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (ex == 0x1Fu) {
        u = sign | 0x7F800000u | (man << 13);
    } else {
        u = sign | ((ex - 15 + 127) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline float o_fp16rt(float f) { return o_f16tof32(o_f16bits(f)); }

static inline void o_put16(uint8_t *p, uint16_t v) { p[0] = (uint8_t)(v & 0xFF); p[1] = (uint8_t)(v >> 8); }
static inline uint16_t o_get16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* ------------------------------------------------------------------ fitters */

/* kquant.py:42-94 make_qkx_quants (qkx2 / qkx3), one block of n (16 or 32) values. */
static void o_make_qkx(const float *x, const float *w, int n, int nmax, float rmin, float rdelta,
                       int nstep, int use_mad, int qkx3, float *o_scale, float *o_negmin, uint8_t *L) {
    float t[32];
    float mn = o_min(x, n);
    float mx = o_max(x, n);
    float sum_w = o_sum(w, n);
    for (int i = 0; i < n; i++) t[i] = w[i] * x[i];
    float sum_x = o_sum(t, n);
    mn = o_minimum(mn, 0.0f);
    int dead = qkx3 ? (mx <= mn) : (mx == mn);
    float span = dead ? 1.0f : mx - mn;
    float iscale = (float)nmax / span;
    float scale = 1.0f / iscale;
    for (int i = 0; i < n; i++) {
        int32_t l = o_clampi(o_nint(iscale * (x[i] - mn)), 0, nmax);
        L[i] = (uint8_t)l;
        float d = scale * (float)l + mn - x[i];
        d = use_mad ? fabsf(d) : d * d;
        t[i] = w[i] * d;
    }
    float best = o_sum(t, n);
    uint8_t laux[32];
    float lf[32], wl[32];
    for (int step = 0; step <= nstep; step++) {
        float span_cur = mx - mn;
        if (!(span_cur > 0.0f)) span_cur = 1.0f;
        float isc = (rmin + rdelta * (float)step + (float)nmax) / span_cur;
        for (int i = 0; i < n; i++) {
            int32_t l = o_clampi(o_nint(isc * (x[i] - mn)), 0, nmax);
            laux[i] = (uint8_t)l;
            lf[i] = (float)l;
            wl[i] = w[i] * lf[i];
        }
        float sum_l = o_sum(wl, n);
        for (int i = 0; i < n; i++) t[i] = wl[i] * lf[i];
        float sum_l2 = o_sum(t, n);
        for (int i = 0; i < n; i++) t[i] = wl[i] * x[i];
        float sum_xl = o_sum(t, n);
        float D = sum_w * sum_l2 - sum_l * sum_l;
        int ok = D > 0.0f;
        float this_scale = (sum_w * sum_xl - sum_x * sum_l) / D;
        float this_min = (sum_l2 * sum_x - sum_l * sum_xl) / D;
        float alt_scale = sum_xl / sum_l2;
        if (this_min > 0.0f) { this_min = 0.0f; this_scale = alt_scale; }
        for (int i = 0; i < n; i++) {
            float d = this_scale * lf[i] + this_min - x[i];
            d = use_mad ? fabsf(d) : d * d;
            t[i] = w[i] * d;
        }
        float cur = o_sum(t, n);
        if (ok && cur < best && !dead) {
            memcpy(L, laux, (size_t)n);
            best = cur;
            scale = this_scale;
            mn = this_min;
        }
    }
    if (dead) {
        scale = 0.0f;
        memset(L, 0, (size_t)n);
    }
    *o_scale = scale;
    *o_negmin = -mn;
}

/* kquant.py:97-133 make_qx_quants (rmse_type 1).  w == NULL means w = x*x.
 * Returns codes offset by +nmax. */
static float o_make_qx(const float *x, const float *wq, int n, int nmax, int32_t *Lout) {
    float w[32], t[32], lf[32];
    int32_t L[32], l[32];
    int idx = o_argmax_abs(x, n);
    float amax = fabsf(x[idx]);
    float mx = x[idx];
    int dead = amax < EPS_GROUP;
    if (dead) mx = 1.0f;
    for (int i = 0; i < n; i++) w[i] = wq ? wq[i] : x[i] * x[i];
    float iscale = -(float)nmax / mx;
    float sumlx, suml2;
    for (int i = 0; i < n; i++) {
        L[i] = o_clampi(o_nint(iscale * x[i]), -nmax, nmax - 1);
        lf[i] = (float)L[i];
    }
    for (int i = 0; i < n; i++) t[i] = w[i] * x[i] * lf[i];
    sumlx = o_sum(t, n);
    for (int i = 0; i < n; i++) t[i] = w[i] * lf[i] * lf[i];
    suml2 = o_sum(t, n);
    float scale = (suml2 != 0.0f) ? sumlx / suml2 : 0.0f;
    float best = scale * sumlx;
    for (int s = -9; s <= 9; s++) {
        if (s == 0) continue;
        float isc = -((float)nmax + 0.1f * (float)s) / mx;
        for (int i = 0; i < n; i++) {
            l[i] = o_clampi(o_nint(isc * x[i]), -nmax, nmax - 1);
            lf[i] = (float)l[i];
        }
        for (int i = 0; i < n; i++) t[i] = w[i] * x[i] * lf[i];
        float slx = o_sum(t, n);
        for (int i = 0; i < n; i++) t[i] = w[i] * lf[i] * lf[i];
        float sl2 = o_sum(t, n);
        if (sl2 > 0.0f && slx * slx > best * sl2 && !dead) {
            float ns = slx / sl2;
            memcpy(L, l, sizeof(int32_t) * (size_t)n);
            scale = ns;
            best = ns * slx;
        }
    }
    if (dead) {
        scale = 0.0f;
        for (int i = 0; i < n; i++) L[i] = 0;
    }
    for (int i = 0; i < n; i++) Lout[i] = L[i] + nmax;
    return scale;
}

/* kquant.py:136-179 make_q3_quants (Q3_K reference path), codes offset by +nmax. */
static float o_make_q3(const float *x, int n, int nmax, int32_t *Lout) {
    float w[32], t[32], L[32];
    int idx = o_argmax_abs(x, n);
    float amax = fabsf(x[idx]);
    float mx = x[idx];
    int dead = amax < EPS_GROUP;
    if (dead) mx = 1.0f;
    float iscale = -(float)nmax / mx;
    for (int i = 0; i < n; i++) L[i] = (float)o_clampi(o_nint(iscale * x[i]), -nmax, nmax - 1);
    for (int i = 0; i < n; i++) w[i] = x[i] * x[i];
    for (int i = 0; i < n; i++) t[i] = w[i] * x[i] * L[i];
    float sumlx = o_sum(t, n);
    for (int i = 0; i < n; i++) t[i] = w[i] * L[i] * L[i];
    float suml2 = o_sum(t, n);
    int active = !dead;
    for (int it = 0; it < 5 && active; it++) {
        int changed = 0;
        for (int i = 0; i < n; i++) {
            float wi = w[i], xi = x[i], Li = L[i];
            float slx = sumlx - wi * xi * Li;
            int cond = slx > 0.0f;
            float sl2 = suml2 - wi * Li * Li;
            float den = (slx == 0.0f) ? 1.0f : slx;
            float nl = (float)o_clampi(o_nint(xi * sl2 / den), -nmax, nmax - 1);
            float slx2 = slx + wi * xi * nl;
            float sl22 = sl2 + wi * nl * nl;
            if (cond && nl != Li && sl22 > 0.0f && slx2 * slx2 * suml2 > sumlx * sumlx * sl22) {
                L[i] = nl;
                sumlx = slx2;
                suml2 = sl22;
                changed = 1;
            }
        }
        active = changed;
    }
    float scale = (suml2 > 0.0f) ? sumlx / suml2 : 0.0f;
    if (dead) scale = 0.0f;
    for (int i = 0; i < n; i++) Lout[i] = (dead ? 0 : (int32_t)L[i]) + nmax;
    return scale;
}

/* kquant.py:182-235 make_qp_quants (non-negative super-scales); n is 16 or 8. */
static float o_make_qp(const float *x, const float *w, int n, int nmax, uint8_t *Lout) {
    float t[16], L[16], diff[16];
    float mx = o_max(x, n);
    int dead = mx < EPS_GROUP;
    float mxs = dead ? 1.0f : mx;
    float iscale = (float)nmax / mxs;
    float scale = 1.0f / iscale;
    for (int i = 0; i < n; i++) {
        float l0 = (float)o_nint(iscale * x[i]);
        diff[i] = x[i] - scale * l0;
    }
    for (int i = 0; i < n; i++) t[i] = w[i] * diff[i] * diff[i];
    float best_mse = o_sum(t, n);
    for (int s = -4; s <= 4; s++) {
        if (s == 0) continue;
        float isc = (0.1f * (float)s + (float)nmax) / mxs;
        float sc = 1.0f / isc;
        for (int i = 0; i < n; i++) {
            int32_t l = o_nint(isc * x[i]);
            if (l > nmax) l = nmax;
            diff[i] = x[i] - sc * (float)l;
        }
        for (int i = 0; i < n; i++) t[i] = w[i] * diff[i] * diff[i];
        float mse = o_sum(t, n);
        if (mse < best_mse && !dead) {
            best_mse = mse;
            iscale = isc;
        }
    }
    for (int i = 0; i < n; i++) {
        int32_t l = o_nint(iscale * x[i]);
        if (l > nmax) l = nmax;
        L[i] = (float)l;
    }
    for (int i = 0; i < n; i++) t[i] = w[i] * x[i] * L[i];
    float sumlx = o_sum(t, n);
    for (int i = 0; i < n; i++) t[i] = w[i] * L[i] * L[i];
    float suml2 = o_sum(t, n);
    int active = !dead;
    for (int it = 0; it < 5 && active; it++) {
        int changed = 0;
        for (int i = 0; i < n; i++) {
            float wi = w[i], xi = x[i], Li = L[i];
            float slx = sumlx - wi * xi * Li;
            float sl2 = suml2 - wi * Li * Li;
            int cond = slx > 0.0f && sl2 > 0.0f;
            float den = (slx == 0.0f) ? 1.0f : slx;
            int32_t l = o_nint(xi * sl2 / den);
            if (l > nmax) l = nmax;
            float nl = (float)l;
            float slx2 = slx + wi * xi * nl;
            float sl22 = sl2 + wi * nl * nl;
            if (cond && nl != Li && slx2 * slx2 * suml2 > sumlx * sumlx * sl22) {
                L[i] = nl;
                sumlx = slx2;
                suml2 = sl22;
                changed = 1;
            }
        }
        active = changed;
    }
    float d = (suml2 > 0.0f) ? sumlx / suml2 : 0.0f;
    if (dead) d = 0.0f;
    for (int i = 0; i < n; i++) Lout[i] = dead ? 0 : o_f2u8(L[i]);
    return d;
}

/* ------------------------------------------------------------------ packers */

/* kquant.py:240-249: 2-bit codes, each 128-chunk interleaved as l, l+32, l+64, l+96. */
static void o_pack_2bit(const uint8_t *L, uint8_t *qs) {
    for (int h = 0; h < 2; h++)
        for (int l = 0; l < 32; l++) {
            const uint8_t *s = L + h * 128 + l;
            qs[h * 32 + l] = (uint8_t)(s[0] | (s[32] << 2) | (s[64] << 4) | (s[96] << 6));
        }
}

static void o_unpack_2bit(const uint8_t *qs, uint8_t *L) {
    for (int h = 0; h < 2; h++)
        for (int k = 0; k < 4; k++)
            for (int l = 0; l < 32; l++) L[h * 128 + k * 32 + l] = (qs[h * 32 + l] >> (2 * k)) & 3;
}

/* kquant.py:264-276 */
static void o_pack_scales_q3(const int32_t *Ls, uint8_t *out) {
    memset(out, 0, 12);
    for (int j = 0; j < 16; j++) {
        uint8_t lj = (uint8_t)Ls[j];
        if (j < 8) out[j] |= lj & 0xF;
        else out[j - 8] |= (uint8_t)((lj & 0xF) << 4);
        out[8 + j % 4] |= (uint8_t)((lj >> 4) << (2 * (j / 4)));
    }
}

/* kquant.py:279-290 */
static void o_unpack_scales_q3(const uint8_t *sc, int32_t *out) {
    for (int j = 0; j < 16; j++) {
        int32_t lo = (j < 8) ? (sc[j] & 0xF) : (sc[j - 8] >> 4);
        int32_t hi = (sc[8 + j % 4] >> (2 * (j / 4))) & 3;
        out[j] = lo | (hi << 4);
    }
}

/* kquant.py:293-307 */
static void o_pack_scales_k4(const uint8_t *ls, const uint8_t *lm, uint8_t *out) {
    memset(out, 0, 12);
    for (int j = 0; j < 8; j++) {
        if (j < 4) {
            out[j] = ls[j];
            out[j + 4] = lm[j];
        } else {
            out[j + 4] = (uint8_t)((ls[j] & 0xF) | ((lm[j] & 0xF) << 4));
            out[j - 4] |= (uint8_t)((ls[j] >> 4) << 6);
            out[j] |= (uint8_t)((lm[j] >> 4) << 6);
        }
    }
}

/* kquant.py:310-322 get_scale_min_k4 */
static void o_unpack_scales_k4(const uint8_t *sc, int32_t *d, int32_t *m) {
    for (int j = 0; j < 8; j++) {
        if (j < 4) {
            d[j] = sc[j] & 63;
            m[j] = sc[j + 4] & 63;
        } else {
            d[j] = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
            m[j] = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
        }
    }
}

/* kquant.py:325-332 */
static void o_pack_nibbles(const uint8_t *L, uint8_t *qs) {
    for (int c = 0; c < 4; c++)
        for (int l = 0; l < 32; l++)
            qs[c * 32 + l] = (uint8_t)((L[c * 64 + l] & 0xF) | ((L[c * 64 + 32 + l] & 0xF) << 4));
}

static void o_unpack_nibbles(const uint8_t *qs, uint8_t *L) {
    for (int c = 0; c < 4; c++)
        for (int l = 0; l < 32; l++) {
            L[c * 64 + l] = qs[c * 32 + l] & 0xF;
            L[c * 64 + 32 + l] = qs[c * 32 + l] >> 4;
        }
}

/* Q3_K codes 0..7 -> hmask + 2-bit qs (kquant.py:474-483, ef.py:137-145). */
static void o_pack_q3_codes(const int32_t *L, uint8_t *hmask, uint8_t *qs) {
    uint8_t lq[QK];
    memset(hmask, 0, 32);
    for (int i = 0; i < QK; i++) {
        int high = L[i] > 3;
        lq[i] = (uint8_t)(high ? L[i] - 4 : L[i]);
        if (high) hmask[i % 32] |= (uint8_t)(1u << (i / 32));
    }
    o_pack_2bit(lq, qs);
}

/* Q5_K codes 0..31 -> qh + nibbles (kquant.py:573-584, ef.py:153-161). */
static void o_pack_q5_codes(const uint8_t *L, uint8_t *qh, uint8_t *qs) {
    uint8_t ll[QK];
    memset(qh, 0, 32);
    for (int c = 0; c < 4; c++)
        for (int l = 0; l < 32; l++) {
            int a = c * 64 + l, b = c * 64 + 32 + l;
            qh[l] |= (uint8_t)(((L[a] > 15) ? 1 : 0) << (2 * c));
            qh[l] |= (uint8_t)(((L[b] > 15) ? 1 : 0) << (2 * c + 1));
        }
    for (int i = 0; i < QK; i++) ll[i] = (uint8_t)(L[i] > 15 ? L[i] - 16 : L[i]);
    o_pack_nibbles(ll, qs);
}

/* Q6_K codes 0..63 -> ql + qh (kquant.py:664-672, ef.py:163-174). */
static void o_pack_q6_codes(const uint8_t *L, uint8_t *ql, uint8_t *qh) {
    for (int h = 0; h < 2; h++)
        for (int l = 0; l < 32; l++) {
            const uint8_t *s = L + h * 128 + l;
            ql[h * 64 + l] = (uint8_t)((s[0] & 0xF) | ((s[64] & 0xF) << 4));
            ql[h * 64 + 32 + l] = (uint8_t)((s[32] & 0xF) | ((s[96] & 0xF) << 4));
            qh[h * 32 + l] = (uint8_t)((s[0] >> 4) | ((s[32] >> 4) << 2) | ((s[64] >> 4) << 4) |
                                       ((s[96] >> 4) << 6));
        }
}

/* ------------------------------------------------------------------ superblock encoders */

/* kquant.py:347-413 quantize_q2_K, one superblock. */
static void o_q2k_block(const float *x, const float *qw, uint8_t *out) {
    float scales[16], mins[16], w[QK];
    uint8_t L[QK];
    int32_t sc_i[16], mn_i[16];
    uint16_t d16, dmin16;
    if (!qw) {
        for (int i = 0; i < QK; i++) w[i] = fabsf(x[i]);
        for (int j = 0; j < 16; j++)
            o_make_qkx(x + 16 * j, w + 16 * j, 16, 3, -0.5f, 0.1f, 15, 1, 0, &scales[j], &mins[j],
                       L + 16 * j);
        float max_scale = o_max(scales, 16);
        float max_min = o_max(mins, 16);
        int pos = max_scale > 0.0f, posm = max_min > 0.0f;
        float isc = pos ? 15.0f / max_scale : 0.0f;
        float iscm = posm ? 15.0f / max_min : 0.0f;
        for (int j = 0; j < 16; j++) {
            sc_i[j] = pos ? o_nint(isc * scales[j]) : 0;
            mn_i[j] = posm ? o_nint(iscm * mins[j]) : 0;
        }
        d16 = o_f16bits(pos ? max_scale / 15.0f : 0.0f);
        dmin16 = o_f16bits(posm ? max_min / 15.0f : 0.0f);
    } else {
        float t[QK], sw[16];
        for (int i = 0; i < QK; i++) t[i] = x[i] * x[i];
        float sigma2 = o_sum(t, QK) / 256.0f;
        for (int i = 0; i < QK; i++) w[i] = qw[i] * sqrtf(sigma2 + x[i] * x[i]);
        for (int j = 0; j < 16; j++) sw[j] = o_sum(w + 16 * j, 16);
        for (int j = 0; j < 16; j++)
            o_make_qkx(x + 16 * j, w + 16 * j, 16, 3, -0.9f, 0.05f, 36, 0, 1, &scales[j], &mins[j],
                       L + 16 * j);
        uint8_t Ls[16], Lm[16];
        float dm = o_make_qp(scales, sw, 16, 15, Ls);
        float mm = o_make_qp(mins, sw, 16, 15, Lm);
        for (int j = 0; j < 16; j++) { sc_i[j] = Ls[j]; mn_i[j] = Lm[j]; }
        d16 = o_f16bits(dm);
        dmin16 = o_f16bits(mm);
    }
    float d = o_f16tof32(d16), dmin = o_f16tof32(dmin16);
    for (int j = 0; j < 16; j++) {
        float dl = d * (float)sc_i[j];
        float ml = dmin * (float)mn_i[j];
        if (dl != 0.0f)
            for (int i = 16 * j; i < 16 * j + 16; i++)
                L[i] = (uint8_t)o_clampi(o_nint((x[i] + ml) / dl), 0, 3);
        out[j] = (uint8_t)(((uint8_t)sc_i[j] & 0xF) | (((uint8_t)mn_i[j] & 0xF) << 4));
    }
    o_pack_2bit(L, out + 16);
    o_put16(out + 80, d16);
    o_put16(out + 82, dmin16);
}

/* kquant.py:432-486 quantize_q3_K, one superblock. */
static void o_q3k_block(const float *x, const float *qw, uint8_t *out) {
    float scales[16];
    int32_t L[QK], Ls[16];
    float d;
    if (!qw) {
        for (int j = 0; j < 16; j++) scales[j] = o_make_q3(x + 16 * j, 16, 4, L + 16 * j);
        int ai = o_argmax_abs(scales, 16);
        float max_scale = scales[ai];
        int nz = max_scale != 0.0f;
        float isc = nz ? -32.0f / max_scale : 0.0f;
        for (int j = 0; j < 16; j++) Ls[j] = nz ? o_clampi(o_nint(isc * scales[j]), -32, 31) + 32 : 0;
        d = nz ? 1.0f / isc : 0.0f;
        if (!isfinite(d)) d = 0.0f;
    } else {
        float t[QK], w[QK], sw[16];
        for (int i = 0; i < QK; i++) t[i] = x[i] * x[i];
        float sigma2 = 2.0f * o_sum(t, QK) / 256.0f;
        for (int i = 0; i < QK; i++) w[i] = qw[i] * sqrtf(sigma2 + x[i] * x[i]);
        for (int j = 0; j < 16; j++) sw[j] = o_sum(w + 16 * j, 16);
        for (int j = 0; j < 16; j++) scales[j] = o_make_qx(x + 16 * j, w + 16 * j, 16, 4, L + 16 * j);
        d = o_make_qx(scales, sw, 16, 32, Ls);
    }
    uint8_t *hmask = out, *qs = out + 32, *scp = out + 96;
    o_pack_scales_q3(Ls, scp);
    uint16_t d16 = o_f16bits(d);
    float df = o_f16tof32(d16);
    int32_t scu[16];
    o_unpack_scales_q3(scp, scu);
    for (int j = 0; j < 16; j++) {
        float ds = df * (float)(scu[j] - 32);
        if (ds != 0.0f)
            for (int i = 16 * j; i < 16 * j + 16; i++) L[i] = o_clampi(o_nint(x[i] / ds), -4, 3) + 4;
    }
    o_pack_q3_codes(L, hmask, qs);
    o_put16(out + 108, d16);
}

/* kquant.py:508-585 _quantize_q45_K, one superblock. */
static void o_q45k_block(const float *x, const float *qw, int nmax, int is_q5, uint8_t *out) {
    float scales[8], mins[8];
    uint8_t L[QK], Ls[8], Lm[8];
    float d, dmin;
    if (!qw) {
        float w[QK], t[32];
        for (int j = 0; j < 8; j++) {
            for (int i = 0; i < 32; i++) t[i] = x[32 * j + i] * x[32 * j + i];
            float av_x = sqrtf(o_sum(t, 32) / 32.0f);
            for (int i = 0; i < 32; i++) w[32 * j + i] = av_x + fabsf(x[32 * j + i]);
        }
        float rmin = is_q5 ? -0.5f : -1.0f;
        int nstep = is_q5 ? 15 : 20;
        for (int j = 0; j < 8; j++)
            o_make_qkx(x + 32 * j, w + 32 * j, 32, nmax, rmin, 0.1f, nstep, 0, 0, &scales[j], &mins[j],
                       L + 32 * j);
        float max_scale = o_max(scales, 8);
        float max_min = o_max(mins, 8);
        float inv_scale = max_scale > 0.0f ? 63.0f / max_scale : 0.0f;
        float inv_min = max_min > 0.0f ? 63.0f / max_min : 0.0f;
        for (int j = 0; j < 8; j++) {
            uint8_t a = (uint8_t)o_nint(inv_scale * scales[j]);
            uint8_t b = (uint8_t)o_nint(inv_min * mins[j]);
            Ls[j] = a < 63 ? a : 63;
            Lm[j] = b < 63 ? b : 63;
        }
        d = max_scale / 63.0f;
        dmin = max_min / 63.0f;
    } else {
        float t[QK], w[QK], sw[8];
        for (int i = 0; i < QK; i++) t[i] = x[i] * x[i];
        float sigma2 = 2.0f * o_sum(t, QK) / 256.0f;
        for (int i = 0; i < QK; i++) w[i] = qw[i] * sqrtf(sigma2 + x[i] * x[i]);
        for (int j = 0; j < 8; j++) sw[j] = o_sum(w + 32 * j, 32);
        for (int j = 0; j < 8; j++)
            o_make_qkx(x + 32 * j, w + 32 * j, 32, nmax, -0.9f, 0.05f, 36, 0, 1, &scales[j], &mins[j],
                       L + 32 * j);
        d = o_make_qp(scales, sw, 8, 63, Ls);
        dmin = o_make_qp(mins, sw, 8, 63, Lm);
        if (is_q5)
            for (int j = 0; j < 8; j++) {
                if (Ls[j] > 63) Ls[j] = 63;
                if (Lm[j] > 63) Lm[j] = 63;
            }
    }
    uint16_t d16 = o_f16bits(d), dmin16 = o_f16bits(dmin);
    uint8_t scp[12];
    o_pack_scales_k4(Ls, Lm, scp);
    int32_t su[8], mu[8];
    o_unpack_scales_k4(scp, su, mu);
    float df = o_f16tof32(d16), dmf = o_f16tof32(dmin16);
    for (int j = 0; j < 8; j++) {
        float ds = df * (float)su[j];
        float ms = dmf * (float)mu[j];
        if (ds != 0.0f)
            for (int i = 32 * j; i < 32 * j + 32; i++)
                L[i] = (uint8_t)o_clampi(o_nint((x[i] + ms) / ds), 0, nmax);
    }
    o_put16(out, d16);
    o_put16(out + 2, dmin16);
    memcpy(out + 4, scp, 12);
    if (!is_q5) {
        o_pack_nibbles(L, out + 16);
    } else {
        o_pack_q5_codes(L, out + 16, out + 48);
    }
}

/* kquant.py:632-678 quantize_q6_K, one superblock. */
static void o_q6k_block(const float *x, const float *qw, uint8_t *out) {
    float scales[16];
    int32_t Li[QK];
    for (int j = 0; j < 16; j++)
        scales[j] = o_make_qx(x + 16 * j, qw ? qw + 16 * j : NULL, 16, 32, Li + 16 * j);
    int ai = o_argmax_abs(scales, 16);
    float max_abs = fabsf(scales[ai]);
    float max_scale = scales[ai];
    int dead = max_abs < EPS_GROUP;
    float mxs = dead ? 1.0f : max_scale;
    float iscale = -128.0f / mxs;
    float d = 1.0f / iscale;
    int8_t sc[16];
    for (int j = 0; j < 16; j++) {
        int32_t v = o_nint(iscale * scales[j]);
        if (v > 127) v = 127;
        sc[j] = (int8_t)v;
    }
    uint16_t d16 = o_f16bits(dead ? 0.0f : d);
    float df = o_f16tof32(d16);
    uint8_t L[QK];
    for (int j = 0; j < 16; j++) {
        float ds = df * (float)sc[j];
        for (int i = 16 * j; i < 16 * j + 16; i++) {
            int32_t v = Li[i];
            if (ds != 0.0f && !dead) v = o_clampi(o_nint(x[i] / ds), -32, 31) + 32;
            if (dead) v = 0;
            L[i] = (uint8_t)v;
        }
    }
    if (dead) memset(sc, 0, 16);
    o_pack_q6_codes(L, out, out + 128);
    memcpy(out + 192, sc, 16);
    o_put16(out + 208, d16);
}

/* kquant.py:706-718 quantize_q8_0, one block of 32. */
static void o_q80_block(const float *x, uint8_t *out) {
    float ax[32];
    for (int i = 0; i < 32; i++) ax[i] = fabsf(x[i]);
    float amax = o_max(ax, 32);
    float d = amax / 127.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    o_put16(out, o_f16bits(d));
    for (int i = 0; i < 32; i++) {
        float x0 = x[i] * id;
        float sg = x0 > 0.0f ? 1.0f : (x0 < 0.0f ? -1.0f : x0);
        float q = sg * floorf(fabsf(x0) + 0.5f);
        out[2 + i] = (uint8_t)(int8_t)(int32_t)q;
    }
}

/* ------------------------------------------------------------------ exported API */

static int o_block_bytes(int type) {
    switch (type) {
    case T_Q2_K: return 84;
    case T_Q3_K: return 110;
    case T_Q4_K: return 144;
    case T_Q5_K: return 176;
    case T_Q6_K: return 210;
    case T_Q8_0: return 34;
    default: return 0;
    }
}

static int o_block_elems(int type) { return type == T_Q8_0 ? 32 : QK; }

int kqo_block_bytes(int type) { return o_block_bytes(type); }

static void o_set_threads(int nthreads) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
}

/* QUANTIZE[type](x, qw): x [nrow, n] f32 row-major, qw [n] or NULL, out [nrow, n/QK*bytes]. */
int kqo_quantize(int type, const float *x, int64_t nrow, int64_t n, const float *qw, uint8_t *out,
                 int nthreads) {
    int bb = o_block_bytes(type), be = o_block_elems(type);
    if (!bb) return 1;
    if (n % be) return 2;
    int64_t nsb = n / be, total = nrow * nsb;
    o_set_threads(nthreads);
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < total; b++) {
        const float *xb = x + b * be;
        const float *qb = qw ? qw + (b % nsb) * be : NULL;
        uint8_t *ob = out + b * bb;
        switch (type) {
        case T_Q2_K: o_q2k_block(xb, qb, ob); break;
        case T_Q3_K: o_q3k_block(xb, qb, ob); break;
        case T_Q4_K: o_q45k_block(xb, qb, 15, 0, ob); break;
        case T_Q5_K: o_q45k_block(xb, qb, 31, 1, ob); break;
        case T_Q6_K: o_q6k_block(xb, qb, ob); break;
        case T_Q8_0: o_q80_block(xb, ob); break;
        }
    }
    return 0;
}

/* Per-(superblock, sub-block) dl/ml of committed bytes (ef.py:87-127, the decoders'
 * scalars).  dl, ml: [nrow*nsb*nsub]; ml may be NULL; for Q3_K/Q6_K ml is written as 0. */
static int o_grid_block(int type, const uint8_t *b, float *dl, float *ml) {
    switch (type) {
    case T_Q2_K: {
        float d = o_f16tof32(o_get16(b + 80)), dm = o_f16tof32(o_get16(b + 82));
        for (int j = 0; j < 16; j++) {
            dl[j] = d * (float)(b[j] & 0xF);
            ml[j] = dm * (float)(b[j] >> 4);
        }
        return 16;
    }
    case T_Q3_K: {
        float d = o_f16tof32(o_get16(b + 108));
        int32_t s[16];
        o_unpack_scales_q3(b + 96, s);
        for (int j = 0; j < 16; j++) { dl[j] = d * (float)(s[j] - 32); ml[j] = 0.0f; }
        return 16;
    }
    case T_Q4_K:
    case T_Q5_K: {
        float d = o_f16tof32(o_get16(b)), dm = o_f16tof32(o_get16(b + 2));
        int32_t s[8], m[8];
        o_unpack_scales_k4(b + 4, s, m);
        for (int j = 0; j < 8; j++) { dl[j] = d * (float)s[j]; ml[j] = dm * (float)m[j]; }
        return 8;
    }
    case T_Q6_K: {
        float d = o_f16tof32(o_get16(b + 208));
        for (int j = 0; j < 16; j++) { dl[j] = d * (float)(int8_t)b[192 + j]; ml[j] = 0.0f; }
        return 16;
    }
    }
    return 0;
}

/* Integer codes of one superblock in the signed range used by ef.py (_grid_params lo..hi). */
static void o_codes_block(int type, const uint8_t *b, int32_t *q) {
    uint8_t L[QK];
    switch (type) {
    case T_Q2_K:
        o_unpack_2bit(b + 16, L);
        for (int i = 0; i < QK; i++) q[i] = L[i];
        break;
    case T_Q3_K:
        o_unpack_2bit(b + 32, L);
        for (int i = 0; i < QK; i++) q[i] = (int32_t)L[i] - (((b[i % 32] >> (i / 32)) & 1) ? 0 : 4);
        break;
    case T_Q4_K:
        o_unpack_nibbles(b + 16, L);
        for (int i = 0; i < QK; i++) q[i] = L[i];
        break;
    case T_Q5_K:
        o_unpack_nibbles(b + 48, L);
        for (int c = 0; c < 4; c++)
            for (int l = 0; l < 32; l++) {
                q[c * 64 + l] = L[c * 64 + l] + 16 * ((b[16 + l] >> (2 * c)) & 1);
                q[c * 64 + 32 + l] = L[c * 64 + 32 + l] + 16 * ((b[16 + l] >> (2 * c + 1)) & 1);
            }
        break;
    case T_Q6_K:
        for (int h = 0; h < 2; h++)
            for (int l = 0; l < 32; l++) {
                const uint8_t *ql = b + h * 64, *qh = b + 128 + h * 32;
                q[h * 128 + l] = ((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                q[h * 128 + 32 + l] = ((ql[32 + l] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                q[h * 128 + 64 + l] = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                q[h * 128 + 96 + l] = ((ql[32 + l] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
            }
        break;
    }
}

/* DEQUANTIZE[type](raw, n) (kquant.py:416-701): y = dl*q - ml, or dl*q without a min. */
int kqo_dequantize(int type, const uint8_t *raw, int64_t nrow, int64_t n, float *out, int nthreads) {
    int bb = o_block_bytes(type), be = o_block_elems(type);
    if (!bb) return 1;
    if (n % be) return 2;
    int64_t total = nrow * (n / be);
    o_set_threads(nthreads);
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < total; b++) {
        const uint8_t *blk = raw + b * bb;
        float *y = out + b * be;
        if (type == T_Q8_0) {
            float d = o_f16tof32(o_get16(blk));
            for (int i = 0; i < 32; i++) y[i] = d * (float)(int8_t)blk[2 + i];
            continue;
        }
        float dl[16], ml[16];
        int32_t q[QK];
        int nsub = o_grid_block(type, blk, dl, ml);
        int sw = QK / nsub;
        o_codes_block(type, blk, q);
        int has_min = (type == T_Q2_K || type == T_Q4_K || type == T_Q5_K);
        for (int i = 0; i < QK; i++) {
            float v = dl[i / sw] * (float)q[i];
            y[i] = has_min ? v - ml[i / sw] : v;
        }
    }
    return 0;
}

int kqo_grid_params(int type, const uint8_t *raw, int64_t nrow, int64_t n, float *dl, float *ml) {
    int bb = o_block_bytes(type);
    if (!bb || type == T_Q8_0) return 1;
    if (n % QK) return 2;
    int64_t total = nrow * (n / QK);
    for (int64_t b = 0; b < total; b++) {
        float a[16], m[16];
        int nsub = o_grid_block(type, raw + b * bb, a, m);
        memcpy(dl + b * nsub, a, sizeof(float) * (size_t)nsub);
        memcpy(ml + b * nsub, m, sizeof(float) * (size_t)nsub);
    }
    return 0;
}

/* Signed codes [nrow, n] (ef.py's L) of committed bytes. */
int kqo_codes(int type, const uint8_t *raw, int64_t nrow, int64_t n, int32_t *codes) {
    int bb = o_block_bytes(type);
    if (!bb || type == T_Q8_0) return 1;
    if (n % QK) return 2;
    int64_t total = nrow * (n / QK);
    for (int64_t b = 0; b < total; b++) o_codes_block(type, raw + b * bb, codes + b * QK);
    return 0;
}

/* ef.py:130-176 _repack: write signed codes L [nrow, n] into committed bytes (in place). */
int kqo_repack(int type, uint8_t *raw, const int32_t *codes, int64_t nrow, int64_t n) {
    int bb = o_block_bytes(type);
    if (!bb || type == T_Q8_0) return 1;
    if (n % QK) return 2;
    int64_t total = nrow * (n / QK);
    for (int64_t b = 0; b < total; b++) {
        uint8_t *blk = raw + b * bb;
        const int32_t *q = codes + b * QK;
        uint8_t L[QK];
        int32_t L3[QK];
        switch (type) {
        case T_Q2_K:
            for (int i = 0; i < QK; i++) L[i] = (uint8_t)q[i];
            o_pack_2bit(L, blk + 16);
            break;
        case T_Q3_K:
            for (int i = 0; i < QK; i++) L3[i] = q[i] + 4;
            o_pack_q3_codes(L3, blk, blk + 32);
            break;
        case T_Q4_K:
            for (int i = 0; i < QK; i++) L[i] = (uint8_t)q[i];
            o_pack_nibbles(L, blk + 16);
            break;
        case T_Q5_K:
            for (int i = 0; i < QK; i++) L[i] = (uint8_t)q[i];
            o_pack_q5_codes(L, blk + 16, blk + 48);
            break;
        case T_Q6_K:
            for (int i = 0; i < QK; i++) L[i] = (uint8_t)(q[i] + 32);
            o_pack_q6_codes(L, blk, blk + 128);
            break;
        }
    }
    return 0;
}

/* ------------------------------------------------------------------ EF column sweep */

/* One iteration of ef.py:197-213 for every row: wp = x[:, order]; for jj ascending,
 * quantize column order[jj] against its committed (dl, ml), e = (w - recon) / U[jj,jj],
 * wp[:, jj+1:] -= e (x) U[jj, jj+1:] with one rounding per multiply and per subtract.
 *   x      [nrow, n] f32 (storage order), order [n] int64, U [n, n] f32 row-major (upper),
 *   dl/ml  [nrow, n/sbw] (ml NULL for Q3_K/Q6_K), codes out [nrow, n] int32 (storage order),
 *   wfinal out [nrow, n] f32 (storage order, the compensated weights ef.py feeds back). */
int kqo_ef_sweep(const float *x, int64_t nrow, int64_t n, const int64_t *order, const float *U,
                 const float *dl, const float *ml, int sbw, int lo, int hi, int32_t *codes,
                 float *wfinal, int nthreads) {
    if (n <= 0 || sbw <= 0 || n % sbw) return 2;
    int64_t nsub = n / sbw;
    o_set_threads(nthreads);
#pragma omp parallel
    {
        float *wp = (float *)malloc(sizeof(float) * (size_t)n);
#pragma omp for schedule(dynamic, 1)
        for (int64_t r = 0; r < nrow; r++) {
            const float *xr = x + r * n;
            for (int64_t k = 0; k < n; k++) wp[k] = xr[order[k]];
            const float *dlr = dl + r * nsub;
            const float *mlr = ml ? ml + r * nsub : NULL;
            for (int64_t jj = 0; jj < n; jj++) {
                int64_t j = order[jj];
                float dlj = dlr[j / sbw];
                float mlj = mlr ? mlr[j / sbw] : 0.0f;
                int32_t q = 0;
                float e = 0.0f;
                if (dlj != 0.0f) {
                    q = o_clampi(o_nint((wp[jj] + mlj) / dlj), lo, hi);
                    float recon = dlj * (float)q - mlj;
                    e = (wp[jj] - recon) / U[jj * n + jj];
                }
                codes[r * n + j] = q;
                const float *urow = U + jj * n;
                for (int64_t k = jj + 1; k < n; k++) wp[k] = wp[k] - e * urow[k];
            }
            for (int64_t k = 0; k < n; k++) wfinal[r * n + order[k]] = wp[k];
        }
        free(wp);
    }
    return 0;
}
