// Device arithmetic of the LNS hot path (xlns16, xlns32, Monte, LPVIP).
//
// Every function here is integer arithmetic plus lookups into the host-built
// tables of lnsb_tables.cpp, so results do not depend on the GPU's floating
// point.  The semantics are those of the reference's LNS16/LNS32 CPU
// backends (xlnscpp configured with xlns16_table + xlns16_alt, xlns32_alt):
// lns-backend/cuda/lns-cuda-xlns16.cu:61-161, lns-cuda-xlns32.cu:30-67.
#pragma once

#include <cstdint>

#include "lnsb_tables.h"

namespace lnsb {

#ifndef LNSB_SUM_MODE
#define LNSB_SUM_MODE 0
#endif
enum : int { M_BASE = 0, M_MONTE = 1, M_MONTE_BYLPVIP = 2, M_LPVIP = 3, M_SUM32 = 4 };
constexpr int  k_mode       = LNSB_SUM_MODE;
constexpr bool k_stochastic = k_mode == M_MONTE || k_mode == M_MONTE_BYLPVIP;
constexpr bool k_acc32      = k_mode == M_LPVIP || k_mode == M_SUM32;

// Device copies of the tables, one set per GPU (lnsb_upload_tables).
struct dev_tables {
    const int16_t *  sbdb16;     // k16_tab_bytes, see lnsb_tables.h
    const uint16_t * conv16;     // 131072, indexed by a float's bits >> 15
    const float *    dec16;      // 65536
    const uint16_t * exp16;      // 65536
    const uint16_t * sig16;      // 65536
    const int16_t *  monte16;    // 2 * k16_monte_n
    const int32_t *  key16;      // k16_key_bytes / 4
    const int32_t *  mkey16;     // k16m_key_bytes / 4
    const int32_t *  key16s;     // k16s_bytes / 4
    const int32_t *  sb32;
    const int32_t *  db32;
    const int32_t *  db32_hi;    // 2048
    const int32_t *  db32_lo;    // 4096
    const int32_t *  flat32;     // k32f_words (flat xlns32 addition image)
    const uint32_t * logm32;     // 2^23 or null
    const float *    expm32;     // 2^23 or null
    const int32_t *  lpvip_db;   // 2^23 or null
    const uint16_t * lfsr_log;   // 65536
    const uint16_t * lfsr_alog;  // 65535
};

// ============================== xlns16 ====================================

__device__ __forceinline__ uint32_t mul16(uint32_t a, uint32_t b) {
    int p = (int) (a & 0x7FFFu) + (int) (b & 0x7FFFu) - 0x4000;
    p = min(max(p, 0), 0x7FFF);
    return ((a ^ b) & 0x8000u) | (uint32_t) p;
}

__device__ __forceinline__ uint32_t div16(uint32_t a, uint32_t b) {
    int p = (int) (a & 0x7FFFu) - (int) (b & 0x7FFFu) + 0x4000;
    p = min(max(p, 0), 0x7FFF);
    return ((a ^ b) & 0x8000u) | (uint32_t) p;
}

// xlns16_add ("alt" form).  tab: the sbdb16 image (shared or global memory).
__device__ __forceinline__ uint32_t add16(uint32_t a, uint32_t b, const int16_t * tab) {
    const int al = (int) (a & 0x7FFFu), bl = (int) (b & 0x7FFFu);
    const uint32_t mx = al > bl ? a : b;
    const int n = abs(al - bl);
    const uint32_t usedb = (a ^ b) & 0x8000u;
    if (n == 0 && usedb) return 0u;
    const int idx = (usedb ? (k16_sign_off / 2) : 0) + min(n, k16_ess + 1);
    const int adj = tab[idx] >> 1;
    const int p = min(max((int) (mx & 0x7FFFu) + adj, 0), 0x7FFF);
    return (mx & 0x8000u) | (uint32_t) p;
}

__device__ __forceinline__ uint32_t sub16(uint32_t a, uint32_t b, const int16_t * tab) {
    return add16(a, b ^ 0x8000u, tab);
}

// halve the signed log, odd logs rounded away from zero (xlns16_sqrt)
__device__ __forceinline__ uint32_t sqrt16(uint32_t a) {
    const int s = (int) (int16_t) (uint16_t) (a << 1);
    const int q = s / 4;
    return ((uint32_t) q & 0x7FFFu) ^ 0x2000u;
}

__device__ __forceinline__ uint32_t recip16(uint32_t a) {
    return (a & 0x8000u) | ((~a + 1u) & 0x7FFFu);
}

__device__ __forceinline__ uint32_t canon16(uint32_t v) {
    return (v & 0x8000u) ? (~v & 0xFFFFu) : (v | 0x10000u);
}
__device__ __forceinline__ bool gt16(uint32_t a, uint32_t b) { return canon16(a) > canon16(b); }
__device__ __forceinline__ bool is_zero16(uint32_t v) { return (v & 0x7FFFu) == 0; }

__device__ __forceinline__ uint32_t from_f32_16(const dev_tables & T, float x) {
    return __ldg(T.conv16 + (__float_as_uint(x) >> 15));
}
__device__ __forceinline__ float to_f32_16(const dev_tables & T, uint32_t v) { return __ldg(T.dec16 + (v & 0xFFFFu)); }

#ifndef LNSB_X32_CONV_FAST
#define LNSB_X32_CONV_FAST 1
#endif

// ============================== xlns32 ====================================

__device__ __forceinline__ uint32_t mul32(uint32_t a, uint32_t b) {
    long long p = (long long) (a & 0x7FFFFFFFu) + (long long) (b & 0x7FFFFFFFu) - 0x40000000LL;
    p = p < 0 ? 0 : (p > 0x7FFFFFFFLL ? 0x7FFFFFFFLL : p);
    return ((a ^ b) & 0x80000000u) | (uint32_t) p;
}

__device__ __forceinline__ uint32_t div32(uint32_t a, uint32_t b) {
    long long p = (long long) (a & 0x7FFFFFFFu) - (long long) (b & 0x7FFFFFFFu) + 0x40000000LL;
    p = p < 0 ? 0 : (p > 0x7FFFFFFFLL ? 0x7FFFFFFFLL : p);
    return ((a ^ b) & 0x80000000u) | (uint32_t) p;
}

// sb(z) and db(z) between knots every 2^-9 octave (k32_sh), floored (z: sb
// [0, ess], db [1, ess]; z = ess reads the last knot, 0, with fraction 0)
__host__ __device__ __forceinline__ int32_t lerp32(int32_t v0, int32_t v1, uint32_t z) {
    const int32_t f = (int32_t) (z & ((1u << k32_sh) - 1u));
    return v0 + (((v1 - v0) * f) >> k32_sh);
}

__device__ __forceinline__ int32_t sb32(const dev_tables & T, uint32_t d) {
    if (d >= k32_ess) return 0;
    const int32_t i = (int32_t) (d >> k32_sh);
    return lerp32(__ldg(T.sb32 + i), __ldg(T.sb32 + i + 1), d);
}

__device__ __forceinline__ int32_t db32(const dev_tables & T, uint32_t d) {   // d > 0
    if (d >= k32_ess) return 0;
    if (d >= k32_one) {
        const int32_t i = (int32_t) ((d - k32_one) >> k32_sh);
        return lerp32(__ldg(T.db32 + i), __ldg(T.db32 + i + 1), d);
    }
    // cotransformation: 1 - 2^z = (1 - 2^z2) + 2^z2 (1 - 2^z1)
    const uint32_t d1 = d >> 12, d2 = d & 4095u;
    if (d1 == 0) return __ldg(T.db32_lo + d2);
    if (d2 == 0) return __ldg(T.db32_hi + d1);
    const int32_t la = __ldg(T.db32_lo + d2);
    const int32_t lb = -(int32_t) d2 + __ldg(T.db32_hi + d1);
    const int32_t hi = la > lb ? la : lb;
    const uint32_t gap = (uint32_t) (la > lb ? la - lb : lb - la);
    return hi + sb32(T, gap);
}

__device__ __forceinline__ uint32_t add32(const dev_tables & T, uint32_t a, uint32_t b) {
    const uint32_t al = a & 0x7FFFFFFFu, bl = b & 0x7FFFFFFFu;
    const uint32_t mx = al > bl ? a : b;
    const uint32_t d  = al > bl ? al - bl : bl - al;
    const bool usedb = ((a ^ b) & 0x80000000u) != 0;
    if (d == 0 && usedb) return 0u;
    const int32_t adj = usedb ? db32(T, d) : sb32(T, d);
    long long p = (long long) (mx & 0x7FFFFFFFu) + adj;
    p = p < 0 ? 0 : (p > 0x7FFFFFFFLL ? 0x7FFFFFFFLL : p);
    return (mx & 0x80000000u) | (uint32_t) p;
}

// add32 over the flat image F (k32f_sb; shared memory in the kernels), without
// branches: every lane makes the cotransformation lookups and the result is
// selected afterwards, so the chains of a warp and of one thread interleave
// instead of diverging.  Same bits as add32:
//   cot (opposite signs, d < 1): db(d) = max(la, lb) + sb(|la - lb|) with
//     la = db(d & 4095), lb = db(d & ~4095) - (d & 4095); the k32f_none
//     entries reproduce the cases d < 4096 and d % 4096 == 0 (|la - lb| >= ess)
//   otherwise sb(d) or db(d) by interpolation; z >= ess lands on the last
//     knot (value 0) with fraction 0
// The interpolation product fits in 32 bits (checked when the image is built).
__host__ __device__ __forceinline__ uint32_t add32f(const int32_t * F, uint32_t a, uint32_t b) {
    const uint32_t al = a & 0x7FFFFFFFu, bl = b & 0x7FFFFFFFu;
    const bool     agt   = al > bl;
    const uint32_t d     = agt ? al - bl : bl - al;
    const uint32_t mx    = agt ? a : b;
    const bool     usedb = (int32_t) (a ^ b) < 0;
    const bool     cot   = usedb && d < k32_one;
    const int32_t  d2 = (int32_t) (d & 4095u);
    const int32_t  la = F[k32f_lo + d2];
    const int32_t  lb = F[k32f_hi + (int32_t) ((d >> 12) & 2047u)] - d2;
    const int32_t  hi = la > lb ? la : lb;
    const uint32_t gap = (uint32_t) (la > lb ? la - lb : lb - la);
    uint32_t z = cot ? gap : d;
    z = z < k32_ess ? z : k32_ess;
    const bool     isdb = usedb && !cot;
    const int32_t  i    = (int32_t) (z >> k32_sh) + (isdb ? k32f_db0 : k32f_sb);
    const int32_t  adj  = lerp32(F[i], F[i + 1], z) + (cot ? hi : 0);
    const uint32_t u = (mx & 0x7FFFFFFFu) + (uint32_t) adj;      // adj > -2^28: wrap means negative
    uint32_t p = u < 0x7FFFFFFFu ? u : 0x7FFFFFFFu;
    if (u >= 0xC0000000u) p = 0;
    const uint32_t r = (mx & 0x80000000u) | p;
    return (usedb && d == 0) ? 0u : r;
}

// sb(z) (db = false) or db(z) (db = true, z >= 1) over the flat image
__device__ __forceinline__ int32_t interp32f(const int32_t * F, uint32_t z, bool db) {
    const int32_t i = (int32_t) (z >> k32_sh) + (db ? k32f_db0 : k32f_sb);
    return lerp32(F[i], F[i + 1], z);
}

// the cotransformed db of the throughput adder's rare branch: opposite signs, d < 1
__device__ __forceinline__ uint32_t add32f_cot(const int32_t * F, uint32_t mx, uint32_t d) {
    const int32_t  d2 = (int32_t) (d & 4095u);
    const int32_t  la = F[k32f_lo + d2];
    const int32_t  lb = F[k32f_hi + (int32_t) (d >> 12)] - d2;
    const int32_t  hi = la > lb ? la : lb;
    uint32_t       z  = (uint32_t) (la > lb ? la - lb : lb - la);
    z = z < k32_ess ? z : k32_ess;
    const int32_t  p = (int32_t) (mx & 0x7FFFFFFFu) + hi + interp32f(F, z, false);   // hi + sb < 0
    const uint32_t r = (mx & 0x80000000u) | (uint32_t) (p > 0 ? p : 0);
    return d == 0 ? 0u : r;
}

// add32 over the flat image for throughput kernels, in two parts so a thread
// can interleave several chains: add32f_main for every chain, then a branch
// per chain for the lanes that need add32f_cot.  The main part is sb(d), or
// db(d) for d >= 1, and needs no clamp from below: 0 <= sb <= 2^23, and
// d + db(d) >= 0 for every d >= 1 (checked exhaustively over the table), so
// |mx| + adj >= 0.  Above, |mx| + adj > 0x7FFFFFFF carries into the sign bit
// (mx + adj then differs from mx in bit 31) and saturates to 0x7FFFFFFF.  The
// cotransformed db (opposite signs, d < 1, exact cancellation included) is
// the cot part.  Same bits as add32.
struct add32f_part {
    uint32_t r, mx, d;
    bool     cot;
};
__device__ __forceinline__ add32f_part add32f_main(const int32_t * F, uint32_t a, uint32_t b) {
    add32f_part o;
    const uint32_t al = a & 0x7FFFFFFFu, bl = b & 0x7FFFFFFFu;
    const bool     agt   = al > bl;
    o.d  = agt ? al - bl : bl - al;
    o.mx = agt ? a : b;
    const bool     usedb = (int32_t) (a ^ b) < 0;
    const uint32_t z     = o.d < k32_ess ? o.d : k32_ess;
    const uint32_t r     = o.mx + (uint32_t) interp32f(F, z, usedb);
    o.r   = (int32_t) (r ^ o.mx) < 0 ? (o.mx | 0x7FFFFFFFu) : r;
    o.cot = usedb && o.d < k32_one;
    return o;
}

// add32 over the flat image for a chain's latency: the main result (sb(d),
// or db(d) for d >= 1) and the cotransformed one (sb of the gap) are computed
// independently and selected, so the dependent path is two table levels
// deep instead of three.  Same bits as add32.
__device__ __forceinline__ uint32_t add32f_sel(const int32_t * F, uint32_t a, uint32_t b) {
    const uint32_t al = a & 0x7FFFFFFFu, bl = b & 0x7FFFFFFFu;
    const bool     agt   = al > bl;
    const uint32_t d     = agt ? al - bl : bl - al;
    const uint32_t mx    = agt ? a : b;
    const bool     usedb = (int32_t) (a ^ b) < 0;
    const bool     cot   = usedb && d < k32_one;
    // main: |mx| + sb(d) or db(d); above 0x7FFFFFFF the carry reaches the sign bit
    const uint32_t z    = d < k32_ess ? d : k32_ess;
    const uint32_t r0   = mx + (uint32_t) interp32f(F, z, usedb);
    const uint32_t rm   = (int32_t) (r0 ^ mx) < 0 ? (mx | 0x7FFFFFFFu) : r0;
    // cot: max(la, lb) + sb(|la - lb|), clamped at zero
    const int32_t  d2 = (int32_t) (d & 4095u);
    const int32_t  la = F[k32f_lo + d2];
    const int32_t  lb = F[k32f_hi + (int32_t) ((d >> 12) & 2047u)] - d2;
    const int32_t  hi = la > lb ? la : lb;
    uint32_t       zc = (uint32_t) (la > lb ? la - lb : lb - la);
    zc = zc < k32_ess ? zc : k32_ess;
    const int32_t  p   = (int32_t) (mx & 0x7FFFFFFFu) + hi + interp32f(F, zc, false);
    const uint32_t rc  = (mx & 0x80000000u) | (uint32_t) (p > 0 ? p : 0);
    return cot ? (d == 0 ? 0u : rc) : rm;
}

__device__ __forceinline__ uint32_t sub32(const dev_tables & T, uint32_t a, uint32_t b) {
    return add32(T, a, b ^ 0x80000000u);
}

__device__ __forceinline__ uint32_t sqrt32(uint32_t a) {
    const int32_t s = (int32_t) (a << 1);
    const int32_t q = s / 4;
    return ((uint32_t) q & 0x7FFFFFFFu) ^ 0x20000000u;
}
__device__ __forceinline__ uint32_t recip32(uint32_t a) { return (a & 0x80000000u) | ((~a + 1u) & 0x7FFFFFFFu); }
__device__ __forceinline__ unsigned long long canon32(uint32_t v) {
    return (v & 0x80000000u) ? (unsigned long long) (~v) : ((unsigned long long) v | 0x100000000ull);
}
__device__ __forceinline__ bool gt32(uint32_t a, uint32_t b) { return canon32(a) > canon32(b); }
__device__ __forceinline__ bool is_zero32(uint32_t v) { return (v & 0x7FFFFFFFu) == 0; }

// float -> xlns32, truncation toward zero of log2|x| * 2^23 (exact: mantissa table)
// floor(log2(1 + man / 2^23) * 2^23), the entry man of the 2^23-entry table
// T.logm32.  Computed in double precision (log2, at most an ulp or two off:
// far below the 2^-20 margin kept from the integers); the rare values within
// the margin of an integer, where the floor could go either way, read the
// table.  Same value as the table for every man (checked exhaustively on the
// GPU); the table is 32 MB, so the computation saves a memory round trip.
__device__ __forceinline__ uint32_t logm32_of(const dev_tables & T, uint32_t man) {
#if LNSB_X32_CONV_FAST
    const double v = log2(1.0 + (double) man * 0x1p-23) * 0x1p23;
    const double fl = floor(v);
    const double fr = v - fl;
    if (fr > 0x1p-20 && fr < 1.0 - 0x1p-20) return (uint32_t) fl;
#endif
    return __ldg(T.logm32 + man);
}
// the float nearest 2^(f / 2^23), f < 2^23: the entry f of T.expm32, computed
// in double precision (exp2) and rounded to float, except within a 2^-21 float
// ulp of a rounding midpoint, where the table is read
__device__ __forceinline__ float expm32_of(const dev_tables & T, uint32_t f) {
#if LNSB_X32_CONV_FAST
    const double d = exp2((double) f * 0x1p-23);
    const double t = d * 0x1p24;                         // floats of [1, 2) at even t, midpoints at odd t
    if (fabs(t - rint(t)) > 0x1p-21) return __double2float_rn(d);
#endif
    return __ldg(T.expm32 + f);
}

__device__ __forceinline__ uint32_t from_f32_32(const dev_tables & T, float x) {
    const uint32_t b = __float_as_uint(x);
    const uint32_t sign = b & 0x80000000u;
    uint32_t ex = (b >> 23) & 0xFFu, man = b & 0x7FFFFFu;
    if (ex == 0xFFu) return man ? 0u : (sign | 0x7FFFFFFFu);
    if (ex == 0 && man == 0) return 0u;
    int e;
    if (ex == 0) {
        const int lz = __clz(man) - 8;          // shifts to bring the msb to bit 23
        man = (man << lz) & 0x7FFFFFu;
        e = -126 - lz;
    } else {
        e = (int) ex - 127;
    }
    long long l = (long long) e * (long long) k32_one + (long long) logm32_of(T, man);
    if (e < 0 && man != 0) l += 1;
    return sign | (uint32_t) ((l + 0x40000000LL) & 0x7FFFFFFFLL);
}

// float in [1,2) times 2^e, round-to-nearest-even into subnormals
__device__ __forceinline__ float scale_pow2(float m, int e) {
    const uint32_t mant = (__float_as_uint(m) & 0x7FFFFFu) | 0x800000u;
    uint32_t out;
    if (e > 127) {
        out = 0x7F800000u;
    } else if (e >= -126) {
        out = ((uint32_t) (e + 127) << 23) | (mant & 0x7FFFFFu);
    } else {
        const int sh = -126 - e;
        if (sh > 25) {
            out = 0;
        } else {
            uint32_t q = mant >> sh;
            const uint32_t rem = mant & ((1u << sh) - 1u), half = 1u << (sh - 1);
            if (rem > half || (rem == half && (q & 1u))) q++;
            out = q;
        }
    }
    return __uint_as_float(out);
}

__device__ __forceinline__ float to_f32_32(const dev_tables & T, uint32_t v) {
    if ((v & 0x7FFFFFFFu) == 0) return 0.0f;
    const int32_t l = (int32_t) (v & 0x7FFFFFFFu) - 0x40000000;
    const int e = l >> 23;
    const float r = scale_pow2(expm32_of(T, (uint32_t) l & 0x7FFFFFu), e);
    return (v & 0x80000000u) ? -r : r;
}

// own float exp: range reduction by 2^n, Taylor series of e^r to degree 14 in
// double with explicit fused multiply-adds, one rounding to float
__device__ __forceinline__ float lnsb_expf(float x) {
    if (x != x) return x;
    double xd = (double) x;
    xd = xd > 200.0 ? 200.0 : (xd < -200.0 ? -200.0 : xd);
    const double t = __dmul_rn(xd, 1.4426950408889634074);
    const double n = rint(t);
    const double r = __dmul_rn(__dsub_rn(t, n), 0.69314718055994530942);
    const double c[15] = {
        1.0, 1.0, 1.0 / 2, 1.0 / 6, 1.0 / 24, 1.0 / 120, 1.0 / 720, 1.0 / 5040, 1.0 / 40320,
        1.0 / 362880, 1.0 / 3628800, 1.0 / 39916800, 1.0 / 479001600, 1.0 / 6227020800.0,
        1.0 / 87178291200.0 };
    double p = c[14];
#pragma unroll
    for (int i = 13; i >= 0; i--) p = __fma_rn(p, r, c[i]);
    return __double2float_rn(scalbn(p, (int) n));
}

// e^x in double: the same series as lnsb_expf without the float rounding,
// |x| clamped to 700 (the device twin of host_exp_d)
__device__ __forceinline__ double lnsb_exp_d(double xd) {
    if (xd != xd) return xd;
    xd = xd > 700.0 ? 700.0 : (xd < -700.0 ? -700.0 : xd);
    const double t = __dmul_rn(xd, 1.4426950408889634074);
    const double n = rint(t);
    const double r = __dmul_rn(__dsub_rn(t, n), 0.69314718055994530942);
    const double c[15] = {
        1.0, 1.0, 1.0 / 2, 1.0 / 6, 1.0 / 24, 1.0 / 120, 1.0 / 720, 1.0 / 5040, 1.0 / 40320,
        1.0 / 362880, 1.0 / 3628800, 1.0 / 39916800, 1.0 / 479001600, 1.0 / 6227020800.0,
        1.0 / 87178291200.0 };
    double p = c[14];
#pragma unroll
    for (int i = 13; i >= 0; i--) p = __fma_rn(p, r, c[i]);
    return scalbn(p, (int) n);
}

// tanh(y) = (e^2y - 1) / (e^2y + 1) in double
__device__ __forceinline__ double lnsb_tanh_d(double y) {
    const double e = lnsb_exp_d(__dmul_rn(2.0, y));
    return __ddiv_rn(__dsub_rn(e, 1.0), __dadd_rn(e, 1.0));
}

__device__ __forceinline__ uint32_t exp32(const dev_tables & T, uint32_t v) {
    return from_f32_32(T, lnsb_expf(to_f32_32(T, v)));
}

// ============================== LPVIP ======================================

__device__ __forceinline__ uint32_t mitchell_exp2_neg(uint32_t d) {
    const uint32_t q = (d + k32_one - 1u) >> 23;
    const uint32_t frac = (q << 23) - d;
    if (q >= 32) return 0;
    return (k32_one + frac) >> q;
}
__device__ __forceinline__ int32_t mitchell_log2(uint32_t v) {
    const int k = 31 - __clz(v);
    const int e = k - 23;
    const uint32_t m = e >= 0 ? (v >> e) : (v << -e);
    return e * (int32_t) k32_one + (int32_t) (m - k32_one);
}
__device__ __forceinline__ uint32_t add32_lpvip(const dev_tables & T, uint32_t a, uint32_t b) {
    const uint32_t al = a & 0x7FFFFFFFu, bl = b & 0x7FFFFFFFu;
    const uint32_t mx = al > bl ? a : b;
    const uint32_t d  = al > bl ? al - bl : bl - al;
    const bool usedb = ((a ^ b) & 0x80000000u) != 0;
    if (d == 0 && usedb) return 0u;
    int32_t adj;
    const uint32_t u = mitchell_exp2_neg(d);
    if (!usedb) {
        adj = mitchell_log2(k32_one + u);
    } else if (d < k32_one) {
        adj = __ldg(T.lpvip_db + d);
    } else {
        adj = (k32_one - u) ? mitchell_log2(k32_one - u) : 0;
    }
    long long p = (long long) (mx & 0x7FFFFFFFu) + adj;
    p = p < 0 ? 0 : (p > 0x7FFFFFFFLL ? 0x7FFFFFFFLL : p);
    return (mx & 0x80000000u) | (uint32_t) p;
}

// add32_lpvip in two parts for the throughput kernels.  Mitchell's
// approximations collapse on the main path: 1 + u lies in [1, 2], so its
// Mitchell log2 is u itself, and for d >= 1 (u <= 1/2) 1 - u lies in
// [1/2, 1), whose Mitchell log2 is -2u exactly.  So sb = u, db = -2u with
// u = mitchell_exp2_neg(d).  On that path db never goes below zero
// (|mx| >= d >= 1 >= 2u) and sb can only carry into the sign bit, which then
// saturates.  The singular case (opposite signs, d < 1) reads the exact db
// table (lpvip_sing).  Same bits as add32_lpvip.
struct lpvip_part {
    uint32_t r, mx, d;
    bool     sing;
};
__host__ __device__ __forceinline__ lpvip_part lpvip_main(uint32_t a, uint32_t b) {
    lpvip_part o;
    const uint32_t al = a & 0x7FFFFFFFu, bl = b & 0x7FFFFFFFu;
    const bool     agt   = al > bl;
    o.d  = agt ? al - bl : bl - al;
    o.mx = agt ? a : b;
    const bool     usedb = (int32_t) (a ^ b) < 0;
    const uint32_t q  = (o.d >> 23) + ((o.d & (k32_one - 1u)) != 0u ? 1u : 0u);   // ceil(d / 2^23)
    const uint32_t qs = q < 31u ? q : 31u;
    uint32_t       u  = (k32_one + ((qs << 23) - o.d)) >> qs;
    if (q >= 32u) u = 0u;
    const uint32_t r = o.mx + (usedb ? 0u - 2u * u : u);
    o.r    = (int32_t) (r ^ o.mx) < 0 ? (o.mx | 0x7FFFFFFFu) : r;
    o.sing = usedb && o.d < k32_one;
    return o;
}
__host__ __device__ __forceinline__ uint32_t lpvip_sing(const int32_t * lpvip_db, uint32_t mx, uint32_t d) {
    if (d == 0) return 0u;
#ifdef __CUDA_ARCH__
    const int32_t adj = __ldg(lpvip_db + d);
#else
    const int32_t adj = lpvip_db[d];
#endif
    const int32_t p = (int32_t) (mx & 0x7FFFFFFFu) + adj;
    return (mx & 0x80000000u) | (uint32_t) (p > 0 ? p : 0);
}

// ===================== additions of non-negative terms =====================
// The normalisers sum non-negative terms only (squares in rms_norm, exp values
// in soft_max), so their chains never take db, the cotransformation or the
// exact cancellation: for a, b >= 0 these are add16 and add32 exactly.
// tab: the sbdb16 image; F: a flat xlns32 image whose sb knots and
// descriptors are filled (the rest is never read here).
__device__ __forceinline__ uint32_t padd16(uint32_t a, uint32_t b, const int16_t * tab) {
    const int d = abs((int) a - (int) b);
    const int adj = tab[min(d, k16_ess + 1)] >> 1;
    return (uint32_t) min(max((int) a, (int) b) + adj, 0x7FFF);
}
// padd32f: sb by interpolation, one table level on the chain's dependent path
__device__ __forceinline__ uint32_t padd32f(const int32_t * F, uint32_t a, uint32_t b) {
    const uint32_t d  = a > b ? a - b : b - a;
    const uint32_t mx = a > b ? a : b;
    const uint32_t z  = d < k32_ess ? d : k32_ess;
    const uint32_t r  = mx + (uint32_t) interp32f(F, z, false);
    return (int32_t) r < 0 ? 0x7FFFFFFFu : r;                      // saturation: the carry into bit 31
}

// ============================== Monte ======================================

__device__ __forceinline__ uint32_t lfsr_step(uint32_t s) { return (s >> 1) ^ ((s & 1u) ? 0xB400u : 0u); }

__device__ __forceinline__ uint32_t lfsr_jump(const dev_tables & T, uint32_t s, unsigned long long n) {
    if (s == 0) return 0;
    const unsigned long long k = ((unsigned long long) __ldg(T.lfsr_log + s) + n % 65535ull) % 65535ull;
    return __ldg(T.lfsr_alog + k);
}

// Monte-Carlo LNS addition: sb/db at 8 extra bits, rounded with the low byte
// of the next LFSR state (one draw per addition)
__device__ __forceinline__ uint32_t add16_monte(uint32_t a, uint32_t b, uint32_t & st, const int16_t * fine) {
    st = lfsr_step(st);
    const int al = (int) (a & 0x7FFFu), bl = (int) (b & 0x7FFFu);
    const uint32_t mx = al > bl ? a : b;
    const int n = abs(al - bl);
    const uint32_t usedb = (a ^ b) & 0x8000u;
    if (n == 0 && usedb) return 0u;
    const int f = n < k16_monte_n ? (int) fine[(usedb ? k16_monte_n : 0) + n] : 0;
    const int adj = (f + (int) (st & 0xFFu)) >> 8;
    const int p = min(max((int) (mx & 0x7FFFu) + adj, 0), 0x7FFF);
    return (mx & 0x8000u) | (uint32_t) p;
}

__device__ __forceinline__ uint32_t add16_monte_bylpvip(const dev_tables & T, uint32_t a, uint32_t b, uint32_t & st) {
    st = lfsr_step(st);
    const uint32_t r = add32_lpvip(T, a << 16, (b << 16) | st);
    return r >> 16;
}

// ====================== reduction policy (GGML_LNS16_SUM) ===================
//   from(v): accumulator from the first term; add(acc, t, st); finish(acc)
// tab16: sbdb16 image, fine16: Monte fine tables (shared or global memory)

struct red16 {
    const dev_tables * T;
    const int16_t *    tab16;
    const int16_t *    fine16;

    __device__ __forceinline__ uint32_t from(uint32_t v) const { return k_acc32 ? (v << 16) : v; }
    __device__ __forceinline__ uint32_t add(uint32_t acc, uint32_t t, uint32_t & st) const {
        if constexpr (k_mode == M_MONTE)         return add16_monte(acc, t, st, fine16);
        if constexpr (k_mode == M_MONTE_BYLPVIP) return add16_monte_bylpvip(*T, acc, t, st);
        if constexpr (k_mode == M_LPVIP)         return add32_lpvip(*T, acc, t << 16);
        if constexpr (k_mode == M_SUM32)         return add32(*T, acc, t << 16);
        return add16(acc, t, tab16);
    }
    __device__ __forceinline__ uint32_t finish(uint32_t acc) const {
        if constexpr (k_mode == M_SUM32) {
            if ((acc & 0x7FFFFFFFu) >= 0x7FFF8000u) return ((acc >> 16) | 0x7FFFu) & 0xFFFFu;
            return (acc + 0x8000u) >> 16;
        }
        if constexpr (k_mode == M_LPVIP) return acc >> 16;
        return acc;
    }
};

}  // namespace lnsb
