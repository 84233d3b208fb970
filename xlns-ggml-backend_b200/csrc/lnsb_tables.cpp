// Host table builder of the product library (see lnsb_tables.h).
#include "lnsb_tables.h"

#include <algorithm>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

namespace lnsb {

// e^x in double: range reduction by 2^n (n = x log2(e) rounded to nearest),
// then the Taylor series of e^r, r = (x log2(e) - n) ln 2, to degree 14 by
// Horner's rule with explicit fused multiply-adds; |x| clamped to 700.  The
// device's lnsb_exp_d is the same sequence of correctly rounded operations,
// so both give the same bits.
double host_exp_d(double xd) {
    if (xd != xd) return xd;
    if (xd > 700.0) xd = 700.0;
    if (xd < -700.0) xd = -700.0;
    const double t = xd * 1.4426950408889634074;
    const double n = std::nearbyint(t);
    const double r = (t - n) * 0.69314718055994530942;
    static const double c[15] = {
        1.0, 1.0, 1.0 / 2, 1.0 / 6, 1.0 / 24, 1.0 / 120, 1.0 / 720, 1.0 / 5040, 1.0 / 40320,
        1.0 / 362880, 1.0 / 3628800, 1.0 / 39916800, 1.0 / 479001600, 1.0 / 6227020800.0,
        1.0 / 87178291200.0 };
    double p = c[14];
    for (int i = 13; i >= 0; i--) p = std::fma(p, r, c[i]);
    return std::ldexp(p, (int) n);
}

// float e^x: the same series from the float argument clamped to 200, one
// rounding to float (the host twin of the device's lnsb_expf)
float host_expf(float x) {
    if (x != x) return x;
    double xd = (double) x;
    if (xd > 200.0) xd = 200.0;
    if (xd < -200.0) xd = -200.0;
    return (float) host_exp_d(xd);
}

namespace {

constexpr long double k_ln2 = 0.693147180559945309417232121458176568L;

void build16(host_tables & t) {
    t.sbdb16.assign(k16_tab_bytes / 2, 0);
    for (int n = 0; n <= k16_ess; n++) {
        const double sb = std::log(1.0 + std::pow(2.0, -(double) n / 128.0)) / std::log(2.0) * 128.0;
        const int sbv = (int) (uint16_t) (sb + .5);
        int dbv = 0;
        if (n > 0) {
            const double dbneg = std::log(std::pow(2.0, (double) n / 128.0) - 1.0) / std::log(2.0) * 128.0;
            dbv = -n + (int) (int16_t) (dbneg + .5);
        }
        t.sbdb16[n]                      = (int16_t) (2 * sbv);
        t.sbdb16[k16_sign_off / 2 + n]   = (int16_t) (2 * dbv);
    }
    // entries n = 1281 of both halves stay 0 (essential zero)

    t.key16.assign(k16_key_bytes / 4, 0);
    for (int n = 0; n <= k16_ess; n++) {
        t.key16[(16 * n) / 4] = 8 * t.sbdb16[n];                                 // 16 * sb(n)
        if (n == 0) {
            t.key16[1] = k16_key_cancel;                                          // byte 4: x + (-x)
        } else {
            t.key16[(16 * n - 4) / 4] = 8 * t.sbdb16[k16_sign_off / 2 + n];      // 16 * db(n)
            t.key16[(16 * n + 4) / 4] = 8 * t.sbdb16[k16_sign_off / 2 + n];
        }
    }

    t.key16s.assign(k16s_bytes / 4, 0);
    for (int i = 0; i < k16s_bytes / 4; i++) {
        const int d = i * 4 - k16_key_max, ad = d < 0 ? -d : d;
        if (ad <= k16_key_max) t.key16s[i] = t.key16[ad / 4];
    }
    t.sbdb16.resize(k16_tab_bytes16 / 2, 0);               // padded to 16 bytes for cp.async copies

    // float -> xlns16, indexed by the float's upper 17 bits (bits >> 15: the
    // sign, the 8 exponent bits and the top 8 mantissa bits).  The log field
    // is the truncating conversion (int)(log2(b) * 128) of the bucket's lower
    // edge b; the sign is the float's.  This is the reference's 65536-entry
    // magnitude table (README.md:75-76) with the sign folded in, so a
    // conversion is one load; it reproduces the reference's conversion
    // statistics (experiments/dot-product-scaling/results/convert.jsonl:1).
    // Zeros and NaNs give the unsigned zero code; |x| >= 2^128 saturates.
    t.conv16.resize(131072);
    for (uint32_t i = 0; i < 131072; i++) {
        const uint32_t bits = (i & 0xFFFFu) << 15;
        float a;
        std::memcpy(&a, &bits, 4);
        const uint16_t sign = (i & 0x10000u) ? 0x8000u : 0;
        uint16_t code;
        if (a == 0.0f || a != a) {
            code = 0;
        } else if (std::isinf(a)) {
            code = (uint16_t) (sign | 0x7FFFu);
        } else {
            const double l = std::log((double) a) / std::log(2.0) * 128.0;
            long c = (long) l + 0x4000L;          // truncation toward zero, then offset
            if (c < 0) c = 0;
            if (c > 0x7FFF) c = 0x7FFF;
            code = (uint16_t) (sign | (uint16_t) c);
        }
        t.conv16[i] = code;
    }

    // xlns16 -> float: 2^(l/128) rounded to float, held to 7 significant
    // decimal digits, rounded to float again (the precision the reference's
    // decodes carry: 2^(491/128) reads 14.280130)
    t.dec16.resize(65536);
    for (uint32_t c = 0; c < 65536; c++) {
        if ((c & 0x7FFFu) == 0) {
            t.dec16[c] = 0.0f;
            continue;
        }
        const float f = (float) std::pow(2.0, (double) ((int) (c & 0x7FFFu) - 0x4000) / 128.0);
        char buf[32];
        std::snprintf(buf, sizeof buf, "%.7g", (double) f);
        const double v = std::strtod(buf, nullptr);
        t.dec16[c] = (float) ((c & 0x8000u) ? -v : v);
    }

    // exp: the log of e^x is x log2(e), taken to F=7 by truncation toward zero
    // from the value's float x = xlns162fp(c) (the rule the reference's
    // printed softmax, tanh and geglu figures pin)
    t.exp16.resize(65536);
    for (uint32_t c = 0; c < 65536; c++) {
        long q = (long) ((double) t.dec16[c] * 1.4426950408889634 * 128.0) + 0x4000L;
        if (q < 0) q = 0;
        if (q > 0x7FFF) q = 0x7FFF;
        t.exp16[c] = (uint16_t) q;
    }

    // sigmoid: entry c = the float 1 / (1 + e^-x), x = xlns162fp(c), through
    // the conversion table (e^-x from host_expf); silu(x) = x * sigmoid(x)
    // reproduces the reference's printed swiglu
    t.sig16.resize(65536);
    for (uint32_t c = 0; c < 65536; c++) {
        const float sg = 1.0f / (1.0f + host_expf(-t.dec16[c]));
        uint32_t b;
        std::memcpy(&b, &sg, 4);
        t.sig16[c] = t.conv16[b >> 15];
    }

    t.monte16.assign(2 * k16_monte_n, 0);
    for (int n = 0; n < k16_monte_n; n++) {
        const long double x  = (long double) n / 128.0L;
        const long double sb = log1pl(exp2l(-x)) / k_ln2;
        t.monte16[n] = (int16_t) llroundl(sb * 32768.0L);
        if (n > 0) {
            const long double db = log1pl(-exp2l(-x)) / k_ln2;
            long double r = roundl(db * 32768.0L);
            if (r < -32768.0L) r = -32768.0L;
            t.monte16[k16_monte_n + n] = (int16_t) r;
        }
    }

    t.mkey16.assign(k16m_key_bytes / 4, 0);
    for (int n = 0; n < k16_monte_n; n++) {
        t.mkey16[(16 * n) / 4] = t.monte16[n];
        if (n == 0) {
            t.mkey16[1] = k16_key_cancel;
        } else {
            t.mkey16[(16 * n - 4) / 4] = t.monte16[k16_monte_n + n];
            t.mkey16[(16 * n + 4) / 4] = t.monte16[k16_monte_n + n];
        }
    }

    t.lfsr_log.assign(65536, 0);
    t.lfsr_alog.assign(65535, 0);
    uint16_t s = 1;
    for (uint32_t i = 0; i < 65535; i++) {
        t.lfsr_alog[i] = s;
        t.lfsr_log[s]  = (uint16_t) i;
        const uint16_t bit = s & 1u;
        s >>= 1;
        if (bit) s ^= 0xB400u;
    }
}

// xlns32 knots are the exact functions truncated toward zero at F=23
int32_t knot(long double v) { return (int32_t) (v * (long double) k32_one); }
int32_t knot_sb(uint32_t d) { return knot(log1pl(exp2l(-(long double) d / (long double) k32_one)) / k_ln2); }
int32_t knot_db(uint32_t d) { return knot(log1pl(-exp2l(-(long double) d / (long double) k32_one)) / k_ln2); }

// The flat image of k32f_sb.  Checks that every interpolation product
// (right - left) * f fits in 32 bits, so the kernels' 32-bit multiply equals
// the 64-bit definition, and that z + db(z) >= 0 at
// every db knot (the main path's result needs no clamp from below); on a
// failed check the image stays empty and lnsb_upload_tables reports it.
void build_flat32(host_tables & t) {
    auto & f = t.flat32;
    f.clear();
    if ((int) t.sb32.size() != k32_sb_knots + 1 || (int) t.db32.size() != k32_db_knots + 1) return;
    f.assign(k32f_words, 0);
    std::copy(t.sb32.begin(), t.sb32.end(), f.begin() + k32f_sb);
    std::copy(t.db32.begin(), t.db32.end(), f.begin() + k32f_db);
    std::copy(t.db32_lo.begin(), t.db32_lo.end(), f.begin() + k32f_lo);
    std::copy(t.db32_hi.begin(), t.db32_hi.end(), f.begin() + k32f_hi);
    f[k32f_lo] = k32f_none;
    f[k32f_hi] = k32f_none;
    auto fits = [&](const std::vector<int32_t> & v) {
        for (size_t i = 0; i + 1 < v.size(); i++) {
            const long long dv = (long long) v[i + 1] - v[i];
            if ((dv < 0 ? -dv : dv) * ((1ll << k32_sh) - 1) >= (1ll << 31)) return false;
        }
        return true;
    };
    bool ok = fits(t.sb32) && fits(t.db32);
    for (int n = 0; n < k32_db_knots; n++) ok = ok && (long long) k32_one + ((long long) n << k32_sh) + t.db32[n] >= 0;
    if (!ok) f.clear();
}

void build32(host_tables & t, bool need32, bool need_lpvip) {
    t.sb32.assign(k32_sb_knots + 1, 0);
    for (int n = 0; n < k32_sb_knots; n++) t.sb32[n] = knot_sb((uint32_t) n << k32_sh);
    t.db32.assign(k32_db_knots + 1, 0);
    for (int n = 0; n < k32_db_knots; n++) t.db32[n] = knot_db(k32_one + ((uint32_t) n << k32_sh));
    t.db32_hi.assign(2048, 0);
    for (int j = 1; j < 2048; j++) t.db32_hi[j] = knot_db((uint32_t) j << 12);
    t.db32_lo.assign(4096, 0);
    for (int k = 1; k < 4096; k++) t.db32_lo[k] = knot_db((uint32_t) k);
    build_flat32(t);

    if (need32) {
        t.logm32.resize((size_t) 1 << 23);
        t.expm32.resize((size_t) 1 << 23);
        for (uint32_t j = 0; j < (1u << 23); j++) {
            const long double m = 1.0L + (long double) j / (long double) k32_one;
            t.logm32[j] = (uint32_t) floorl(log2l(m) * (long double) k32_one);
            t.expm32[j] = (float) exp2l((long double) j / (long double) k32_one);
        }
    }
    if (need_lpvip) {
        t.lpvip_db.resize((size_t) 1 << 23);
        t.lpvip_db[0] = 0;
        for (uint32_t j = 1; j < (1u << 23); j++) t.lpvip_db[j] = knot_db(j);
    }
}

}  // namespace

const host_tables & get_host_tables(bool need32, bool need_lpvip) {
    static std::mutex mu;
    static host_tables t;
    static bool built16 = false, built32 = false, have32 = false, have_lpvip = false;
    std::lock_guard<std::mutex> lock(mu);
    if (!built16) {
        build16(t);
        built16 = true;
    }
    if (!built32 || (need32 && !have32) || (need_lpvip && !have_lpvip)) {
        build32(t, need32 || have32, need_lpvip || have_lpvip);
        built32    = true;
        have32     = have32 || need32;
        have_lpvip = have_lpvip || need_lpvip;
    }
    return t;
}

}  // namespace lnsb
