/*
 * lns_oracle.c -- CPU restatement of the LNS16/LNS32 reduction hot path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the product).  Written in
 * plain C from the published LNS mathematics and the reference's call sites;
 * no reference source is copied (the reference's arithmetic library xlnscpp
 * is not in its checkout at all).  Each function names the reference code
 * whose behaviour it restates.
 *
 * Number formats (format facts: lns-backend/tests/test-lns16-sum32.cpp:37-51,
 * lns-backend/src/lns16-sum32.h:54-81):
 *   xlns16: bit 15 sign, bits 14..0 = round(log2|x| * 128) + 0x4000.
 *           0x0000 / 0x8000 are zero, 0x7FFF / 0xFFFF saturate; -inf = 0xFFFF.
 *   xlns32: bit 31 sign, bits 30..0 = log2|x| * 2^23 + 0x40000000.
 */
#include "lns_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ===================================================================== */
/* xlns16                                                                 */
/* ===================================================================== */

#define X16_LOGMASK  0x7FFFu
#define X16_SIGNMASK 0x8000u
#define X16_OFFSET   0x4000u
#define X16_ZERO     0x0000u
#define X16_NEG_INF  0xFFFFu
#define X16_ESSZER   1280      /* sb/db are zero for |z| > 1280 (0x500) */

static int      g_ready;
static uint16_t g_sb16[X16_ESSZER + 1];      /* sb(-n), n = 0..1280            */
static int16_t  g_db16[X16_ESSZER + 1];      /* db(-n) adjustment, n = 1..1280 */
static uint16_t g_conv16[65536];             /* |float| bits 30..15 -> log field */
static float    g_dec16[65536];              /* xlns16 -> float                */
static uint16_t g_exp16[65536];              /* xlns16 exp                     */
static uint16_t g_sig16[65536];              /* xlns16 sigmoid                 */

/*
 * Gaussian logarithms at F=7.  The reference adds through a table of the
 * ideal sb/db functions (docs/CUDA.md:138-143, "1280-entry sb/db table";
 * essential zero 0x500).  The table values are the ideal functions rounded
 * with the C idiom (int)(v + 0.5); for the db branch the value rounded is
 * log2(2^n - 1), which is negative for n < 128, where that idiom rounds one
 * step high.  This is what reproduces the reference's printed two-term
 * statistics (results/sum32-evidence/standalone-sum32-invariants.txt:4:
 * "base max 1 ULP (mean 0.025)"; the exactly rounded table gives 0 / 0.000).
 */
static void build16(void) {
    for (int n = 0; n <= X16_ESSZER; n++) {
        double sb = log(1.0 + pow(2.0, -(double)n / 128.0)) / log(2.0) * 128.0;
        g_sb16[n] = (uint16_t)(sb + .5);
        if (n == 0) {
            g_db16[n] = 0;
        } else {
            double dbneg = log(pow(2.0, (double)n / 128.0) - 1.0) / log(2.0) * 128.0;
            g_db16[n] = (int16_t)(-n + (int16_t)(dbneg + .5));
        }
    }
    /*
     * float -> xlns16: a 65536-entry table (README.md:75-76 "65536-entry
     * lookup table") indexed by the float's 8 exponent bits and its top 8
     * mantissa bits, (bits >> 15) & 0xFFFF; the sign bit is copied, not
     * looked up.  Each entry is the truncating conversion (int)(log2(b)*128)
     * of the bucket's lower edge b = the float with those 16 bits and zeros
     * below.  This is the construction that reproduces every figure of the
     * reference's conversion statistics over 4 M log-uniform values
     * (experiments/dot-product-scaling/results/convert.jsonl:1, protocol
     * dot-bench.cpp:186-213): mean log2 error -2.07e-3, 63.4 % rounded down,
     * rms relative error 3.54e-3, 49.4 % / 49.2 % of codes changed by a second /
     * third round trip, each change exactly one ulp down.  Indexing by the
     * bfloat16 pattern instead (7 mantissa bits) gives -4.2e-3 and 76 %.
     * Out-of-range logs saturate (|x| >= 2^128 -> 0x7FFF, below 2^-128 -> 0,
     * keeping the sign); zeros and NaNs whose top 8 mantissa bits are not all
     * zero convert to the unsigned zero code, marked 0xFFFF in the table.
     */
    for (uint32_t i = 0; i < 65536; i++) {
        uint32_t bits = i << 15;
        float a;
        memcpy(&a, &bits, 4);
        uint16_t code;
        if (a == 0.0f || a != a) {
            code = 0xFFFFu;                       /* unsigned zero */
        } else if (isinf(a)) {
            code = X16_LOGMASK;
        } else {
            double l = log((double)a) / log(2.0) * 128.0;
            long t = (long)l;                     /* truncation toward zero */
            long c = t + (long)X16_OFFSET;
            if (c < 0) c = 0;
            if (c > (long)X16_LOGMASK) c = X16_LOGMASK;
            code = (uint16_t)c;
        }
        g_conv16[i] = code;
    }
    /*
     * xlns16 -> float: 2^(l/128) rounded to float, that float held to 7
     * significant decimal digits, then rounded to float again; zero log field
     * -> 0.0f.  The reference's decodes carry that precision, not the
     * correctly rounded float: 2^(491/128) prints as 14.280130 (results/
     * sum32-evidence/unit-tests-lns16-base.txt:23, correctly rounded:
     * 14.280133) and 2^(1355/128) as 1537.0380 (standalone-sum32-
     * invariants.txt:9).  Rounding to float before taking the 7 digits is
     * what reproduces the reference's conversion statistics exactly
     * (convert.jsonl:1: 28 of 4,194,304 values round-trip to themselves, 63.3988 %
     * round down); taking the digits of the double gives 30 and 63.3989 %.  A
     * float powf in place of the double pow gives the same statistics (116
     * codes differ; the evidence does not decide between the two).
     */
    for (uint32_t c = 0; c < 65536; c++) {
        if ((c & X16_LOGMASK) == 0) {
            g_dec16[c] = 0.0f;
        } else {
            const float f = (float) pow(2.0, (double)((int)(c & X16_LOGMASK) - (int)X16_OFFSET) / 128.0);
            char buf[32];
            snprintf(buf, sizeof buf, "%.7g", (double) f);    /* 7 significant digits */
            const double v = strtod(buf, NULL);
            g_dec16[c] = (float)((c & X16_SIGNMASK) ? -v : v);
        }
    }
    /* exp as a 65536-entry table (docs/CUDA.md:138-140, "exp ... table
     * lookups"): the log of e^x is x log2(e), taken to F=7 by truncation
     * toward zero -- the same truncation as the conversion table -- from the
     * code's float x = xlns162fp(c).  Pinned by the reference's softmax
     * printouts (results/sum32-evidence/unit-tests-lns16-{base,sum32}.txt:
     * short/long/scaled/masked/masked-scaled max abs error, all ten figures)
     * and by its tanh and geglu printouts (unit-tests-lns16-base.txt:65-86),
     * which go through exp; flooring instead misses four of those figures. */
    for (uint32_t c = 0; c < 65536; c++) {
        long q = (long) ((double) g_dec16[c] * 1.4426950408889634 * 128.0) + (long) X16_OFFSET;
        if (q < 0) q = 0;
        if (q > (long) X16_LOGMASK) q = (long) X16_LOGMASK;
        g_exp16[c] = (uint16_t) q;
    }
    /* sigmoid as a 65536-entry table (docs/CUDA.md:138-140, "sigmoid ...
     * table lookups"): entry c = fp2xlns16 of the float 1 / (1 + e^-x), x =
     * xlns162fp(c), e^-x from this file's own float exp.  silu(x) = x *
     * sigmoid(x) through it reproduces the reference's swiglu printout
     * (unit-tests-lns16-base.txt:44-63) to every digit; x / (1 + exp(-x)) in
     * xlns16 arithmetic misses one of the eight values. */
    for (uint32_t c = 0; c < 65536; c++) {
        const float x = g_dec16[c];
        g_sig16[c] = orc16_from_f32(1.0f / (1.0f + orc_expf(-x)));
    }
}

uint16_t orc16_from_f32(float x) {
    uint32_t bits;
    memcpy(&bits, &x, 4);
    uint16_t m = g_conv16[(bits >> 15) & 0xFFFFu];
    return m == 0xFFFFu ? (uint16_t)X16_ZERO : (uint16_t)(m | ((bits >> 16) & X16_SIGNMASK));
}

float orc16_to_f32(uint16_t v) { return g_dec16[v]; }

/* xlns16_mul: add the log fields; underflow -> signed zero, overflow -> saturate */
uint16_t orc16_mul(uint16_t a, uint16_t b) {
    int p = (int)(a & X16_LOGMASK) + (int)(b & X16_LOGMASK) - (int)X16_OFFSET;
    if (p < 0) p = 0;
    if (p > (int)X16_LOGMASK) p = X16_LOGMASK;
    return (uint16_t)(((a ^ b) & X16_SIGNMASK) | (uint16_t)p);
}

uint16_t orc16_div(uint16_t a, uint16_t b) {
    int p = (int)(a & X16_LOGMASK) - (int)(b & X16_LOGMASK) + (int)X16_OFFSET;
    if (p < 0) p = 0;
    if (p > (int)X16_LOGMASK) p = X16_LOGMASK;
    return (uint16_t)(((a ^ b) & X16_SIGNMASK) | (uint16_t)p);
}

/*
 * xlns16_add in its "alt" form: the result is the larger operand scaled by
 * 2^(adjust/128), adjust = sb or db of z = min - max; z == 0 with opposite
 * signs is exact cancellation (xlns16 zero); |z| > 1280 adds nothing.
 * Ties in magnitude keep the second operand's sign.
 */
uint16_t orc16_add(uint16_t a, uint16_t b) {
    int al = a & X16_LOGMASK, bl = b & X16_LOGMASK;
    uint16_t mx = (al > bl) ? a : b;
    int n = al > bl ? al - bl : bl - al;
    int usedb = (a ^ b) & X16_SIGNMASK;
    if (n == 0 && usedb) return X16_ZERO;
    int adj = 0;
    if (n <= X16_ESSZER) adj = usedb ? g_db16[n] : g_sb16[n];
    int p = (int)(mx & X16_LOGMASK) + adj;
    if (p < 0) p = 0;
    if (p > (int)X16_LOGMASK) p = X16_LOGMASK;
    return (uint16_t)((mx & X16_SIGNMASK) | (uint16_t)p);
}

uint16_t orc16_sub(uint16_t a, uint16_t b) { return orc16_add(a, (uint16_t)(b ^ X16_SIGNMASK)); }
uint16_t orc16_exp(uint16_t a) { return g_exp16[a]; }

/* xlns16_sqrt: halve the signed log (rounding odd logs away from zero) */
uint16_t orc16_sqrt(uint16_t a) {
    int16_t s = (int16_t)(uint16_t)(a << 1);
    int q = s / 4;                                   /* C division truncates */
    return (uint16_t)(((uint16_t)q & X16_LOGMASK) ^ 0x2000u);
}

/* xlns16_recip: negate the log, keep the sign */
uint16_t orc16_recip(uint16_t a) {
    return (uint16_t)((a & X16_SIGNMASK) | ((uint16_t)(~a + 1u) & X16_LOGMASK));
}

static inline uint32_t canon16(uint16_t v) {
    return (v & X16_SIGNMASK) ? (uint32_t)(~v & 0xFFFFu) : (uint32_t)(v | 0x10000u);
}
int orc16_gt(uint16_t a, uint16_t b) { return canon16(a) > canon16(b); }
static inline int is_zero16(uint16_t v) { return (v & X16_LOGMASK) == 0; }

uint16_t orc16_mask_from_f32(float m) { return m <= -3.0e38f ? X16_NEG_INF : orc16_from_f32(m); }

/* ===================================================================== */
/* xlns32                                                                 */
/* ===================================================================== */

#define X32_LOGMASK  0x7FFFFFFFu
#define X32_SIGNMASK 0x80000000u
#define X32_OFFSET   0x40000000u
#define X32_NEG_INF  0xFFFFFFFFu
#define X32_ONE_OCT  (1u << 23)
#define X32_ESS      (26u << 23)

/*
 * Addition tables for xlns32 (the reference's LNS32 configuration,
 * "xlns32_alt": table sb with linear interpolation, cotransformed db;
 * docs/CUDA.md:141-143, lns-backend/src/lns16-sum32.h:22-24; the library
 * itself, xlnscpp's xlns32.cpp, is an un-vendored submodule).  This is a
 * restatement of that scheme, not the library's table layout:
 *   sb: knots every 2^-9 octave on [0,26), truncated toward zero,
 *       interpolation floored;
 *   db: on (0,1) the cotransformation
 *       db(z) = log2(A + B),  A = 1 - 2^z2,  B = 2^z2 (1 - 2^z1)
 *       with z1 = z rounded to 2^-11 octave and z2 = z - z1 (exact tables);
 *       on [1,26) knots every 2^-9 octave, truncated, interpolation floored.
 * The reference's CPU printouts fix the sb choice: with it the sum32 sums of
 * N ones (results/sum32-evidence/standalone-sum32-invariants.txt:6-11, all
 * six N) and the LNS32 rms_norm error (unit-tests-lns32.txt) are reproduced,
 * which the previous segmented layout (2^-10 / 2^-7 octave) and any rounded
 * interpolation do not.  Of the reference CUDA backend's synthetic sum32
 * records (experiments/dot-product-scaling/results/synth.jsonl) it reproduces
 * signed K = 16, 32, softmax-weighted K = 16..64 and positive K = 64; the
 * other positive records need the sb interpolation rounded to nearest, i.e.
 * that backend's device port of the adder rounds where the CPU library
 * floors.  Mixed-sign records beyond K = 64 differ in the fifth digit: the db
 * above one octave is not pinned.
 */
typedef struct { uint32_t lo, hi; int shift; int round; } seg_t;
static const seg_t k_sb_seg[1] = { {0u, 26u << 23, 14, 0} };   /* floored */
static const seg_t k_db_seg[1] = { {1u << 23, 26u << 23, 14, 0} };
static int32_t * g_sb32;   /* concatenated knots of both sb segments */
static int32_t * g_db32;   /* concatenated knots of the 4 db segments */
static int       g_sb_base[1], g_db_base[1];
static int32_t   g_db32_hi[2048];    /* db at z1 = -j * 2^-11 octave, j = 1..2047 */
static int32_t   g_db32_lo[4096];    /* db at z2 = -k * 2^-23 octave, k = 1..4095 */
static uint32_t * g_logm32;          /* floor(log2(1 + j/2^23) * 2^23), j < 2^23 */
static float    * g_expm32;          /* float nearest 2^(f/2^23), f < 2^23     */
static int32_t  * g_lpvip_db;        /* exact db on the LPVIP singular branch  */
static int16_t    g_sbf[2304], g_dbf[2304];  /* Monte: sb/db at 8 extra bits  */

static int KNOT_MODE = 1;
static int32_t knot_round(long double v) {
    v *= (long double)X32_ONE_OCT;
    if (KNOT_MODE == 0) return (int32_t)llroundl(v);
    if (KNOT_MODE == 1) return (int32_t)v;            /* truncation toward zero */
    return (int32_t)floorl(v);
}
static int32_t knot_sb(uint32_t d) {
    long double x = (long double)d / (long double)X32_ONE_OCT;
    return knot_round(log1pl(exp2l(-x)) / 0.693147180559945309417232121458176568L);
}
static int32_t knot_db(uint32_t d) {
    long double x = (long double)d / (long double)X32_ONE_OCT;
    return knot_round(log1pl(-exp2l(-x)) / 0.693147180559945309417232121458176568L);
}
void orc_set_knot_mode(int m) { KNOT_MODE = m; }

static int build32(void) {
    int tot = 0;
    for (int s = 0; s < 1; s++) { g_sb_base[s] = tot; tot += (int)((k_sb_seg[s].hi - k_sb_seg[s].lo) >> k_sb_seg[s].shift) + 1; }
    g_sb32 = (int32_t *)malloc(sizeof(int32_t) * (size_t)tot);
    for (int s = 0; s < 1; s++) {
        int n = (int)((k_sb_seg[s].hi - k_sb_seg[s].lo) >> k_sb_seg[s].shift);
        for (int i = 0; i <= n; i++) g_sb32[g_sb_base[s] + i] = knot_sb(k_sb_seg[s].lo + ((uint32_t)i << k_sb_seg[s].shift));
    }
    tot = 0;
    for (int s = 0; s < 1; s++) { g_db_base[s] = tot; tot += (int)((k_db_seg[s].hi - k_db_seg[s].lo) >> k_db_seg[s].shift) + 1; }
    g_db32 = (int32_t *)malloc(sizeof(int32_t) * (size_t)tot);
    for (int s = 0; s < 1; s++) {
        int n = (int)((k_db_seg[s].hi - k_db_seg[s].lo) >> k_db_seg[s].shift);
        for (int i = 0; i <= n; i++) g_db32[g_db_base[s] + i] = knot_db(k_db_seg[s].lo + ((uint32_t)i << k_db_seg[s].shift));
    }
    g_db32_hi[0] = 0;
    for (int j = 1; j < 2048; j++) g_db32_hi[j] = knot_db((uint32_t)j << 12);
    g_db32_lo[0] = 0;
    for (int k = 1; k < 4096; k++) g_db32_lo[k] = knot_db((uint32_t)k);

    /* LNS32 conversions, exact by construction */
    g_logm32 = (uint32_t *)malloc(sizeof(uint32_t) << 23);
    g_expm32 = (float *)malloc(sizeof(float) << 23);
    g_lpvip_db = (int32_t *)malloc(sizeof(int32_t) << 23);
    if (!g_logm32 || !g_expm32 || !g_lpvip_db) return -1;
    #pragma omp parallel for schedule(static)
    for (int32_t jj = 0; jj < (1 << 23); jj++) {
        const uint32_t j = (uint32_t)jj;
        long double m = 1.0L + (long double)j / (long double)X32_ONE_OCT;
        long double v = log2l(m) * (long double)X32_ONE_OCT;
        g_logm32[j] = (uint32_t)floorl(v);
        g_expm32[j] = (float)exp2l((long double)j / (long double)X32_ONE_OCT);
        g_lpvip_db[j] = j == 0 ? 0 : knot_db(j);
    }
    /* Monte fine tables: 256 sub-steps per xlns16 ULP */
    for (int n = 0; n < 2304; n++) {
        long double x = (long double)n / 128.0L;
        long double sb = log1pl(exp2l(-x)) / 0.693147180559945309417232121458176568L;
        g_sbf[n] = (int16_t)llroundl(sb * 32768.0L);
        if (n == 0) {
            g_dbf[n] = 0;
        } else {
            long double db = log1pl(-exp2l(-x)) / 0.693147180559945309417232121458176568L;
            long double r = roundl(db * 32768.0L);
            g_dbf[n] = (int16_t)(r < -32768.0L ? -32768 : r);
        }
    }
    return 0;
}

static inline int32_t interp(const int32_t * t, const seg_t * sg, int base, uint32_t d) {
    uint32_t off = d - sg->lo;
    uint32_t i = off >> sg->shift;
    uint32_t f = off & ((1u << sg->shift) - 1u);
    int32_t a = t[base + (int)i], b = t[base + (int)i + 1];
    return a + (int32_t)((((int64_t)(b - a) * (int64_t)f) + (sg->round ? (1LL << (sg->shift - 1)) : 0)) >> sg->shift);
}

static inline int32_t sb32(uint32_t d) {
    if (d >= X32_ESS) return 0;
    return interp(g_sb32, &k_sb_seg[0], g_sb_base[0], d);
}

static inline int32_t db32(uint32_t d) {   /* d > 0 */
    if (d >= X32_ESS) return 0;
    if (d >= X32_ONE_OCT) {
        return interp(g_db32, &k_db_seg[0], g_db_base[0], d);
    }
    uint32_t d1 = d >> 12, d2 = d & 4095u;
    if (d1 == 0) return g_db32_lo[d2];
    if (d2 == 0) return g_db32_hi[d1];
    int32_t la = g_db32_lo[d2];
    int32_t lb = -(int32_t)d2 + g_db32_hi[d1];
    int32_t hi = la > lb ? la : lb;
    uint32_t gap = (uint32_t)(la > lb ? la - lb : lb - la);
    return hi + sb32(gap);
}

static inline uint32_t mul32(uint32_t a, uint32_t b) {
    int64_t p = (int64_t)(a & X32_LOGMASK) + (int64_t)(b & X32_LOGMASK) - (int64_t)X32_OFFSET;
    if (p < 0) p = 0;
    if (p > (int64_t)X32_LOGMASK) p = X32_LOGMASK;
    return ((a ^ b) & X32_SIGNMASK) | (uint32_t)p;
}
uint32_t orc32_mul(uint32_t a, uint32_t b) { return mul32(a, b); }

static inline uint32_t div32(uint32_t a, uint32_t b) {
    int64_t p = (int64_t)(a & X32_LOGMASK) - (int64_t)(b & X32_LOGMASK) + (int64_t)X32_OFFSET;
    if (p < 0) p = 0;
    if (p > (int64_t)X32_LOGMASK) p = X32_LOGMASK;
    return ((a ^ b) & X32_SIGNMASK) | (uint32_t)p;
}

/* xlns32_add ("alt" form, same structure as xlns16's) */
static inline uint32_t add32(uint32_t a, uint32_t b) {
    uint32_t al = a & X32_LOGMASK, bl = b & X32_LOGMASK;
    uint32_t mx = al > bl ? a : b;
    uint32_t d = al > bl ? al - bl : bl - al;
    int usedb = ((a ^ b) & X32_SIGNMASK) != 0;
    if (d == 0 && usedb) return 0;
    int32_t adj = usedb ? db32(d) : sb32(d);
    int64_t p = (int64_t)(mx & X32_LOGMASK) + adj;
    if (p < 0) p = 0;
    if (p > (int64_t)X32_LOGMASK) p = X32_LOGMASK;
    return (mx & X32_SIGNMASK) | (uint32_t)p;
}
uint32_t orc32_add(uint32_t a, uint32_t b) { return add32(a, b); }
static inline uint32_t sub32(uint32_t a, uint32_t b) { return add32(a, b ^ X32_SIGNMASK); }

static inline uint32_t sqrt32(uint32_t a) {
    int32_t s = (int32_t)(a << 1);
    int32_t q = s / 4;
    return ((uint32_t)q & X32_LOGMASK) ^ 0x20000000u;
}
static inline uint32_t recip32(uint32_t a) { return (a & X32_SIGNMASK) | ((~a + 1u) & X32_LOGMASK); }
static inline uint64_t canon32(uint32_t v) {
    return (v & X32_SIGNMASK) ? (uint64_t)(~v) : ((uint64_t)v | 0x100000000ull);
}
static inline int gt32(uint32_t a, uint32_t b) { return canon32(a) > canon32(b); }
static inline int is_zero32(uint32_t v) { return (v & X32_LOGMASK) == 0; }

/*
 * float -> xlns32: (int)(log2|x| * 2^23), truncation toward zero
 * (lns-backend/src32/lns32-ops.cpp:58-62 uses libm log per element).  Here
 * the truncation is exact: log2 of the 24-bit mantissa comes from a table
 * built in long double, the exponent is added as an integer.
 */
uint32_t orc32_from_f32(float x) {
    uint32_t b;
    memcpy(&b, &x, 4);
    uint32_t sign = b & 0x80000000u;
    uint32_t ex = (b >> 23) & 0xFFu, man = b & 0x7FFFFFu;
    if (ex == 0xFFu) return man ? 0u : (sign | X32_LOGMASK);
    if (ex == 0 && man == 0) return 0u;
    int e;
    if (ex == 0) {                         /* subnormal: normalise */
        e = -126;
        while (!(man & 0x800000u)) { man <<= 1; e--; }
        man &= 0x7FFFFFu;
    } else {
        e = (int)ex - 127;
    }
    int64_t l = (int64_t)e * (int64_t)X32_ONE_OCT + (int64_t)g_logm32[man];
    if (e < 0 && man != 0) l += 1;         /* ceil for |x| < 1 */
    return sign | (uint32_t)((l + (int64_t)X32_OFFSET) & (int64_t)X32_LOGMASK);
}

/* scale a float in [1,2) by 2^e, rounding to nearest even into subnormals */
static float scale_pow2(float m, int e) {
    uint32_t mb;
    memcpy(&mb, &m, 4);
    uint32_t mant = (mb & 0x7FFFFFu) | 0x800000u;     /* 24-bit significand */
    uint32_t out;
    if (e > 127) {
        out = 0x7F800000u;
    } else if (e >= -126) {
        out = ((uint32_t)(e + 127) << 23) | (mant & 0x7FFFFFu);
    } else {
        int sh = -126 - e;                             /* >= 1 */
        if (sh > 25) {
            out = 0;
        } else {
            uint32_t q = mant >> sh, rem = mant & ((1u << sh) - 1u), half = 1u << (sh - 1);
            if (rem > half || (rem == half && (q & 1u))) q++;
            out = q;                                   /* may carry into the normal range */
        }
    }
    float r;
    memcpy(&r, &out, 4);
    return r;
}

float orc32_to_f32(uint32_t v) {
    if ((v & X32_LOGMASK) == 0) return 0.0f;
    int32_t l = (int32_t)(v & X32_LOGMASK) - (int32_t)X32_OFFSET;
    int e = l >> 23;                                   /* floor */
    uint32_t f = (uint32_t)l & 0x7FFFFFu;
    float r = scale_pow2(g_expm32[f], e);
    return (v & X32_SIGNMASK) ? -r : r;
}

uint32_t orc32_mask_from_f32(float m) { return m <= -3.0e38f ? X32_NEG_INF : orc32_from_f32(m); }

/*
 * Float exp used by xlns32's exp (the reference evaluates it with float
 * libm, docs/CUDA.md:159-161).  Own definition so host and device agree bit
 * for bit: range reduction by 2^n, Taylor series of e^r (|r| <= ln2/2) to
 * degree 14 in double with explicit fused multiply-adds, one rounding to
 * float at the end.
 */
float orc_expf(float x) {
    if (x != x) return x;
    double xd = (double)x;
    if (xd > 200.0) xd = 200.0;
    if (xd < -200.0) xd = -200.0;
    double t = xd * 1.4426950408889634074;
    double n = nearbyint(t);
    double r = (t - n) * 0.69314718055994530942;
    static const double c[15] = {
        1.0, 1.0, 1.0 / 2, 1.0 / 6, 1.0 / 24, 1.0 / 120, 1.0 / 720, 1.0 / 5040, 1.0 / 40320,
        1.0 / 362880, 1.0 / 3628800, 1.0 / 39916800, 1.0 / 479001600, 1.0 / 6227020800.0,
        1.0 / 87178291200.0 };
    double p = c[14];
    for (int i = 13; i >= 0; i--) p = fma(p, r, c[i]);
    return (float)ldexp(p, (int)n);
}

static inline uint32_t exp32(uint32_t v) { return orc32_from_f32(orc_expf(orc32_to_f32(v))); }

/* ===================================================================== */
/* LPVIP: 32-bit accumulator with Mitchell-approximated sb/db            */
/* ===================================================================== */

/*
 * Restatement of the LPVIP accumulator the reference takes from xlnscpp's
 * xlns32lpvip.cpp (README.md:113 "32-bit LPVIP accumulator", test-lns-backend.cpp:48-55
 * "Mitchell-approximated adds"; docs/CUDA.md:176-180: the singular branch of
 * the subtraction is evaluated exactly).  Mitchell: 2^z ~ 2^floor(z)(1 + frac z),
 * log2(m 2^k) ~ k + (m - 1).  Opposite signs closer than one octave use the
 * exact db (tabulated for all 2^23 inputs).
 */
static inline uint32_t mitchell_exp2_neg(uint32_t d) {      /* ~2^(-d) at F=23, d >= 0 */
    uint32_t q = (d + X32_ONE_OCT - 1u) >> 23;               /* ceil(d) in octaves */
    uint32_t frac = (q << 23) - d;                           /* z - floor(z) */
    if (q >= 32) return 0;
    return (X32_ONE_OCT + frac) >> q;
}
static inline int32_t mitchell_log2(uint32_t v) {             /* ~log2(v / 2^23), v > 0 */
    int k = 31 - __builtin_clz(v);                             /* msb position */
    int e = k - 23;
    uint32_t m = e >= 0 ? (v >> e) : (v << -e);                /* [2^23, 2^24) */
    return (int32_t)(e * (int32_t)X32_ONE_OCT) + (int32_t)(m - X32_ONE_OCT);
}
uint32_t orc32_add_lpvip(uint32_t a, uint32_t b) {
    uint32_t al = a & X32_LOGMASK, bl = b & X32_LOGMASK;
    uint32_t mx = al > bl ? a : b;
    uint32_t d = al > bl ? al - bl : bl - al;
    int usedb = ((a ^ b) & X32_SIGNMASK) != 0;
    if (d == 0 && usedb) return 0;
    int32_t adj;
    uint32_t u = mitchell_exp2_neg(d);
    if (!usedb) {
        adj = mitchell_log2(X32_ONE_OCT + u);
    } else if (d < X32_ONE_OCT) {
        adj = g_lpvip_db[d];
    } else {
        adj = (X32_ONE_OCT - u) ? mitchell_log2(X32_ONE_OCT - u) : 0;
    }
    int64_t p = (int64_t)(mx & X32_LOGMASK) + adj;
    if (p < 0) p = 0;
    if (p > (int64_t)X32_LOGMASK) p = X32_LOGMASK;
    return (mx & X32_SIGNMASK) | (uint32_t)p;
}

/* ===================================================================== */
/* Monte LFSR (lns-backend/src/lns-ops.cpp:178-195)                      */
/* ===================================================================== */

static uint16_t g_lfsr_log[65536], g_lfsr_alog[65535];

uint16_t orc_lfsr_step(uint16_t s) {
    uint16_t bit = s & 1u;
    s >>= 1;
    if (bit) s ^= 0xB400u;
    return s;
}

static void build_lfsr(void) {
    uint16_t s = 1;
    for (uint32_t i = 0; i < 65535; i++) {
        g_lfsr_alog[i] = s;
        g_lfsr_log[s] = (uint16_t)i;
        s = orc_lfsr_step(s);
    }
}

/* state after n steps: the step is multiplication by a field generator */
uint16_t orc_lfsr_jump(uint16_t s, uint64_t n) {
    if (s == 0) return 0;
    return g_lfsr_alog[((uint64_t)g_lfsr_log[s] + n % 65535u) % 65535u];
}

/*
 * Monte add (restatement of Monte-Carlo LNS, xlnscpp's xlns16monte.cpp;
 * README.md:112 "unbiased in expectation"): the Gaussian-log adjustment at
 * 8 extra fraction bits is rounded stochastically with the low byte of the
 * next LFSR state (one draw per addition, lns-ops.cpp:89-92).
 */
static inline uint16_t add16_monte(uint16_t a, uint16_t b, uint16_t * st) {
    *st = orc_lfsr_step(*st);
    int al = a & X16_LOGMASK, bl = b & X16_LOGMASK;
    uint16_t mx = (al > bl) ? a : b;
    int n = al > bl ? al - bl : bl - al;
    int usedb = (a ^ b) & X16_SIGNMASK;
    if (n == 0 && usedb) return X16_ZERO;
    int fine = n < 2304 ? (usedb ? g_dbf[n] : g_sbf[n]) : 0;
    int adj = (fine + (int)(*st & 0xFFu)) >> 8;
    int p = (int)(mx & X16_LOGMASK) + adj;
    if (p < 0) p = 0;
    if (p > (int)X16_LOGMASK) p = X16_LOGMASK;
    return (uint16_t)((mx & X16_SIGNMASK) | (uint16_t)p);
}

/* Monte by LPVIP: the term's 16 dither bits ride below the xlns16 LSB */
static inline uint16_t add16_monte_bylpvip(uint16_t a, uint16_t b, uint16_t * st) {
    *st = orc_lfsr_step(*st);
    uint32_t r = orc32_add_lpvip((uint32_t)a << 16, ((uint32_t)b << 16) | *st);
    return (uint16_t)(r >> 16);
}

/* ===================================================================== */
/* Reductions (the GGML_LNS16_SUM policies, lns-cuda-xlns16.cu:67-130)   */
/* ===================================================================== */

static inline uint16_t narrow_sum32(uint32_t s) {          /* lns16-sum32.h:76-81 */
    if ((s & X32_LOGMASK) >= 0x7FFF8000u) return (uint16_t)((s >> 16) | X16_LOGMASK);
    return (uint16_t)((s + 0x8000u) >> 16);
}

typedef struct { uint32_t acc; uint16_t st; } red_t;

static inline void red_from(int mode, red_t * r, uint16_t v) {
    r->acc = (mode == ORC_LPVIP || mode == ORC_SUM32) ? ((uint32_t)v << 16) : v;
}
static inline void red_add(int mode, red_t * r, uint16_t t) {
    switch (mode) {
        case ORC_MONTE:         r->acc = add16_monte((uint16_t)r->acc, t, &r->st); break;
        case ORC_MONTE_BYLPVIP: r->acc = add16_monte_bylpvip((uint16_t)r->acc, t, &r->st); break;
        case ORC_LPVIP:         r->acc = orc32_add_lpvip(r->acc, (uint32_t)t << 16); break;
        case ORC_SUM32:         r->acc = add32(r->acc, (uint32_t)t << 16); break;
        default:                r->acc = orc16_add((uint16_t)r->acc, t); break;
    }
}
static inline uint16_t red_finish(int mode, const red_t * r) {
    if (mode == ORC_SUM32) return narrow_sum32(r->acc);
    if (mode == ORC_LPVIP) return (uint16_t)(r->acc >> 16);
    return (uint16_t)r->acc;
}
static inline int stochastic(int mode) { return mode == ORC_MONTE || mode == ORC_MONTE_BYLPVIP; }

uint16_t orc16_sum(int mode, const uint16_t * a, int64_t n, uint16_t * lfsr) {
    if (n == 0) return X16_ZERO;
    red_t r;
    r.st = lfsr ? *lfsr : 7;
    red_from(mode, &r, a[0]);
    for (int64_t i = 1; i < n; i++) red_add(mode, &r, a[i]);
    if (lfsr) *lfsr = r.st;
    return red_finish(mode, &r);
}

uint16_t orc16_vec_dot(int mode, const uint16_t * a, const uint16_t * b, int64_t n, uint16_t * lfsr) {
    if (n == 0) return X16_ZERO;
    red_t r;
    r.st = lfsr ? *lfsr : 7;
    red_from(mode, &r, orc16_mul(a[0], b[0]));
    for (int64_t i = 1; i < n; i++) red_add(mode, &r, orc16_mul(a[i], b[i]));
    if (lfsr) *lfsr = r.st;
    return red_finish(mode, &r);
}

uint64_t orc_mul_mat_draws(int mode, int64_t K, int64_t M, int64_t N, int64_t ne12, int64_t ne13) {
    if (!stochastic(mode) || K == 0) return 0;
    return (uint64_t)ne12 * (uint64_t)ne13 * (uint64_t)M * (uint64_t)N * (uint64_t)(K - 1);
}
uint64_t orc_soft_max_draws(int mode, int64_t ncols, int64_t nrows) {
    return stochastic(mode) && ncols > 0 ? (uint64_t)nrows * (uint64_t)(ncols - 1) : 0;
}
uint64_t orc_rms_norm_draws(int mode, int64_t ncols, int64_t nrows) {
    return stochastic(mode) ? (uint64_t)nrows * (uint64_t)ncols : 0;
}

/* ===================================================================== */
/* Ops                                                                    */
/* ===================================================================== */

/* lns_mul_mat (lns-ops.cpp:293-384): one sequential dot per output; outputs
 * are independent, so threads split them without changing any bit. */
void orc16_mul_mat(int mode, const uint16_t * w, const uint16_t * x, uint16_t * dst,
                   int64_t K, int64_t M, int64_t N, int64_t ne02, int64_t ne03, int64_t ne12, int64_t ne13,
                   uint16_t monte_seed, int nthreads) {
    const int64_t r2 = ne12 / ne02, r3 = ne13 / ne03;
    const int64_t total = ne12 * ne13 * M * N;
    (void)nthreads;
#ifdef _OPENMP
    #pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
#endif
    for (int64_t o = 0; o < total; o++) {
        /* o = ((z * M + m) * N + n), the CPU loop order (i13, i12, i0, i1) */
        const int64_t n = o % N, m = (o / N) % M, z = o / (N * M);
        const int64_t i12 = z % ne12, i13 = z / ne12;
        const uint16_t * wr = w + (((i13 / r3) * ne02 + i12 / r2) * M + m) * K;
        const uint16_t * xr = x + (z * N + n) * K;
        uint16_t out;
        if (K == 0) {
            out = X16_ZERO;
        } else {
            red_t r;
            r.st = stochastic(mode) ? orc_lfsr_jump(monte_seed, (uint64_t)o * (uint64_t)(K - 1)) : 0;
            red_from(mode, &r, orc16_mul(wr[0], xr[0]));
            for (int64_t k = 1; k < K; k++) red_add(mode, &r, orc16_mul(wr[k], xr[k]));
            out = red_finish(mode, &r);
        }
        dst[(z * N + n) * M + m] = out;
    }
}

void orc32_mul_mat(const uint32_t * w, const uint32_t * x, uint32_t * dst,
                   int64_t K, int64_t M, int64_t N, int64_t ne02, int64_t ne03, int64_t ne12, int64_t ne13,
                   int nthreads) {
    const int64_t r2 = ne12 / ne02, r3 = ne13 / ne03;
    const int64_t total = ne12 * ne13 * M * N;
    (void)nthreads;
#ifdef _OPENMP
    #pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
#endif
    for (int64_t o = 0; o < total; o++) {
        const int64_t n = o % N, m = (o / N) % M, z = o / (N * M);
        const int64_t i12 = z % ne12, i13 = z / ne12;
        const uint32_t * wr = w + (((i13 / r3) * ne02 + i12 / r2) * M + m) * K;
        const uint32_t * xr = x + (z * N + n) * K;
        uint32_t acc = 0;
        if (K > 0) {
            acc = mul32(wr[0], xr[0]);
            for (int64_t k = 1; k < K; k++) acc = add32(acc, mul32(wr[k], xr[k]));
        }
        dst[(z * N + n) * M + m] = acc;
    }
}

/* MUL_MAT_ID (lns-backend/src/lns-ops.cpp:394-462): for token t and slot s,
 * dst[t][s][m] = vec_dot(w[ids[t][s]][m], x[t][s % ne11]) (slot-based
 * broadcast of the activation rows), the chains in the loop order (t, s, m),
 * so the Monte chain o = (t * n_used + s) * M + m starts o * (K - 1) draws
 * after the seed.  w: [n_expert][M][K] weight rows, x: [n_tokens][ne11][K],
 * ids: ids[t * ids_stride + s].  Returns the number of out-of-range ids (their
 * outputs are the zero code; the reference aborts on them). */
int64_t orc16_mul_mat_id(int mode, const uint16_t * w, const uint16_t * x, const int32_t * ids, uint16_t * dst,
                         int64_t K, int64_t M, int64_t n_expert, int64_t ne11, int64_t n_used, int64_t n_tokens,
                         int64_t ids_stride, uint16_t monte_seed, int nthreads) {
    const int64_t total = n_tokens * n_used * M;
    int64_t bad = 0;
    (void)nthreads;
#ifdef _OPENMP
    #pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1) reduction(+:bad)
#endif
    for (int64_t o = 0; o < total; o++) {
        const int64_t m = o % M, z = o / M, s = z % n_used, t = z / n_used;
        const int32_t e = ids[t * ids_stride + s];
        uint16_t out = X16_ZERO;
        if (e < 0 || e >= n_expert) {
            if (m == 0) bad++;
        } else if (K > 0) {
            const uint16_t * wr = w + ((int64_t)e * M + m) * K;
            const uint16_t * xr = x + (t * ne11 + s % ne11) * K;
            red_t r;
            r.st = stochastic(mode) ? orc_lfsr_jump(monte_seed, (uint64_t)o * (uint64_t)(K - 1)) : 0;
            red_from(mode, &r, orc16_mul(wr[0], xr[0]));
            for (int64_t k = 1; k < K; k++) red_add(mode, &r, orc16_mul(wr[k], xr[k]));
            out = red_finish(mode, &r);
        }
        dst[o] = out;
    }
    return bad;
}

int64_t orc32_mul_mat_id(const uint32_t * w, const uint32_t * x, const int32_t * ids, uint32_t * dst,
                         int64_t K, int64_t M, int64_t n_expert, int64_t ne11, int64_t n_used, int64_t n_tokens,
                         int64_t ids_stride, int nthreads) {
    const int64_t total = n_tokens * n_used * M;
    int64_t bad = 0;
    (void)nthreads;
#ifdef _OPENMP
    #pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1) reduction(+:bad)
#endif
    for (int64_t o = 0; o < total; o++) {
        const int64_t m = o % M, z = o / M, s = z % n_used, t = z / n_used;
        const int32_t e = ids[t * ids_stride + s];
        uint32_t acc = 0;
        if (e < 0 || e >= n_expert) {
            if (m == 0) bad++;
        } else if (K > 0) {
            const uint32_t * wr = w + ((int64_t)e * M + m) * K;
            const uint32_t * xr = x + (t * ne11 + s % ne11) * K;
            acc = mul32(wr[0], xr[0]);
            for (int64_t k = 1; k < K; k++) acc = add32(acc, mul32(wr[k], xr[k]));
        }
        dst[o] = acc;
    }
    return bad;
}

/* k_soft_max (lns-cuda-kernels.cuh:255-325) = xlns16_softmax[_masked]
 * (lns16-sum32.h:158-198 shows the control flow) */
void orc16_soft_max(int mode, const uint16_t * src, const int64_t ne[4], const uint16_t * mask,
                    const int64_t mne[4], uint16_t scale, uint16_t * dst, uint16_t monte_seed, int nthreads) {
    const int64_t n = ne[0], nrows = ne[1] * ne[2] * ne[3];
    (void)nthreads;
    if (n == 0) return;
#ifdef _OPENMP
    #pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
#endif
    for (int64_t row = 0; row < nrows; row++) {
        const int64_t i1 = row % ne[1], i2 = (row / ne[1]) % ne[2], i3 = row / (ne[1] * ne[2]);
        const uint16_t * xs = src + row * n;
        const uint16_t * ms = mask ? mask + (((i3 % mne[3]) * mne[2] + i2 % mne[2]) * mne[1] + i1) * n : NULL;
        uint16_t * c = dst + row * n;
        uint16_t mx = X16_NEG_INF;
        for (int64_t i = 0; i < n; i++) {
            uint16_t v = xs[i];
            if (v != X16_NEG_INF) {
                v = orc16_mul(v, scale);
                if (ms) {
                    if (ms[i] == X16_NEG_INF) v = X16_NEG_INF;
                    else if (!is_zero16(ms[i])) v = orc16_add(v, ms[i]);
                }
            }
            c[i] = v;
            if (orc16_gt(v, mx)) mx = v;
        }
        for (int64_t i = 0; i < n; i++) c[i] = orc16_exp(orc16_sub(c[i], mx));
        red_t r;
        r.st = stochastic(mode) ? orc_lfsr_jump(monte_seed, (uint64_t)row * (uint64_t)(n - 1)) : 0;
        red_from(mode, &r, c[0]);
        for (int64_t i = 1; i < n; i++) red_add(mode, &r, c[i]);
        const uint16_t total = red_finish(mode, &r);
        for (int64_t i = 0; i < n; i++) c[i] = orc16_div(c[i], total);
    }
}

void orc32_soft_max(const uint32_t * src, const int64_t ne[4], const uint32_t * mask,
                    const int64_t mne[4], uint32_t scale, uint32_t * dst, int nthreads) {
    const int64_t n = ne[0], nrows = ne[1] * ne[2] * ne[3];
    (void)nthreads;
    if (n == 0) return;
#ifdef _OPENMP
    #pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
#endif
    for (int64_t row = 0; row < nrows; row++) {
        const int64_t i1 = row % ne[1], i2 = (row / ne[1]) % ne[2], i3 = row / (ne[1] * ne[2]);
        const uint32_t * xs = src + row * n;
        const uint32_t * ms = mask ? mask + (((i3 % mne[3]) * mne[2] + i2 % mne[2]) * mne[1] + i1) * n : NULL;
        uint32_t * c = dst + row * n;
        uint32_t mx = X32_NEG_INF;
        for (int64_t i = 0; i < n; i++) {
            uint32_t v = xs[i];
            if (v != X32_NEG_INF) {
                v = mul32(v, scale);
                if (ms) {
                    if (ms[i] == X32_NEG_INF) v = X32_NEG_INF;
                    else if (!is_zero32(ms[i])) v = add32(v, ms[i]);
                }
            }
            c[i] = v;
            if (gt32(v, mx)) mx = v;
        }
        for (int64_t i = 0; i < n; i++) c[i] = exp32(sub32(c[i], mx));
        uint32_t total = c[0];
        for (int64_t i = 1; i < n; i++) total = add32(total, c[i]);
        for (int64_t i = 0; i < n; i++) c[i] = div32(c[i], total);
    }
}

/* k_rms_norm (lns-cuda-kernels.cuh:225-250) = xlns16_rms_norm[_sum32]
 * (lns16-sum32.h:142-151): sum of squares from zero, n additions */
void orc16_rms_norm(int mode, const uint16_t * src, uint16_t * dst, int64_t ncols, int64_t nrows,
                    float eps, uint16_t monte_seed, int nthreads) {
    (void)nthreads;
    if (ncols == 0) return;
    const uint16_t eps_l = orc16_from_f32(eps);
    const uint16_t inv_n = orc16_from_f32(1.0f / (float)ncols);
#ifdef _OPENMP
    #pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
#endif
    for (int64_t row = 0; row < nrows; row++) {
        const uint16_t * xs = src + row * ncols;
        red_t r;
        r.st = stochastic(mode) ? orc_lfsr_jump(monte_seed, (uint64_t)row * (uint64_t)ncols) : 0;
        red_from(mode, &r, X16_ZERO);
        for (int64_t i = 0; i < ncols; i++) red_add(mode, &r, orc16_mul(xs[i], xs[i]));
        const uint16_t mean = orc16_mul(red_finish(mode, &r), inv_n);
        const uint16_t inv = orc16_recip(orc16_sqrt(orc16_add(mean, eps_l)));
        for (int64_t i = 0; i < ncols; i++) dst[row * ncols + i] = orc16_mul(xs[i], inv);
    }
}

void orc32_rms_norm(const uint32_t * src, uint32_t * dst, int64_t ncols, int64_t nrows, float eps, int nthreads) {
    (void)nthreads;
    if (ncols == 0) return;
    const uint32_t eps_l = orc32_from_f32(eps);
    const uint32_t inv_n = orc32_from_f32(1.0f / (float)ncols);
#ifdef _OPENMP
    #pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
#endif
    for (int64_t row = 0; row < nrows; row++) {
        const uint32_t * xs = src + row * ncols;
        uint32_t acc = 0;
        for (int64_t i = 0; i < ncols; i++) acc = add32(acc, mul32(xs[i], xs[i]));
        const uint32_t mean = mul32(acc, inv_n);
        const uint32_t inv = recip32(sqrt32(add32(mean, eps_l)));
        for (int64_t i = 0; i < ncols; i++) dst[row * ncols + i] = mul32(xs[i], inv);
    }
}

void orc16_from_f32_n(const float * src, uint16_t * dst, int64_t n) { for (int64_t i = 0; i < n; i++) dst[i] = orc16_from_f32(src[i]); }
void orc16_to_f32_n(const uint16_t * src, float * dst, int64_t n) { for (int64_t i = 0; i < n; i++) dst[i] = g_dec16[src[i]]; }
void orc32_from_f32_n(const float * src, uint32_t * dst, int64_t n) { for (int64_t i = 0; i < n; i++) dst[i] = orc32_from_f32(src[i]); }
void orc32_to_f32_n(const uint32_t * src, float * dst, int64_t n) { for (int64_t i = 0; i < n; i++) dst[i] = orc32_to_f32(src[i]); }

int orc_init(void) {
    if (g_ready) return 0;
    build16();
    if (build32() != 0) return -1;
    build_lfsr();
    g_ready = 1;
    return 0;
}

/* ===================================================================== */
/* Elementwise ops at the F32 op boundary (lns-backend/src/lns-ops.cpp:   */
/* 468-599, 786-868, 1199-1281): each operand is converted with fp2xlns16, */
/* the op runs in xlns16 and the result is written back with xlns162fp.   */
/* ===================================================================== */

/* silu(x) = x * sigmoid(x), the sigmoid from its table (see build16) */
uint16_t orc16_silu(uint16_t x) { return orc16_mul(x, g_sig16[x]); }
/* tanh(x) = (e^2x - 1) / (e^2x + 1) in xlns16 arithmetic over the exp table;
 * reproduces the reference's tanh printout (unit-tests-lns16-base.txt:86),
 * including tanh(-0.01) = -0.008158 */
uint16_t orc16_tanh(uint16_t x) {
    const uint16_t e = orc16_exp(orc16_mul(x, (uint16_t) (X16_OFFSET + 128)));
    return orc16_div(orc16_sub(e, (uint16_t) X16_OFFSET), orc16_add(e, (uint16_t) X16_OFFSET));
}
/* gelu(x) = 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))), ggml's tanh
 * form, in xlns16 arithmetic with the constants converted by fp2xlns16;
 * reproduces the reference's geglu printout (unit-tests-lns16-base.txt:65-84) */
uint16_t orc16_gelu(uint16_t x) {
    const uint16_t s = orc16_from_f32(0.79788456080286535588f), a = orc16_from_f32(0.044715f), h = orc16_from_f32(0.5f);
    const uint16_t x3 = orc16_mul(orc16_mul(x, x), x);
    const uint16_t in = orc16_mul(s, orc16_add(x, orc16_mul(a, x3)));
    return orc16_mul(orc16_mul(h, x), orc16_add((uint16_t) X16_OFFSET, orc16_tanh(in)));
}
/* relu(x): x where x > 0, else the zero code */
uint16_t orc16_relu(uint16_t x) {
    return ((x & X16_SIGNMASK) || (x & X16_LOGMASK) == 0) ? (uint16_t) X16_ZERO : x;
}

static inline uint16_t f2c(float f) { return orc16_from_f32(f); }
static inline float c2f(uint16_t c) { return orc16_to_f32(c); }

/* dst = a op b, b repeated to a's shape (lns_add / lns_mul / lns_div) */
void orc16_binary_f32(int op, const float * a, const int64_t ane[4], const float * b, const int64_t bne[4], float * dst) {
    for (int64_t i3 = 0; i3 < ane[3]; i3++)
        for (int64_t i2 = 0; i2 < ane[2]; i2++)
            for (int64_t i1 = 0; i1 < ane[1]; i1++) {
                const int64_t ra = ((i3 * ane[2] + i2) * ane[1] + i1) * ane[0];
                const int64_t rb = (((i3 % bne[3]) * bne[2] + (i2 % bne[2])) * bne[1] + (i1 % bne[1])) * bne[0];
                for (int64_t i0 = 0; i0 < ane[0]; i0++) {
                    const uint16_t x = f2c(a[ra + i0]), y = f2c(b[rb + i0 % bne[0]]);
                    const uint16_t r = op == ORC_ADD ? orc16_add(x, y) : op == ORC_MUL ? orc16_mul(x, y) : orc16_div(x, y);
                    dst[ra + i0] = c2f(r);
                }
            }
}

/* dst = src * s (+ b when b != 0) (lns_scale) */
void orc16_scale_f32(const float * src, float * dst, int64_t n, float s, float b) {
    const uint16_t sl = f2c(s), bl = f2c(b);
    for (int64_t i = 0; i < n; i++) {
        uint16_t v = orc16_mul(f2c(src[i]), sl);
        if (b != 0.0f) v = orc16_add(v, bl);
        dst[i] = c2f(v);
    }
}

void orc16_unary_f32(int op, const float * src, float * dst, int64_t n) {
    for (int64_t i = 0; i < n; i++) {
        const uint16_t v = f2c(src[i]);
        dst[i] = c2f(op == ORC_SILU ? orc16_silu(v) : op == ORC_GELU ? orc16_gelu(v) : op == ORC_TANH ? orc16_tanh(v)
                                                                                             : orc16_relu(v));
    }
}

/* dst[r][c] = silu(gate[r*gs + c]) * up[r*us + c] (lns_swiglu) */
void orc16_swiglu_f32(const float * gate, const float * up, int64_t gs, int64_t us, float * dst, int64_t nc, int64_t nr) {
    for (int64_t r = 0; r < nr; r++)
        for (int64_t c = 0; c < nc; c++)
            dst[r * nc + c] = c2f(orc16_mul(orc16_silu(f2c(gate[r * gs + c])), f2c(up[r * us + c])));
}

/* dst[r][c] = gelu(gate[r*gs + c]) * up[r*us + c] (lns_geglu, lns-ops.cpp:865-918) */
void orc16_geglu_f32(const float * gate, const float * up, int64_t gs, int64_t us, float * dst, int64_t nc, int64_t nr) {
    for (int64_t r = 0; r < nr; r++)
        for (int64_t c = 0; c < nc; c++)
            dst[r * nc + c] = c2f(orc16_mul(orc16_gelu(f2c(gate[r * gs + c])), f2c(up[r * us + c])));
}

/* rotary embedding of rows of ne[0] (lns_rope): pairs (2j, 2j+1), or (j, j +
 * n_dims/2) for neox, rotated by cos_sin[(i2 * n_dims/2 + j) * 2 + {0,1}] of
 * the row's position i2; dimensions past n_dims pass through xlns16. */
void orc16_rope_f32(const float * src, const int64_t ne[4], const float * cos_sin, int n_dims, int neox, float * dst) {
    const int64_t half = n_dims / 2;
    for (int64_t i3 = 0; i3 < ne[3]; i3++)
        for (int64_t i2 = 0; i2 < ne[2]; i2++)
            for (int64_t i1 = 0; i1 < ne[1]; i1++) {
                const int64_t row = ((i3 * ne[2] + i2) * ne[1] + i1) * ne[0];
                for (int64_t j = 0; j < half; j++) {
                    const uint16_t c = f2c(cos_sin[(i2 * half + j) * 2]), sn = f2c(cos_sin[(i2 * half + j) * 2 + 1]);
                    const int64_t i0 = neox ? j : 2 * j, i1b = neox ? j + half : 2 * j + 1;
                    const uint16_t x0 = f2c(src[row + i0]), x1 = f2c(src[row + i1b]);
                    dst[row + i0]  = c2f(orc16_sub(orc16_mul(x0, c), orc16_mul(x1, sn)));
                    dst[row + i1b] = c2f(orc16_add(orc16_mul(x0, sn), orc16_mul(x1, c)));
                }
                for (int64_t j = n_dims; j < ne[0]; j++) dst[row + j] = c2f(f2c(src[row + j]));
            }
}

/* ---- the same ops in xlns32 (lns-backend/src32/lns32-ops.cpp) ---- */

/* silu(x) = x / (1 + exp(-x)) in xlns32 arithmetic, exp through float as in
 * the xlns32 softmax (exp32) */
uint32_t orc32_silu(uint32_t x) {
    return div32(x, add32(0x40000000u, exp32(x ^ X32_SIGNMASK)));
}

static inline uint32_t f2c32(float f) { return orc32_from_f32(f); }
static inline float c2f32(uint32_t c) { return orc32_to_f32(c); }

/* e^x in double: the same range reduction and degree-14 Taylor series as
 * orc_expf, without the float rounding; |x| clamped to 700 */
double orc_exp_d(double xd) {
    if (xd != xd) return xd;
    if (xd > 700.0) xd = 700.0;
    if (xd < -700.0) xd = -700.0;
    const double t = xd * 1.4426950408889634074;
    const double n = nearbyint(t);
    const double r = (t - n) * 0.69314718055994530942;
    static const double c[15] = {
        1.0, 1.0, 1.0 / 2, 1.0 / 6, 1.0 / 24, 1.0 / 120, 1.0 / 720, 1.0 / 5040, 1.0 / 40320,
        1.0 / 362880, 1.0 / 3628800, 1.0 / 39916800, 1.0 / 479001600, 1.0 / 6227020800.0,
        1.0 / 87178291200.0 };
    double p = c[14];
    for (int i = 13; i >= 0; i--) p = fma(p, r, c[i]);
    return ldexp(p, (int)n);
}
/* tanh(y) = (e^2y - 1) / (e^2y + 1) in double */
double orc_tanh_d(double y) {
    const double e = orc_exp_d(2.0 * y);
    return (e - 1.0) / (e + 1.0);
}
/* xlns32 tanh and gelu go through floating point, as xlns32's activations do
 * in the reference (docs/CUDA.md:159-166: float tanhf there; this build's
 * own double tanh, identical on host and device, so the GPU is bit-exact).
 * Both reproduce the reference's LNS32 tanh and geglu printouts
 * (results/sum32-evidence/unit-tests-lns32.txt); gelu in xlns32 arithmetic
 * misses one geglu digit. */
uint32_t orc32_tanh(uint32_t x) { return orc32_from_f32((float) orc_tanh_d((double) orc32_to_f32(x))); }
uint32_t orc32_gelu(uint32_t x) {
    const double d = (double) orc32_to_f32(x);
    const double u = 0.79788456080286535588 * (d + 0.044715 * d * d * d);
    return orc32_from_f32((float) (0.5 * d * (1.0 + orc_tanh_d(u))));
}

uint32_t orc32_relu(uint32_t x) {
    return ((x & X32_SIGNMASK) || (x & ~X32_SIGNMASK) == 0) ? 0u : x;
}

void orc32_unary_f32(int op, const float * src, float * dst, int64_t n) {
    for (int64_t i = 0; i < n; i++) {
        const uint32_t v = f2c32(src[i]);
        dst[i] = c2f32(op == ORC_SILU ? orc32_silu(v) : op == ORC_GELU ? orc32_gelu(v) : op == ORC_TANH ? orc32_tanh(v)
                                                                                                : orc32_relu(v));
    }
}

void orc32_binary_f32(int op, const float * a, const int64_t ane[4], const float * b, const int64_t bne[4], float * dst) {
    for (int64_t i3 = 0; i3 < ane[3]; i3++)
        for (int64_t i2 = 0; i2 < ane[2]; i2++)
            for (int64_t i1 = 0; i1 < ane[1]; i1++) {
                const int64_t ra = ((i3 * ane[2] + i2) * ane[1] + i1) * ane[0];
                const int64_t rb = (((i3 % bne[3]) * bne[2] + (i2 % bne[2])) * bne[1] + (i1 % bne[1])) * bne[0];
                for (int64_t i0 = 0; i0 < ane[0]; i0++) {
                    const uint32_t x = f2c32(a[ra + i0]), y = f2c32(b[rb + i0 % bne[0]]);
                    const uint32_t r = op == ORC_ADD ? add32(x, y) : op == ORC_MUL ? mul32(x, y) : div32(x, y);
                    dst[ra + i0] = c2f32(r);
                }
            }
}

void orc32_scale_f32(const float * src, float * dst, int64_t n, float s, float b) {
    const uint32_t sl = f2c32(s), bl = f2c32(b);
    for (int64_t i = 0; i < n; i++) {
        uint32_t v = mul32(f2c32(src[i]), sl);
        if (b != 0.0f) v = add32(v, bl);
        dst[i] = c2f32(v);
    }
}

void orc32_swiglu_f32(const float * gate, const float * up, int64_t gs, int64_t us, float * dst, int64_t nc, int64_t nr) {
    for (int64_t r = 0; r < nr; r++)
        for (int64_t c = 0; c < nc; c++)
            dst[r * nc + c] = c2f32(mul32(orc32_silu(f2c32(gate[r * gs + c])), f2c32(up[r * us + c])));
}

void orc32_geglu_f32(const float * gate, const float * up, int64_t gs, int64_t us, float * dst, int64_t nc, int64_t nr) {
    for (int64_t r = 0; r < nr; r++)
        for (int64_t c = 0; c < nc; c++)
            dst[r * nc + c] = c2f32(mul32(orc32_gelu(f2c32(gate[r * gs + c])), f2c32(up[r * us + c])));
}

void orc32_rope_f32(const float * src, const int64_t ne[4], const float * cos_sin, int n_dims, int neox, float * dst) {
    const int64_t half = n_dims / 2;
    for (int64_t i3 = 0; i3 < ne[3]; i3++)
        for (int64_t i2 = 0; i2 < ne[2]; i2++)
            for (int64_t i1 = 0; i1 < ne[1]; i1++) {
                const int64_t row = ((i3 * ne[2] + i2) * ne[1] + i1) * ne[0];
                for (int64_t j = 0; j < half; j++) {
                    const uint32_t c = f2c32(cos_sin[(i2 * half + j) * 2]), sn = f2c32(cos_sin[(i2 * half + j) * 2 + 1]);
                    const int64_t i0 = neox ? j : 2 * j, i1b = neox ? j + half : 2 * j + 1;
                    const uint32_t x0 = f2c32(src[row + i0]), x1 = f2c32(src[row + i1b]);
                    dst[row + i0]  = c2f32(add32(mul32(x0, c), mul32(x1, sn) ^ X32_SIGNMASK));
                    dst[row + i1b] = c2f32(add32(mul32(x0, sn), mul32(x1, c)));
                }
                for (int64_t j = n_dims; j < ne[0]; j++) dst[row + j] = c2f32(f2c32(src[row + j]));
            }
}
