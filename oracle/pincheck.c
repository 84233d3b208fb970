/*
 * pincheck.c -- replays the reference's deterministic test programs through
 * the oracle and prints, as JSON, every figure those programs print.  Test
 * infrastructure: tests/test_oracle_pins.py compares the output with the
 * reference's committed outputs (tests/golden/reference_pins.json).
 *
 * Replayed programs (same generators, same shapes, same metrics):
 *   lns-backend/tests/test-lns16-sum32.cpp:24-220  (standalone sum32 checks)
 *   lns-backend/tests/test-lns-backend.cpp:83-215   (4x3 mul_mat)
 *                                        :221-285   (mul mat long, K=1536)
 *                                        :886-1001  (softmax cases)
 *                                        :1003-1051 (rms_norm cases)
 */
#include "lns_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static uint64_t g_rng = 0x2545F4914F6CDD1DULL;
static double rnd_uniform(void) {
    g_rng = g_rng * 6364136223846793005ULL + 1442695040888963407ULL;
    return (double)((g_rng >> 11) & ((1ULL << 53) - 1)) / (double)(1ULL << 53);
}
static uint16_t ideal16(double v) {
    if (v == 0.0) return 0;
    long code = lround(log2(fabs(v)) * 128.0) + 0x4000;
    if (code < 0) code = 0;
    if (code > 0x7FFF) code = 0x7FFF;
    return (uint16_t)((v < 0 ? 0x8000 : 0) | (unsigned)code);
}
static int ulp_diff(uint16_t a, uint16_t b) {
    if ((a ^ b) & 0x8000) return 0x7FFF;
    return abs((int)(a & 0x7FFF) - (int)(b & 0x7FFF));
}
static double dec(uint16_t v) { return (double)orc16_to_f32(v); }

static void standalone(void) {
    /* 1. round trip through the sum32 accumulator */
    int rt_ok = 1;
    for (int i = 0; i < 65536; i++) {
        uint16_t x = (uint16_t)i;
        if (orc16_sum(ORC_SUM32, &x, 1, NULL) != x) rt_ok = 0;
    }
    printf("\"roundtrip_ok\": %d,\n", rt_ok);

    /* 2. two-term sums */
    int wb = 0, ws = 0;
    long long tb = 0, ts = 0, cnt = 0;
    for (int i = 0; i < 200000; i++) {
        const double ea = rnd_uniform() * 40.0 - 20.0;
        const double eb = ea + rnd_uniform() * 40.0 - 20.0;
        double va = pow(2.0, ea), vb = pow(2.0, eb);
        if (rnd_uniform() < 0.5) va = -va;
        if (rnd_uniform() < 0.5) vb = -vb;
        const uint16_t a = orc16_from_f32((float)va), b = orc16_from_f32((float)vb);
        const double exact = dec(a) + dec(b);
        if (exact == 0.0) continue;
        const uint16_t want = ideal16(exact);
        const uint16_t pair[2] = { a, b };
        const int db = ulp_diff(orc16_add(a, b), want);
        const int ds = ulp_diff(orc16_sum(ORC_SUM32, pair, 2, NULL), want);
        if (db > wb) wb = db;
        if (ds > ws) ws = ds;
        tb += db; ts += ds; cnt++;
    }
    printf("\"two_term\": {\"n\": %lld, \"base_max\": %d, \"base_mean\": %.3f, \"sum32_max\": %d, \"sum32_mean\": %.3f},\n",
           cnt, wb, (double)tb / cnt, ws, (double)ts / cnt);

    /* 3. stagnation */
    const int sizes[] = { 128, 370, 512, 1536, 8960, 65536 };
    printf("\"ones\": {");
    for (int k = 0; k < 6; k++) {
        const int n = sizes[k];
        uint16_t * v = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)n);
        for (int i = 0; i < n; i++) v[i] = 0x4000;
        printf("%s\"%d\": [%.4f, %.4f]", k ? ", " : "", n, dec(orc16_sum(ORC_BASE, v, n, NULL)),
               dec(orc16_sum(ORC_SUM32, v, n, NULL)));
        free(v);
    }
    printf("},\n");

    /* 4. long mixed-sign dots */
    const int Ks[] = { 1536, 8960 };
    printf("\"long_dot\": {");
    for (int kk = 0; kk < 2; kk++) {
        const int K = Ks[kk];
        double srb = 0, srs = 0;
        int wins = 0;
        uint16_t * a = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)K);
        uint16_t * b = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)K);
        for (int t = 0; t < 64; t++) {
            double exact = 0.0;
            for (int i = 0; i < K; i++) {
                const float fa = (float)(rnd_uniform() * 2.0 - 1.0);
                const float fb = (float)(rnd_uniform() * 2.0 - 1.0);
                a[i] = orc16_from_f32(fa);
                b[i] = orc16_from_f32(fb);
                exact += dec(a[i]) * dec(b[i]);
            }
            const double gb = dec(orc16_vec_dot(ORC_BASE, a, b, K, NULL));
            const double gs = dec(orc16_vec_dot(ORC_SUM32, a, b, K, NULL));
            const double rb = fabs(gb - exact) / fabs(exact), rs = fabs(gs - exact) / fabs(exact);
            srb += rb; srs += rs;
            if (rs < rb) wins++;
        }
        printf("%s\"%d\": [%.3f, %.3f, %d]", kk ? ", " : "", K, srb / 64 * 100.0, srs / 64 * 100.0, wins);
        free(a); free(b);
    }
    printf("},\n");

    /* 5. rms_norm */
    const int rs_n[] = { 576, 1536 };
    printf("\"rms_standalone\": {");
    for (int kk = 0; kk < 2; kk++) {
        const int n = rs_n[kk];
        uint16_t * x = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)n);
        uint16_t * yb = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)n);
        uint16_t * ys = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)n);
        double sq = 0.0;
        for (int i = 0; i < n; i++) {
            x[i] = orc16_from_f32((float)(rnd_uniform() * 2.0 - 1.0));
            sq += dec(x[i]) * dec(x[i]);
        }
        const double inv = 1.0 / sqrt(sq / (double)n + 1e-6);
        orc16_rms_norm(ORC_BASE, x, yb, n, 1, 1e-6f, 7, 1);
        orc16_rms_norm(ORC_SUM32, x, ys, n, 1, 1e-6f, 7, 1);
        double mb = 0, ms = 0;
        for (int i = 0; i < n; i++) {
            const double want = dec(x[i]) * inv;
            const double eb = fabs(dec(yb[i]) - want) / fmax(fabs(want), 1e-6);
            const double es = fabs(dec(ys[i]) - want) / fmax(fabs(want), 1e-6);
            if (eb > mb) mb = eb;
            if (es > ms) ms = es;
        }
        printf("%s\"%d\": [%.3f, %.3f]", kk ? ", " : "", n, mb * 100.0, ms * 100.0);
        free(x); free(yb); free(ys);
    }
    printf("},\n");
}

/* ---- ggml suite cases, per mode (mode 100 = LNS32) ---- */

static float max_scaled(const float * got, const float * want, int n) {
    float m = 0.0f;
    for (int i = 0; i < n; i++) {
        const float e = fabsf(got[i] - want[i]) / fmaxf(fabsf(want[i]), 1.0f);
        if (e > m) m = e;
    }
    return m;
}

/* dst[N][M] = A[M][K] . B[N][K], through the oracle in `mode` */
static void lns_mm(int mode, const float * A, const float * B, float * out, int K, int M, int N, uint16_t * seed) {
    if (mode == 100) {
        uint32_t * a = malloc(sizeof(uint32_t) * (size_t)M * K), * b = malloc(sizeof(uint32_t) * (size_t)N * K);
        uint32_t * d = malloc(sizeof(uint32_t) * (size_t)M * N);
        orc32_from_f32_n(A, a, (int64_t)M * K);
        orc32_from_f32_n(B, b, (int64_t)N * K);
        orc32_mul_mat(a, b, d, K, M, N, 1, 1, 1, 1, 1);
        orc32_to_f32_n(d, out, (int64_t)M * N);
        free(a); free(b); free(d);
        return;
    }
    uint16_t * a = malloc(sizeof(uint16_t) * (size_t)M * K), * b = malloc(sizeof(uint16_t) * (size_t)N * K);
    uint16_t * d = malloc(sizeof(uint16_t) * (size_t)M * N);
    orc16_from_f32_n(A, a, (int64_t)M * K);
    orc16_from_f32_n(B, b, (int64_t)N * K);
    orc16_mul_mat(mode, a, b, d, K, M, N, 1, 1, 1, 1, *seed, 1);
    *seed = orc_lfsr_jump(*seed, orc_mul_mat_draws(mode, K, M, N, 1, 1));
    orc16_to_f32_n(d, out, (int64_t)M * N);
    free(a); free(b); free(d);
}

static void suite(int mode) {
    uint16_t seed = 7;
    /* 4x3 mul_mat, K=2 */
    const float A[8] = { 2, 8, 5, 1, 4, 2, 8, 6 }, B[6] = { 10, 5, 9, 9, 5, 4 };
    const float expected[12] = { 60, 55, 50, 110, 90, 54, 54, 126, 42, 29, 28, 64 };
    float out[12];
    lns_mm(mode, A, B, out, 2, 4, 3, &seed);
    printf("\"mm4x3\": [");
    for (int i = 0; i < 12; i++) printf("%s%.2f", i ? ", " : "", out[i]);
    printf("], \"mm4x3_err\": %.4f, ", max_scaled(out, expected, 12) * 100.0f);

    /* mul mat long */
    {
        const int K = 1536, M = 8, N = 4;
        uint64_t rng = 0x9E3779B97F4A7C15ull;
        float * a = malloc(sizeof(float) * M * K), * b = malloc(sizeof(float) * N * K), * o = malloc(sizeof(float) * M * N);
        for (int i = 0; i < M * K; i++) { rng = rng * 6364136223846793005ull + 1442695040888963407ull; a[i] = (float)((double)(uint32_t)(rng >> 32) / 2147483648.0 - 1.0); }
        for (int i = 0; i < N * K; i++) { rng = rng * 6364136223846793005ull + 1442695040888963407ull; b[i] = (float)((double)(uint32_t)(rng >> 32) / 2147483648.0 - 1.0); }
        lns_mm(mode, a, b, o, K, M, N, &seed);
        double se = 0, sr = 0, mx = 0;
        for (int n = 0; n < N; n++) for (int m = 0; m < M; m++) {
            double ref = 0;
            for (int k = 0; k < K; k++) ref += (double)a[m * K + k] * (double)b[n * K + k];
            const double err = o[n * M + m] - ref;
            se += err * err; sr += ref * ref;
            if (fabs(err) > mx) mx = fabs(err);
        }
        printf("\"mm_long\": [%.4f, %.4f, %.4f], ", mx / sqrt(sr / (M * N)) * 100.0, sqrt(sr / (M * N)), sqrt(se / sr) * 100.0);
        free(a); free(b); free(o);
    }

    /* softmax cases */
    {
        const struct { int ne00, ne01; float scale; int masked; } cs[5] = {
            { 8, 4, 1.0f, 0 }, { 512, 4, 1.0f, 0 }, { 512, 4, 0.125f, 0 }, { 64, 8, 1.0f, 1 }, { 256, 4, 0.125f, 1 } };
        printf("\"softmax\": [");
        for (int c = 0; c < 5; c++) {
            const int ne00 = cs[c].ne00, ne01 = cs[c].ne01, nn = ne00 * ne01;
            float * a = malloc(sizeof(float) * nn), * mk = malloc(sizeof(float) * nn), * ex = malloc(sizeof(float) * nn), * got = malloc(sizeof(float) * nn);
            for (int r = 0; r < ne01; r++) for (int i = 0; i < ne00; i++) {
                const float u = (float)((i * 37 + r * 101) % 97) / 97.0f;
                a[r * ne00 + i] = 8.0f * (u - 0.5f);
                mk[r * ne00 + i] = (cs[c].masked && (i >= ne00 - 1 - r || (i % 13) == 5)) ? -INFINITY : 0.0f;
            }
            for (int r = 0; r < ne01; r++) {
                float maxv = -INFINITY, sum = 0.0f;
                float * t = ex + r * ne00;
                for (int i = 0; i < ne00; i++) {
                    t[i] = a[r * ne00 + i] * cs[c].scale + (cs[c].masked ? mk[r * ne00 + i] : 0.0f);
                    if (t[i] > maxv) maxv = t[i];
                }
                for (int i = 0; i < ne00; i++) { t[i] = expf(t[i] - maxv); sum += t[i]; }
                for (int i = 0; i < ne00; i++) t[i] = t[i] / sum;
            }
            const int64_t ne[4] = { ne00, ne01, 1, 1 };
            if (mode == 100) {
                uint32_t * s = malloc(4 * (size_t)nn), * m = malloc(4 * (size_t)nn), * d = malloc(4 * (size_t)nn);
                for (int i = 0; i < nn; i++) { s[i] = orc32_from_f32(a[i]); m[i] = orc32_mask_from_f32(mk[i]); }
                orc32_soft_max(s, ne, cs[c].masked ? m : NULL, ne, orc32_from_f32(cs[c].scale), d, 1);
                orc32_to_f32_n(d, got, nn);
                free(s); free(m); free(d);
            } else {
                uint16_t * s = malloc(2 * (size_t)nn), * m = malloc(2 * (size_t)nn), * d = malloc(2 * (size_t)nn);
                for (int i = 0; i < nn; i++) { s[i] = orc16_from_f32(a[i]); m[i] = orc16_mask_from_f32(mk[i]); }
                orc16_soft_max(mode, s, ne, cs[c].masked ? m : NULL, ne, orc16_from_f32(cs[c].scale), d, seed, 1);
                seed = orc_lfsr_jump(seed, orc_soft_max_draws(mode, ne00, ne01));
                orc16_to_f32_n(d, got, nn);
                free(s); free(m); free(d);
            }
            float mae = 0.0f;
            for (int i = 0; i < nn; i++) { const float e = fabsf(got[i] - ex[i]); if (e > mae) mae = e; }
            printf("%s%.6f", c ? ", " : "", mae);
            free(a); free(mk); free(ex); free(got);
        }
        printf("], ");
    }

    /* rms_norm cases */
    {
        const int ns[2] = { 16, 576 };
        printf("\"rms_norm\": [");
        for (int c = 0; c < 2; c++) {
            const int ne00 = ns[c], ne01 = 3, nn = ne00 * ne01;
            float * a = malloc(sizeof(float) * nn), * ex = malloc(sizeof(float) * nn), * got = malloc(sizeof(float) * nn);
            for (int r = 0; r < ne01; r++) {
                double ss = 0.0;
                for (int i = 0; i < ne00; i++) {
                    const float u = (float)((i * 53 + r * 19) % 89) / 89.0f;
                    a[r * ne00 + i] = 6.0f * (u - 0.5f);
                    ss += (double)a[r * ne00 + i] * (double)a[r * ne00 + i];
                }
                const float inv = 1.0f / sqrtf((float)(ss / (double)ne00) + 1e-5f);
                for (int i = 0; i < ne00; i++) ex[r * ne00 + i] = a[r * ne00 + i] * inv;
            }
            if (mode == 100) {
                uint32_t * s = malloc(4 * (size_t)nn), * d = malloc(4 * (size_t)nn);
                orc32_from_f32_n(a, s, nn);
                orc32_rms_norm(s, d, ne00, ne01, 1e-5f, 1);
                orc32_to_f32_n(d, got, nn);
                free(s); free(d);
            } else {
                uint16_t * s = malloc(2 * (size_t)nn), * d = malloc(2 * (size_t)nn);
                orc16_from_f32_n(a, s, nn);
                orc16_rms_norm(mode, s, d, ne00, ne01, 1e-5f, seed, 1);
                seed = orc_lfsr_jump(seed, orc_rms_norm_draws(mode, ne00, ne01));
                orc16_to_f32_n(d, got, nn);
                free(s); free(d);
            }
            printf("%s%.4f", c ? ", " : "", max_scaled(got, ex, nn) * 100.0f);
            free(a); free(ex); free(got);
        }
        printf("]");
    }
}

static void lfsr(void) {
    uint16_t s = 7;
    uint16_t one = orc_lfsr_step(s);
    uint32_t period = 0;
    uint16_t t = 1;
    do { t = orc_lfsr_step(t); period++; } while (t != 1 && period < 70000);
    printf("\"lfsr\": {\"step7\": %u, \"period\": %u, \"zero_absorbing\": %d, \"jump_ok\": %d},\n",
           one, period, orc_lfsr_step(0) == 0, orc_lfsr_jump(7, 1) == one && orc_lfsr_jump(7, 65535) == 7);
}

int main(void) {
    if (getenv("KNOT")) orc_set_knot_mode(atoi(getenv("KNOT")));
    if (orc_init() != 0) { fprintf(stderr, "oracle init failed\n"); return 1; }
    printf("{\n");
    standalone();
    lfsr();
    const char * names[6] = { "base", "monte", "monte_bylpvip", "lpvip", "sum32", "lns32" };
    const int modes[6] = { ORC_BASE, ORC_MONTE, ORC_MONTE_BYLPVIP, ORC_LPVIP, ORC_SUM32, 100 };
    printf("\"suite\": {\n");
    for (int i = 0; i < 6; i++) {
        printf("  \"%s\": {", names[i]);
        suite(modes[i]);
        printf("}%s\n", i < 5 ? "," : "");
    }
    printf("}\n}\n");
    return 0;
}
