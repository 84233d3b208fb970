// synthstat.cpp -- the reference's dot-product error statistics, replayed
// through the oracle.  TEST INFRASTRUCTURE ONLY.
//
// Protocol of experiments/dot-product-scaling/dot-bench.cpp synth() (run by
// run.py:62-75 with its defaults: seed 1, 4096 outputs = 1024 weight rows x 4
// tokens, one repetition): for each K, std::mt19937_64(seed + K) and
// std::normal_distribution<float>(0, 1) draw the weights a0 [M][K], then the
// activations x0 [N][K] ("signed"), |a0| and |N(0,1)| ("positive"), or a
// softmax over K of 2 N(0,1) per token ("attn").  a = x = the round trip of
// the inputs through the LNS format (the backend's scale by 1.0); the product
// is the mul_mat of the original F32 inputs in the configuration (Monte: LFSR
// state 1 + (seed * 7919 + K) % 65535 before it).  Errors per output against
// the exact long-double sums:
//   acc         (got - sum(a x)) / sum|a x|
//   acc_l2scale (got - sum(a x)) / sqrt(sum (a x)^2)
//   total       (got - sum(a0 x0)) / sum|a0 x0|
// each with bias, sd, rms, mean_abs, rel_l2 as the reference prints them.
//
//   synthstat <base|monte|lpvip|sum32|monte_bylpvip|xlns32> <signed|positive|attn> <K>  -> one JSON line
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "lns_oracle.h"

namespace {

struct err_stats {
    double n = 0, sum = 0, sumsq = 0, abs_sum = 0, num = 0, den = 0;
    void add(long double got, long double ref, long double scale) {
        const double e = scale > 0 ? (double) ((got - ref) / scale) : 0.0;
        n++;
        sum += e;
        sumsq += e * e;
        abs_sum += std::fabs(e);
        num += (double) ((got - ref) * (got - ref));
        den += (double) (ref * ref);
    }
    double mean() const { return sum / n; }
    double rms() const { return std::sqrt(sumsq / n); }
    double sd() const { return std::sqrt(std::max(0.0, sumsq / n - mean() * mean())); }
    double rel_l2() const { return den > 0 ? std::sqrt(num / den) : 0.0; }
};

void print(const char * key, const err_stats & s) {
    std::printf("\"%s\":{\"bias\":%.6g,\"sd\":%.6g,\"rms\":%.6g,\"mean_abs\":%.6g,\"rel_l2\":%.6g}", key, s.mean(),
                s.sd(), s.rms(), s.abs_sum / s.n, s.rel_l2());
}

void gen(const std::string & dist, int64_t K, int64_t M, int64_t N, std::mt19937_64 & rng, std::vector<float> & a,
         std::vector<float> & x) {
    std::normal_distribution<float> g(0.0f, 1.0f);
    a.resize((size_t) (K * M));
    x.resize((size_t) (K * N));
    for (auto & v : a) v = g(rng);
    if (dist == "signed") {
        for (auto & v : x) v = g(rng);
    } else if (dist == "positive") {
        for (auto & v : a) v = std::fabs(v);
        for (auto & v : x) v = std::fabs(g(rng));
    } else {
        for (int64_t n = 0; n < N; n++) {
            float mx = -1e30f;
            for (int64_t k = 0; k < K; k++) {
                x[n * K + k] = 2.0f * g(rng);
                mx = std::max(mx, x[n * K + k]);
            }
            double s = 0;
            for (int64_t k = 0; k < K; k++) {
                x[n * K + k] = std::exp(x[n * K + k] - mx);
                s += x[n * K + k];
            }
            for (int64_t k = 0; k < K; k++) x[n * K + k] = (float) (x[n * K + k] / s);
        }
    }
}

}  // namespace

int main(int argc, char ** argv) {
    if (argc < 4) {
        std::fprintf(stderr, "usage: synthstat <config> <dist> <K> [seed]\n");
        return 2;
    }
    const std::string cfg = argv[1], dist = argv[2];
    const int64_t K = std::atoll(argv[3]);
    const uint64_t seed = argc > 4 ? std::strtoull(argv[4], nullptr, 10) : 1;
    if (orc_init() != 0) return 1;
    const bool x32 = cfg == "xlns32";
    const int mode = cfg == "monte" ? ORC_MONTE : cfg == "monte_bylpvip" ? ORC_MONTE_BYLPVIP : cfg == "lpvip" ? ORC_LPVIP
                   : cfg == "sum32" ? ORC_SUM32 : ORC_BASE;
    const int64_t N = 4, M = 1024;
    std::mt19937_64 rng(seed + (uint64_t) K);
    std::vector<float> a0, x0;
    gen(dist, K, M, N, rng, a0, x0);
    // the inputs as the kernel uses them (the backend's round trip), and the product
    std::vector<float> a(a0.size()), x(x0.size()), out((size_t) (M * N));
    if (x32) {
        std::vector<uint32_t> ac(a0.size()), xc(x0.size()), oc((size_t) (M * N));
        orc32_from_f32_n(a0.data(), ac.data(), (int64_t) a0.size());
        orc32_from_f32_n(x0.data(), xc.data(), (int64_t) x0.size());
        orc32_to_f32_n(ac.data(), a.data(), (int64_t) a.size());
        orc32_to_f32_n(xc.data(), x.data(), (int64_t) x.size());
        orc32_mul_mat(ac.data(), xc.data(), oc.data(), K, M, N, 1, 1, 1, 1, 16);
        orc32_to_f32_n(oc.data(), out.data(), M * N);
    } else {
        std::vector<uint16_t> ac(a0.size()), xc(x0.size()), oc((size_t) (M * N));
        orc16_from_f32_n(a0.data(), ac.data(), (int64_t) a0.size());
        orc16_from_f32_n(x0.data(), xc.data(), (int64_t) x0.size());
        orc16_to_f32_n(ac.data(), a.data(), (int64_t) a.size());
        orc16_to_f32_n(xc.data(), x.data(), (int64_t) x.size());
        const uint16_t st = (uint16_t) (1 + (seed * 7919 + (uint64_t) K) % 65535);
        orc16_mul_mat(mode, ac.data(), xc.data(), oc.data(), K, M, N, 1, 1, 1, 1, st, 16);
        orc16_to_f32_n(oc.data(), out.data(), M * N);
    }
    err_stats acc, acc2, total;
    for (int64_t n = 0; n < N; n++) {
        for (int64_t m = 0; m < M; m++) {
            long double s = 0, s1 = 0, s2 = 0, t = 0, t1 = 0;
            for (int64_t k = 0; k < K; k++) {
                const long double p = (long double) a[m * K + k] * (long double) x[n * K + k];
                s += p;
                s1 += fabsl(p);
                s2 += p * p;
                const long double p0 = (long double) a0[m * K + k] * (long double) x0[n * K + k];
                t += p0;
                t1 += fabsl(p0);
            }
            const long double got = out[n * M + m];
            acc.add(got, s, s1);
            acc2.add(got, s, sqrtl(s2));
            total.add(got, t, t1);
        }
    }
    std::printf("{\"config\":\"%s\",\"dist\":\"%s\",\"K\":%lld,\"outputs\":%lld,", cfg.c_str(), dist.c_str(),
                (long long) K, (long long) (M * N));
    print("acc", acc);
    std::printf(",");
    print("acc_l2scale", acc2);
    std::printf(",");
    print("total", total);
    std::printf("}\n");
    return 0;
}
