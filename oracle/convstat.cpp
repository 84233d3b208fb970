// convstat.cpp -- the reference's F32 -> LNS conversion statistics, replayed
// through the oracle.  TEST INFRASTRUCTURE ONLY.
//
// Protocol of experiments/dot-product-scaling/dot-bench.cpp:186-213 (run with
// its default --seed 1 and --outputs 4194304, run.py:85-95): n values with
// log-uniform magnitudes 2^-20 .. 2^20 and a random sign from one
// std::mt19937_64, each converted to LNS and back once, twice and three
// times; the statistics are the ones that program prints, over the values
// whose round trips stay finite and non-zero.  The sign bit and the exponent
// are drawn in one expression whose operand order C++ leaves to the
// compiler, so both orders are available (argument 3: 0 = the exponent's
// draw first, as GCC evaluates it; 1 = the sign's first).
//
//   convstat <16|32> [n] [order]   -> one JSON line
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <vector>

#include "lns_oracle.h"

static float round_trip(int fmt, float x) {
    return fmt == 16 ? orc16_to_f32(orc16_from_f32(x)) : orc32_to_f32(orc32_from_f32(x));
}

int main(int argc, char ** argv) {
    const int fmt = argc > 1 ? std::atoi(argv[1]) : 16;
    const long long n = argc > 2 ? std::atoll(argv[2]) : 4194304;
    const int order = argc > 3 ? std::atoi(argv[3]) : 0;
    if (orc_init() != 0) return 1;
    std::mt19937_64 rng(1);
    std::uniform_real_distribution<double> e(-20.0, 20.0);
    std::vector<float> v((size_t) n);
    for (auto & x : v) {
        double s, m;
        if (order == 0) { m = std::exp2(e(rng)); s = (rng() & 1) ? -1.0 : 1.0; }
        else            { s = (rng() & 1) ? -1.0 : 1.0; m = std::exp2(e(rng)); }
        x = (float) (s * m);
    }
    double mean = 0, sq = 0, lg = 0, d12 = 0, d23 = 0;
    long long up = 0, down = 0, same = 0, ch12 = 0, ch23 = 0, cnt = 0;
    for (size_t i = 0; i < v.size(); i++) {
        const float r1 = round_trip(fmt, v[i]), r2 = round_trip(fmt, r1), r3 = round_trip(fmt, r2);
        if (!std::isfinite(r1) || !std::isfinite(r3) || r1 == 0 || r2 == 0 || r3 == 0) continue;
        const double rel = ((double) r1 - v[i]) / v[i];
        mean += rel;
        sq += rel * rel;
        lg += std::log2(std::fabs((double) r1 / v[i]));
        up += std::fabs(r1) > std::fabs(v[i]);
        down += std::fabs(r1) < std::fabs(v[i]);
        same += r1 == v[i];
        ch12 += r2 != r1;
        ch23 += r3 != r2;
        d12 += std::log2(std::fabs((double) r2 / r1));
        d23 += std::log2(std::fabs((double) r3 / r2));
        cnt++;
    }
    std::printf("{\"values\": %lld, \"mean_rel\": %.6g, \"rms_rel\": %.6g, \"mean_log2\": %.6g, \"frac_up\": %.6g, "
                "\"frac_down\": %.6g, \"frac_exact\": %.6g, \"frac_changed_round2\": %.6g, \"frac_changed_round3\": %.6g, "
                "\"drift_log2_round2\": %.6g, \"drift_log2_round3\": %.6g}\n",
                cnt, mean / cnt, std::sqrt(sq / cnt), lg / cnt, (double) up / cnt, (double) down / cnt,
                (double) same / cnt, (double) ch12 / cnt, (double) ch23 / cnt, d12 / cnt, d23 / cnt);
    return 0;
}
