// Host check: the flat image's branch-free xlns32 addition (add32f,
// lnsb_arith.cuh) equals the branching addition over the separate tables
// (add32: sb32 / db32 knots, db32_lo / db32_hi cotransformation), restated
// here on the host tables step for step.  Built host-only with nvcc (the
// header's __host__ __device__ functions) and linked with lnsb_tables.cpp.
// Usage: flat_adder_check [random pairs]  -> prints "<n> pairs, <k> differ".
#include <cstdio>
#include <cstdlib>
#include <random>

#include "lnsb_arith.cuh"

using namespace lnsb;

static const host_tables * H;

static int32_t host_sb(uint32_t d) {
    if (d >= k32_ess) return 0;
    const int32_t i = (int32_t) (d >> k32_sh);
    return lerp32(H->sb32[i], H->sb32[i + 1], d);
}

static int32_t host_db(uint32_t d) {                   // d > 0
    if (d >= k32_ess) return 0;
    if (d >= k32_one) {
        const int32_t i = (int32_t) ((d - k32_one) >> k32_sh);
        return lerp32(H->db32[i], H->db32[i + 1], d);
    }
    const uint32_t d1 = d >> 12, d2 = d & 4095u;
    if (d1 == 0) return H->db32_lo[d2];
    if (d2 == 0) return H->db32_hi[d1];
    const int32_t la = H->db32_lo[d2], lb = -(int32_t) d2 + H->db32_hi[d1];
    const int32_t hi = la > lb ? la : lb;
    return hi + host_sb((uint32_t) (la > lb ? la - lb : lb - la));
}

static uint32_t host_add32(uint32_t a, uint32_t b) {
    const uint32_t al = a & 0x7FFFFFFFu, bl = b & 0x7FFFFFFFu;
    const uint32_t mx = al > bl ? a : b, d = al > bl ? al - bl : bl - al;
    const bool usedb = ((a ^ b) & 0x80000000u) != 0;
    if (d == 0 && usedb) return 0u;
    const long long p = (long long) (mx & 0x7FFFFFFFu) + (usedb ? host_db(d) : host_sb(d));
    return (mx & 0x80000000u) | (uint32_t) (p < 0 ? 0 : (p > 0x7FFFFFFFLL ? 0x7FFFFFFFLL : p));
}

int main(int argc, char ** argv) {
    const long nrand = argc > 1 ? atol(argv[1]) : 20000000L;
    H = &get_host_tables(true, false);
    const int32_t * F = H->flat32.data();
    long n = 0, bad = 0;
    auto check = [&](uint32_t a, uint32_t b) {
        n++;
        const uint32_t x = add32f(F, a, b), y = host_add32(a, b);
        if (x != y) {
            if (bad < 10) printf("a=%08x b=%08x flat %08x tables %08x\n", a, b, x, y);
            bad++;
        }
    };
    // differences: every one below 2^18 (the cotransformation's octave in
    // full detail), every 64th up to three octaves, at several magnitudes,
    // for all four sign pairs; then the end of the tables (26 octaves)
    const uint32_t bases[] = { 0u, 1u, 0x00800000u, 0x3F000000u, 0x40000000u, 0x40000123u, 0x7F000000u, 0x7FF00000u };
    for (uint32_t base : bases)
        for (uint32_t d = 0; d < (3u << 23); d++) {
            if (d >= (1u << 18) && (d & 63u)) continue;
            if (base + d > 0x7FFFFFFFu) break;
            for (uint32_t s = 0; s < 4; s++) check(((s & 1u) << 31) | (base + d), ((s >> 1) << 31) | base);
        }
    for (uint32_t d = (26u << 23) - 4096; d < (26u << 23) + 4096; d++)
        for (uint32_t s = 0; s < 4; s++) check(((s & 1u) << 31) | (0x50000000u + d), ((s >> 1) << 31) | 0x50000000u);
    // random pairs, and random pairs less than 2^25 apart
    std::mt19937_64 g(1);
    for (long k = 0; k < nrand; k++) {
        const uint64_t r = g();
        check((uint32_t) r, (uint32_t) (r >> 32));
        const uint32_t a = (uint32_t) g() & 0x7FFFFFFFu, d = (uint32_t) (r >> 39);
        if (a + d <= 0x7FFFFFFFu) check((a + d) | ((uint32_t) (r >> 63) << 31), a);
    }
    printf("%ld pairs, %ld differ\n", n, bad);
    return bad != 0;
}
