// Parity of the C++ host interface (include/lnsb200_kernel_set.hpp) with the
// CPU oracle, the way the reference's own parity test drives its kernel_set
// (lns-backend/tests/test-lns-cuda-parity.cpp): seeded inputs, every op
// through kernel_set, results compared bit for bit.  Linked against one
// liblnsb200_<mode>.so; the oracle (test infrastructure) is the checker.
// Exit status 0 = every case matched.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include <cuda_fp16.h>

#include "lnsb200_kernel_set.hpp"

extern "C" {
#include "lns_oracle.h"
}

namespace {

int g_fail = 0, g_pass = 0;

void check(bool ok, const char * what) {
    std::printf("%s %s\n", ok ? "PASS" : "FAIL", what);
    (ok ? g_pass : g_fail)++;
}

// seeded normal floats: 64-bit LCG + Box-Muller
struct rng {
    uint64_t s;
    explicit rng(uint64_t seed) : s(seed * 0x9E3779B97F4A7C15ull + 1) {}
    double uni() {
        s = s * 6364136223846793005ull + 1442695040888963407ull;
        return ((double) (s >> 11) + 0.5) / 9007199254740992.0;
    }
    std::vector<float> normal(size_t n, double sigma) {
        std::vector<float> v(n);
        for (size_t i = 0; i < n; i++) v[i] = (float) (sigma * std::sqrt(-2.0 * std::log(uni())) * std::cos(6.283185307179586 * uni()));
        return v;
    }
};

template <class T> struct dev {
    T * p = nullptr;
    size_t n = 0;
    explicit dev(size_t n_) : n(n_) { cudaMalloc((void **) &p, n * sizeof(T) + 16); }
    explicit dev(const std::vector<T> & h) : dev(h.size()) { cudaMemcpy(p, h.data(), n * sizeof(T), cudaMemcpyHostToDevice); }
    ~dev() { cudaFree(p); }
    std::vector<T> get() const {
        std::vector<T> h(n);
        cudaMemcpy(h.data(), p, n * sizeof(T), cudaMemcpyDeviceToHost);
        return h;
    }
};

int oracle_mode(const char * m, const char * impl) {
    const std::string s = m ? m : "", i = impl ? impl : "";
    if (s == "monte") return i == "bylpvip" ? ORC_MONTE_BYLPVIP : ORC_MONTE;
    if (s == "lpvip") return ORC_LPVIP;
    if (s == "sum32") return ORC_SUM32;
    return ORC_BASE;
}

std::vector<uint16_t> codes16(const std::vector<float> & f) {
    std::vector<uint16_t> c(f.size());
    orc16_from_f32_n(f.data(), c.data(), (int64_t) f.size());
    return c;
}
std::vector<uint32_t> codes32(const std::vector<float> & f) {
    std::vector<uint32_t> c(f.size());
    orc32_from_f32_n(f.data(), c.data(), (int64_t) f.size());
    return c;
}
template <class T> std::vector<T> kmajor(const std::vector<T> & rows, int64_t M, int64_t K) {
    std::vector<T> t((size_t) (M * K));
    for (int64_t m = 0; m < M; m++)
        for (int64_t k = 0; k < K; k++) t[(size_t) (k * M + m)] = rows[(size_t) (m * K + k)];
    return t;
}

void test_mul_mat16(const lnsb200::kernel_set & ks, int mode, int64_t K, int64_t M, int64_t N, uint16_t seed) {
    rng r((uint64_t) (K * 7919 + M * 31 + N));
    const auto w = codes16(r.normal((size_t) (M * K), 0.02));
    const auto x = codes16(r.normal((size_t) (N * K), 1.0));
    dev<uint16_t> dw(kmajor(w, M, K)), dx(x), dout((size_t) (N * M));
    dev<float> df((size_t) (N * M));
    lnsb200::mul_mat_args a{ dw.p, dx.p, df.p, K, M, N, 1, 1, 1, 1, seed };
    const bool ok1 = ks.mul_mat_lns(a, dout.p, nullptr) == cudaSuccess;
    const bool ok2 = ks.mul_mat(a, nullptr) == cudaSuccess;
    cudaDeviceSynchronize();
    std::vector<uint16_t> want((size_t) (N * M));
    orc16_mul_mat(mode, w.data(), x.data(), want.data(), K, M, N, 1, 1, 1, 1, seed, 8);
    std::vector<float> wantf(want.size());
    orc16_to_f32_n(want.data(), wantf.data(), (int64_t) want.size());
    const auto got = dout.get();
    const auto gotf = df.get();
    char buf[128];
    std::snprintf(buf, sizeof buf, "mul_mat xlns16 K=%lld M=%lld N=%lld (codes)", (long long) K, (long long) M, (long long) N);
    check(ok1 && got == want, buf);
    std::snprintf(buf, sizeof buf, "mul_mat xlns16 K=%lld M=%lld N=%lld (F32 out)", (long long) K, (long long) M, (long long) N);
    check(ok2 && std::memcmp(gotf.data(), wantf.data(), gotf.size() * 4) == 0, buf);
}

void test_soft_max16(const lnsb200::kernel_set & ks, int mode) {
    const int64_t ne0 = 96, ne1 = 40;
    rng r(5);
    const auto src = codes16(r.normal((size_t) (ne0 * ne1), 3.0));
    std::vector<float> mf((size_t) (ne0 * ne1), 0.0f);
    for (int64_t q = 0; q < ne1; q++)
        for (int64_t k = q + ne0 - ne1 + 1; k < ne0; k++) mf[(size_t) (q * ne0 + k)] = -INFINITY;
    std::vector<uint16_t> mask(mf.size());
    for (size_t i = 0; i < mf.size(); i++) mask[i] = orc16_mask_from_f32(mf[i]);
    const int64_t ne[4] = { ne0, ne1, 1, 1 };
    const uint16_t scale = orc16_from_f32(0.125f);
    dev<uint16_t> ds(src), dm(mask), dd(src.size()), dwk(src.size());
    const bool ok = ks.soft_max_lns(ds.p, ne, dm.p, ne, scale, dd.p, dwk.p, 7, nullptr) == cudaSuccess;
    cudaDeviceSynchronize();
    std::vector<uint16_t> want(src.size());
    orc16_soft_max(mode, src.data(), ne, mask.data(), ne, scale, want.data(), 7, 8);
    check(ok && dd.get() == want, "soft_max xlns16 96 x 40, causal mask, scale 0.125");
}

void test_rms_norm16(const lnsb200::kernel_set & ks, int mode) {
    const int64_t nc = 576, nr = 16;
    rng r(9);
    const auto src = codes16(r.normal((size_t) (nc * nr), 1.0));
    dev<uint16_t> ds(src), dd(src.size());
    const bool ok = ks.rms_norm_lns(ds.p, dd.p, nc, nr, 1e-5f, 7, nullptr) == cudaSuccess;
    cudaDeviceSynchronize();
    std::vector<uint16_t> want(src.size());
    orc16_rms_norm(mode, src.data(), want.data(), nc, nr, 1e-5f, 7, 8);
    check(ok && dd.get() == want, "rms_norm xlns16 576 x 16, eps 1e-5");
}

void test_conversions(const lnsb200::kernel_set & ks16, const lnsb200::kernel_set & ks32) {
    rng r(13);
    const auto f = r.normal(4096, 2.0);
    dev<float> df(f);
    dev<uint16_t> d16(f.size());
    dev<uint32_t> d32(f.size());
    const bool ok = ks16.to_lns(df.p, d16.p, (int64_t) f.size(), nullptr) == cudaSuccess &&
                    ks32.to_lns(df.p, d32.p, (int64_t) f.size(), nullptr) == cudaSuccess;
    cudaDeviceSynchronize();
    check(ok && d16.get() == codes16(f) && d32.get() == codes32(f), "to_lns xlns16 and xlns32, 4096 values");
}

void test_mul_mat32(const lnsb200::kernel_set & ks, int64_t K, int64_t M, int64_t N) {
    rng r((uint64_t) (K + M + N));
    const auto w = codes32(r.normal((size_t) (M * K), 0.02));
    const auto x = codes32(r.normal((size_t) (N * K), 1.0));
    dev<uint32_t> dw(kmajor(w, M, K)), dx(x), dout((size_t) (N * M));
    lnsb200::mul_mat_args a{ dw.p, dx.p, nullptr, K, M, N, 1, 1, 1, 1, 7 };
    const bool ok = ks.mul_mat_lns(a, dout.p, nullptr) == cudaSuccess;
    cudaDeviceSynchronize();
    std::vector<uint32_t> want((size_t) (N * M));
    orc32_mul_mat(w.data(), x.data(), want.data(), K, M, N, 1, 1, 1, 1, 8);
    char buf[96];
    std::snprintf(buf, sizeof buf, "mul_mat xlns32 K=%lld M=%lld N=%lld", (long long) K, (long long) M, (long long) N);
    check(ok && dout.get() == want, buf);
}

void test_mul_mat_id16(const lnsb200::kernel_set & ks, int mode) {
    const int64_t n_expert = 4, K = 200, M = 70, n_tokens = 3, n_used = 2, ne11 = 1;
    rng r(21);
    const auto w = codes16(r.normal((size_t) (n_expert * M * K), 0.02));     // [e][m][k]
    const auto x = codes16(r.normal((size_t) (n_tokens * ne11 * K), 1.0));
    std::vector<int32_t> ids = { 3, 1, 0, 0, 2, 3 };
    std::vector<uint16_t> wk((size_t) (n_expert * K * M));
    for (int64_t e = 0; e < n_expert; e++)
        for (int64_t m = 0; m < M; m++)
            for (int64_t k = 0; k < K; k++) wk[(size_t) ((e * K + k) * M + m)] = w[(size_t) ((e * M + m) * K + k)];
    dev<uint16_t> dw(wk), dx(x), dout((size_t) (n_tokens * n_used * M));
    dev<int32_t> di(ids);
    lnsb_mul_mat_id_args a{ dw.p, dx.p, di.p, nullptr, K, M, n_expert, ne11, n_used, n_tokens, n_used, 0xB403 };
    const bool ok = ks.mul_mat_id_lns(a, dout.p, nullptr) == cudaSuccess;
    cudaDeviceSynchronize();
    std::vector<uint16_t> want(dout.n);
    orc16_mul_mat_id(mode, w.data(), x.data(), ids.data(), want.data(), K, M, n_expert, ne11, n_used, n_tokens, n_used,
                     0xB403, 8);
    check(ok && dout.get() == want, "mul_mat_id xlns16 4 experts, 3 tokens x 2 slots, K=200 M=70");
}

void test_weight_cache(const lnsb200::kernel_set & ks) {
    const int64_t rows = 96, cols = 512;
    rng r(23);
    const auto f = r.normal((size_t) (rows * cols), 0.05);
    std::vector<uint16_t> h16(f.size());
    for (size_t i = 0; i < f.size(); i++) {                // F16 rows on the host (round to nearest even)
        const __half v = __float2half_rn(f[i]);
        std::memcpy(&h16[i], &v, 2);
    }
    lnsb200::weight_cache cache(ks, 1 << 20);
    cudaError_t st = cudaErrorUnknown;
    const void * img = cache.get(h16.data(), LNSB_TYPE_F16, rows, cols, nullptr, nullptr, &st);
    const void * again = cache.get(h16.data(), LNSB_TYPE_F16, rows, cols, nullptr, nullptr);
    std::vector<uint16_t> got((size_t) (rows * cols));
    if (img != nullptr) cudaMemcpy(got.data(), img, got.size() * 2, cudaMemcpyDeviceToHost);
    std::vector<uint16_t> want(got.size());
    for (int64_t m = 0; m < rows; m++)
        for (int64_t k = 0; k < cols; k++) {
            __half hv;
            std::memcpy(&hv, &h16[(size_t) (m * cols + k)], 2);
            want[(size_t) (k * rows + m)] = orc16_from_f32(__half2float(hv));
        }
    check(st == cudaSuccess && img != nullptr && img == again && cache.entries() == 1 && got == want,
          "weight_cache: F16 host rows, converted once, k-major image");
}

}  // namespace

int main() {
    if (orc_init() != 0) {
        std::printf("FAIL oracle init\n");
        return 2;
    }
    const auto & k16 = lnsb200::xlns16_kernels();
    const auto & k32 = lnsb200::xlns32_kernels();
    const int mode = oracle_mode(k16.sum_mode(), k16.monte_impl());
    std::printf("library: %s\n", k16.description());
    check(std::string(k16.format_name()) == "xlns16" && k16.value_size() == 2 &&
          std::string(k32.format_name()) == "xlns32" && k32.value_size() == 4, "identity");

    // calls before upload_tables report an error and do not abort
    {
        dev<uint16_t> dw(16), dx(16), dout(16);
        lnsb200::mul_mat_args a{ dw.p, dx.p, nullptr, 4, 4, 4, 1, 1, 1, 1, 7 };
        const cudaError_t e = k16.mul_mat_lns(a, dout.p, nullptr);
        check(e == cudaErrorInitializationError && lnsb200::kernel_set::last_status() == LNSB_E_NO_TABLES,
              "mul_mat before upload_tables -> cudaErrorInitializationError (LNSB_E_NO_TABLES)");
    }
    check(k16.upload_tables() == cudaSuccess && k32.upload_tables() == cudaSuccess, "upload_tables");
    {
        lnsb200::mul_mat_args a{ nullptr, nullptr, nullptr, -1, 4, 4, 1, 1, 1, 1, 7 };
        const cudaError_t e = k16.mul_mat_lns(a, nullptr, nullptr);
        check(e == cudaErrorInvalidValue && lnsb200::kernel_set::last_status() == LNSB_E_INVALID,
              "negative K -> cudaErrorInvalidValue (LNSB_E_INVALID)");
    }

    test_conversions(k16, k32);
    test_mul_mat16(k16, mode, 1536, 576, 8, 7);
    test_mul_mat16(k16, mode, 576, 1536, 64, 7);       // configs[1] weights, 64 tokens
    test_mul_mat16(k16, mode, 100, 37, 5, 0xB403);     // ragged
    test_soft_max16(k16, mode);
    test_rms_norm16(k16, mode);
    test_mul_mat_id16(k16, mode);
    test_weight_cache(k16);
    test_mul_mat32(k32, 576, 96, 9);
    test_mul_mat32(k32, 129, 33, 4);

    // Monte state: reserve hands out the current state and advances it by the draws
    {
        const uint16_t s0 = lnsb200::monte_get_state();
        lnsb200::mul_mat_args a{ nullptr, nullptr, nullptr, 576, 1536, 8, 1, 1, 1, 1, 0 };
        const uint64_t draws = k16.mul_mat_draws(a);
        const uint16_t start = lnsb200::monte_reserve(draws);
        check(start == s0 && lnsb200::monte_get_state() == orc_lfsr_jump(s0, draws), "Monte reserve");
        lnsb200::monte_set_state(7);
    }

    std::printf("%d passed, %d failed (sum mode %s)\n", g_pass, g_fail, k16.sum_mode() ? k16.sum_mode() : "-");
    return g_fail == 0 ? 0 : 1;
}
