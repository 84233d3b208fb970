// C++ host interface of the B200 LNS hot path: the reference's kernel_set
// (lns-backend/cuda/lns-cuda-kernels.h:85-139) restated over the C ABI of
// lnsb200.h.  Method names, argument meanings and the cudaError_t results
// follow that interface, so host code written against it (the reference's
// context, lns-backend/cuda/lns-cuda-context.cpp) reads the same; the
// namespace is this library's own.  Header-only: link one
// liblnsb200_<mode>.so, which fixes the GGML_LNS16_SUM mode as the
// reference's build does.  The interface's elementwise ops (binary, scale,
// unary, glu, rope; :117-138) are not on this hot path and are not mirrored.
//
// Error behaviour: every call returns cudaSuccess or an error and never
// aborts.  C ABI statuses map as: > 0 -> that cudaError_t, LNSB_E_NO_TABLES
// -> cudaErrorInitializationError, LNSB_E_NO_DEVICE -> cudaErrorNoDevice,
// LNSB_E_UNSUPPORTED -> cudaErrorNotSupported, other negatives ->
// cudaErrorInvalidValue.  last_status() keeps the C ABI's own code.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "lnsb200.h"

namespace lnsb200 {

// lns-cuda-kernels.h:39-58: four ggml dimensions; mul_mat operands (weights
// k-major per slice, w[k*M + m]; activations [slice][N][K]; dst F32 [slice][N][M])
struct shape4 {
    int64_t ne[4];
};

struct mul_mat_args {
    const void * w;
    const void * x;
    float *      dst;
    int64_t      K, M, N;
    int64_t      ne02, ne03, ne12, ne13;
    uint16_t     monte_seed;
};

// lns-cuda-kernels.h:60-83: F32 source and mask, LNS work buffer of src's size
struct soft_max_args {
    const float * src;
    shape4        src_shape;
    const float * mask;
    shape4        mask_shape;
    float         scale;
    float *       dst;
    void *        work;
    uint16_t      monte_seed;
};

static_assert(sizeof(mul_mat_args) == sizeof(lnsb_mul_mat_args), "mul_mat_args mirrors lnsb_mul_mat_args");
static_assert(sizeof(soft_max_args) == sizeof(lnsb_soft_max_args), "soft_max_args mirrors lnsb_soft_max_args");

inline cudaError_t to_cuda(int st) {
    if (st == LNSB_OK) return cudaSuccess;
    if (st > 0) return (cudaError_t) st;
    switch (st) {
        case LNSB_E_NO_TABLES:   return cudaErrorInitializationError;
        case LNSB_E_NO_DEVICE:   return cudaErrorNoDevice;
        case LNSB_E_UNSUPPORTED: return cudaErrorNotSupported;
        default:                 return cudaErrorInvalidValue;
    }
}

class kernel_set {
public:
    explicit kernel_set(int fmt) : fmt_(fmt) {}

    // identity (lns-cuda-kernels.h:89-95)
    const char * format_name() const { return lnsb_format_name(fmt_); }
    size_t       value_size() const { return lnsb_value_size(fmt_); }
    const char * sum_mode() const { return lnsb_sum_mode(fmt_); }
    const char * monte_impl() const { return lnsb_monte_impl(fmt_); }
    const char * description() const { return lnsb_description(fmt_); }

    // Monte draws each op consumes (lns-cuda-kernels.h:97-100)
    uint64_t mul_mat_draws(const mul_mat_args & a) const { return lnsb_mul_mat_draws(fmt_, c_args(a)); }
    uint64_t soft_max_draws(int64_t ncols, int64_t nrows) const { return lnsb_soft_max_draws(fmt_, ncols, nrows); }
    uint64_t rms_norm_draws(int64_t ncols, int64_t nrows) const { return lnsb_rms_norm_draws(fmt_, ncols, nrows); }

    // once per device before any op on it (lns-cuda-kernels.h:102-104)
    cudaError_t upload_tables() const { return ret(lnsb_upload_tables(fmt_)); }

    // conversions (lns-cuda-kernels.h:106-112)
    cudaError_t to_lns(const float * src, void * dst, int64_t n, cudaStream_t stream) const {
        return ret(lnsb_to_lns(fmt_, src, dst, n, stream));
    }
    cudaError_t to_lns_transposed(const float * src, void * dst, int64_t rows, int64_t cols, int64_t dst_ld,
                                  cudaStream_t stream) const {
        return ret(lnsb_to_lns_transposed(fmt_, src, dst, rows, cols, dst_ld, stream));
    }
    cudaError_t to_f32(const void * src, float * dst, int64_t n, cudaStream_t stream) const {
        return ret(lnsb_to_f32(fmt_, src, dst, n, stream));
    }

    // the reduction ops (lns-cuda-kernels.h:114-136)
    cudaError_t mul_mat(const mul_mat_args & a, cudaStream_t stream) const {
        return ret(lnsb_mul_mat(fmt_, c_args(a), stream));
    }
    cudaError_t rms_norm(const float * src, float * dst, int64_t ncols, int64_t nrows, float eps, uint16_t monte_seed,
                         cudaStream_t stream) const {
        return ret(lnsb_rms_norm(fmt_, src, dst, ncols, nrows, eps, monte_seed, stream));
    }
    cudaError_t soft_max(const soft_max_args & a, cudaStream_t stream) const {
        lnsb_soft_max_args b;
        std::memcpy(&b, &a, sizeof b);
        return ret(lnsb_soft_max(fmt_, &b, stream));
    }

    // the MUL_MAT op over F32 activations (to_lns of src1 and mul_mat in one call,
    // lns-cuda-ops.cpp:57-75); a.x holds F32 values, x_work N*K codes
    cudaError_t mul_mat_xf32(const mul_mat_args & a, void * x_work, cudaStream_t stream) const {
        return ret(lnsb_mul_mat_xf32(fmt_, c_args(a), x_work, stream));
    }

    // LNS-resident forms (codes in and out; not in the reference's interface)
    cudaError_t mul_mat_lns(const mul_mat_args & a, void * dst, cudaStream_t stream) const {
        return ret(lnsb_mul_mat_lns(fmt_, c_args(a), dst, stream));
    }
    cudaError_t soft_max_lns(const void * src, const int64_t ne[4], const void * mask, const int64_t mne[4],
                             uint32_t scale, void * dst, void * work, uint16_t monte_seed, cudaStream_t stream) const {
        return ret(lnsb_soft_max_lns(fmt_, src, ne, mask, mne, scale, dst, work, monte_seed, stream));
    }
    cudaError_t rms_norm_lns(const void * src, void * dst, int64_t ncols, int64_t nrows, float eps,
                             uint16_t monte_seed, cudaStream_t stream) const {
        return ret(lnsb_rms_norm_lns(fmt_, src, dst, ncols, nrows, eps, monte_seed, stream));
    }

    // MUL_MAT_ID (lns-backend/src/lns-ops.cpp:394-462; the reference's GPU
    // backend declines it), F32 out to a.dst or LNS codes out to dst
    cudaError_t mul_mat_id(const lnsb_mul_mat_id_args & a, cudaStream_t stream) const {
        return ret(lnsb_mul_mat_id(fmt_, &a, stream));
    }
    cudaError_t mul_mat_id_lns(const lnsb_mul_mat_id_args & a, void * dst, cudaStream_t stream) const {
        return ret(lnsb_mul_mat_id_lns(fmt_, &a, dst, stream));
    }
    uint64_t mul_mat_id_draws(const lnsb_mul_mat_id_args & a) const { return lnsb_mul_mat_id_draws(fmt_, &a); }

    // weights in ggml storage types (LNSB_TYPE_*), decoded on the device
    cudaError_t to_lns_transposed_typed(int type, const void * src, void * dst, int64_t rows, int64_t cols,
                                        int64_t dst_ld, cudaStream_t stream) const {
        return ret(lnsb_to_lns_transposed_typed(fmt_, type, src, dst, rows, cols, dst_ld, stream));
    }

    // the C ABI status of this thread's last call through any kernel_set
    static int last_status() { return last_(); }

private:
    static const lnsb_mul_mat_args * c_args(const mul_mat_args & a) {
        return reinterpret_cast<const lnsb_mul_mat_args *>(&a);   // same fields, same order (static_assert above)
    }
    static int & last_() {
        thread_local int st = LNSB_OK;
        return st;
    }
    static cudaError_t ret(int st) {
        last_() = st;
        return to_cuda(st);
    }
    int fmt_;
};

// the reference's accessors (lns-cuda-kernels.h:141-142); its per-mode
// accessors (:145-147) correspond here to loading another liblnsb200_<mode>.so
inline const kernel_set & xlns16_kernels() {
    static const kernel_set k(LNSB_XLNS16);
    return k;
}
inline const kernel_set & xlns32_kernels() {
    static const kernel_set k(LNSB_XLNS32);
    return k;
}

// The weight cache (lns-cuda-context.h:79-113) as an owning handle: get()
// returns the cached k-major LNS image of a weight, converting it on a miss.
class weight_cache {
public:
    // budget_bytes < 0: GGML_LNS_CUDA_CACHE_MB, else free device memory less 1 GiB
    explicit weight_cache(const kernel_set & ks, int64_t budget_bytes = -1)
        : h_(lnsb_weight_cache_create(ks.value_size() == 2 ? LNSB_XLNS16 : LNSB_XLNS32, budget_bytes)) {}
    ~weight_cache() { lnsb_weight_cache_destroy(h_); }
    weight_cache(const weight_cache &) = delete;
    weight_cache & operator=(const weight_cache &) = delete;

    bool valid() const { return h_ != nullptr; }
    // nullptr on failure (status in *st when st is given)
    const void * get(const void * src, int type, int64_t rows, int64_t cols, void * scratch, cudaStream_t stream,
                     cudaError_t * st = nullptr) const {
        const void * out = nullptr;
        const int r = lnsb_weight_cache_get(h_, src, type, rows, cols, scratch, &out, stream);
        if (st != nullptr) *st = to_cuda(r);
        return r == LNSB_OK ? out : nullptr;
    }
    int64_t entries() const { int64_t e = 0; lnsb_weight_cache_stats(h_, &e, nullptr, nullptr); return e; }
    int64_t used() const { int64_t u = 0; lnsb_weight_cache_stats(h_, nullptr, &u, nullptr); return u; }

private:
    lnsb_weight_cache * h_;
};

// Monte LFSR state of the process (ggml_backend_lns16_monte_*, lns-backend/include/ggml-lns.h:13-24)
inline uint16_t monte_get_state() {
    uint16_t s = 0;
    lnsb_monte_get_state(&s);
    return s;
}
inline bool monte_set_state(uint16_t s) { return lnsb_monte_set_state(s) == LNSB_OK; }
inline uint16_t monte_reserve(uint64_t draws) {
    uint16_t start = 0;
    lnsb_monte_reserve(draws, &start);
    return start;
}

}  // namespace lnsb200
