// B200 (sm_100a) kernels of the LNSCUDA16 / LNSCUDA32 hot path and the C ABI
// of include/lnsb200.h.
//
// The hot path is the reduction inside three ops (lns-backend/cuda/
// lns-cuda-kernels.cuh:80-157, 225-250, 255-325): every output is one
// sequential chain of LNS additions, in element order, because LNS addition
// is not associative.  Parallelism therefore comes only from independent
// outputs; each kernel below is organised around keeping as many chains in
// flight as possible per SM, with operands staged in shared memory and the
// Gaussian-log table resident there.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <array>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>

#include "lnsb200.h"
#include "lnsb200_graph.h"
#include "lnsb_arith.cuh"
#include "lnsb_tables.h"

// Scratch of lnsb_soft_max_lns_noalloc: a file-scope device array, so that
// entry point never allocates.  Host code must not use this name as a device
// address (in host code it is only a stand-in); the device address is looked
// up per device with cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[LNSB_NOALLOC_SCRATCH_BYTES];

namespace lnsb {

uint32_t host_from_f32_32(float x);   // defined below; the host twin of from_f32_32

namespace {

constexpr int k_max_devices = 64;

// ============================ table registry ===============================

struct device_slot {
    bool       ready16 = false, ready32 = false;
    dev_tables t{};
};
std::mutex                                 g_mu;
std::array<device_slot, k_max_devices>     g_slots;

template <class T>
cudaError_t upload(const std::vector<T> & v, const T ** out) {
    if (v.empty()) { *out = nullptr; return cudaSuccess; }
    void * p = nullptr;
    cudaError_t e = cudaMalloc(&p, v.size() * sizeof(T));
    if (e != cudaSuccess) return e;
    e = cudaMemcpy(p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) { cudaFree(p); return e; }
    *out = static_cast<const T *>(p);
    return cudaSuccess;
}

int current_device(int * dev) {
    const cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) return (int) e;
    if (*dev < 0 || *dev >= k_max_devices) return LNSB_E_NO_DEVICE;
    return 0;
}

// the current device's tables, or an error if lnsb_upload_tables did not run
int tables_for(int fmt, const dev_tables ** out) {
    int dev = 0;
    const int st = current_device(&dev);
    if (st != 0) return st;
    std::lock_guard<std::mutex> lock(g_mu);
    const device_slot & s = g_slots[dev];
    if (fmt == LNSB_XLNS16 ? !s.ready16 : !s.ready32) return LNSB_E_NO_TABLES;
    *out = &s.t;
    return 0;
}

__host__ __device__ __forceinline__ int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }

int status_of(cudaError_t e) { return e == cudaSuccess ? 0 : (int) e; }
int launch_status() { return status_of(cudaGetLastError()); }

// Programmatic dependent launch.  Every kernel of this library is launched
// with programmatic stream serialisation and begins with pdl_entry(): it
// waits there for the grid before it in the stream to complete (and its
// writes to be visible) before touching any data, then lets the grid after
// it launch.  The next kernel's launch and block scheduling so overlap this
// kernel's run instead of following its last block -- in a decode step of
// ~1,000 dependent launches that latency is a visible share.  A kernel
// launched without the attribute (torch's, say) is ordered as usual.
#ifndef LNSB_PDL
#define LNSB_PDL 1
#endif
__device__ __forceinline__ void pdl_entry() {
#if LNSB_PDL
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;\n" :::);
#endif
}
template <typename... KArgs, typename... Args>
void launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args &&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = LNSB_PDL;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    (void) cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);   // an error stays in cudaGetLastError
}

bool valid_fmt(int fmt) { return fmt == LNSB_XLNS16 || fmt == LNSB_XLNS32; }

unsigned grid_for(int64_t n, int block) {
    int64_t b = (n + block - 1) / block;
    if (b < 1) b = 1;
    if (b > 148 * 64) b = 148 * 64;     // grid-stride beyond 64 blocks per SM
    return (unsigned) b;
}

// ============================ conversions ==================================

template <int FMT>
__global__ void k_to_lns(dev_tables T, const float * __restrict__ src, void * __restrict__ dst, int64_t n) {
    pdl_entry();
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t) blockDim.x * gridDim.x) {
        if constexpr (FMT == 16) static_cast<uint16_t *>(dst)[i] = (uint16_t) from_f32_16(T, src[i]);
        else                     static_cast<uint32_t *>(dst)[i] = from_f32_32(T, src[i]);
    }
}

// dst[c * dst_ld + r] = lns(src[r * cols + c]), through a 32x32 shared tile so
// both the F32 reads and the LNS writes are coalesced
template <int FMT>
__global__ void k_to_lns_transposed(dev_tables T, const float * __restrict__ src, void * __restrict__ dst,
                                    int64_t rows, int64_t cols, int64_t dst_ld) {
    pdl_entry();
    using V = typename std::conditional<FMT == 16, uint16_t, uint32_t>::type;
    __shared__ V tile[32][33];
    const int64_t r0 = (int64_t) blockIdx.y * 32, c0 = (int64_t) blockIdx.x * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int64_t r = r0 + i, c = c0 + threadIdx.x;
        if (r < rows && c < cols) {
            const float f = src[r * cols + c];
            tile[i][threadIdx.x] = FMT == 16 ? (V) from_f32_16(T, f) : (V) from_f32_32(T, f);
        }
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int64_t c = c0 + i, r = r0 + threadIdx.x;
        if (r < rows && c < cols) static_cast<V *>(dst)[c * dst_ld + r] = tile[threadIdx.x][i];
    }
}

// ===================== weights in ggml storage types =======================
// ggml's block layouts (the formats ggml writes in GGUF files), decoded one
// value at a time: every value of a row is a function of its block's header
// and its own quant bits, so a thread computes value (r, c) directly and the
// transposing conversion keeps its coalesced tile structure.  Float steps are
// plain IEEE multiplies and subtractions (no contraction), in the order of
// ggml's reference dequantisers:
//   F16, BF16        the value widened
//   Q8_0  (34 B/32)  d (f16), 32 x int8 q:  d * q
//   Q4_0  (18 B/32)  d (f16), 16 bytes: value j < 16 low nibbles, j >= 16 high:
//                    d * (nibble - 8)
//   Q4_K  (144 B/256) d, dmin (f16), 12 bytes of 6-bit scales/mins for 8
//                    sub-blocks of 32, 128 bytes of nibbles (64 values per 32
//                    bytes: low nibbles then high): (d * sc) * q - (dmin * m)
//   Q6_K  (210 B/256) 128 bytes low 4 bits, 64 bytes high 2 bits, 16 int8
//                    scales, d (f16): (d * sc) * (q - 32)
__device__ __forceinline__ float f16_at(const unsigned char * p) {
    return __half2float(__ushort_as_half((unsigned short) (p[0] | (p[1] << 8))));
}
__device__ __forceinline__ void q4k_scale_min(int j, const unsigned char * q, int & sc, int & m) {
    if (j < 4) {
        sc = q[j] & 63;
        m  = q[j + 4] & 63;
    } else {
        sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        m  = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}
template <int TYPE>
__device__ __forceinline__ float dequant_at_t(const unsigned char * __restrict__ row, int64_t c);
__device__ __forceinline__ float dequant_at(int type, const unsigned char * __restrict__ row, int64_t c) {
    switch (type) {
        case LNSB_TYPE_F32:  return reinterpret_cast<const float *>(row)[c];
        case LNSB_TYPE_F16:  return f16_at(row + 2 * c);
        case LNSB_TYPE_BF16: return __uint_as_float((uint32_t) (row[2 * c] | (row[2 * c + 1] << 8)) << 16);
        case LNSB_TYPE_Q8_0: {
            const unsigned char * b = row + (c / 32) * 34;
            return __fmul_rn((float) (int8_t) b[2 + c % 32], f16_at(b));
        }
        case LNSB_TYPE_Q4_0: {
            const unsigned char * b = row + (c / 32) * 18;
            const int j = (int) (c % 32);
            const int byte = b[2 + (j & 15)];
            return __fmul_rn((float) ((j < 16 ? byte & 0xF : byte >> 4) - 8), f16_at(b));
        }
        case LNSB_TYPE_Q4_K: {
            const unsigned char * b = row + (c / 256) * 144;
            const int j = (int) (c % 256), chunk = j / 64, w = j % 64, sub = 2 * chunk + (w >= 32);
            const int q = b[16 + chunk * 32 + (w % 32)];
            int sc, m;
            q4k_scale_min(sub, b + 4, sc, m);
            const float d1 = __fmul_rn(f16_at(b), (float) sc), m1 = __fmul_rn(f16_at(b + 2), (float) m);
            return __fsub_rn(__fmul_rn(d1, (float) (w < 32 ? q & 0xF : q >> 4)), m1);
        }
        case LNSB_TYPE_Q6_K: {
            const unsigned char * b = row + (c / 256) * 210;
            const int j = (int) (c % 256), n = j / 128, quarter = (j % 128) / 32, l = j % 32;
            const unsigned char * ql = b + n * 64;
            const unsigned char * qh = b + 128 + n * 32;
            const int8_t * sc = reinterpret_cast<const int8_t *>(b + 192) + n * 8;
            const int lo = quarter & 1 ? ql[l + 32] : ql[l];
            const int q  = ((quarter < 2 ? lo & 0xF : lo >> 4) | (((qh[l] >> (2 * quarter)) & 3) << 4)) - 32;
            return __fmul_rn(__fmul_rn(f16_at(b + 208), (float) sc[l / 16 + 2 * quarter]), (float) q);
        }
        default: return 0.0f;
    }
}
template <int TYPE>
__device__ __forceinline__ float dequant_at_t(const unsigned char * __restrict__ row, int64_t c) {
    if constexpr (TYPE == LNSB_TYPE_F32) {
        return reinterpret_cast<const float *>(row)[c];
    } else if constexpr (TYPE == LNSB_TYPE_F16) {
        return __half2float(reinterpret_cast<const __half *>(row)[c]);          // rows are 2-byte aligned
    } else if constexpr (TYPE == LNSB_TYPE_BF16) {
        return __uint_as_float((uint32_t) reinterpret_cast<const uint16_t *>(row)[c] << 16);
    } else {
        return dequant_at(TYPE, row, c);
    }
}

// dst[c * dst_ld + r] = lns(dequant(row r)[c]); rows `row_bytes` apart
template <int FMT, int TYPE>
__global__ void k_to_lns_transposed_typed(dev_tables T, int type, const unsigned char * __restrict__ src,
                                          int64_t row_bytes, void * __restrict__ dst, int64_t rows, int64_t cols,
                                          int64_t dst_ld) {
    pdl_entry();
    using V = typename std::conditional<FMT == 16, uint16_t, uint32_t>::type;
    __shared__ V tile[32][33];
    // persistent over the 32 x 32 tiles (a grid of a few per SM, not one CTA per tile)
    const int64_t tc = (cols + 31) / 32, ntiles = tc * ((rows + 31) / 32);
    for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
        const int64_t r0 = (t / tc) * 32, c0 = (t % tc) * 32;
        for (int i = threadIdx.y; i < 32; i += blockDim.y) {
            const int64_t r = r0 + i, c = c0 + threadIdx.x;
            if (r < rows && c < cols) {
                const float f = dequant_at_t<TYPE>(src + r * row_bytes, c);
                tile[i][threadIdx.x] = FMT == 16 ? (V) from_f32_16(T, f) : (V) from_f32_32(T, f);
            }
        }
        __syncthreads();
        for (int i = threadIdx.y; i < 32; i += blockDim.y) {
            const int64_t c = c0 + i, r = r0 + threadIdx.x;
            if (r < rows && c < cols) static_cast<V *>(dst)[c * dst_ld + r] = tile[threadIdx.x][i];
        }
        __syncthreads();                                 // the tile is reused
    }
}

__global__ void k_dequantize(int type, const unsigned char * __restrict__ src, int64_t row_bytes, float * __restrict__ dst,
                             int64_t rows, int64_t cols) {
    pdl_entry();
    const int64_t n = rows * cols;
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t) blockDim.x * gridDim.x) {
        const int64_t r = i / cols, c = i - r * cols;
        dst[i] = dequant_at(type, src + r * row_bytes, c);
    }
}

template <int FMT>
__global__ void k_to_f32(dev_tables T, const void * __restrict__ src, float * __restrict__ dst, int64_t n) {
    pdl_entry();
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t) blockDim.x * gridDim.x) {
        if constexpr (FMT == 16) dst[i] = to_f32_16(T, static_cast<const uint16_t *>(src)[i]);
        else                     dst[i] = to_f32_32(T, static_cast<const uint32_t *>(src)[i]);
    }
}

// ============================ MUL_MAT (xlns16) =============================
//
// Three kernels cover the xlns16 modes: base and Monte run on packed keys
// (k_mul_mat16_fast, k_mul_mat16_lat), sum32 / lpvip / Monte-by-LPVIP on the
// 32-bit accumulator kernel k_mul_mat_a32 further down.
constexpr int MM_TABPAD  = (k16_tab_bytes + 15) / 16 * 16;       // the packed table, 16-byte padded

__device__ __forceinline__ void cp_async16(void * smem, const void * gmem) {
    const unsigned s = (unsigned) __cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
// zero-fills the 16 bytes beyond src_bytes (0 or 16 here)
__device__ __forceinline__ void cp_async16_zfill(void * smem, const void * gmem, int src_bytes) {
    const unsigned s = (unsigned) __cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
// `bytes` (a multiple of 16; both addresses 16-byte aligned) from global to
// shared memory by the whole block, every piece in flight at once; the caller
// commits, waits and synchronises
__device__ __forceinline__ void stage_async(void * smem, const void * gmem, int bytes);
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }
__device__ __forceinline__ void stage_async(void * smem, const void * gmem, int bytes) {
    for (int i = threadIdx.x; i < bytes / 16; i += blockDim.x)
        cp_async16(static_cast<unsigned char *>(smem) + 16 * i, static_cast<const unsigned char *>(gmem) + 16 * i);
}

// ---- the xlns16 image of a typed weight at HBM speed ----------------------
//
// float -> xlns16 without the 256 KB table: for a normal float (biased
// exponent e in 1..254, top 8 mantissa bits m) the table entry is
//     clamp(128 (e - 127) + G[m] + 0x4000, 0, 0x7FFF) | sign,
// G[m] = 128 log2(1 + m/256) truncated toward zero: floored for |x| >= 1,
// rounded up below.  G is read off the table itself (entries at e = 127 and
// e = 126) and the split is checked against every entry on the host before
// this path is used (conv16_splits); subnormals, infinities and NaNs keep the
// table lookup.  A CTA keeps G in shared memory, one copy per bank (word
// m * 32 + lane holds G for |x| >= 1 in byte 0, for |x| < 1 in byte 1), so a
// warp's lookups never conflict.  A value's index u is its float's bits >> 15
// (17 bits: sign, exponent, top 8 mantissa bits).
constexpr int TW_ROWS = 64, TW_THREADS = 1024, TW_STAGES = 4;
constexpr int TW_OP = TW_ROWS + 2;                       // codes per column of the transposed tile (33 words)
constexpr int TW_GTAB = 256 * 32 * 4;

template <int TYPE> struct tw_geom {
    static constexpr int cols  = TYPE == LNSB_TYPE_F32 ? 128 : 256;     // a tile's columns: whole blocks
    static constexpr int blk   = (TYPE == LNSB_TYPE_Q4_K || TYPE == LNSB_TYPE_Q6_K) ? 256
                               : (TYPE == LNSB_TYPE_Q8_0 || TYPE == LNSB_TYPE_Q4_0) ? 32 : 1;
    static constexpr int bb    = TYPE == LNSB_TYPE_F32 ? 4 : TYPE == LNSB_TYPE_Q8_0 ? 34 : TYPE == LNSB_TYPE_Q4_0 ? 18
                               : TYPE == LNSB_TYPE_Q4_K ? 144 : TYPE == LNSB_TYPE_Q6_K ? 210 : 2;
    static constexpr int seg   = cols / blk * bb;                           // raw bytes of a tile row
    static constexpr int rawp  = (seg + 15 + 15) / 16 * 16;                 // staged row pitch (16-byte window slack)
    static constexpr int stage = TW_ROWS * rawp;
    static constexpr int smem  = TW_GTAB + TW_STAGES * stage + cols * TW_OP * 2;
};

// a normal float's index u = bits >> 15 -> xlns16 through the shared copies of G
__device__ __forceinline__ uint32_t conv16_fast(const uint32_t * __restrict__ glane, uint32_t u) {
    const uint32_t g = __byte_perm(glane[(u & 0xFFu) << 5], 0u, (u & 0xFFFFu) < (127u << 8) ? 0x4441u : 0x4440u);
    return ((u >> 1) & 0x8000u) | min(((u & 0xFF00u) >> 1) + g + 128u, 0x7FFFu);   // 128 (e - 127) + 0x4000 = 128 e + 128
}
__device__ __forceinline__ bool conv16_normal(uint32_t u) { return (u & 0xFF00u) - 0x100u < 0xFE00u; }
__device__ __forceinline__ uint32_t conv16_split(const dev_tables & T, const uint32_t * __restrict__ glane, uint32_t u) {
    return conv16_normal(u) ? conv16_fast(glane, u) : (uint32_t) __ldg(T.conv16 + u);
}

// the upper 17 bits of value c's float (the conversion table's index)
template <int TYPE>
__device__ __forceinline__ uint32_t f32_hi_at(const unsigned char * row, int c) {
    if constexpr (TYPE == LNSB_TYPE_BF16) {
        return (uint32_t) reinterpret_cast<const uint16_t *>(row)[c] << 1;
    } else if constexpr (TYPE == LNSB_TYPE_F16) {
        return __float_as_uint(__half2float(reinterpret_cast<const __half *>(row)[c])) >> 15;   // exact widening
    } else {
        return __float_as_uint(dequant_at_t<TYPE>(row, c)) >> 15;
    }
}

// dst[c * dst_ld + r] = xlns16(dequant(row r)[c]), rows `row_bytes` apart.
// One CTA per SM walks tiles of 64 rows x tw_geom::cols columns through a
// ring of TW_STAGES staging buffers: each tile's raw row segments are copied
// with 16-byte cp.async (vec_in: src and row_bytes 16-byte aligned; the
// window is rounded out to 16 bytes, never past the row), so the next
// TW_STAGES - 1 tiles' copies are in flight while one tile is decoded and
// converted from shared memory into a transposed tile (33-word column pitch:
// conflict-free both ways) and stored, each column's 64 codes as 128
// contiguous bytes (vec_out: dst and dst_ld 16-byte aligned).
template <int TYPE>
__global__ void __launch_bounds__(TW_THREADS, 1)
k_to_lns16_typed_tiled(dev_tables T, const unsigned char * __restrict__ src, int64_t row_bytes,
                       uint16_t * __restrict__ dst, int64_t rows, int64_t cols, int64_t dst_ld, int vec_in, int vec_out) {
    using G = tw_geom<TYPE>;
    pdl_entry();
    extern __shared__ __align__(16) unsigned char smem[];
    uint32_t *      gtab = reinterpret_cast<uint32_t *>(smem);
    unsigned char * raw  = smem + TW_GTAB;
    uint16_t *      tile = reinterpret_cast<uint16_t *>(smem + TW_GTAB + TW_STAGES * G::stage);
    const int tid = threadIdx.x, lane = tid & 31;

    // G from the table's entries at e = 127 (|x| >= 1) and e = 126 (|x| < 1):
    // one load each by the first 128 threads, then one copy per bank
    uint32_t * g0 = reinterpret_cast<uint32_t *>(tile);
    if (tid < 256) {
        const uint32_t gp = (uint32_t) __ldg(T.conv16 + ((127 << 8) | tid)) - 0x4000u;
        const uint32_t gn = (uint32_t) __ldg(T.conv16 + ((126 << 8) | tid)) - 0x4000u + 128u;
        g0[tid] = gp | (gn << 8);
    }

    // tile t: row block t / nct, column block t % nct (the launcher keeps the tile count below 2^31)
    const uint32_t nct = (uint32_t) ((cols + G::cols - 1) / G::cols);
    const int64_t ntiles = (int64_t) nct * ((rows + TW_ROWS - 1) / TW_ROWS);
    // window of a tile's row segment: bytes [cb0, cb1) of each row
    auto window = [&](int64_t t, int64_t & r0, int64_t & c0, int64_t & a0, int & nch, int & off) {
        const uint32_t rt = (uint32_t) t / nct;
        r0 = (int64_t) rt * TW_ROWS;
        c0 = (int64_t) ((uint32_t) t - rt * nct) * G::cols;
        const int64_t cb0 = c0 / G::blk * G::bb, cb1 = imin64(cb0 + G::seg, row_bytes);
        if (vec_in) {
            a0 = cb0 & ~(int64_t) 15;
            nch = (int) ((((cb1 + 15) & ~(int64_t) 15) - a0) >> 4);
            off = (int) (cb0 - a0);
        } else {
            a0 = cb0;
            nch = (int) (cb1 - cb0);        // bytes
            off = 0;
        }
    };
    // stages tile t (when it exists) into ring slot `slot`; always closes a
    // cp.async group, so the groups in flight count tiles
    auto stage = [&](int64_t t, int slot) {
        if (t < ntiles) {
            int64_t r0, c0, a0; int nch, off;
            window(t, r0, c0, a0, nch, off);
            const int rv = (int) imin64(TW_ROWS, rows - r0);
            unsigned char * rs = raw + slot * G::stage;
            if (vec_in) {                                  // a warp per row
                for (int r = tid >> 5; r < rv; r += TW_THREADS / 32)
                    for (int q = lane; q < nch; q += 32)
                        cp_async16(rs + r * G::rawp + 16 * q, src + (r0 + r) * row_bytes + a0 + 16 * q);
            } else {
                for (int r = tid >> 5; r < rv; r += TW_THREADS / 32)
                    for (int q = lane; q < nch; q += 32) rs[r * G::rawp + q] = src[(r0 + r) * row_bytes + a0 + q];
            }
        }
        cp_async_commit();
    };

#pragma unroll
    for (int k = 0; k < TW_STAGES - 1; k++) stage((int64_t) blockIdx.x + (int64_t) k * gridDim.x, k);
    __syncthreads();                                       // g0 written
    uint32_t gw[256 * 32 / TW_THREADS];
#pragma unroll
    for (int j = 0; j < 256 * 32 / TW_THREADS; j++) gw[j] = g0[(tid + j * TW_THREADS) >> 5];
    __syncthreads();                                       // g0 read: the tile is free
#pragma unroll
    for (int j = 0; j < 256 * 32 / TW_THREADS; j++) gtab[tid + j * TW_THREADS] = gw[j];
    const uint32_t * glane = gtab + lane;

    int slot = 0;
    for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
        int64_t r0, c0, a0; int nch, off;
        window(t, r0, c0, a0, nch, off);
        const int rv = (int) imin64(TW_ROWS, rows - r0), cv = (int) imin64(G::cols, cols - c0);
        cp_async_wait<TW_STAGES - 2>();                    // this tile's group has landed
        __syncthreads();                                   // ... for every thread; the tile and the slot
                                                           // read last time are free again
        stage(t + (int64_t) (TW_STAGES - 1) * gridDim.x, slot == 0 ? TW_STAGES - 1 : slot - 1);
        const unsigned char * rs = raw + slot * G::stage + off;
        // a thread converts column c of row pairs p0, p0 + TW_PPS, ... and
        // writes each pair as one word of the transposed tile; a warp covers
        // 32 consecutive columns.  The branch-free path covers zeros and every
        // value whose float is normal (subnormal halves widen to normal
        // floats); a value outside it (infinity, NaN, a subnormal float) is
        // patched afterwards from the table.  Rows past the matrix hold stale
        // bytes: harmless, they are never stored.
        constexpr int TW_PPS = TW_THREADS / G::cols;       // row pairs per step
        constexpr int TW_NP  = TW_ROWS / 2 / TW_PPS;       // steps
        const int c = tid % G::cols, p0 = tid / G::cols;
        if (c < cv) {
            uint32_t bad = 0;                              // bit k: pair k holds a value outside the fast path
#pragma unroll 4
            for (int k = 0; k < TW_NP; k++) {
                const int r = 2 * (p0 + k * TW_PPS);
                const uint32_t u0 = f32_hi_at<TYPE>(rs + r * G::rawp, c), u1 = f32_hi_at<TYPE>(rs + (r + 1) * G::rawp, c);
                const bool ok = (conv16_normal(u0) || (u0 & 0xFFFFu) == 0) && (conv16_normal(u1) || (u1 & 0xFFFFu) == 0);
                bad |= ok ? 0u : 1u << k;
                const uint32_t v0 = (u0 & 0xFFFFu) ? conv16_fast(glane, u0) : 0u;
                const uint32_t v1 = (u1 & 0xFFFFu) ? conv16_fast(glane, u1) : 0u;
                *reinterpret_cast<uint32_t *>(tile + c * TW_OP + r) = v0 | (v1 << 16);
            }
            while (bad) {
                const int k = __ffs(bad) - 1;
                bad &= bad - 1;
                const int r = 2 * (p0 + k * TW_PPS);
                const uint32_t v0 = conv16_split(T, glane, f32_hi_at<TYPE>(rs + r * G::rawp, c));
                const uint32_t v1 = conv16_split(T, glane, f32_hi_at<TYPE>(rs + (r + 1) * G::rawp, c));
                *reinterpret_cast<uint32_t *>(tile + c * TW_OP + r) = v0 | (v1 << 16);
            }
        }
        __syncthreads();                                   // the tile complete
        slot = slot == TW_STAGES - 1 ? 0 : slot + 1;
        if (vec_out && rv == TW_ROWS) {
            for (int i = tid; i < cv * 8; i += TW_THREADS) {
                const int c = i >> 3, j = i & 7;
                const uint32_t * w = reinterpret_cast<const uint32_t *>(tile) + c * (TW_OP / 2) + 4 * j;
                *reinterpret_cast<uint4 *>(dst + (c0 + c) * dst_ld + r0 + 8 * j) = make_uint4(w[0], w[1], w[2], w[3]);
            }
        } else {
            for (int i = tid; i < cv * TW_ROWS; i += TW_THREADS) {
                const int c = i / TW_ROWS, r = i % TW_ROWS;
                if (r < rv) dst[(c0 + c) * dst_ld + r0 + r] = tile[c * TW_OP + r];
            }
        }
    }
    cp_async_wait<0>();
}

// ===================== MUL_MAT (xlns16, base mode, key form) ================
//
// The base-mode (and Monte) tiled kernels.  Every chain carries its accumulator as a key
// (lnsb_tables.h): key = 16 * log + 4 * sign.  One LNS addition of a
// product p is then
//     d   = |a - p|                 one signed difference gives n and the sign case
//     adj = T[min(d, KEYMAX)]       sb or db (or the cancellation sentinel), * 16
//     a   = max(max(a, p) + adj, 0) max() picks the larger magnitude (a tie of
//                                   equal signs is harmless); for x + (-x) the
//                                   sentinel drives the sum below 0 and the clamp
//                                   gives key 0 = +0, as xlns16_add does
// and the product key is wkey + xkey with one mask fixing the sign flag, so an
// addition costs 8 integer instructions instead of ~30 on packed codes.
// This form drops the saturation of the product and of the sum, so it is
// used for a K chunk only when that chunk's operands prove neither can
// happen: every product >= 2^-120 (log >= 964, beyond the largest db step, so
// no sum underflows either) and every product small enough that K additions
// cannot reach 2^127.  Otherwise the chain continues on packed codes with the
// full xlns16 semantics -- the bits are the same either way.
//
// Tile: 64 weight rows x 32 tokens, 128 threads, 4 x 4 chains per thread;
// K chunks of 32 staged with cp.async (double buffered) and converted to key
// form once per chunk in shared memory; the 20 KB key table replicas sit from
// shared offset 0, so a byte index needs no address arithmetic beyond the
// replica offset folded into its clamp.  k_mul_mat16_fast runs one tile body
// per CTA with two replicas (the Monte build); k_mul_mat16_fast4 runs four
// tile bodies per CTA, one CTA per SM, over four replicas (the base build,
// the peer-store gather included).
constexpr int FB_BM = 64, FB_BN = 32, FB_KC = 32, FB_TM = 4, FB_TN = 4;
constexpr int FB_THREADS = (FB_BM / FB_TM) * (FB_BN / FB_TN);      // 128
constexpr int FB_XP  = FB_KC + 8;                                  // x code pitch, halfwords
constexpr int FB_XKP = FB_KC + 4;                                  // x key pitch, words
constexpr int FB_WCODES = FB_KC * FB_BM;                           // halfwords
constexpr int FB_XCODES = FB_BN * FB_XP;                           // halfwords
// Monte (GGML_LNS16_SUM=monte) runs the same kernel over the fine tables in
// key form (k16m_key_max): adj = 16 * floor((fine + low byte of the chain's
// next LFSR state) / 256), one LFSR step per addition and chain.  A dithered
// step exceeds the exact sum by at most one ulp and falls short by at most one,
// so the chunk range check below holds for it unchanged.
constexpr bool FB_MONTE   = k_mode == M_MONTE;
constexpr int  FB_KEYB    = FB_MONTE ? k16m_key_bytes : k16_key_bytes;
constexpr int  FB_KEYMAX  = FB_MONTE ? k16m_key_max : k16_key_max;
constexpr int FB_REPL     = FB_KEYB + 36;                         // replica stride: word offset = 1 mod 4
constexpr int FB_OFF_WKEY = (2 * FB_REPL + 15) / 16 * 16;
constexpr int FB_OFF_XKEY = FB_OFF_WKEY + FB_KC * FB_BM * 4;
constexpr int FB_OFF_RED  = FB_OFF_XKEY + FB_BN * FB_XKP * 4;
constexpr int FB_OFF_CODE = FB_OFF_RED + 128;
constexpr int FB_SMEM     = FB_OFF_CODE + 2 * (FB_WCODES + FB_XCODES) * 2;

template <int BN>
__device__ __forceinline__ void fb_stage(uint16_t * wc, uint16_t * xc, const uint16_t * __restrict__ W,
                                         const uint16_t * __restrict__ X, int64_t K, int64_t M, int64_t N,
                                         int64_t m0, int64_t n0, int64_t k0, bool vec, int tid) {
    if (vec) {
#pragma unroll
        for (int it = 0; it < 2; it++) {           // weights: 32 k-rows x 128 B = 256 x 16 B
            const int c = tid + it * FB_THREADS;
            const int r = c >> 3, q = c & 7;
            if (k0 + r < K) cp_async16(wc + r * FB_BM + q * 8, W + (k0 + r) * M + m0 + q * 8);
        }
        {                                          // tokens: BN rows x 64 B (at most 128 x 16 B)
            const int r = tid >> 2, q = tid & 3;
            if (r < BN && n0 + r < N && k0 + q * 8 < K) cp_async16(xc + r * FB_XP + q * 8, X + (n0 + r) * K + k0 + q * 8);
        }
    } else {
        for (int i = tid; i < FB_WCODES; i += FB_THREADS) {
            const int r = i / FB_BM, c = i % FB_BM;
            const int64_t k = k0 + r, m = m0 + c;
            wc[r * FB_BM + c] = (k < K && m < M) ? W[k * M + m] : (uint16_t) 0x4000;
        }
        for (int i = tid; i < BN * FB_KC; i += FB_THREADS) {
            const int r = i / FB_KC, c = i % FB_KC;
            const int64_t n = n0 + r, k = k0 + c;
            xc[r * FB_XP + c] = (n < N && k < K) ? X[n * K + k] : (uint16_t) 0x4000;
        }
    }
}

// one addition in key form (see above); rbase: byte offset of this thread's
// table replica, folded into the clamp; st: the chain's LFSR state (Monte)
__device__ __forceinline__ int key_step(int a, int p, const unsigned char * tab, int rbase, uint32_t & st) {
    const int d   = __viaddmin_s32(abs(a - p), rbase, FB_KEYMAX + rbase);
    int adj = *reinterpret_cast<const int *>(tab + d);
    if constexpr (FB_MONTE) {
        st  = lfsr_step(st);
        adj = ((adj + (int) (st & 0xFFu)) >> 4) & ~15;
    }
    return __viaddmax_s32(max(a, p), adj, 0);
}
// Largest growth of a sum's log (units of 2^-7 octave) over n additions whose
// terms are no larger than max(|sum|, |term|): each xlns16 addition returns the
// exact sum times at most 2^(1/128), so |sum_n| <= 2^(n/128) (n+1) max, i.e.
// growth <= 128 ceil(log2(n+1)) + n.  One more 128 covers the last addition.
__host__ __device__ constexpr int growth_bound(int n) {
    int lg = 0;
    while ((1 << lg) < n + 1) lg++;
    return 128 * lg + n + 128;
}

__device__ __forceinline__ int key_of_code_w(uint32_t c) {      // weight operand: 16 * log + 4 * sign
    return (int) (((c << 4) & 0x7FFF0u) | ((c >> 13) & 4u));
}
__device__ __forceinline__ int key_of_code_x(uint32_t c) {      // activation operand carries the -0x4000 bias
    return (int) (((c << 4) & 0x7FFF0u) | ((c >> 13) & 4u)) - 16 * 0x4000;
}
// sign flags add to 4 * (ws + xs); bit 3 is set only for two negatives
__device__ __forceinline__ int key_of_product(int wkey, int xkey) { return (wkey + xkey) & ~8; }
__device__ __forceinline__ uint32_t code_of_key(int key) {
    return ((uint32_t) (key >> 4) & 0x7FFFu) | (((uint32_t) key & 4u) << 13);
}
__device__ __forceinline__ int key_of_code(uint32_t c) { return key_of_code_w(c); }

// the all-gather of output-row shards fused into the store: every code goes
// to each peer's buffer (peer memory over NVLink, plain stores) at
// [z][n][off + m] with rows of ld codes; n == 0: the local dst as usual
struct peer_out_dev {
    uint16_t * const * ptrs;     // device array of n buffer pointers
    int                n;
    int64_t            ld, off;
};

// A group of FB_THREADS threads synchronises on its own named barrier when
// several groups share a CTA (bar: 1 + group), on the CTA barrier otherwise.
template <int NG>
__device__ __forceinline__ void fb_sync(int bar) {
    if constexpr (NG == 1) __syncthreads();
    else asm volatile("bar.sync %0, %1;\n" ::"r"(bar), "n"(FB_THREADS) : "memory");
}

// One tile: 64 weight rows x 8 * TN tokens from (m0, n0) of slice z, run by
// one group of FB_THREADS threads (tid: the thread's index in the group); a
// thread runs 4 rows x TN tokens (tokens tn, tn + 8, ...).  tab: the key
// table replicas, rbase: the byte offset of this thread's replica; gsm: the
// group's operand buffers (the layout from FB_OFF_WKEY on).
template <bool OUT_F32, int TN, int NG>
__device__ __forceinline__ void fb_tile(const dev_tables & T, const unsigned char * tab, unsigned char * gsm, int tid,
                                        int rbase, int bar, const uint16_t * __restrict__ W,
                                        const uint16_t * __restrict__ X, void * __restrict__ dst, int64_t K, int64_t M,
                                        int64_t N, int64_t ne02, int64_t ne12, int64_t r2, int64_t r3,
                                        uint32_t monte_seed, int vec, const peer_out_dev & peers, int64_t z,
                                        int64_t m0, int64_t n0) {
    constexpr int BN = 8 * TN;                          // tokens of the tile
    int *      wkeys = reinterpret_cast<int *>(gsm);
    int *      xkeys = reinterpret_cast<int *>(gsm + (FB_OFF_XKEY - FB_OFF_WKEY));
    int *      red   = reinterpret_cast<int *>(gsm + (FB_OFF_RED - FB_OFF_WKEY));
    uint16_t * codes = reinterpret_cast<uint16_t *>(gsm + (FB_OFF_CODE - FB_OFF_WKEY));


    const int64_t i12 = z % ne12, i13 = z / ne12;
    const uint16_t * Wz = W + ((i13 / r3) * ne02 + i12 / r2) * K * M;
    const uint16_t * Xz = X + z * N * K;
    const int tm = tid % (FB_BM / FB_TM), tn = tid / (FB_BM / FB_TM);
    const int mloc = tm * FB_TM;                        // rows mloc .. mloc+3
    const int warp = tid >> 5;
    // tokens tn, tn + 8, tn + 16, tn + 24

    int      akey[FB_TM][TN];
    uint32_t acc[FB_TM][TN];
    uint32_t st[FB_TM][TN];                          // Monte: each chain's LFSR state
    bool fast = true;                                   // uniform across the block
    const int nchunks = (int) ((K + FB_KC - 1) / FB_KC);
    const int64_t nvalid = imin64(BN, N - n0);
    red16 R{ &T, T.sbdb16, T.monte16 };                 // slow path reads the packed tables from L1/L2
#pragma unroll
    for (int i = 0; i < FB_TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++) {
            st[i][j] = 0;
            if constexpr (FB_MONTE) {
                // the chain of output (z, m, n) starts (its index in the CPU's loop
                // order z, m, n) * (K - 1) draws after the seed
                const int64_t m = imin64(m0 + mloc + i, M - 1), n = imin64(n0 + tn + 8 * j, N - 1);
                const unsigned long long out = ((unsigned long long) z * (unsigned long long) M + (unsigned long long) m) *
                                               (unsigned long long) N + (unsigned long long) n;
                if (K > 1) st[i][j] = lfsr_jump(T, monte_seed, out * (unsigned long long) (K - 1));
            }
        }

    if (nchunks > 0) {
        fb_stage<BN>(codes, codes + FB_WCODES, Wz, Xz, K, M, N, m0, n0, 0, vec != 0, tid);
        cp_async_commit();
    }
    for (int c = 0; c < nchunks; c++) {
        uint16_t * wc = codes + (c & 1) * (FB_WCODES + FB_XCODES);
        uint16_t * xc = wc + FB_WCODES;
        if (c + 1 < nchunks) {
            uint16_t * wn = codes + ((c + 1) & 1) * (FB_WCODES + FB_XCODES);
            fb_stage<BN>(wn, wn + FB_WCODES, Wz, Xz, K, M, N, m0, n0, (int64_t) (c + 1) * FB_KC, vec != 0, tid);
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        fb_sync<NG>(bar);
        const int kvalid = (int) imin64(FB_KC, K - (int64_t) c * FB_KC);
        if (fast) {
            // convert this chunk to key form; operand log ranges for the range check
            int wmin = 0x7FFF, wmax = 0, xmin = 0x7FFF, xmax = 0;
            for (int i = tid; i < FB_KC * FB_BM; i += FB_THREADS) {
                const int r = i / FB_BM;
                const uint32_t cw = wc[i];
                wkeys[i] = key_of_code_w(cw);
                if (r < kvalid) { const int l = (int) (cw & 0x7FFFu); wmin = min(wmin, l); wmax = max(wmax, l); }
            }
            for (int i = tid; i < BN * FB_KC; i += FB_THREADS) {
                const int r = i / FB_KC, col = i % FB_KC;
                const uint32_t cx = xc[r * FB_XP + col];
                xkeys[r * FB_XKP + col] = key_of_code_x(cx);
                if (r < nvalid && col < kvalid) { const int l = (int) (cx & 0x7FFFu); xmin = min(xmin, l); xmax = max(xmax, l); }
            }
            // the largest accumulator log entering this chunk
            int amax = 0;
            if (c > 0) {
#pragma unroll
                for (int i = 0; i < FB_TM; i++)
#pragma unroll
                    for (int j = 0; j < TN; j++) amax = max(amax, akey[i][j] >> 4);
            }
            wmin = __reduce_min_sync(0xFFFFFFFFu, wmin);
            wmax = __reduce_max_sync(0xFFFFFFFFu, wmax);
            xmin = __reduce_min_sync(0xFFFFFFFFu, xmin);
            xmax = __reduce_max_sync(0xFFFFFFFFu, xmax);
            amax = __reduce_max_sync(0xFFFFFFFFu, amax);
            if ((tid & 31) == 0) {
                red[warp * 8 + 0] = wmin; red[warp * 8 + 1] = wmax; red[warp * 8 + 2] = xmin; red[warp * 8 + 3] = xmax;
                red[warp * 8 + 4] = amax;
            }
            fb_sync<NG>(bar);
            int a0 = 0x7FFF, a1 = 0, b0 = 0x7FFF, b1 = 0, am = 0;
#pragma unroll
            for (int w = 0; w < FB_THREADS / 32; w++) {
                a0 = min(a0, red[w * 8 + 0]); a1 = max(a1, red[w * 8 + 1]);
                b0 = min(b0, red[w * 8 + 2]); b1 = max(b1, red[w * 8 + 3]);
                am = max(am, red[w * 8 + 4]);
            }
            // exact in key form: every product >= 2^-120 (no sum can underflow)
            // and no sum can reach 2^127 within this chunk (growth_bound)
            const bool ok = a0 + b0 - 0x4000 >= 964 && max(am, a1 + b1 - 0x4000) + growth_bound(FB_KC) <= 0x7FFF;
            if (!ok) {
                fast = false;
                if (c > 0) {
#pragma unroll
                    for (int i = 0; i < FB_TM; i++)
#pragma unroll
                        for (int j = 0; j < TN; j++) acc[i][j] = code_of_key(akey[i][j]);
                }
            }
        }
        int k = 0;
        if (fast) {
            if (c == 0) {
                const int4 w4 = *reinterpret_cast<const int4 *>(wkeys + mloc);
                const int wv[4] = { w4.x, w4.y, w4.z, w4.w };
#pragma unroll
                for (int i = 0; i < FB_TM; i++)
#pragma unroll
                    for (int j = 0; j < TN; j++) akey[i][j] = key_of_product(wv[i], xkeys[(tn + 8 * j) * FB_XKP]);
                k = 1;
                for (; k < 4 && k < kvalid; k++) {
                    const int4 wk = *reinterpret_cast<const int4 *>(wkeys + k * FB_BM + mloc);
                    const int w2[4] = { wk.x, wk.y, wk.z, wk.w };
#pragma unroll
                    for (int i = 0; i < FB_TM; i++)
#pragma unroll
                        for (int j = 0; j < TN; j++)
                            akey[i][j] = key_step(akey[i][j], key_of_product(w2[i], xkeys[(tn + 8 * j) * FB_XKP + k]), tab, rbase, st[i][j]);
                }
            }
            for (; k + 4 <= kvalid; k += 4) {
                int4 xv[TN];
#pragma unroll
                for (int j = 0; j < TN; j++) xv[j] = *reinterpret_cast<const int4 *>(xkeys + (tn + 8 * j) * FB_XKP + k);
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int4 wk = *reinterpret_cast<const int4 *>(wkeys + (k + u) * FB_BM + mloc);
                    const int w2[4] = { wk.x, wk.y, wk.z, wk.w };
#pragma unroll
                    for (int i = 0; i < FB_TM; i++)
#pragma unroll
                        for (int j = 0; j < TN; j++) {
                            const int xk = u == 0 ? xv[j].x : u == 1 ? xv[j].y : u == 2 ? xv[j].z : xv[j].w;
                            akey[i][j] = key_step(akey[i][j], key_of_product(w2[i], xk), tab, rbase, st[i][j]);
                        }
                }
            }
            for (; k < kvalid; k++) {
                const int4 wk = *reinterpret_cast<const int4 *>(wkeys + k * FB_BM + mloc);
                const int w2[4] = { wk.x, wk.y, wk.z, wk.w };
#pragma unroll
                for (int i = 0; i < FB_TM; i++)
#pragma unroll
                    for (int j = 0; j < TN; j++)
                        akey[i][j] = key_step(akey[i][j], key_of_product(w2[i], xkeys[(tn + 8 * j) * FB_XKP + k]), tab, rbase, st[i][j]);
            }
        } else {
            // packed codes, full xlns16 semantics
            if (c == 0) {
#pragma unroll
                for (int i = 0; i < FB_TM; i++)
#pragma unroll
                    for (int j = 0; j < TN; j++) acc[i][j] = mul16(wc[mloc + i], xc[(tn + 8 * j) * FB_XP]);
                k = 1;
            }
            for (; k < kvalid; k++) {
#pragma unroll
                for (int i = 0; i < FB_TM; i++) {
                    const uint32_t w = wc[k * FB_BM + mloc + i];
#pragma unroll
                    for (int j = 0; j < TN; j++) acc[i][j] = R.add(acc[i][j], mul16(w, xc[(tn + 8 * j) * FB_XP + k]), st[i][j]);
                }
            }
        }
        fb_sync<NG>(bar);
    }

    if (!OUT_F32 && peers.n > 0) {
        // 4 consecutive rows per thread and token: one 8-byte store per peer
        // (16 threads cover a token's 64 rows: 128 contiguous bytes)
#pragma unroll
        for (int j = 0; j < TN; j++) {
            const int64_t n = n0 + tn + 8 * j;
            if (n >= N) continue;
            uint32_t v[FB_TM];
#pragma unroll
            for (int i = 0; i < FB_TM; i++) v[i] = K == 0 ? 0u : (fast ? code_of_key(akey[i][j]) : acc[i][j]);
            const int64_t o = (z * N + n) * peers.ld + peers.off + m0 + mloc;
            const bool whole = m0 + mloc + FB_TM <= M && (o & 3) == 0;
            for (int p = 0; p < peers.n; p++) {
                uint16_t * d = peers.ptrs[p];
                if (whole) {
                    *reinterpret_cast<uint2 *>(d + o) = make_uint2(v[0] | (v[1] << 16), v[2] | (v[3] << 16));
                } else {
#pragma unroll
                    for (int i = 0; i < FB_TM; i++)
                        if (m0 + mloc + i < M) d[o + i] = (uint16_t) v[i];
                }
            }
        }
        return;
    }
#pragma unroll
    for (int i = 0; i < FB_TM; i++) {
        const int64_t m = m0 + mloc + i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < TN; j++) {
            const int64_t n = n0 + tn + 8 * j;
            if (n >= N) continue;
            const uint32_t v = K == 0 ? 0u : (fast ? code_of_key(akey[i][j]) : acc[i][j]);
            const int64_t o = (z * N + n) * M + m;
            if constexpr (OUT_F32) static_cast<float *>(dst)[o] = to_f32_16(T, v);
            else                   static_cast<uint16_t *>(dst)[o] = (uint16_t) v;
        }
    }
}

// Blocks [0, nfull) run whole 64 x 32 tiles (tile b at (b % gx, b / gx));
// the blocks after them run the remaining tiles in quarters of 8 tokens (one
// token per thread).  The launcher makes nfull a multiple of the SM count, so
// whole tiles fill whole waves and the last, partial wave is dealt out in
// quarter-size pieces that even out the work per SM.
template <bool OUT_F32>
__global__ void __launch_bounds__(FB_THREADS, FB_MONTE ? 2 : 4)
k_mul_mat16_fast(dev_tables T, const uint16_t * __restrict__ W, const uint16_t * __restrict__ X,
                 void * __restrict__ dst, int64_t K, int64_t M, int64_t N, int64_t ne02, int64_t ne12,
                 int64_t r2, int64_t r3, uint32_t monte_seed, int vec, peer_out_dev peers, int64_t gx, int64_t nfull) {
    pdl_entry();
    extern __shared__ __align__(16) unsigned char smem[];
    // two replicas of the key table, one per lane parity: same-sign lookups
    // of one replica fall in banks 4j, the other's in 4j + 1 (made visible by
    // the tile's first barrier)
    const int32_t * keytab = FB_MONTE ? T.mkey16 : T.key16;
    for (int i = threadIdx.x; i < FB_KEYB / 4; i += FB_THREADS) {
        const int v = keytab[i];
        reinterpret_cast<int *>(smem)[i] = v;
        reinterpret_cast<int *>(smem + FB_REPL)[i] = v;
    }
    const int rbase = (threadIdx.x & 1) * FB_REPL;
    unsigned char * gsm = smem + FB_OFF_WKEY;
    const int64_t b = blockIdx.x, z = blockIdx.z;
    if (b < nfull) {
        fb_tile<OUT_F32, FB_TN, 1>(T, smem, gsm, threadIdx.x, rbase, 0, W, X, dst, K, M, N, ne02, ne12, r2, r3,
                                   monte_seed, vec, peers, z, (b % gx) * FB_BM, (b / gx) * FB_BN);
    } else {
        const int64_t q = b - nfull, t = nfull + q / 4;
        const int64_t n0 = (t / gx) * FB_BN + (q % 4) * 8;
        if (n0 < N)
            fb_tile<OUT_F32, 1, 1>(T, smem, gsm, threadIdx.x, rbase, 0, W, X, dst, K, M, N, ne02, ne12, r2, r3,
                                   monte_seed, vec, peers, z, (t % gx) * FB_BM, n0);
    }
}

// One CTA per SM: FB4_GROUPS groups of FB_THREADS threads share
// four replicas of the key table, chosen by lane & 3.  Replica r starts r
// words past a multiple of 4 (0, 17, 2, 19 mod 32),
// so the same-sign entries (words 4n) of the four lane groups fall in four
// disjoint sets of 8 banks and a warp's 32 random lookups spread over all 32
// banks rather than crowding into half of them.  Items (whole tiles; from
// nfull on, quarter tiles as in k_mul_mat16_fast) are dealt to the CTAs
// round-robin and taken in turn by each CTA's groups.
constexpr int FB4_OFF_GROUP = (4 * FB_REPL + 15) / 16 * 16;
constexpr int FB_GROUP_BYTES = FB_SMEM - FB_OFF_WKEY;                 // one group's operand buffers
constexpr int FB4_GROUPS = FB_MONTE ? 2 : 4;                          // as many as fit beside the replicas
                                                                      // (the launcher uses it for base only)
constexpr int FB4_THREADS = FB4_GROUPS * FB_THREADS;
constexpr int FB4_SMEM = FB4_OFF_GROUP + FB4_GROUPS * FB_GROUP_BYTES;

template <bool OUT_F32>
__global__ void __launch_bounds__(FB4_THREADS, 1)
k_mul_mat16_fast4(dev_tables T, const uint16_t * __restrict__ W, const uint16_t * __restrict__ X,
                  void * __restrict__ dst, int64_t K, int64_t M, int64_t N, int64_t ne02, int64_t ne12,
                  int64_t r2, int64_t r3, uint32_t monte_seed, int vec, peer_out_dev peers, int64_t gx,
                  int64_t nfull, int64_t nblk) {
    pdl_entry();
    extern __shared__ __align__(16) unsigned char smem[];
    const int32_t * keytab = FB_MONTE ? T.mkey16 : T.key16;
    for (int i = threadIdx.x; i < FB_KEYB / 4; i += FB4_THREADS) {
        const int v = keytab[i];
#pragma unroll
        for (int r = 0; r < 4; r++) reinterpret_cast<int *>(smem + r * FB_REPL)[i] = v;
    }
    __syncthreads();
    const int g = threadIdx.x / FB_THREADS, tid = threadIdx.x % FB_THREADS;
    const int rbase = (threadIdx.x & 3) * FB_REPL;
    unsigned char * gsm = smem + FB4_OFF_GROUP + g * FB_GROUP_BYTES;
    const int64_t z = blockIdx.z;
    for (int64_t b = blockIdx.x + (int64_t) g * gridDim.x; b < nblk; b += (int64_t) FB4_GROUPS * gridDim.x) {
        if (b < nfull) {
            fb_tile<OUT_F32, FB_TN, FB4_GROUPS>(T, smem, gsm, tid, rbase, 1 + g, W, X, dst, K, M, N, ne02, ne12, r2,
                                                r3, monte_seed, vec, peers, z, (b % gx) * FB_BM, (b / gx) * FB_BN);
        } else {
            const int64_t q = b - nfull, t = nfull + q / 4;
            const int64_t n0 = (t / gx) * FB_BN + (q % 4) * 8;
            if (n0 < N)
                fb_tile<OUT_F32, 1, FB4_GROUPS>(T, smem, gsm, tid, rbase, 1 + g, W, X, dst, K, M, N, ne02, ne12, r2,
                                                r3, monte_seed, vec, peers, z, (t % gx) * FB_BM, n0);
        }
        fb_sync<FB4_GROUPS>(1 + g);                     // the group's buffers are reused by its next item
    }
}

// ============== MUL_MAT (xlns16, base mode, few outputs: latency form) ========
//
// When M*N is too small to fill the GPU with the tiled kernel (decode, the
// reference's K=1536 x N=8 case), time is one chain's latency: K dependent
// additions.  This kernel minimises that latency: one chain per thread (128
// consecutive weight rows of one token per CTA), the token's row resident in
// shared memory, W streamed through cp.async in 64-step chunks, and the key
// form with a signed 41 KB table, so the dependent path of one addition is
//     t = min(a - p, KM)  (DPX add-min)  ->  max(t, -KM)  ->  table load
//       ->  a = max(max(a, p) + adj, 4)  (DPX add-max)
// Range safety is decided per K chunk for the whole block (as in
// k_mul_mat16_fast), so the chunk's steps carry no branch and consecutive
// steps overlap; a chunk that fails the check runs on packed codes.
constexpr int LT_ROWS = 128, LT_KC = 128;
constexpr int LT_KM   = k16_key_max;                              // 20500
constexpr int LT_TABS = k16s_bytes;                               // signed table bytes
constexpr int LT_OFF_TAB2 = LT_TABS;
constexpr int LT_OFF_W    = LT_OFF_TAB2 + MM_TABPAD;              // 2 stages of W codes
constexpr int LT_WSTAGE   = LT_KC * LT_ROWS;                      // halfwords
constexpr int LT_OFF_X    = LT_OFF_W + 2 * LT_WSTAGE * 2;         // x keys (K words) then x codes (K halfwords)
constexpr int LT_MAX_K    = 16384;                               // one token per thread
constexpr int LT_MAX_K2   = 8192;                                // two tokens per thread
inline int lt_smem(int64_t K, int tn) { return LT_OFF_X + (int) ((K + 3) & ~3) * 6 * tn + 16; }

__device__ __forceinline__ void lt_stage(uint16_t * ws, const uint16_t * __restrict__ W, int64_t K, int64_t M,
                                         int64_t m0, int64_t k0, bool vec) {
    if (vec) {
#pragma unroll
        for (int it = 0; it < (LT_KC * LT_ROWS / 8) / LT_ROWS; it++) {   // 1024 copies of 16 B
            const int c = threadIdx.x + it * LT_ROWS;
            const int r = c >> 4, q = c & 15;
            if (k0 + r < K) {
                if (m0 + q * 8 < M) cp_async16(ws + r * LT_ROWS + q * 8, W + (k0 + r) * M + m0 + q * 8);
                else *reinterpret_cast<uint4 *>(ws + r * LT_ROWS + q * 8) = make_uint4(0x40004000u, 0x40004000u, 0x40004000u, 0x40004000u);
            }
        }
    } else {
        for (int i = threadIdx.x; i < LT_WSTAGE; i += LT_ROWS) {
            const int r = i / LT_ROWS, c = i % LT_ROWS;
            const int64_t k = k0 + r, m = m0 + c;
            ws[i] = (k < K && m < M) ? W[k * M + m] : (uint16_t) 0x4000;
        }
    }
}

// the signed key table at shared offset 0 and the packed table at LT_OFF_TAB2,
// as 16-byte asynchronous copies (the caller commits and waits)
__device__ __forceinline__ void lt_tables_async(const dev_tables & T, unsigned char * smem) {
    for (int i = threadIdx.x; i < LT_TABS / 16; i += blockDim.x)
        cp_async16(smem + i * 16, reinterpret_cast<const unsigned char *>(T.key16s) + i * 16);
    for (int i = threadIdx.x; i < MM_TABPAD / 16; i += blockDim.x)
        cp_async16(smem + LT_OFF_TAB2 + i * 16, reinterpret_cast<const unsigned char *>(T.sbdb16) + i * 16);
}

// TN tokens per thread (1 or 2): a thread runs the chains of its weight row
// against TN tokens, sharing the weight load and key conversion, and the TN
// independent chains interleave, hiding the dependent path of each.
template <bool OUT_F32, int TN>
__global__ void __launch_bounds__(LT_ROWS)
k_mul_mat16_lat(dev_tables T, const uint16_t * __restrict__ W, const uint16_t * __restrict__ X,
                void * __restrict__ dst, int64_t K, int64_t M, int64_t N, int64_t ne02, int64_t ne12,
                int64_t r2, int64_t r3, int vec) {
    pdl_entry();
    extern __shared__ __align__(16) unsigned char smem[];
    int16_t *  tab2  = reinterpret_cast<int16_t *>(smem + LT_OFF_TAB2);
    uint16_t * wst   = reinterpret_cast<uint16_t *>(smem + LT_OFF_W);
    const int KP = (int) ((K + 3) & ~3);                // token row pitch: 16-byte aligned rows (K <= LT_MAX_K)
    int *      xkeys = reinterpret_cast<int *>(smem + LT_OFF_X);                  // [TN][KP]
    uint16_t * xcod  = reinterpret_cast<uint16_t *>(smem + LT_OFF_X + TN * KP * 4); // [TN][KP]
    __shared__ int red[LT_ROWS / 32][4];

    lt_tables_async(T, smem);                           // signed key table, packed table
    cp_async_commit();

    const int64_t z = blockIdx.z, i12 = z % ne12, i13 = z / ne12;
    const int64_t n0 = (int64_t) blockIdx.y * TN;
    const int64_t m0 = (int64_t) blockIdx.x * LT_ROWS;
    const int64_t m = m0 + threadIdx.x;
    const int warp = threadIdx.x >> 5;
    const uint16_t * Wz = W + ((i13 / r3) * ne02 + i12 / r2) * K * M;
    int xmin = 0x7FFF, xmax = 0;
#pragma unroll
    for (int t = 0; t < TN; t++) {
        const bool tok = n0 + t < N;                    // a missing token runs on 1.0 and is not stored
        const uint16_t * xr = X + (z * N + (tok ? n0 + t : N - 1)) * K;
        for (int64_t k = threadIdx.x; k < K; k += LT_ROWS) {
            const uint32_t c = tok ? xr[k] : 0x4000u;
            xcod[t * KP + k]  = (uint16_t) c;
            xkeys[t * KP + k] = key_of_code_x(c);
            xmin = min(xmin, (int) (c & 0x7FFFu));
            xmax = max(xmax, (int) (c & 0x7FFFu));
        }
    }
    xmin = __reduce_min_sync(0xFFFFFFFFu, xmin);
    xmax = __reduce_max_sync(0xFFFFFFFFu, xmax);
    if ((threadIdx.x & 31) == 0) { red[warp][0] = xmin; red[warp][1] = xmax; }
    __syncthreads();
#pragma unroll
    for (int w = 0; w < LT_ROWS / 32; w++) { xmin = min(xmin, red[w][0]); xmax = max(xmax, red[w][1]); }

    const int nchunks = (int) ((K + LT_KC - 1) / LT_KC);
    if (nchunks > 0) {
        lt_stage(wst, Wz, K, M, m0, 0, vec != 0);
        cp_async_commit();
    }
    int a[TN];                                          // accumulator keys
#pragma unroll
    for (int t = 0; t < TN; t++) a[t] = 0;
    for (int c = 0; c < nchunks; c++) {
        const uint16_t * ws = wst + (c & 1) * LT_WSTAGE;
        if (c + 1 < nchunks) {
            lt_stage(wst + ((c + 1) & 1) * LT_WSTAGE, Wz, K, M, m0, (int64_t) (c + 1) * LT_KC, vec != 0);
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const int kb = c * LT_KC;
        const int kvalid = (int) imin64(LT_KC, K - kb);
        const int * xkc[TN];                            // this chunk's token keys
#pragma unroll
        for (int t = 0; t < TN; t++) xkc[t] = xkeys + t * KP + kb;
        // block-wide range check of this chunk (see k_mul_mat16_fast): 16x2
        // SIMD min/max over the staged codes (columns past M hold 1.0)
        unsigned vmin = 0x7FFF7FFFu, vmax = 0u;
#pragma unroll
        for (int it = 0; it < LT_WSTAGE / 8 / LT_ROWS; it++) {
            const int v = threadIdx.x + it * LT_ROWS;           // 16-byte vector index
            if ((v >> 4) < kvalid) {
                const uint4 q = *reinterpret_cast<const uint4 *>(ws + v * 8);
                const unsigned w0 = q.x & 0x7FFF7FFFu, w1 = q.y & 0x7FFF7FFFu, w2 = q.z & 0x7FFF7FFFu, w3 = q.w & 0x7FFF7FFFu;
                vmin = __vminu2(vmin, __vminu2(__vminu2(w0, w1), __vminu2(w2, w3)));
                vmax = __vmaxu2(vmax, __vmaxu2(__vmaxu2(w0, w1), __vmaxu2(w2, w3)));
            }
        }
        int wmin = (int) min(vmin & 0xFFFFu, vmin >> 16), wmax = (int) max(vmax & 0xFFFFu, vmax >> 16);
        int amax = 0;
        if (c > 0) {
#pragma unroll
            for (int t = 0; t < TN; t++) amax = max(amax, a[t] >> 4);
        }
        wmin = __reduce_min_sync(0xFFFFFFFFu, wmin);
        wmax = __reduce_max_sync(0xFFFFFFFFu, wmax);
        amax = __reduce_max_sync(0xFFFFFFFFu, m < M ? amax : 0);
        __syncthreads();                                // red[] reuse
        if ((threadIdx.x & 31) == 0) { red[warp][0] = wmin; red[warp][1] = wmax; red[warp][2] = amax; }
        __syncthreads();
        int w0 = 0x7FFF, w1 = 0, am = 0;
#pragma unroll
        for (int w = 0; w < LT_ROWS / 32; w++) { w0 = min(w0, red[w][0]); w1 = max(w1, red[w][1]); am = max(am, red[w][2]); }
        const bool fast = w0 + xmin - 0x4000 >= 964 && max(am, w1 + xmax - 0x4000) + growth_bound(LT_KC) <= 0x7FFF;

        int k = 0;
        if (fast) {
            // one dependent step of chain t with product key p
            auto step = [&](int t, int p) {
                const int d   = max(__viaddmin_s32(a[t], -p, LT_KM), -LT_KM);
                const int adj = *reinterpret_cast<const int *>(smem + LT_KM + d);
                a[t] = __viaddmax_s32(max(a[t], p), adj, 0);
            };
            if (c == 0) {
                const int wk = key_of_code_w(ws[threadIdx.x]);
#pragma unroll
                for (int t = 0; t < TN; t++) a[t] = key_of_product(wk, xkc[t][0]);
                for (k = 1; k < 8 && k < kvalid; k++) {
                    const int wk2 = key_of_code_w(ws[k * LT_ROWS + threadIdx.x]);
#pragma unroll
                    for (int t = 0; t < TN; t++) step(t, key_of_product(wk2, xkc[t][k]));
                }
            }
            // blocks of 8 steps with constant trip counts: the 8 products are
            // formed first, so the dependent chain runs without operand waits
            for (; k + 8 <= kvalid; k += 8) {
                int wk8[8];
#pragma unroll
                for (int u = 0; u < 8; u++) wk8[u] = key_of_code_w(ws[(k + u) * LT_ROWS + threadIdx.x]);
#pragma unroll
                for (int t = 0; t < TN; t++) {
                    const int4 x0 = *reinterpret_cast<const int4 *>(xkc[t] + k);
                    const int4 x1 = *reinterpret_cast<const int4 *>(xkc[t] + k + 4);
                    const int xk8[8] = { x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w };
                    int p8[8];
#pragma unroll
                    for (int u = 0; u < 8; u++) p8[u] = key_of_product(wk8[u], xk8[u]);
#pragma unroll
                    for (int u = 0; u < 8; u++) step(t, p8[u]);
                }
            }
            for (; k < kvalid; k++) {
                const int wk = key_of_code_w(ws[k * LT_ROWS + threadIdx.x]);
#pragma unroll
                for (int t = 0; t < TN; t++) step(t, key_of_product(wk, xkc[t][k]));
            }
        } else {
#pragma unroll
            for (int t = 0; t < TN; t++) {
                uint32_t ac = c == 0 ? mul16(ws[threadIdx.x], xcod[t * KP]) : code_of_key(a[t]);
                for (int kk = c == 0 ? 1 : 0; kk < kvalid; kk++)
                    ac = add16(ac, mul16(ws[kk * LT_ROWS + threadIdx.x], xcod[t * KP + kb + kk]), tab2);
                a[t] = key_of_code(ac);
            }
        }
        __syncthreads();
    }
    if (m < M) {
#pragma unroll
        for (int t = 0; t < TN; t++) {
            if (n0 + t >= N) continue;
            const uint32_t v = K == 0 ? 0u : code_of_key(a[t]);
            const int64_t o = (z * N + n0 + t) * M + m;
            if constexpr (OUT_F32) static_cast<float *>(dst)[o] = to_f32_16(T, v);
            else                   static_cast<uint16_t *>(dst)[o] = (uint16_t) v;
        }
    }
}

// Segments of the key form's range check in the weight-resident latency
// kernels (k_mul_mat16_res2): the check is made per LR_SEG steps.
constexpr int LR_SEG    = 256;
constexpr int LR_MAXSEG = 16;                                     // K <= LR_SEG * LR_MAXSEG

// ======= MUL_MAT (xlns16, base mode, few outputs, weight keys resident) =====
//
// The latency form of the chain with less work on each step.  The
// CTA's weight slice is held as 32-bit keys in [row][k] order (a row's pitch
// r2_pitch(K) words, 4 mod 32, so the 16-byte loads of different rows start
// in different banks), the tokens' rows as keys beside it, so a lane reads
// four steps of weights and four of activations with two 16-byte loads and
// converts nothing inside the loop.  A warp runs R rows x 32/R tokens (lane =
// row + R * token slot): R = 32 for a single token where it fits, else 16
// rows against two tokens.  The table index is clamped with one unsigned
// add-min: the signed table holds the adjustment of a key difference D at
// byte KM + D and both ends (|D| >= KM) hold zero, so a difference below -KM,
// which wraps to a huge unsigned value, may be clamped to the upper end.  The
// dependent path of a step is therefore
//     idx = min(a + (KM - p), 2 KM) (unsigned)  ->  table load
//       ->  a = max(max(a, p) + adj, 0)
// with p and KM - p formed off the path (one-warp measurement on B200: 47
// cycles a step with 32 lanes, 41 with one; the load alone is most of it).
// The range check is per segment of LR_SEG steps and per warp (both token
// slots) from the ranges staging records; a segment that fails runs on packed codes
// rebuilt from the keys.
//
// Warps [0, cw) run the chains; the other 4 - cw warps produce: the whole CTA
// stages the tables, the token rows and the first segment of weights, then
// each producer warp stages later segments (16-byte loads, keys, the
// segment's log range) and signals segment s on hardware named barrier s
// (bar.arrive), which the chain warps wait on (bar.sync) just before they
// reach it -- so the staging of segments 1.. runs under the chain.  With
// cw = 4 there are no producers and everything is staged first.  Output:
// codes, F32, or codes into every peer's buffer (the fused all-gather of
// output-row shards, peers.n > 0).
constexpr int R2_THREADS = 128;
constexpr int R2_OFF_W   = LT_OFF_TAB2 + MM_TABPAD;              // [R][pitch] weight keys, then [tokens][pitch] x keys
__host__ __device__ constexpr int r2_pitch(int64_t K) {     // >= K rounded to 4, and 4 mod 32
    return (int) ((K + 3) & ~3) + (36 - (int) (((K + 3) & ~3) % 32)) % 32;
}
inline int r2_smem(int64_t K, int R, int ntok) { return R2_OFF_W + (R + ntok) * r2_pitch(K) * 4; }
constexpr int R2_SMEM_MAX = 225 * 1024;                          // with the kernel's 1.1 KB of static shared memory

// weight keys of k-rows [k0, k1) of the CTA's R rows, staged by threads t of
// nt: 16-byte loads of 8 codes (vec: M a multiple of 8, W 16-byte aligned),
// eight in flight per thread, otherwise one code per load; rows past M hold
// 1.0.  lo / hi: this thread's smallest / largest log field staged.
template <int R>
__device__ __forceinline__ void r2_stage_w(int * wk, int PW, const uint16_t * __restrict__ Wz, int64_t M, int64_t m0,
                                           int k0, int k1, int t, int nt, int vec, int & lo, int & hi) {
    if (vec) {
        constexpr int QR = R / 8;                        // 16-byte pieces of a k-row
        const int nld = (k1 - k0) * QR;
        for (int base = t; base < nld; base += nt * 8) {
            uint4 q[8];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int i = base + u * nt, k = k0 + i / QR, c8 = (i % QR) * 8;
                q[u] = (i < nld && m0 + c8 < M) ? __ldg(reinterpret_cast<const uint4 *>(Wz + (int64_t) k * M + m0 + c8))
                                                : make_uint4(0x40004000u, 0x40004000u, 0x40004000u, 0x40004000u);
            }
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int i = base + u * nt, k = k0 + i / QR, c8 = (i % QR) * 8;
                if (i >= nld) break;
                const uint32_t wd[4] = { q[u].x, q[u].y, q[u].z, q[u].w };
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    const uint32_t c = (wd[e >> 1] >> (16 * (e & 1))) & 0xFFFFu;
                    wk[(c8 + e) * PW + k] = key_of_code_w(c);
                    lo = min(lo, (int) (c & 0x7FFFu));
                    hi = max(hi, (int) (c & 0x7FFFu));
                }
            }
        }
    } else {
        for (int i = t; i < (k1 - k0) * R; i += nt) {
            const int k = k0 + i / R, r = i % R;
            const int64_t m = m0 + r;
            const uint32_t c = m < M ? (uint32_t) Wz[(int64_t) k * M + m] : 0x4000u;
            wk[r * PW + k] = key_of_code_w(c);
            lo = min(lo, (int) (c & 0x7FFFu));
            hi = max(hi, (int) (c & 0x7FFFu));
        }
    }
}

template <bool OUT_F32, int R, int TPW, bool XF32>
__global__ void __launch_bounds__(R2_THREADS)
k_mul_mat16_res2(dev_tables T, const uint16_t * __restrict__ W, const void * __restrict__ X,
                 void * __restrict__ dst, int64_t K, int64_t M, int64_t N, int64_t ne02, int64_t ne12,
                 int64_t r2, int64_t r3, int cw, int vec, peer_out_dev peers) {
    // TPW token slots per warp: 32 / R, or 1 with R = 16, where lanes 16..31
    // repeat lanes 0..15 (same addresses: the table lookup sees 16 distinct
    // addresses, fewer bank conflicts, a shorter step) and only lanes 0..15 store.
    // XF32: the activations arrive as F32 and are converted (from_f32_16, the
    // conversion of k_to_lns) as they are staged.
    static_assert(R * TPW == 32 || (R == 16 && TPW == 1), "lane layout");
    pdl_entry();
    extern __shared__ __align__(16) unsigned char smem[];
    const int Ki = (int) K, PW = r2_pitch(K);
    const int ntok  = cw * TPW;                          // token rows staged by this CTA
    const int nseg  = (Ki + LR_SEG - 1) / LR_SEG;
    const int nprod = R2_THREADS / 32 - cw;              // producer warps
    const int kpre  = nprod > 0 ? min(Ki, LR_SEG) : Ki;  // weight rows staged before the chains start
    const int16_t * tab2 = reinterpret_cast<const int16_t *>(smem + LT_OFF_TAB2);
    int * wk = reinterpret_cast<int *>(smem + R2_OFF_W);                  // [R][PW]
    int * xk = wk + R * PW;                                                // [ntok][PW]
    __shared__ int wseg[LR_MAXSEG][2];                   // weight log range per segment
    __shared__ int xseg[8][LR_MAXSEG][2];                // token log range per token row and segment
    __shared__ int wred[R2_THREADS / 32][2];             // per-warp weight range of the first staging

    const int64_t z = blockIdx.z, i12 = z % ne12, i13 = z / ne12;
    const int64_t m0 = (int64_t) blockIdx.x * R, n0 = (int64_t) blockIdx.y * ntok;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint16_t * Wz = W + ((i13 / r3) * ne02 + i12 / r2) * K * M;

    lt_tables_async(T, smem);                            // signed key table, packed table
    cp_async_commit();
    // token keys: token row t is token n0 + t (the last token stands in past
    // N); 16-byte loads where K is a multiple of 8 and X 16-byte aligned.  The
    // first batch of token loads is issued before the weights are staged, so
    // the two trips to memory overlap.
    const bool xvec = Ki % 8 == 0 && ((uintptr_t) X % 16) == 0;
    const int  k8n = Ki / 8, nld = xvec ? ntok * k8n : 0;
    constexpr int XQ = XF32 ? 2 : 1;                     // 16-byte words per piece of 8 values
    auto xload = [&](int base, uint4 (&q)[4 * XQ]) {
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int i = base + u * R2_THREADS;
            if (i < nld) {
                const int t = i / k8n;
                const int64_t n = min(n0 + t, N - 1), o = (z * N + n) * K + (int64_t) (i - t * k8n) * 8;
                if constexpr (XF32) {
                    const uint4 * p = reinterpret_cast<const uint4 *>(static_cast<const float *>(X) + o);
                    q[2 * u] = __ldg(p);
                    q[2 * u + 1] = __ldg(p + 1);
                } else {
                    q[u] = __ldg(reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(X) + o));
                }
            }
        }
    };
    auto xstore = [&](int base, const uint4 (&q)[4 * XQ]) {
        if constexpr (XF32) {
            uint32_t c[4][8];                            // the pieces' codes, every lookup issued first
#pragma unroll
            for (int u = 0; u < 4; u++) {
                if (base + u * R2_THREADS >= nld) continue;
                const uint32_t wd[8] = { q[2 * u].x, q[2 * u].y, q[2 * u].z, q[2 * u].w,
                                         q[2 * u + 1].x, q[2 * u + 1].y, q[2 * u + 1].z, q[2 * u + 1].w };
#pragma unroll
                for (int e = 0; e < 8; e++) c[u][e] = from_f32_16(T, __uint_as_float(wd[e]));
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int i = base + u * R2_THREADS;
                if (i >= nld) break;
                const int t = i / k8n, k = (i - t * k8n) * 8;
                int key[8];
#pragma unroll
                for (int e = 0; e < 8; e++) key[e] = key_of_code_x(c[u][e]);
                *reinterpret_cast<int4 *>(xk + t * PW + k)     = make_int4(key[0], key[1], key[2], key[3]);
                *reinterpret_cast<int4 *>(xk + t * PW + k + 4) = make_int4(key[4], key[5], key[6], key[7]);
            }
        } else {
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int i = base + u * R2_THREADS;
                if (i >= nld) break;
                const int t = i / k8n, k = (i - t * k8n) * 8;
                const uint32_t wd[4] = { q[u].x, q[u].y, q[u].z, q[u].w };
                int key[8];
#pragma unroll
                for (int e = 0; e < 8; e++) key[e] = key_of_code_x((wd[e >> 1] >> (16 * (e & 1))) & 0xFFFFu);
                *reinterpret_cast<int4 *>(xk + t * PW + k)     = make_int4(key[0], key[1], key[2], key[3]);
                *reinterpret_cast<int4 *>(xk + t * PW + k + 4) = make_int4(key[4], key[5], key[6], key[7]);
            }
        }
    };
    uint4 xq0[4 * XQ];
    if (xvec) xload(tid, xq0);
    {
        int lo = 0x7FFF, hi = 0;
        r2_stage_w<R>(wk, PW, Wz, M, m0, 0, kpre, tid, R2_THREADS, vec, lo, hi);
        lo = __reduce_min_sync(0xFFFFFFFFu, lo);
        hi = __reduce_max_sync(0xFFFFFFFFu, hi);
        if (lane == 0) { wred[warp][0] = lo; wred[warp][1] = hi; }
    }
    if (xvec) {
        xstore(tid, xq0);
        for (int base = tid + R2_THREADS * 4; base < nld; base += R2_THREADS * 4) {
            uint4 q[4 * XQ];
            xload(base, q);
            xstore(base, q);
        }
    } else {
        for (int i = tid; i < ntok * Ki; i += R2_THREADS) {
            const int t = i / Ki, k = i - t * Ki;
            const int64_t o = (z * N + min(n0 + t, N - 1)) * K + k;
            xk[t * PW + k] = key_of_code_x(XF32 ? from_f32_16(T, static_cast<const float *>(X)[o])
                                                : (uint32_t) static_cast<const uint16_t *>(X)[o]);
        }
    }
    __syncthreads();
    // log ranges: the tokens' per token row and segment; the weights' of the
    // first staging (segment 0, or every segment without producers)
    const int wsegs = nprod > 0 ? min(nseg, 1) : nseg;
    for (int j = warp; j < nseg * ntok + (nprod > 0 ? 0 : nseg); j += R2_THREADS / 32) {
        const bool wj = j >= nseg * ntok;
        const int sg = j % nseg, t = j / nseg;
        const int k0 = sg * LR_SEG, k1 = min(Ki, k0 + LR_SEG);
        int lo = 0x7FFF, hi = 0;
        if (wj) {
            for (int i = lane; i < (k1 - k0) * R; i += 32) {
                const int l = (wk[(i % R) * PW + k0 + i / R] >> 4) & 0x7FFF;
                lo = min(lo, l); hi = max(hi, l);
            }
        } else {
            for (int k = k0 + lane; k < k1; k += 32) {
                const int l = ((xk[t * PW + k] + 16 * 0x4000) >> 4) & 0x7FFF;
                lo = min(lo, l); hi = max(hi, l);
            }
        }
        lo = __reduce_min_sync(0xFFFFFFFFu, lo);
        hi = __reduce_max_sync(0xFFFFFFFFu, hi);
        if (lane == 0) {
            if (wj) { wseg[sg][0] = lo; wseg[sg][1] = hi; }
            else    { xseg[t][sg][0] = lo; xseg[t][sg][1] = hi; }
        }
    }
    if (nprod > 0 && tid == 0 && wsegs > 0) {
        int lo = 0x7FFF, hi = 0;
        for (int w = 0; w < R2_THREADS / 32; w++) { lo = min(lo, wred[w][0]); hi = max(hi, wred[w][1]); }
        wseg[0][0] = lo; wseg[0][1] = hi;
    }
    cp_async_wait<0>();
    __syncthreads();                                     // the last block-wide barrier

    if (warp >= cw) {
        // producer: segments s = 1 + (warp - cw), then every nprod-th, each
        // signalled on named barrier s (ids 1..15: K <= 16 segments)
        for (int sg = 1 + (warp - cw); sg < nseg; sg += nprod) {
            const int k0 = sg * LR_SEG, k1 = min(Ki, k0 + LR_SEG);
            int lo = 0x7FFF, hi = 0;
            r2_stage_w<R>(wk, PW, Wz, M, m0, k0, k1, lane, 32, vec, lo, hi);
            lo = __reduce_min_sync(0xFFFFFFFFu, lo);
            hi = __reduce_max_sync(0xFFFFFFFFu, hi);
            if (lane == 0) { wseg[sg][0] = lo; wseg[sg][1] = hi; }
            __threadfence_block();
            asm volatile("bar.arrive %0, %1;\n" ::"r"(sg), "r"(32 * (cw + 1)) : "memory");
        }
        return;
    }

    const int row = lane % R, slot = (lane / R) % TPW, t = warp * TPW + slot;
    const int64_t n = n0 + t;
    const bool store_lane = lane < R * TPW;
    const int * wr = wk + row * PW;
    const int * xr = xk + t * PW;
    uint32_t v = 0;
    if (Ki > 0) {
        constexpr int KM = LT_KM;
        int      a  = 0;                                 // key (fast)
        uint32_t ac = 0;                                 // code (slow)
        bool     fast = true;                            // uniform across the warp
        auto step = [&](int p) {
            const uint32_t idx = __viaddmin_u32((uint32_t) a, (uint32_t) (KM - p), 2u * KM);
            const int adj = *reinterpret_cast<const int *>(smem + idx);
            a = __viaddmax_s32(max(a, p), adj, 0);
        };
        for (int sg = 0; sg < nseg; sg++) {
            const int s0 = sg * LR_SEG, s1 = min(Ki, s0 + LR_SEG);
            if (sg > 0 && nprod > 0)                     // segment sg staged by its producer
                asm volatile("bar.sync %0, %1;\n" ::"r"(sg), "r"(32 * (cw + 1)) : "memory");
            {
                // exact in key form over this segment: every product >= 2^-120 and
                // no sum able to reach 2^127 within it (growth_bound); decided for
                // the warp (both token slots), both ways
                const int am = __reduce_max_sync(0xFFFFFFFFu, sg == 0 ? 0 : fast ? (a >> 4) : (int) (ac & 0x7FFFu));
                const bool mine = wseg[sg][0] + xseg[t][sg][0] - 0x4000 >= 964 &&
                                  max(am, wseg[sg][1] + xseg[t][sg][1] - 0x4000) + growth_bound(LR_SEG) <= 0x7FFF;
                const bool ok = __all_sync(0xFFFFFFFFu, mine);
                if (sg > 0 && ok != fast) {
                    if (ok) a = key_of_code(ac);
                    else    ac = code_of_key(a);
                }
                fast = ok;
            }
            int k = s0;
            if (fast) {
                if (sg == 0) {
                    a = key_of_product(wr[0], xr[0]);
                    for (k = 1; k < 4 && k < s1; k++) step(key_of_product(wr[k], xr[k]));
                }
                if (k + 4 <= s1) {
                    // four steps per pair of 16-byte loads, the next four loaded first
                    int4 w4 = *reinterpret_cast<const int4 *>(wr + k), x4 = *reinterpret_cast<const int4 *>(xr + k);
                    for (; k + 8 <= s1; k += 4) {
                        const int4 wn = *reinterpret_cast<const int4 *>(wr + k + 4), xn = *reinterpret_cast<const int4 *>(xr + k + 4);
                        step(key_of_product(w4.x, x4.x));
                        step(key_of_product(w4.y, x4.y));
                        step(key_of_product(w4.z, x4.z));
                        step(key_of_product(w4.w, x4.w));
                        w4 = wn; x4 = xn;
                    }
                    step(key_of_product(w4.x, x4.x));
                    step(key_of_product(w4.y, x4.y));
                    step(key_of_product(w4.z, x4.z));
                    step(key_of_product(w4.w, x4.w));
                    k += 4;
                }
                for (; k < s1; k++) step(key_of_product(wr[k], xr[k]));
            } else {
                auto wc = [&](int kk) { return code_of_key(wr[kk]); };
                auto xc = [&](int kk) { return code_of_key(xr[kk] + 16 * 0x4000); };
                if (sg == 0) { ac = mul16(wc(0), xc(0)); k = 1; }
                for (; k < s1; k++) ac = add16(ac, mul16(wc(k), xc(k)), tab2);
            }
        }
        v = fast ? code_of_key(a) : ac;
    }
    const int64_t m = m0 + row;
    if (store_lane && n < N && m < M) {
        if (peers.n > 0) {
            const int64_t o = (z * N + n) * peers.ld + peers.off + m;
            for (int p = 0; p < peers.n; p++) peers.ptrs[p][o] = (uint16_t) v;
        } else {
            const int64_t o = (z * N + n) * M + m;
            if constexpr (OUT_F32) static_cast<float *>(dst)[o] = to_f32_16(T, v);
            else                   static_cast<uint16_t *>(dst)[o] = (uint16_t) v;
        }
    }
}

// ================= MUL_MAT over the flat xlns32 addition ====================
//
// xlns16 in sum32 mode (acc32 = add32(acc32, t << 16), narrowed once at the
// end; lns-backend/cuda/lns-cuda-xlns16.cu:75-130, lns16-sum32.h:59-107) and
// the xlns32 format (lns-backend/cuda/lns-cuda-xlns32.cu:30-67) share this
// kernel.  The flat addition image (k32f_words, ~126 KB) is resident in shared
// memory, one CTA per SM (32 warps for xlns16, 16 for xlns32).  A warp runs
// 32 x TN chains side by side: 32 consecutive weight rows (one per lane)
// against TN tokens (two once there are enough units of work, so a lane has
// two independent chains to interleave).  Units of work (slice, 32-row block,
// token group) are dealt to warps round-robin with the CTA index fastest, so a
// small problem spreads over every SM; all units cost the same K steps, so the
// static deal is balanced.  Operands stream through a per-warp cp.async ring
// of 8-step chunks (the warp's 32 consecutive rows of the k-major weights, and
// each token's 8 values), A32_STAGES - 1 chunks ahead; unaligned operands take
// a register-prefetch path instead.  Each step is add32f_main for every chain
// (ALU work moved to the multiply pipe where the interpolation allows) and a
// branch per chain for the rare cotransformed case (add32f_cot).
constexpr int A32_THREADS = 512;
// threads per CTA: 32 warps per SM where the per-warp rings fit beside the
// table (xlns16), else 16
__host__ __device__ constexpr int a32_threads(int fmt, bool ring) { return fmt == 16 && ring ? 1024 : A32_THREADS; }
#ifndef LNSB_A32_SEL_WARPS
// at most this many units per SM: the SM is latency bound and the chains take
// the selected adder (add32f_sel, two table levels deep, more instructions);
// beyond it issue binds and they take the main path with a branch for the
// cotransformed case
#define LNSB_A32_SEL_WARPS 16
#endif
#ifndef LNSB_A32_LAT_ADDER
// the adder of the latency regime: 0 the selected one (add32f_sel: main and
// cotransformed results side by side), 1 the single-path one (add32f: the
// cotransformation lookups, then one interpolation, fewer instructions)
#define LNSB_A32_LAT_ADDER 0
#endif
#ifndef LNSB_A32_LV
// 1: products with few units per SM (sum32, xlns32) run k_mat_vec_lat
#define LNSB_A32_LV 1
#endif
#ifndef LNSB_A32_LV_PAIRS
// ... up to this many units per SM (at most LV_MAX_PAIRS).  Measured per step
// at N = 16 against k_mul_mat_a32: 189 / 223 / 227 / 227 cycles at 1 / 2 / 3 / 4
// units per SM against 232-234; 287 / 358 at 5 / 6 against 276
#define LNSB_A32_LV_PAIRS 4
#endif
#ifndef LNSB_A32_TN2_MIN_QUARTERS
// two tokens per lane once the two-token units fill this many quarters of the
// warps (W 8192 x 4096, sum32: N = 32 runs 443 -> 549 G-LNSadd/s with two
// tokens, 0.86 of the warps busy; N = 16 falls 465 -> 331, 0.43 busy)
#define LNSB_A32_TN2_MIN_QUARTERS 3
#endif

// Accumulation policy of the kernel: the flat xlns32 addition (xlns32, and
// xlns16 in sum32 mode), LPVIP (xlns16 lpvip: acc32 = add32_lpvip(acc32,
// t << 16), truncated to 16 bits at the end) or Monte-by-LPVIP (xlns16 monte
// with GGML_LNS16_MONTE_BYLPVIP: a 16-bit accumulator, each addition
// add32_lpvip(acc << 16, (t << 16) | next LFSR state) >> 16;
// lns-backend/src/lns-ops.cpp:93-97).
enum : int { A32_FLAT = 0, A32_LPVIP = 1, A32_MBL = 2 };
template <int FMT> __host__ __device__ constexpr int a32_kind() {
    return FMT == 32 || k_mode == M_SUM32 ? A32_FLAT : (k_mode == M_LPVIP ? A32_LPVIP : A32_MBL);
}

template <int FMT> struct a32_fmt;
template <> struct a32_fmt<16> {
    using elem = uint16_t;
    static constexpr int xvec = 1;    // uint4 per 8 values
    __device__ static __forceinline__ uint32_t term(uint32_t w, uint32_t x) {
        return a32_kind<16>() == A32_MBL ? mul16(w, x) : mul16(w, x) << 16;
    }
    __device__ static __forceinline__ uint32_t finish(uint32_t acc) {
        if constexpr (a32_kind<16>() == A32_FLAT) {
            if ((acc & 0x7FFFFFFFu) >= 0x7FFF8000u) return ((acc >> 16) | 0x7FFFu) & 0xFFFFu;
            return (acc + 0x8000u) >> 16;
        }
        if constexpr (a32_kind<16>() == A32_LPVIP) return acc >> 16;
        return acc;
    }
    __device__ static __forceinline__ void store(const dev_tables & T, void * dst, int64_t o, uint32_t v, bool f32) {
        if (f32) static_cast<float *>(dst)[o] = to_f32_16(T, v);
        else     static_cast<uint16_t *>(dst)[o] = (uint16_t) v;
    }
};
template <> struct a32_fmt<32> {
    using elem = uint32_t;
    static constexpr int xvec = 2;
    __device__ static __forceinline__ uint32_t term(uint32_t w, uint32_t x) { return mul32(w, x); }
    __device__ static __forceinline__ uint32_t finish(uint32_t acc) { return acc; }
    __device__ static __forceinline__ void store(const dev_tables & T, void * dst, int64_t o, uint32_t v, bool f32) {
        if (f32) static_cast<float *>(dst)[o] = to_f32_32(T, v);
        else     static_cast<uint32_t *>(dst)[o] = v;
    }
};

template <int FMT, int TN>
struct a32_chunk {
    uint32_t w[8];
    uint4    x[TN][a32_fmt<FMT>::xvec];
    __device__ __forceinline__ uint32_t xv(int t, int j) const {
        const uint32_t * p = reinterpret_cast<const uint32_t *>(&x[t][0]);
        if constexpr (FMT == 16) return (p[j >> 1] >> (16 * (j & 1))) & 0xFFFFu;
        else                     return p[j];
    }
};

template <int FMT, int TN>
__device__ __forceinline__ void a32_load(a32_chunk<FMT, TN> & c, const typename a32_fmt<FMT>::elem * __restrict__ wl,
                                         const typename a32_fmt<FMT>::elem * const (&xt)[TN], int64_t k0, int64_t K,
                                         int64_t M, bool vecx) {
    using E = typename a32_fmt<FMT>::elem;
    if (k0 + 8 <= K) {
#pragma unroll
        for (int j = 0; j < 8; j++) c.w[j] = __ldg(wl + (k0 + j) * M);
    } else {
#pragma unroll
        for (int j = 0; j < 8; j++) c.w[j] = k0 + j < K ? (uint32_t) __ldg(wl + (k0 + j) * M) : 0u;
    }
#pragma unroll
    for (int t = 0; t < TN; t++) {
        if (vecx && k0 + 8 <= K) {
#pragma unroll
            for (int v = 0; v < a32_fmt<FMT>::xvec; v++) c.x[t][v] = __ldg(reinterpret_cast<const uint4 *>(xt[t] + k0) + v);
        } else {
            __align__(16) E tmp[8];
#pragma unroll
            for (int j = 0; j < 8; j++) tmp[j] = k0 + j < K ? __ldg(xt[t] + k0 + j) : (E) 0;
#pragma unroll
            for (int v = 0; v < a32_fmt<FMT>::xvec; v++) c.x[t][v] = reinterpret_cast<const uint4 *>(tmp)[v];
        }
    }
}

// L2 prefetch of the weights of the chunk at k0 (one lane's column)
constexpr int A32_L2PF = 6;        // chunks ahead
template <int FMT>
__device__ __forceinline__ void a32_prefetch_l2(const typename a32_fmt<FMT>::elem * wl, int64_t k0, int64_t K, int64_t M) {
#pragma unroll
    for (int j = 0; j < 8; j++)
        if (k0 + j < K) asm volatile("prefetch.global.L2 [%0];\n" ::"l"(__cvta_generic_to_global(wl + (k0 + j) * M)));
}

// One step of every chain of a lane: the main parts first (independent, so
// they interleave), then a branch per chain for the lanes on the rare path.
// F: the flat image (A32_FLAT); LP: the LPVIP singular-branch table; st: the
// chains' LFSR states (A32_MBL).
template <int FMT, int TN, bool BF = false>
__device__ __forceinline__ void a32_step_x(const int32_t * F, const int32_t * LP, uint32_t (&acc)[TN],
                                           uint32_t (&st)[TN], uint32_t w, const uint32_t (&x)[TN]) {
    using OP = a32_fmt<FMT>;
    if constexpr (a32_kind<FMT>() == A32_FLAT && BF) {
        // latency regime: the selected adder (main and cotransformed results
        // side by side, two table levels deep), no divergence on the dependent path
#pragma unroll
        for (int t = 0; t < TN; t++)
            acc[t] = LNSB_A32_LAT_ADDER ? add32f(F, acc[t], OP::term(w, x[t])) : add32f_sel(F, acc[t], OP::term(w, x[t]));
    } else if constexpr (a32_kind<FMT>() == A32_FLAT) {
        uint32_t    b[TN];
        add32f_part o[TN];
#pragma unroll
        for (int t = 0; t < TN; t++) {
            b[t] = OP::term(w, x[t]);
            o[t] = add32f_main(F, acc[t], b[t]);
        }
#pragma unroll
        for (int t = 0; t < TN; t++) acc[t] = o[t].cot ? add32f_cot(F, o[t].mx, o[t].d) : o[t].r;
    } else {
        lpvip_part o[TN];
#pragma unroll
        for (int t = 0; t < TN; t++) {
            if constexpr (a32_kind<FMT>() == A32_MBL) {
                st[t] = lfsr_step(st[t]);
                o[t]  = lpvip_main(acc[t] << 16, (OP::term(w, x[t]) << 16) | st[t]);
            } else {
                o[t] = lpvip_main(acc[t], OP::term(w, x[t]));
            }
        }
#pragma unroll
        for (int t = 0; t < TN; t++) {
            const uint32_t r = o[t].sing ? lpvip_sing(LP, o[t].mx, o[t].d) : o[t].r;
            acc[t] = a32_kind<FMT>() == A32_MBL ? r >> 16 : r;
        }
    }
}
template <int FMT, int TN, bool BF = false>
__device__ __forceinline__ void a32_step(const int32_t * F, const int32_t * LP, uint32_t (&acc)[TN], uint32_t (&st)[TN],
                                         uint32_t w, const a32_chunk<FMT, TN> & c, int j) {
    uint32_t x[TN];
#pragma unroll
    for (int t = 0; t < TN; t++) x[t] = c.xv(t, j);
    a32_step_x<FMT, TN, BF>(F, LP, acc, st, w, x);
}

// The steps of one 8-step chunk: j in [j0, kv) (kv < 8 only in the last chunk).
template <int FMT, int TN, bool BF = false>
__device__ __forceinline__ void a32_steps(const int32_t * F, const int32_t * LP, const a32_chunk<FMT, TN> & c,
                                          uint32_t (&acc)[TN], uint32_t (&st)[TN], bool first, int64_t kv) {
    using OP = a32_fmt<FMT>;
    if (first) {
#pragma unroll
        for (int t = 0; t < TN; t++) acc[t] = OP::term(c.w[0], c.xv(t, 0));
#pragma unroll
        for (int j = 1; j < 8; j++) {
            if (j < kv) a32_step<FMT, TN, BF>(F, LP, acc, st, c.w[j], c, j);
        }
    } else if (kv >= 8) {
#pragma unroll
        for (int j = 0; j < 8; j++) a32_step<FMT, TN, BF>(F, LP, acc, st, c.w[j], c, j);
    } else {
#pragma unroll
        for (int j = 0; j < 8; j++) {
            if (j < kv) a32_step<FMT, TN, BF>(F, LP, acc, st, c.w[j], c, j);
        }
    }
}

// Per-warp ring of A32_STAGES chunks in shared memory, filled with cp.async:
// chunk c + A32_STAGES - 1 is in flight while chunk c is consumed.  A stage is
// the 8 x 32 weights of the warp's row block ([k][row], as in global memory)
// and the 8 values of each of its TN tokens.  Needs 16-byte aligned weight
// rows (M * size % 16 == 0) and token rows (K * size % 16 == 0).
constexpr int A32_STAGES = 4;
template <int FMT, int TN>
struct a32_ring {
    using E = typename a32_fmt<FMT>::elem;
    static constexpr int es     = (int) sizeof(E);
    static constexpr int wbytes = 8 * 32 * es;
    static constexpr int stage  = wbytes + TN * 8 * es;
    static constexpr int warp_bytes = A32_STAGES * stage;
    static constexpr int table  = a32_kind<FMT>() == A32_FLAT ? k32f_words * 4 : 0;   // flat image bytes
    static constexpr int smem   = table + (a32_threads(FMT, true) / 32) * warp_bytes;

    // issue chunk k0 of the row block starting at row m0 (wb: the slice's k-major weights)
    __device__ static __forceinline__ void issue(unsigned char * st, const E * __restrict__ wb, const E * const (&xt)[TN],
                                                 int64_t m0, int64_t k0, int64_t K, int64_t M, int lane) {
        constexpr int per_k = 32 * es / 16;              // 16-byte pieces per weight row of the block
#pragma unroll
        for (int p = lane; p < 8 * per_k; p += 32) {
            const int     k = p / per_k, q = p % per_k;
            const int64_t kk = k0 + k, mm = m0 + q * (16 / es);
            const bool    ok = kk < K && mm < M;          // M % (16 / es) == 0: pieces are whole
            cp_async16_zfill(st + k * 32 * es + q * 16, ok ? (const void *) (wb + kk * M + mm) : (const void *) wb,
                             ok ? 16 : 0);
        }
        constexpr int per_t = 8 * es / 16;
        if (lane < TN * per_t) {
            const int     t = lane / per_t, q = lane % per_t;
            const int64_t kk = k0 + q * (16 / es);
            const bool    ok = kk < K;
            cp_async16_zfill(st + wbytes + t * 8 * es + q * 16, ok ? (const void *) (xt[t] + kk) : (const void *) xt[t],
                             ok ? 16 : 0);
        }
    }
    __device__ static __forceinline__ void read(a32_chunk<FMT, TN> & c, const unsigned char * st, int lane) {
        const E * ws = reinterpret_cast<const E *>(st);
#pragma unroll
        for (int j = 0; j < 8; j++) c.w[j] = ws[j * 32 + lane];
#pragma unroll
        for (int t = 0; t < TN; t++) {
#pragma unroll
            for (int v = 0; v < a32_fmt<FMT>::xvec; v++)
                c.x[t][v] = reinterpret_cast<const uint4 *>(st + wbytes + t * 8 * es)[v];
        }
    }
};

template <int FMT, int TN, bool OUT_F32, bool RING>
__global__ void __launch_bounds__(a32_threads(FMT, RING), 1)
k_mul_mat_a32(dev_tables T, const typename a32_fmt<FMT>::elem * __restrict__ W,
              const typename a32_fmt<FMT>::elem * __restrict__ X, void * __restrict__ dst, int64_t K, int64_t M,
              int64_t N, int64_t ne02, int64_t ne12, int64_t r2, int64_t r3, int64_t nz, uint32_t monte_seed,
              int vecx, int lat_sel, peer_out_dev peers) {
    using E  = typename a32_fmt<FMT>::elem;
    using OP = a32_fmt<FMT>;
    using RG = a32_ring<FMT, TN>;
    constexpr int KIND = a32_kind<FMT>();
    extern __shared__ __align__(16) int32_t F[];
    constexpr int NT = a32_threads(FMT, RING);
    if constexpr (KIND == A32_FLAT) {
        stage_async(F, T.flat32, k32f_words * 4);          // read-only tables: before the wait
        cp_async_commit();
        cp_async_wait<0>();
        __syncthreads();
    }
    pdl_entry();
    const int32_t * LP = T.lpvip_db;

    const int     lane = threadIdx.x & 31;
    unsigned char * ring = reinterpret_cast<unsigned char *>(F) + RG::table + (threadIdx.x >> 5) * RG::warp_bytes;
    const int64_t RB = (M + 31) / 32, TG = (N + TN - 1) / TN;
    const int64_t units  = nz * RB * TG;
    const int64_t nwarps = (int64_t) gridDim.x * (NT / 32);
    const int64_t nchunks = (K + 7) / 8;
    const bool    lat = units <= nwarps;                 // one round: chain latency bounds the time
    for (int64_t u = (int64_t) (threadIdx.x >> 5) * gridDim.x + blockIdx.x; u < units; u += nwarps) {
        const int64_t tg = u % TG, rest = u / TG, rb = rest % RB, z = rest / RB;
        const int64_t i12 = z % ne12, i13 = z / ne12;
        const int64_t m0 = rb * 32, m = m0 + lane;
        const E * wb = W + ((i13 / r3) * ne02 + i12 / r2) * K * M;
        const E * xt[TN];
#pragma unroll
        for (int t = 0; t < TN; t++) {
            const int64_t n = tg * TN + t;
            xt[t] = X + (z * N + (n < N ? n : N - 1)) * K;
        }
        uint32_t acc[TN], st[TN];
#pragma unroll
        for (int t = 0; t < TN; t++) {
            acc[t] = 0;
            st[t]  = 0;
            if constexpr (KIND == A32_MBL) {
                // the chain of output (z, m, n) starts (its index in the CPU's loop
                // order z, m, n) * (K - 1) draws after the seed
                const int64_t mm = m < M ? m : M - 1, nn = imin64(tg * TN + t, N - 1);
                const unsigned long long out = ((unsigned long long) z * (unsigned long long) M + (unsigned long long) mm) *
                                               (unsigned long long) N + (unsigned long long) nn;
                if (K > 1) st[t] = lfsr_jump(T, monte_seed, out * (unsigned long long) (K - 1));
            }
        }
        if (K > 0) {
            a32_chunk<FMT, TN> cur;
            if constexpr (RING) {
#pragma unroll
                for (int s = 0; s < A32_STAGES - 1; s++) {
                    if (s < nchunks) RG::issue(ring + s * RG::stage, wb, xt, m0, s * 8, K, M, lane);
                    cp_async_commit();
                }
                for (int64_t c = 0; c < nchunks; c++) {
                    cp_async_wait<A32_STAGES - 2>();
                    __syncwarp();                       // every lane's copies of chunk c landed
                    const int64_t nx = c + A32_STAGES - 1;   // refills the stage chunk c - 1 used
                    if (nx < nchunks) RG::issue(ring + (int) (nx % A32_STAGES) * RG::stage, wb, xt, m0, nx * 8, K, M, lane);
                    cp_async_commit();
                    const unsigned char * sg = ring + (int) (c % A32_STAGES) * RG::stage;
                    if (lat) {                           // few units: all 8 steps unrolled, operands in registers
                        RG::read(cur, sg, lane);
                        if (lat_sel) a32_steps<FMT, TN, true>(F, LP, cur, acc, st, c == 0, K - c * 8);
                        else         a32_steps<FMT, TN, false>(F, LP, cur, acc, st, c == 0, K - c * 8);
                        continue;
                    }
                    const E * ws = reinterpret_cast<const E *>(sg) + lane;
                    const E * xs = reinterpret_cast<const E *>(sg + RG::wbytes);
                    int j = 0;
                    if (c == 0) {
#pragma unroll
                        for (int t = 0; t < TN; t++) acc[t] = OP::term(ws[0], xs[t * 8]);
                        j = 1;
                    }
                    const int kv = (int) imin64(8, K - c * 8);
#pragma unroll 2
                    for (; j < kv; j++) {
                        uint32_t x[TN];
#pragma unroll
                        for (int t = 0; t < TN; t++) x[t] = xs[t * 8 + j];
                        a32_step_x<FMT, TN>(F, LP, acc, st, ws[j * 32], x);
                    }
                }
                cp_async_wait<0>();
                __syncwarp();                           // the ring is free for the next unit
            } else {
                // registers hold chunk c + 1 while chunk c runs; the weights of chunk
                // c + A32_L2PF are prefetched into L2 so that those loads hit there
                // (a lane's 8 steps are shorter than a DRAM miss in the latency regime)
                const E * wl = wb + (m < M ? m : M - 1);
                a32_chunk<FMT, TN> nxt;
                for (int64_t c = 1; c < A32_L2PF && c < nchunks; c++) a32_prefetch_l2<FMT>(wl, c * 8, K, M);
                a32_load<FMT, TN>(cur, wl, xt, 0, K, M, vecx != 0);
                for (int64_t c = 0; c < nchunks; c++) {
                    if (c + A32_L2PF < nchunks) a32_prefetch_l2<FMT>(wl, (c + A32_L2PF) * 8, K, M);
                    if (c + 1 < nchunks) a32_load<FMT, TN>(nxt, wl, xt, (c + 1) * 8, K, M, vecx != 0);
                    a32_steps<FMT, TN>(F, LP, cur, acc, st, c == 0, K - c * 8);
                    cur = nxt;
                }
            }
        }
        if (m < M) {
#pragma unroll
            for (int t = 0; t < TN; t++) {
                const int64_t n = tg * TN + t;
                if (n >= N) continue;
                const uint32_t v = K == 0 ? 0u : OP::finish(acc[t]);
                if (!OUT_F32 && peers.n > 0) {             // the fused all-gather: codes into every peer's buffer
                    const int64_t o = (z * N + n) * peers.ld + peers.off + m;
                    for (int p = 0; p < peers.n; p++) reinterpret_cast<E *>(peers.ptrs[p])[o] = (E) v;
                } else {
                    OP::store(T, dst, (z * N + n) * M + m, v, OUT_F32);
                }
            }
        }
    }
}

// A chain acc = add(acc, q[i * 32]), i in [i0, n) -- one lane's column of a
// [step][lane] ring in shared memory -- its terms loaded a batch ahead of the
// additions, so a step's dependent path is the addition alone.
template <typename ADD>
__device__ __forceinline__ uint32_t chain_smem_strided(const uint32_t * q, int i0, int n, uint32_t acc, ADD add) {
    constexpr int U = 8;
    uint32_t cur[U];
    int i = i0;
#pragma unroll
    for (int u = 0; u < U; u++) cur[u] = i + u < n ? q[(i + u) * 32] : 0u;
    for (; i + U <= n; i += U) {
        uint32_t nxt[U];
#pragma unroll
        for (int u = 0; u < U; u++) nxt[u] = i + U + u < n ? q[(i + U + u) * 32] : 0u;
#pragma unroll
        for (int u = 0; u < U; u++) acc = add(acc, cur[u]);
#pragma unroll
        for (int u = 0; u < U; u++) cur[u] = nxt[u];
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
        if (i + u < n) acc = add(acc, cur[u]);
    }
    return acc;
}

// ============== latency mat-vec over the flat xlns32 addition ===============
// Up to LV_MAX_PAIRS units (32 weight rows x 1 token each) per SM -- the
// decode's mat-vecs in sum32 and xlns32, the one- and few-token products of
// large ones -- the time is the chain: K dependent additions per lane.  Two
// warps per unit, np units per block sharing the 129 KB addition image.  A
// unit's producer warp streams its 32 rows' weights and the token's values and
// writes the products into its own ring of LV_STAGES stages of LV_STEPS steps
// ([step][lane], one word each); its chain warp reads a product (a batch
// ahead) and adds it (add32f_sel), so the chain warp's instruction stream is
// the addition alone.  Stage s is handed over with named barriers counted over
// the whole block, so the block's units move in step: id 1 + s (every
// producer wrote stage s) and 1 + LV_STAGES + s (every chain warp is done with
// it; arrived only for stages the producers refill, so each wait has its
// arrivals).  Units past the end run on the last unit's operands and store
// nothing.  Same bits as k_mul_mat_a32.
constexpr int LV_STEPS = 32, LV_STAGES = 4, LV_MAX_PAIRS = 6;
constexpr int LV_RING_BYTES = LV_STAGES * LV_STEPS * 32 * 4;     // per unit
template <int FMT, bool OUT_F32>
__global__ void __launch_bounds__(64 * LV_MAX_PAIRS, 1)
k_mat_vec_lat(dev_tables T, const typename a32_fmt<FMT>::elem * __restrict__ W,
              const typename a32_fmt<FMT>::elem * __restrict__ X, void * __restrict__ dst, int64_t K, int64_t M,
              int64_t N, int64_t ne02, int64_t ne12, int64_t r2, int64_t r3, int64_t units, peer_out_dev peers) {
    using E  = typename a32_fmt<FMT>::elem;
    using OP = a32_fmt<FMT>;
    extern __shared__ __align__(16) int32_t F[];
    stage_async(F, T.flat32, k32f_words * 4);              // read-only tables: before the wait
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    pdl_entry();
    const int     lane = threadIdx.x & 31, warp = threadIdx.x >> 5, pair = warp >> 1;
    const int     np = (int) (blockDim.x >> 6), nthr = (int) blockDim.x;
    uint32_t * ring = reinterpret_cast<uint32_t *>(F + k32f_words) + pair * (LV_RING_BYTES / 4);
    const int64_t RB = (M + 31) / 32;
    const int64_t u0 = (int64_t) blockIdx.x * np + pair;
    const bool    valid = u0 < units;
    const int64_t u = valid ? u0 : units - 1;
    const int64_t n = u % N, rest = u / N, rb = rest % RB, z = rest / RB;
    const int64_t i12 = z % ne12, i13 = z / ne12;
    const int64_t m = rb * 32 + lane;
    const E * wb = W + ((i13 / r3) * ne02 + i12 / r2) * K * M;
    const E * xt = X + (z * N + n) * K;
    const int64_t nch = (K + LV_STEPS - 1) / LV_STEPS;
    if (warp & 1) {
        // producer: the products of chunk c into stage c % LV_STAGES
        const E * wl = wb + (m < M ? m : M - 1);
        for (int64_t c = 0; c < nch; c++) {
            const int sidx = (int) (c % LV_STAGES);
            if (c >= LV_STAGES) asm volatile("bar.sync %0, %1;\n" ::"r"(1 + LV_STAGES + sidx), "r"(nthr) : "memory");
            const int64_t k0 = c * LV_STEPS;
            uint32_t * st = ring + sidx * LV_STEPS * 32 + lane;
            uint32_t w[LV_STEPS];
#pragma unroll
            for (int j = 0; j < LV_STEPS; j++) w[j] = k0 + j < K ? (uint32_t) __ldg(wl + (k0 + j) * M) : 0u;
#pragma unroll
            for (int j = 0; j < LV_STEPS; j++) {
                const uint32_t x = k0 + j < K ? (uint32_t) __ldg(xt + k0 + j) : 0u;
                st[j * 32] = OP::term(w[j], x);
            }
            asm volatile("bar.arrive %0, %1;\n" ::"r"(1 + sidx), "r"(nthr) : "memory");
        }
        return;
    }
    // the chain warp
    uint32_t acc = 0;
    for (int64_t c = 0; c < nch; c++) {
        const int sidx = (int) (c % LV_STAGES);
        asm volatile("bar.sync %0, %1;\n" ::"r"(1 + sidx), "r"(nthr) : "memory");
        const uint32_t * q = ring + sidx * LV_STEPS * 32 + lane;
        const int kv = (int) imin64(LV_STEPS, K - c * LV_STEPS);
        if (c == 0) acc = q[0];
        acc = chain_smem_strided(q, c == 0 ? 1 : 0, kv, acc, [&](uint32_t a, uint32_t t) { return add32f_sel(F, a, t); });
        if (c + LV_STAGES < nch) asm volatile("bar.arrive %0, %1;\n" ::"r"(1 + LV_STAGES + sidx), "r"(nthr) : "memory");
    }
    if (valid && m < M) {
        const uint32_t v = K == 0 ? 0u : OP::finish(acc);
        if (!OUT_F32 && peers.n > 0) {                     // the fused all-gather: codes into every peer's buffer
            const int64_t o = (z * N + n) * peers.ld + peers.off + m;
            for (int p = 0; p < peers.n; p++) reinterpret_cast<E *>(peers.ptrs[p])[o] = (E) v;
        } else {
            OP::store(T, dst, (z * N + n) * M + m, v, OUT_F32);
        }
    }
}

// ============================ MUL_MAT_ID ===================================
// The expert-selected product (lns-backend/src/lns-ops.cpp:394-462): output
// (t, s, m) is the chain over k of w[e][k][m] * x[t][s % ne11][k] with e the
// id of slot s of token t.  Units of work are (slot z = t * n_used + s, block
// of 32 rows), one chain per lane, dealt to warps round-robin; the weights of
// a warp's rows are one coalesced 64- or 128-byte row per k (k-major expert
// slices), the activation value is the same for the warp (a broadcast load).
// The reduction is the build's policy with its tables in shared memory: the
// flat xlns32 image (xlns32, sum32), or the packed xlns16 table (and the Monte
// fine tables); LPVIP's singular branch reads its global table.  Monte chain
// (t, s, m) starts ((t * n_used + s) * M + m) * (K - 1) draws after the seed,
// the CPU loop order.  An id out of range gives the zero code and is counted.
__device__ unsigned long long g_bad_ids;      // one per device, as every module variable

template <int FMT> __host__ __device__ constexpr bool mmid_flat() { return FMT == 32 || k_mode == M_SUM32; }
template <int FMT> __host__ __device__ constexpr int  mmid_smem() {
    return mmid_flat<FMT>() ? k32f_words * 4 : k16_tab_bytes16 + (k_mode == M_MONTE ? 2 * k16_monte_n * 2 : 0);
}

template <int FMT, bool OUT_F32>
__global__ void __launch_bounds__(256)
k_mul_mat_id(dev_tables T, const typename a32_fmt<FMT>::elem * __restrict__ W,
             const typename a32_fmt<FMT>::elem * __restrict__ X, const int32_t * __restrict__ ids,
             void * __restrict__ dst, int64_t K, int64_t M, int64_t n_expert, int64_t ne11, int64_t n_used,
             int64_t n_tokens, int64_t ids_stride, uint32_t monte_seed) {
    pdl_entry();
    using E = typename a32_fmt<FMT>::elem;
    extern __shared__ __align__(16) unsigned char mmid_sm[];
    int32_t * F    = reinterpret_cast<int32_t *>(mmid_sm);
    int16_t * tab  = reinterpret_cast<int16_t *>(mmid_sm);
    int16_t * fine = reinterpret_cast<int16_t *>(mmid_sm + k16_tab_bytes16);
    if constexpr (mmid_flat<FMT>()) {
        stage_async(F, T.flat32, k32f_words * 4);
    } else {
        stage_async(tab, T.sbdb16, k16_tab_bytes16);
        if constexpr (k_mode == M_MONTE) stage_async(fine, T.monte16, 2 * k16_monte_n * 2);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    const int     lane = threadIdx.x & 31;
    const int64_t RB = (M + 31) / 32, units = n_tokens * n_used * RB;
    const int64_t nwarps = (int64_t) gridDim.x * (blockDim.x / 32);
    for (int64_t u = (int64_t) (threadIdx.x >> 5) * gridDim.x + blockIdx.x; u < units; u += nwarps) {
        const int64_t z = u / RB, rb = u % RB, t = z / n_used, s = z % n_used;
        const int64_t m = rb * 32 + lane;
        const int32_t e = __ldg(ids + t * ids_stride + s);
        uint32_t out = 0u;                              // the zero code
        if (e < 0 || e >= n_expert) {
            if (lane == 0 && rb == 0) atomicAdd(&g_bad_ids, 1ull);
        } else if (K > 0) {
            const E * wl = W + (int64_t) e * K * M + (m < M ? m : M - 1);
            const E * xr = X + (t * ne11 + s % ne11) * K;
            uint32_t st = 0u;
            if constexpr (FMT == 16 && k_stochastic)
                st = lfsr_jump(T, monte_seed, (unsigned long long) (z * M + (m < M ? m : M - 1)) * (unsigned long long) (K - 1));
            red16 R{ &T, tab, fine };
            uint32_t acc = 0u;
            for (int64_t k0 = 0; k0 < K; k0 += 8) {
                uint32_t w8[8], x8[8];
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const bool in = k0 + j < K;
                    w8[j] = in ? (uint32_t) __ldg(wl + (k0 + j) * M) : 0u;
                    x8[j] = in ? (uint32_t) __ldg(xr + k0 + j) : 0u;
                }
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const int64_t k = k0 + j;
                    if (k >= K) break;
                    if constexpr (FMT == 32) {
                        const uint32_t p = mul32(w8[j], x8[j]);
                        acc = k == 0 ? p : add32f_sel(F, acc, p);
                    } else if constexpr (k_mode == M_SUM32) {
                        const uint32_t p = mul16(w8[j], x8[j]) << 16;
                        acc = k == 0 ? p : add32f_sel(F, acc, p);
                    } else {
                        const uint32_t p = mul16(w8[j], x8[j]);
                        acc = k == 0 ? R.from(p) : R.add(acc, p, st);
                    }
                }
            }
            out = FMT == 16 ? R.finish(acc) : acc;
        }
        if (m < M) a32_fmt<FMT>::store(T, dst, z * M + m, out, OUT_F32);
    }
}

// ============================ RMS_NORM =====================================
// Block = up to 32 rows (rpb).  Each lane runs its row's sum-of-squares chain
// (n additions from zero); the scaling pass is done by the whole block,
// coalesced.  In base and sum32 modes (NNCHAIN) the squares are first formed
// by the whole block into shared memory and the chain is the non-negative
// addition over a shared-memory table (padd16 / padd32f); the other modes
// run the general reduction policy.
constexpr bool NNCHAIN = k_mode == M_BASE || k_mode == M_SUM32;
constexpr int  NN_TAB  = k_mode == M_SUM32 ? k32f_sb_bytes16 : 0;   // sb knot bytes in dynamic smem
// xlns32 normalisers: always the non-negative chain over the sb knots, 4-byte terms
template <int FMT> __host__ __device__ constexpr int nn_tab() { return FMT == 32 ? k32f_sb_bytes16 : NN_TAB; }
template <int FMT> __host__ __device__ constexpr int nn_term_bytes() { return FMT == 32 ? 4 : 2; }
// Row pitch (terms) of a normaliser block's shared terms: each lane runs one
// row's chain, so the rows must start in different banks -- an odd number of
// words apart (a pitch of n itself puts every lane of a 512- or 576-term row
// in one bank: a 32-way conflict on every step).
__host__ __device__ inline int64_t nn_pitch(int64_t n, int term_bytes) {
    if (term_bytes == 4) return n | 1;
    int64_t p = (n + 1) & ~(int64_t) 1;
    return ((p >> 1) & 1) ? p : p + 2;
}

// the sb knots of the flat xlns32 image (all a non-negative chain reads) into
// shared memory, asynchronously (committed with the block's other copies)
template <int FMT = 16>
__device__ __forceinline__ void nn_tables(const dev_tables & T, int32_t * F) {
    if constexpr (FMT == 32 || k_mode == M_SUM32) stage_async(F, T.flat32, k32f_sb_bytes16);
}
// the xlns16 tables a normaliser block keeps in shared memory (sbdb16, and the
// Monte fine tables in monte mode), asynchronously
__device__ __forceinline__ void norm_tables(const dev_tables & T, int16_t * tab, int16_t * fine) {
    stage_async(tab, T.sbdb16, k16_tab_bytes16);
    if constexpr (k_mode == M_MONTE) stage_async(fine, T.monte16, 2 * k16_monte_n * 2);
}
// A chain acc = add(acc, q[i]), i in [i0, n), over terms in shared memory: the
// terms are loaded a batch ahead of the additions (they do not depend on the
// chain), so a step's dependent path is the addition alone.
template <typename E, typename ADD>
__device__ __forceinline__ uint32_t chain_smem(const E * q, int i0, int n, uint32_t acc, ADD add) {
    constexpr int U = 8;
    uint32_t cur[U];
    int i = i0;
#pragma unroll
    for (int u = 0; u < U; u++) cur[u] = i + u < n ? (uint32_t) q[i + u] : 0u;
    for (; i + U <= n; i += U) {
        uint32_t nxt[U];
#pragma unroll
        for (int u = 0; u < U; u++) nxt[u] = i + U + u < n ? (uint32_t) q[i + U + u] : 0u;
#pragma unroll
        for (int u = 0; u < U; u++) acc = add(acc, cur[u]);
#pragma unroll
        for (int u = 0; u < U; u++) cur[u] = nxt[u];
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
        if (i + u < n) acc = add(acc, cur[u]);
    }
    return acc;
}

// one non-negative addition of the mode: accumulator form (sum32: acc32) and term code
__device__ __forceinline__ uint32_t nn_add(const int32_t * F, const int16_t * tab, uint32_t acc, uint32_t t) {
    if constexpr (k_mode == M_SUM32) return padd32f(F, acc, t << 16);
    else                             return padd16(acc, t, tab);
}

// FUSE: the decode graph's norm block in one kernel, each op boundary kept --
// x = src (+ res: the residual add, F32 out), rms_norm(x) (F32 out), times the
// norm weight nw (F32 out), to_lns -> dst codes; x_out (if given) gets x.
template <int FMT, bool IO_F32, bool FUSE = false>
__global__ void __launch_bounds__(256)
k_rms_norm(dev_tables T, const void * __restrict__ src, void * __restrict__ dst, int64_t ncols, int64_t nrows,
           uint32_t eps_l, uint32_t inv_n, uint32_t monte_seed, int rpb, int nn_ok,
           const float * __restrict__ res = nullptr, float * __restrict__ x_out = nullptr,
           const float * __restrict__ nw = nullptr) {
    __shared__ __align__(16) int16_t tab[k16_tab_bytes16 / 2];
    __shared__ __align__(16) int16_t fine[k_mode == M_MONTE ? 2 * k16_monte_n : 8];
    __shared__ uint32_t s_inv[32];
    extern __shared__ __align__(16) int32_t dyn[];          // NNCHAIN: [sb knots (sum32)][squares: rpb x ncols]
    constexpr bool NNC = FMT == 32 || NNCHAIN;
    const bool     NN  = NNC && nn_ok != 0;                 // the squares fit in shared memory
    if constexpr (FMT == 16) norm_tables(T, tab, fine);
    const int64_t row0 = (int64_t) blockIdx.x * rpb;
    const int64_t nr = imin64(rpb, nrows - row0);
    auto f2c = [&](float f) -> uint32_t { return FMT == 16 ? from_f32_16(T, f) : from_f32_32(T, f); };
    auto c2f = [&](uint32_t c) -> float { return FMT == 16 ? to_f32_16(T, c) : to_f32_32(T, c); };
    auto xval = [&](int64_t idx) -> float {              // x: src, or the residual add's F32 result
        const float f = static_cast<const float *>(src)[idx];
        if (!FUSE || res == nullptr) return f;
        const uint32_t a = f2c(f), b = f2c(res[idx]);
        return c2f(FMT == 16 ? add16(a, b, tab) : add32f(T.flat32, a, b));
    };
    auto load = [&](int64_t idx) -> uint32_t {
        if constexpr (IO_F32) {
            return f2c(xval(idx));
        } else {
            return FMT == 16 ? (uint32_t) static_cast<const uint16_t *>(src)[idx] : static_cast<const uint32_t *>(src)[idx];
        }
    };
    uint16_t * sq   = reinterpret_cast<uint16_t *>(reinterpret_cast<unsigned char *>(dyn) + nn_tab<FMT>());
    uint32_t * sq32 = reinterpret_cast<uint32_t *>(reinterpret_cast<unsigned char *>(dyn) + nn_tab<FMT>());
    if (NN) nn_tables<FMT>(T, dyn);
    pdl_entry();                                         // read-only tables above: before the wait
    if constexpr (FUSE) {                                // the residual add reads the packed table
        cp_async_commit();
        cp_async_wait<0>();
        __syncthreads();
    }
    const int64_t P = nn_pitch(ncols, nn_term_bytes<FMT>());   // row pitch of the squares
    if (NN) {
        auto square = [&](int64_t e, uint32_t v) {
            const int r = (int) e / (int) ncols;         // nr * ncols fits the block's shared memory
            const int64_t o = r * P + ((int) e - r * (int) ncols);
            if constexpr (FMT == 16) sq[o] = (uint16_t) mul16(v, v);
            else                     sq32[o] = mul32(v, v);
        };
        const int64_t tot = nr * ncols;
        if (FUSE && x_out != nullptr) {
            // x once (the scaling pass reads it back); a thread's values in
            // batches, so their chains of table lookups interleave
            constexpr int U = 4;
            for (int64_t e0 = threadIdx.x; e0 < tot; e0 += (int64_t) blockDim.x * U) {
                float xf[U];
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int64_t e = e0 + (int64_t) u * blockDim.x;
                    xf[u] = e < tot ? xval(row0 * ncols + e) : 0.0f;
                }
                uint32_t c[U];
#pragma unroll
                for (int u = 0; u < U; u++) c[u] = f2c(xf[u]);
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int64_t e = e0 + (int64_t) u * blockDim.x;
                    if (e < tot) {
                        x_out[row0 * ncols + e] = xf[u];
                        square(e, c[u]);
                    }
                }
            }
        } else {
            constexpr int U = 8;                         // loads in flight per thread
            const int64_t step = (int64_t) blockDim.x * U;
            int64_t e0 = 0;
            for (; e0 + step <= tot; e0 += step) {
                uint32_t v[U];
#pragma unroll
                for (int u = 0; u < U; u++) v[u] = load(row0 * ncols + e0 + u * blockDim.x + threadIdx.x);
#pragma unroll
                for (int u = 0; u < U; u++) square(e0 + u * blockDim.x + threadIdx.x, v[u]);
            }
            for (int64_t e = e0 + threadIdx.x; e < tot; e += blockDim.x) square(e, load(row0 * ncols + e));
        }
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    if (threadIdx.x < nr) {
        const int64_t row = row0 + threadIdx.x;
        if (NN && FMT == 32) {
            const uint32_t * q = sq32 + threadIdx.x * P;
            uint32_t acc = 0u;
            acc = chain_smem(q, 0, (int) ncols, acc, [&](uint32_t a, uint32_t t) { return padd32f(dyn, a, t); });
            const uint32_t mean = mul32(acc, inv_n);
            s_inv[threadIdx.x] = recip32(sqrt32(add32(T, mean, eps_l)));
        } else if (NN) {
            const uint16_t * q = sq + threadIdx.x * P;
            uint32_t acc = 0u;                              // the zero code (acc32 0 in sum32)
            acc = chain_smem(q, 0, (int) ncols, acc, [&](uint32_t a, uint32_t t) { return nn_add(dyn, tab, a, t); });
            red16 R{ &T, tab, fine };
            const uint32_t mean = mul16(R.finish(acc), inv_n);
            s_inv[threadIdx.x] = recip16(sqrt16(add16(mean, eps_l, tab)));
        } else if constexpr (FMT == 16) {
            red16 R{ &T, tab, fine };
            uint32_t st = k_stochastic ? lfsr_jump(T, monte_seed, (unsigned long long) row * (unsigned long long) ncols) : 0u;
            uint32_t acc = R.from(0u);
            for (int64_t i = 0; i < ncols; i++) {
                const uint32_t v = load(row * ncols + i);
                acc = R.add(acc, mul16(v, v), st);
            }
            const uint32_t mean = mul16(R.finish(acc), inv_n);
            s_inv[threadIdx.x] = recip16(sqrt16(add16(mean, eps_l, tab)));
        } else {
            uint32_t acc = 0u;
            for (int64_t i = 0; i < ncols; i++) {
                const uint32_t v = load(row * ncols + i);
                acc = add32(T, acc, mul32(v, v));
            }
            const uint32_t mean = mul32(acc, inv_n);
            s_inv[threadIdx.x] = recip32(sqrt32(add32(T, mean, eps_l)));
        }
    }
    __syncthreads();
    if constexpr (FUSE) {
        if (x_out != nullptr && NN) {
            // the fused block's scaling pass in batches (the x values were
            // written by the squares pass of this block)
            constexpr int U = 4;
            const int64_t tot = nr * ncols;
            for (int64_t e0 = threadIdx.x; e0 < tot; e0 += (int64_t) blockDim.x * U) {
                float yf[U];
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int64_t e = e0 + (int64_t) u * blockDim.x;
                    const int64_t ee = e < tot ? e : tot - 1;
                    const int64_t r = ee / ncols;
                    const int64_t idx = (row0 + r) * ncols + (ee - r * ncols);
                    const uint32_t inv = s_inv[r];
                    const uint32_t v = f2c(x_out[idx]);
                    yf[u] = c2f(FMT == 16 ? mul16(v, inv) : mul32(v, inv));
                    if (nw != nullptr) {
                        const uint32_t yc = f2c(yf[u]), wc = f2c(nw[ee - r * ncols]);
                        yf[u] = c2f(FMT == 16 ? mul16(yc, wc) : mul32(yc, wc));
                    }
                }
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int64_t e = e0 + (int64_t) u * blockDim.x;
                    if (e < tot) {
                        const int64_t r = e / ncols;
                        const int64_t idx = (row0 + r) * ncols + (e - r * ncols);
                        if constexpr (FMT == 16) static_cast<uint16_t *>(dst)[idx] = (uint16_t) f2c(yf[u]);
                        else                     static_cast<uint32_t *>(dst)[idx] = f2c(yf[u]);
                    }
                }
            }
            return;
        }
    }
    for (int64_t e = threadIdx.x; e < nr * ncols; e += blockDim.x) {
        const int64_t r = e / ncols;
        const int64_t idx = (row0 + r) * ncols + (e - r * ncols);
        const uint32_t inv = s_inv[r];
        if constexpr (FUSE) {
            float xf;
            if (x_out != nullptr && NN) {
                xf = x_out[idx];                         // written by the squares pass (same block)
            } else {
                xf = xval(idx);
                if (x_out != nullptr) x_out[idx] = xf;
            }
            const uint32_t v = f2c(xf);
            float yf = c2f(FMT == 16 ? mul16(v, inv) : mul32(v, inv));
            if (nw != nullptr) {
                const uint32_t yc = f2c(yf), wc = f2c(nw[e - r * ncols]);
                yf = c2f(FMT == 16 ? mul16(yc, wc) : mul32(yc, wc));
            }
            if constexpr (FMT == 16) static_cast<uint16_t *>(dst)[idx] = (uint16_t) f2c(yf);
            else                     static_cast<uint32_t *>(dst)[idx] = f2c(yf);
            continue;
        }
        const uint32_t v = load(idx);
        if constexpr (FMT == 16) {
            const uint32_t y = mul16(v, inv);
            if constexpr (IO_F32) static_cast<float *>(dst)[idx] = to_f32_16(T, y);
            else                  static_cast<uint16_t *>(dst)[idx] = (uint16_t) y;
        } else {
            const uint32_t y = mul32(v, inv);
            if constexpr (IO_F32) static_cast<float *>(dst)[idx] = to_f32_32(T, y);
            else                  static_cast<uint32_t *>(dst)[idx] = y;
        }
    }
}

// ============================ SOFT_MAX =====================================
// Block = up to 32 rows, SM_THREADS threads.  Pass 1 (whole block): scale, mask, row max;
// pass 2 (whole block): c = exp(v - max); pass 3 (one lane per row): the
// normaliser chain over c in element order; pass 4 (whole block): dst = c /
// total.  When the block's rows fit in shared memory (ST, every mode) pass 1
// loads each logit once, eight loads in flight per lane, and keeps the scaled,
// masked value there; pass 2 rewrites it in place with c, and passes 3 and 4
// read c there.  Otherwise c goes through the work buffer in global memory.
constexpr int SM_THREADS = 512;
template <int FMT, bool IO_F32>
__global__ void __launch_bounds__(SM_THREADS)
k_soft_max(dev_tables T, const void * __restrict__ src, lnsb_shape4 s, const void * __restrict__ mask,
           lnsb_shape4 ms, uint32_t scale_l, void * __restrict__ dst, void * __restrict__ work,
           uint32_t monte_seed, int rpb, int nn_ok) {
    extern __shared__ __align__(16) int32_t dyn[];          // [sb knots (xlns32, sum32)][terms: rpb x pitch]
    __shared__ __align__(16) int16_t tab[k16_tab_bytes16 / 2];
    __shared__ __align__(16) int16_t fine[k_mode == M_MONTE ? 2 * k16_monte_n : 8];
    __shared__ uint32_t s_max[32][4];
    __shared__ uint32_t s_tot[32];
    constexpr uint32_t NEG_INF = FMT == 16 ? 0xFFFFu : 0xFFFFFFFFu;
    const bool ST = nn_ok != 0;                             // the rows' terms stay in shared memory
    const bool NN = (FMT == 32 || NNCHAIN) && ST;
    if constexpr (FMT == 16) norm_tables(T, tab, fine);
    if (ST) nn_tables<FMT>(T, dyn);
    cp_async_commit();
    pdl_entry();                                            // read-only tables above: before the wait
    cp_async_wait<0>();
    __syncthreads();
    const int64_t n = s.ne[0];
    const int64_t nrows = s.ne[1] * s.ne[2] * s.ne[3];
    const int64_t row0 = (int64_t) blockIdx.x * rpb;
    const int64_t nr = imin64(rpb, nrows - row0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;

    auto ld = [&](const void * p, int64_t idx) -> uint32_t {
        return FMT == 16 ? (uint32_t) static_cast<const uint16_t *>(p)[idx] : static_cast<const uint32_t *>(p)[idx];
    };
    auto mask_row = [&](int64_t row) -> int64_t {           // the mask row a row reads (dims 2, 3 broadcast)
        const int64_t i1 = row % s.ne[1], i2 = (row / s.ne[1]) % s.ne[2], i3 = row / (s.ne[1] * s.ne[2]);
        return ((i3 % ms.ne[3]) * ms.ne[2] + i2 % ms.ne[2]) * ms.ne[1] + i1;
    };
    // a logit in two parts, so a batch's loads are all in flight before any is used:
    // the raw words (the source value, the mask value; IO_F32: float bits), then
    // the scaled, masked code
    auto rawv = [&](int64_t row, int64_t i) -> uint32_t {
        if constexpr (IO_F32) return __float_as_uint(static_cast<const float *>(src)[row * n + i]);
        else                  return ld(src, row * n + i);
    };
    auto rawm = [&](int64_t mrow, int64_t i) -> uint32_t {
        if (mask == nullptr) return 0u;
        if constexpr (IO_F32) return __float_as_uint(static_cast<const float *>(mask)[mrow * n + i]);
        else                  return ld(mask, mrow * n + i);
    };
    auto cook = [&](uint32_t rv, uint32_t rm) -> uint32_t {
        uint32_t v;
        if constexpr (IO_F32) {
            const float f = __uint_as_float(rv);
            v = FMT == 16 ? from_f32_16(T, f) : from_f32_32(T, f);
        } else {
            v = rv;
        }
        if (v != NEG_INF) {
            v = FMT == 16 ? mul16(v, scale_l) : mul32(v, scale_l);
            if (mask != nullptr) {
                uint32_t mk;
                if constexpr (IO_F32) {
                    const float mf = __uint_as_float(rm);
                    mk = mf <= -3.0e38f ? NEG_INF : (FMT == 16 ? from_f32_16(T, mf) : from_f32_32(T, mf));
                } else {
                    mk = rm;
                }
                if (mk == NEG_INF) v = NEG_INF;
                else if (FMT == 16 ? !is_zero16(mk) : !is_zero32(mk)) v = FMT == 16 ? add16(v, mk, tab) : add32f(T.flat32, v, mk);
            }
        }
        return v;
    };
    auto value = [&](int64_t row, int64_t mrow, int64_t i) -> uint32_t { return cook(rawv(row, i), rawm(mrow, i)); };

    uint16_t * cs   = reinterpret_cast<uint16_t *>(reinterpret_cast<unsigned char *>(dyn) + nn_tab<FMT>());
    uint32_t * cs32 = reinterpret_cast<uint32_t *>(reinterpret_cast<unsigned char *>(dyn) + nn_tab<FMT>());
    const int64_t P = nn_pitch(n, nn_term_bytes<FMT>());       // row pitch of the shared terms
    auto put = [&](int r, int64_t i, uint32_t v) {
        if constexpr (FMT == 16) cs[r * P + i] = (uint16_t) v;
        else                     cs32[r * P + i] = v;
    };
    auto get = [&](int r, int64_t i) -> uint32_t { return FMT == 16 ? (uint32_t) cs[r * P + i] : cs32[r * P + i]; };
    constexpr int U = 8;                                     // loads in flight per lane

    // pass 1: row max (each warp takes rows warp, warp + nw, ...); ST: the values into shared memory
    for (int r = warp; r < nr; r += nw) {
        const int64_t row = row0 + r, mrow = mask != nullptr ? mask_row(row) : 0;
        uint32_t mx = NEG_INF;
        if (ST) {
            int64_t i0 = 0;
            for (; i0 + 32 * U <= n; i0 += 32 * U) {
                uint32_t v[U], m[U];
#pragma unroll
                for (int u = 0; u < U; u++) {
                    v[u] = rawv(row, i0 + u * 32 + lane);
                    m[u] = rawm(mrow, i0 + u * 32 + lane);
                }
#pragma unroll
                for (int u = 0; u < U; u++) v[u] = cook(v[u], m[u]);
#pragma unroll
                for (int u = 0; u < U; u++) {
                    put(r, i0 + u * 32 + lane, v[u]);
                    if (FMT == 16 ? gt16(v[u], mx) : gt32(v[u], mx)) mx = v[u];
                }
            }
            for (int64_t i = i0 + lane; i < n; i += 32) {
                const uint32_t v = value(row, mrow, i);
                put(r, i, v);
                if (FMT == 16 ? gt16(v, mx) : gt32(v, mx)) mx = v;
            }
        } else {
            for (int64_t i = lane; i < n; i += 32) {
                const uint32_t v = value(row, mrow, i);
                if (FMT == 16 ? gt16(v, mx) : gt32(v, mx)) mx = v;
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const uint32_t o = __shfl_xor_sync(0xFFFFFFFFu, mx, off);
            if (FMT == 16 ? gt16(o, mx) : gt32(o, mx)) mx = o;
        }
        if (lane == 0) s_max[r][0] = mx;
    }
    __syncthreads();
    // pass 2: c = exp(v - max), in place (ST) or into work
    auto expo = [&](uint32_t v, uint32_t mx) -> uint32_t {
        if constexpr (FMT == 16) return __ldg(T.exp16 + sub16(v, mx, tab));
        else                     return exp32(T, sub32(T, v, mx));
    };
    for (int r = warp; r < nr; r += nw) {
        const int64_t row = row0 + r;
        const uint32_t mx = s_max[r][0];
        if (ST) {
            int64_t i0 = 0;
            for (; i0 + 32 * U <= n; i0 += 32 * U) {
                uint32_t e[U];
#pragma unroll
                for (int u = 0; u < U; u++) e[u] = expo(get(r, i0 + u * 32 + lane), mx);
#pragma unroll
                for (int u = 0; u < U; u++) put(r, i0 + u * 32 + lane, e[u]);
            }
            for (int64_t i = i0 + lane; i < n; i += 32) put(r, i, expo(get(r, i), mx));
        } else {
            const int64_t mrow = mask != nullptr ? mask_row(row) : 0;
            for (int64_t i = lane; i < n; i += 32) {
                const uint32_t e = expo(value(row, mrow, i), mx);
                if constexpr (FMT == 16) static_cast<uint16_t *>(work)[row * n + i] = (uint16_t) e;
                else                     static_cast<uint32_t *>(work)[row * n + i] = e;
            }
        }
    }
    __syncthreads();
    // pass 3: the normaliser, one sequential chain per row (xlns16_sum order)
    if (threadIdx.x < nr) {
        const int r = threadIdx.x;
        const int64_t row = row0 + r;
        if (NN && FMT == 32) {
            const uint32_t * q = cs32 + r * P;
            uint32_t acc = q[0];
            acc = chain_smem(q, 1, (int) n, acc, [&](uint32_t a, uint32_t t) { return padd32f(dyn, a, t); });
            s_tot[r] = acc;
        } else if (NN) {
            const uint16_t * q = cs + r * P;
            red16 R{ &T, tab, fine };
            uint32_t acc = R.from(q[0]);
            acc = chain_smem(q, 1, (int) n, acc, [&](uint32_t a, uint32_t t) { return nn_add(dyn, tab, a, t); });
            s_tot[r] = R.finish(acc);
        } else if constexpr (FMT == 16) {
            red16 R{ &T, tab, fine };
            uint32_t st = k_stochastic ? lfsr_jump(T, monte_seed, (unsigned long long) row * (unsigned long long) (n - 1)) : 0u;
            auto term = [&](int64_t i) -> uint32_t { return ST ? get(r, i) : ld(work, row * n + i); };
            uint32_t acc = R.from(term(0));
            for (int64_t i = 1; i < n; i++) acc = R.add(acc, term(i), st);
            s_tot[r] = R.finish(acc);
        } else {
            uint32_t acc = ld(work, row * n);
            for (int64_t i = 1; i < n; i++) acc = add32(T, acc, ld(work, row * n + i));
            s_tot[r] = acc;
        }
    }
    __syncthreads();
    // pass 4: dst = c / total
    for (int r = warp; r < nr; r += nw) {
        const int64_t row = row0 + r;
        const uint32_t tot = s_tot[r];
        for (int64_t i = lane; i < n; i += 32) {
            const uint32_t cv = ST ? get(r, i) : ld(work, row * n + i);
            if constexpr (FMT == 16) {
                const uint32_t y = div16(cv, tot);
                if constexpr (IO_F32) static_cast<float *>(dst)[row * n + i] = to_f32_16(T, y);
                else                  static_cast<uint16_t *>(dst)[row * n + i] = (uint16_t) y;
            } else {
                const uint32_t y = div32(cv, tot);
                if constexpr (IO_F32) static_cast<float *>(dst)[row * n + i] = to_f32_32(T, y);
                else                  static_cast<uint32_t *>(dst)[row * n + i] = y;
            }
        }
    }
}

// ===================== decode attention, one query position =================
// One decode step's attention for one head in one CTA: what the model graph
// runs as F16 -> F32 K/V conversions, to_lns, mul_mat (kq), soft_max (scale,
// causal mask, normaliser), to_lns and mul_mat (kqv), with every op-boundary
// conversion kept (codes -> F32 -> codes between the ops), so the bits are
// those of the unfused ops:
//   kq[k]  = sum_d K[k][d] q[d]        (K codes from F16 via F32; chains over d)
//   p      = soft_max(kq * scale)      (every key visible: the mask row is zero)
//   out[d] = sum_k V[k][d] p[k]        (chains over k)
// Monte chains start where the unfused calls' chains start: kq chain (h, k)
// at (h * nkv + k) * (D - 1), the softmax row h at h * (nkv - 1), kqv chain
// (h, d) at (h * D + d) * (nkv - 1) draws after the seed.  Chains take the
// build's policy: the selected flat adder (xlns32, sum32) or red16.
template <int FMT> __host__ __device__ constexpr bool attn_flat() { return FMT == 32 || k_mode == M_SUM32; }
template <int FMT> __host__ __device__ constexpr int  attn_tab() {
    return (attn_flat<FMT>() ? k32f_words * 4 : 0) +
           (FMT == 16 ? k16_tab_bytes16 + (k_mode == M_MONTE ? 2 * k16_monte_n * 2 : 0) : 0);
}

template <int FMT>
struct attn_ops {
    const dev_tables & T;
    const int32_t *    F;      // flat image (attn_flat)
    const int16_t *    tab;    // packed xlns16 table
    const int16_t *    fine;   // Monte fine tables
    __device__ uint32_t from(float f) const { return FMT == 16 ? from_f32_16(T, f) : from_f32_32(T, f); }
    __device__ float    to(uint32_t v) const { return FMT == 16 ? to_f32_16(T, v) : to_f32_32(T, v); }
    __device__ uint32_t mul(uint32_t a, uint32_t b) const { return FMT == 16 ? mul16(a, b) : mul32(a, b); }
    // a mul_mat chain: start with the first product, step, finish (the build's policy)
    __device__ uint32_t start(uint32_t p) const {
        if constexpr (FMT == 32) return p;
        else if constexpr (k_mode == M_SUM32) return p << 16;
        else return red16{ &T, tab, fine }.from(p);
    }
    __device__ uint32_t step(uint32_t acc, uint32_t p, uint32_t & st) const {
        if constexpr (FMT == 32) return add32f_sel(F, acc, p);
        else if constexpr (k_mode == M_SUM32) return add32f_sel(F, acc, p << 16);
        else return red16{ &T, tab, fine }.add(acc, p, st);
    }
    __device__ uint32_t finish(uint32_t acc) const {
        if constexpr (FMT == 32) return acc;
        else return red16{ &T, tab, fine }.finish(acc);
    }
};

// keys per tile: the K (then V) codes of a tile of keys sit in shared memory,
// converted by the whole block with coalesced reads of the F16 caches
constexpr int ATTN_KT = 256;

template <int FMT>
__global__ void __launch_bounds__(256)
k_attn_decode(dev_tables T, const float * __restrict__ q, const __half * __restrict__ kc, const __half * __restrict__ vc,
              int64_t kv_ld, int64_t nkv, int H, int HKV, int D, uint32_t scale_l, float * __restrict__ out,
              uint32_t seed, void * __restrict__ out_lns) {
    extern __shared__ __align__(16) unsigned char attn_sm[];
    constexpr int TAB = attn_tab<FMT>();
    constexpr int KTP = ATTN_KT + 1;                                // [d][k] rows, padded
    int32_t * F    = reinterpret_cast<int32_t *>(attn_sm);
    int16_t * tab  = reinterpret_cast<int16_t *>(attn_sm + (attn_flat<FMT>() ? k32f_words * 4 : 0));
    int16_t * fine = tab + k16_tab_bytes16 / 2;
    uint32_t * tile = reinterpret_cast<uint32_t *>(attn_sm + TAB);  // K: [d][KTP]; V: [k][D]
    uint32_t * qc = tile + (int64_t) D * KTP;                       // q codes [D]
    uint32_t * sv = qc + D;                                         // scaled logits, then exp terms [nkv]
    uint32_t * pc = sv + nkv;                                       // p codes [nkv]
    __shared__ uint32_t s_red[8];
    __shared__ uint32_t s_tot;
    if constexpr (attn_flat<FMT>()) stage_async(F, T.flat32, k32f_words * 4);
    if constexpr (FMT == 16) {
        stage_async(tab, T.sbdb16, k16_tab_bytes16);
        if constexpr (k_mode == M_MONTE) stage_async(fine, T.monte16, 2 * k16_monte_n * 2);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    pdl_entry();
    const attn_ops<FMT> O{ T, F, tab, fine };
    constexpr uint32_t NEG_INF = FMT == 16 ? 0xFFFFu : 0xFFFFFFFFu;
    const int h = blockIdx.x, kvh = h / (H / HKV);
    const int tid = threadIdx.x, nt = blockDim.x;
    const __half * kh = kc + (int64_t) kvh * D;
    const __half * vh = vc + (int64_t) kvh * D;
    for (int d = tid; d < D; d += nt) qc[d] = O.from(q[(int64_t) h * D + d]);
    // a tile of nk keys of the F16 cache into codes (F16 -> F32 -> codes), K as
    // [d][k] (kt) or V as [k][d]: each thread's values in batches of eight, the
    // cache loads and then the conversions' table loads all in flight
    auto stage_kv = [&](const __half * src, int64_t t0, int nk, bool kt) {
        constexpr int U = 8;
        const int n = nk * D;
        for (int i0 = tid; i0 < n; i0 += nt * U) {
            float f[U];
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int i = i0 + u * nt;
                const int kk = i / D, d = i - kk * D;
                f[u] = i < n ? __half2float(src[(t0 + kk) * kv_ld + d]) : 0.0f;
            }
            uint32_t c[U];
#pragma unroll
            for (int u = 0; u < U; u++) c[u] = O.from(f[u]);
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int i = i0 + u * nt;
                if (i < n) {
                    const int kk = i / D, d = i - kk * D;
                    tile[kt ? d * KTP + kk : kk * D + d] = c[u];
                }
            }
        }
    };
    // kq: one chain over d per key, a tile of keys at a time
    for (int64_t t0 = 0; t0 < nkv; t0 += ATTN_KT) {
        const int64_t nk = nkv - t0 < ATTN_KT ? nkv - t0 : ATTN_KT;
        __syncthreads();                                             // the previous tile's chains are done
        stage_kv(kh, t0, (int) nk, true);
        __syncthreads();
        for (int64_t kk = tid; kk < nk; kk += nt) {
            const int64_t k = t0 + kk;
            uint32_t st = FMT == 16 && k_stochastic && D > 1
                              ? lfsr_jump(T, seed, (unsigned long long) ((int64_t) h * nkv + k) * (unsigned long long) (D - 1)) : 0u;
            uint32_t acc = O.start(O.mul(tile[kk], qc[0]));
            for (int d = 1; d < D; d++) acc = O.step(acc, O.mul(tile[d * KTP + kk], qc[d]), st);
            uint32_t v = O.from(O.to(O.finish(acc)));            // mul_mat F32 out -> soft_max F32 in
            if (v != NEG_INF) v = O.mul(v, scale_l);
            sv[k] = v;
        }
    }
    __syncthreads();
    // soft_max: row max, exp terms, the normaliser chain in key order, p
    uint32_t mx = NEG_INF;
    for (int64_t k = tid; k < nkv; k += nt) {
        const uint32_t v = sv[k];
        if (FMT == 16 ? gt16(v, mx) : gt32(v, mx)) mx = v;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const uint32_t o = __shfl_xor_sync(0xFFFFFFFFu, mx, off);
        if (FMT == 16 ? gt16(o, mx) : gt32(o, mx)) mx = o;
    }
    if ((tid & 31) == 0) s_red[tid >> 5] = mx;
    __syncthreads();
    mx = s_red[0];
    for (int w = 1; w < nt / 32; w++) if (FMT == 16 ? gt16(s_red[w], mx) : gt32(s_red[w], mx)) mx = s_red[w];
    for (int64_t k = tid; k < nkv; k += nt) {
        const uint32_t v = sv[k];
        if constexpr (FMT == 16) sv[k] = __ldg(T.exp16 + sub16(v, mx, tab));
        else                     sv[k] = exp32(T, sub32(T, v, mx));
    }
    __syncthreads();
    if (tid == 0) {
        uint32_t acc;
        if constexpr (FMT == 32) {
            acc = sv[0];
            acc = chain_smem(sv, 1, (int) nkv, acc, [&](uint32_t a, uint32_t t) { return padd32f(F, a, t); });
        } else if constexpr (NNCHAIN) {
            red16 R{ &T, tab, fine };
            acc = R.from(sv[0]);
            acc = chain_smem(sv, 1, (int) nkv, acc, [&](uint32_t a, uint32_t t) { return nn_add(F, tab, a, t); });
            acc = R.finish(acc);
        } else {
            red16 R{ &T, tab, fine };
            uint32_t st = k_stochastic && nkv > 1 ? lfsr_jump(T, seed, (unsigned long long) h * (unsigned long long) (nkv - 1)) : 0u;
            acc = R.from(sv[0]);
            for (int64_t k = 1; k < nkv; k++) acc = R.add(acc, sv[k], st);
            acc = R.finish(acc);
        }
        s_tot = acc;
    }
    __syncthreads();
    const uint32_t tot = s_tot;
    for (int64_t k = tid; k < nkv; k += nt)             // soft_max F32 out -> to_lns for kqv
        pc[k] = O.from(O.to(FMT == 16 ? div16(sv[k], tot) : div32(sv[k], tot)));
    // kqv: one chain over the keys per d, continued across the tiles
    uint32_t acc = 0u, st = 0u;
    if (tid < D && FMT == 16 && k_stochastic && nkv > 1)
        st = lfsr_jump(T, seed, (unsigned long long) ((int64_t) h * D + tid) * (unsigned long long) (nkv - 1));
    for (int64_t t0 = 0; t0 < nkv; t0 += ATTN_KT) {
        const int64_t nk = nkv - t0 < ATTN_KT ? nkv - t0 : ATTN_KT;
        __syncthreads();
        stage_kv(vh, t0, (int) nk, false);
        __syncthreads();
        if (tid < D) {
            for (int64_t kk = 0; kk < nk; kk++) {
                const uint32_t p = O.mul(tile[kk * D + tid], pc[t0 + kk]);
                acc = t0 + kk == 0 ? O.start(p) : O.step(acc, p, st);
            }
        }
    }
    if (tid < D) {
        const float y = O.to(O.finish(acc));
        if (out != nullptr) out[(int64_t) h * D + tid] = y;
        if (out_lns != nullptr) {                        // to_lns of the output (the wo mat-vec's input)
            if constexpr (FMT == 16) static_cast<uint16_t *>(out_lns)[(int64_t) h * D + tid] = (uint16_t) O.from(y);
            else                     static_cast<uint32_t *>(out_lns)[(int64_t) h * D + tid] = O.from(y);
        }
    }
}

// ===================== group barrier over peer memory ========================
// After lnsb_mul_mat_lns_peers: thread p stores the epoch into peer p's flag
// slot for this rank (system-scope release; the kernel starts after the
// mul_mat has completed, pdl_entry) and waits for peer p's store into this
// rank's slot p (system-scope acquire).  The wait is bounded: past `limit`
// polls it records an error and returns, so a missing peer cannot hang the GPU.
__global__ void k_group_barrier(int32_t * const * __restrict__ flags, int world, int rank, int32_t epoch,
                                int32_t * __restrict__ err, long long limit) {
    pdl_entry();
    const int p = threadIdx.x;
    if (p >= world) return;
    int32_t * peer = flags[p] + rank;
    asm volatile("st.release.sys.global.s32 [%0], %1;\n" ::"l"(peer), "r"(epoch) : "memory");
    const int32_t * mine = flags[rank] + p;
    int32_t v = 0;
    for (long long it = 0; it < limit; it++) {
        asm volatile("ld.acquire.sys.global.s32 %0, [%1];\n" : "=r"(v) : "l"(mine) : "memory");
        if (v >= epoch) return;
        __nanosleep(100);
    }
    atomicExch(err, 1);
}

// ===================== elementwise ops of the model graph ===================
//
// F32 in and out, as at every ggml op boundary of the reference's backends
// (lns-backend/cuda/lns-cuda-kernels.cuh:162-355, lns-backend/src/lns-ops.cpp):
// convert with the F32 -> LNS table, compute in LNS, write back through the
// decode table.  Grid-stride loops over elements; the tables are read through
// the read-only cache (conv16 256 KB, dec16 256 KB, sbdb16 6.7 KB).
template <int FMT> struct ew;
template <> struct ew<16> {
    __device__ static __forceinline__ uint32_t from(const dev_tables & T, float x) { return from_f32_16(T, x); }
    __device__ static __forceinline__ float    to(const dev_tables & T, uint32_t v) { return to_f32_16(T, v); }
    __device__ static __forceinline__ uint32_t add(const dev_tables & T, uint32_t a, uint32_t b) { return add16(a, b, T.sbdb16); }
    __device__ static __forceinline__ uint32_t sub(const dev_tables & T, uint32_t a, uint32_t b) { return add16(a, b ^ 0x8000u, T.sbdb16); }
    __device__ static __forceinline__ uint32_t mul(uint32_t a, uint32_t b) { return mul16(a, b); }
    __device__ static __forceinline__ uint32_t div(uint32_t a, uint32_t b) { return div16(a, b); }
};
template <> struct ew<32> {
    __device__ static __forceinline__ uint32_t from(const dev_tables & T, float x) { return from_f32_32(T, x); }
    __device__ static __forceinline__ float    to(const dev_tables & T, uint32_t v) { return to_f32_32(T, v); }
    // the flat image's branch-free addition (same bits as add32): a warp's
    // lanes take no separate sb / db / cotransformation paths
    __device__ static __forceinline__ uint32_t add(const dev_tables & T, uint32_t a, uint32_t b) { return add32f(T.flat32, a, b); }
    __device__ static __forceinline__ uint32_t sub(const dev_tables & T, uint32_t a, uint32_t b) { return add32f(T.flat32, a, b ^ 0x80000000u); }
    __device__ static __forceinline__ uint32_t mul(uint32_t a, uint32_t b) { return mul32(a, b); }
    __device__ static __forceinline__ uint32_t div(uint32_t a, uint32_t b) { return div32(a, b); }
};

// silu(x) = x * sigmoid(x), the sigmoid from its table (entry c: the float
// 1 / (1 + e^-x) of code c's value, converted)
__device__ __forceinline__ uint32_t silu16(const dev_tables & T, uint32_t x) {
    return mul16(x, __ldg(T.sig16 + x));
}
__device__ __forceinline__ uint32_t relu16(uint32_t x) { return ((x & 0x8000u) || (x & 0x7FFFu) == 0) ? 0u : x; }
// tanh(x) = (e^2x - 1) / (e^2x + 1) in xlns16 arithmetic over the exp table
__device__ __forceinline__ uint32_t tanh16(const dev_tables & T, uint32_t x) {
    const uint32_t e = __ldg(T.exp16 + mul16(x, 0x4080u));
    return div16(add16(e, 0xC000u, T.sbdb16), add16(e, 0x4000u, T.sbdb16));
}
// gelu(x) = 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))) in xlns16
// arithmetic, the constants converted from float like any operand
__device__ __forceinline__ uint32_t gelu16(const dev_tables & T, uint32_t x) {
    const uint32_t s = from_f32_16(T, 0.79788456080286535588f), a = from_f32_16(T, 0.044715f), h = from_f32_16(T, 0.5f);
    const uint32_t x3 = mul16(mul16(x, x), x);
    const uint32_t in = mul16(s, add16(x, mul16(a, x3), T.sbdb16));
    return mul16(mul16(h, x), add16(0x4000u, tanh16(T, in), T.sbdb16));
}
// xlns32: silu in xlns32 arithmetic with exp through float, as in the xlns32
// softmax; tanh and gelu through double precision (lnsb_tanh_d), as xlns32's
// activations go through floating point in the reference
__device__ __forceinline__ uint32_t silu32(const dev_tables & T, uint32_t x) {
    return div32(x, add32f(T.flat32, 0x40000000u, exp32(T, x ^ 0x80000000u)));
}
__device__ __forceinline__ uint32_t relu32(uint32_t x) { return ((x & 0x80000000u) || (x & 0x7FFFFFFFu) == 0) ? 0u : x; }
__device__ __forceinline__ uint32_t tanh32(const dev_tables & T, uint32_t x) {
    return from_f32_32(T, __double2float_rn(lnsb_tanh_d((double) to_f32_32(T, x))));
}
__device__ __forceinline__ uint32_t gelu32(const dev_tables & T, uint32_t x) {
    const double d = (double) to_f32_32(T, x);
    const double u = __dmul_rn(0.79788456080286535588, __dadd_rn(d, __dmul_rn(__dmul_rn(__dmul_rn(0.044715, d), d), d)));
    return from_f32_32(T, __double2float_rn(__dmul_rn(__dmul_rn(0.5, d), __dadd_rn(1.0, lnsb_tanh_d(u)))));
}
template <int FMT, int OP>
__device__ __forceinline__ uint32_t unary_op(const dev_tables & T, uint32_t v) {
    if constexpr (FMT == 16) {
        if constexpr (OP == LNSB_UNARY_SILU) return silu16(T, v);
        else if constexpr (OP == LNSB_UNARY_GELU) return gelu16(T, v);
        else if constexpr (OP == LNSB_UNARY_TANH) return tanh16(T, v);
        else return relu16(v);
    } else {
        if constexpr (OP == LNSB_UNARY_SILU) return silu32(T, v);
        else if constexpr (OP == LNSB_UNARY_GELU) return gelu32(T, v);
        else if constexpr (OP == LNSB_UNARY_TANH) return tanh32(T, v);
        else return relu32(v);
    }
}

#define LNSB_GRID_STRIDE(i, n) \
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < (n); i += (int64_t) blockDim.x * gridDim.x)

template <int FMT, int OP>
__global__ void k_binary(dev_tables T, const float * __restrict__ a, lnsb_shape4 as, const float * __restrict__ b,
                         lnsb_shape4 bs, float * __restrict__ dst) {
    pdl_entry();
    using A = ew<FMT>;
    const int64_t n = as.ne[0] * as.ne[1] * as.ne[2] * as.ne[3];
    LNSB_GRID_STRIDE(i, n) {
        const int64_t i0 = i % as.ne[0], r = i / as.ne[0];
        const int64_t i1 = r % as.ne[1], r2 = r / as.ne[1];
        const int64_t i2 = r2 % as.ne[2], i3 = r2 / as.ne[2];
        const int64_t j = (((i3 % bs.ne[3]) * bs.ne[2] + i2 % bs.ne[2]) * bs.ne[1] + i1 % bs.ne[1]) * bs.ne[0] + i0 % bs.ne[0];
        const uint32_t x = A::from(T, a[i]), y = A::from(T, b[j]);
        const uint32_t v = OP == LNSB_BINARY_ADD ? A::add(T, x, y) : OP == LNSB_BINARY_MUL ? A::mul(x, y) : A::div(x, y);
        dst[i] = A::to(T, v);
    }
}

template <int FMT>
__global__ void k_scale(dev_tables T, const float * __restrict__ src, float * __restrict__ dst, int64_t n, uint32_t sl,
                        uint32_t bl, int has_b) {
    pdl_entry();
    using A = ew<FMT>;
    LNSB_GRID_STRIDE(i, n) {
        uint32_t v = A::mul(A::from(T, src[i]), sl);
        if (has_b) v = A::add(T, v, bl);
        dst[i] = A::to(T, v);
    }
}

template <int FMT, int OP>
__global__ void k_unary(dev_tables T, const float * __restrict__ src, float * __restrict__ dst, int64_t n) {
    pdl_entry();
    using A = ew<FMT>;
    LNSB_GRID_STRIDE(i, n) {
        dst[i] = A::to(T, unary_op<FMT, OP>(T, A::from(T, src[i])));
    }
}

// act(gate) * up with act = silu (swiglu) or gelu (geglu).  OUT_LNS: the glu
// op's F32 result converted again (to_lns of the next mul_mat)
template <int FMT, bool OUT_LNS = false, int ACT = LNSB_UNARY_SILU>
__global__ void k_swiglu(dev_tables T, const float * __restrict__ gate, const float * __restrict__ up, int64_t gs,
                         int64_t us, void * __restrict__ dst, int64_t nc, int64_t nr) {
    pdl_entry();
    using A = ew<FMT>;
    LNSB_GRID_STRIDE(i, nc * nr) {
        const int64_t r = i / nc, c = i - r * nc;
        const uint32_t g = A::from(T, gate[r * gs + c]), u = A::from(T, up[r * us + c]);
        const float y = A::to(T, A::mul(unary_op<FMT, ACT>(T, g), u));
        if constexpr (!OUT_LNS)    static_cast<float *>(dst)[i] = y;
        else if constexpr (FMT == 16) static_cast<uint16_t *>(dst)[i] = (uint16_t) A::from(T, y);
        else                          static_cast<uint32_t *>(dst)[i] = A::from(T, y);
    }
}

// the decode graph's step after the q/k/v mat-vec, one kernel: rope of the q
// and k heads (F32 out, as lnsb_rope), k and v into the F16 caches (as
// lnsb_f32_to_f16).  qkv rows [T][ld]: q heads, then k heads, then v heads.
template <int FMT>
__global__ void k_rope_qkv(dev_tables T, const float * __restrict__ qkv, int64_t ld, const float * __restrict__ cos_sin,
                           int n_dims, int neox, int H, int HKV, int D, int64_t nt, float * __restrict__ q_out,
                           __half * __restrict__ kc, __half * __restrict__ vc, int64_t kv_ld) {
    pdl_entry();
    using A = ew<FMT>;
    const int64_t half = n_dims / 2, per = half + (D - n_dims);
    const int64_t nrope = nt * (H + HKV) * per, nv = nt * (int64_t) HKV * D;
    LNSB_GRID_STRIDE(i, nrope + nv) {
        if (i >= nrope) {                                    // v -> F16 cache
            const int64_t e = i - nrope, t = e / ((int64_t) HKV * D), c = e - t * HKV * D;
            vc[t * kv_ld + c] = __float2half_rn(qkv[t * ld + (int64_t) (H + HKV) * D + c]);
            continue;
        }
        const int64_t row = i / per, j = i - row * per;      // row = t * (H + HKV) + head
        const int64_t t = row / (H + HKV), hd = row - t * (H + HKV);
        const float * x = qkv + t * ld + hd * D;
        float y0, y1 = 0.0f;
        int64_t a0, a1 = -1;
        if (j < half) {
            a0 = neox ? j : 2 * j;
            a1 = neox ? j + half : 2 * j + 1;
            const uint32_t c = A::from(T, cos_sin[(t * half + j) * 2]), sn = A::from(T, cos_sin[(t * half + j) * 2 + 1]);
            const uint32_t x0 = A::from(T, x[a0]), x1 = A::from(T, x[a1]);
            y0 = A::to(T, A::sub(T, A::mul(x0, c), A::mul(x1, sn)));
            y1 = A::to(T, A::add(T, A::mul(x0, sn), A::mul(x1, c)));
        } else {
            a0 = n_dims + (j - half);
            y0 = A::to(T, A::from(T, x[a0]));
        }
        if (hd < H) {
            float * y = q_out + t * (int64_t) H * D + hd * D;
            y[a0] = y0;
            if (a1 >= 0) y[a1] = y1;
        } else {
            __half * y = kc + t * kv_ld + (hd - H) * D;
            y[a0] = __float2half_rn(y0);
            if (a1 >= 0) y[a1] = __float2half_rn(y1);
        }
    }
}

// one thread per rotated pair or passed-through dimension (lns-cuda-kernels.cuh:330-355)
template <int FMT>
__global__ void k_rope(dev_tables T, const float * __restrict__ src, lnsb_shape4 s, const float * __restrict__ cos_sin,
                       int n_dims, int neox, float * __restrict__ dst) {
    pdl_entry();
    using A = ew<FMT>;
    const int64_t half = n_dims / 2, per = half + (s.ne[0] - n_dims);
    const int64_t nrows = s.ne[1] * s.ne[2] * s.ne[3];
    LNSB_GRID_STRIDE(i, nrows * per) {
        const int64_t row = i / per, j = i - row * per;
        const int64_t i2 = (row / s.ne[1]) % s.ne[2];
        const float * x = src + row * s.ne[0];
        float *       y = dst + row * s.ne[0];
        if (j < half) {
            const int64_t a0 = neox ? j : 2 * j, a1 = neox ? j + half : 2 * j + 1;
            const uint32_t c = A::from(T, cos_sin[(i2 * half + j) * 2]), sn = A::from(T, cos_sin[(i2 * half + j) * 2 + 1]);
            const uint32_t x0 = A::from(T, x[a0]), x1 = A::from(T, x[a1]);
            y[a0] = A::to(T, A::sub(T, A::mul(x0, c), A::mul(x1, sn)));
            y[a1] = A::to(T, A::add(T, A::mul(x0, sn), A::mul(x1, c)));
        } else {
            const int64_t a0 = n_dims + (j - half);
            y[a0] = A::to(T, A::from(T, x[a0]));
        }
    }
}

__global__ void k_f32_to_f16(const float * __restrict__ src, __half * __restrict__ dst, int64_t n) {
    pdl_entry();
    LNSB_GRID_STRIDE(i, n) dst[i] = __float2half_rn(src[i]);
}
__global__ void k_f16_to_f32(const __half * __restrict__ src, float * __restrict__ dst, int64_t n) {
    pdl_entry();
    LNSB_GRID_STRIDE(i, n) dst[i] = __half2float(src[i]);
}

// ============================ launch helpers ===============================

int sm_count(int dev) {
    static int sms[k_max_devices] = {};
    if (sms[dev] == 0) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
        sms[dev] = v;
    }
    return sms[dev];
}

template <int FMT, int TN, bool OUT_F32, bool RING>
int launch_a32(const dev_tables & T, const lnsb_mul_mat_args * a, void * dst, int64_t r2, int64_t r3, int64_t units,
               int dev, bool vecx, cudaStream_t stream, const peer_out_dev & peers) {
    static bool attr[k_max_devices] = {};
    auto kern = k_mul_mat_a32<FMT, TN, OUT_F32, RING>;
    constexpr int smem = RING ? a32_ring<FMT, TN>::smem : a32_ring<FMT, TN>::table;
    if (!attr[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return (int) e;
        attr[dev] = true;
    }
    using E = typename a32_fmt<FMT>::elem;
    const int64_t grid = units < sm_count(dev) ? units : sm_count(dev);
    launch_k(kern, (unsigned) grid, a32_threads(FMT, RING), smem, stream, T, static_cast<const E *>(a->w), static_cast<const E *>(a->x),
                                                       dst, a->K, a->M, a->N, a->ne02, a->ne12, r2, r3,
                                                       a->ne12 * a->ne13, a->monte_seed, vecx ? 1 : 0,
                                                       units <= (int64_t) sm_count(dev) * LNSB_A32_SEL_WARPS ? 1 : 0, peers);
    return launch_status();
}

template <int FMT, int TN>
int launch_a32_by(const dev_tables & T, const lnsb_mul_mat_args * a, void * dst, bool out_f32, bool ring, int64_t r2,
                  int64_t r3, int64_t units, int dev, bool vecx, cudaStream_t stream, const peer_out_dev & peers) {
    if (ring) return out_f32 ? launch_a32<FMT, TN, true, true>(T, a, dst, r2, r3, units, dev, vecx, stream, peers)
                             : launch_a32<FMT, TN, false, true>(T, a, dst, r2, r3, units, dev, vecx, stream, peers);
    return out_f32 ? launch_a32<FMT, TN, true, false>(T, a, dst, r2, r3, units, dev, vecx, stream, peers)
                   : launch_a32<FMT, TN, false, false>(T, a, dst, r2, r3, units, dev, vecx, stream, peers);
}

// the latency mat-vec (k_mat_vec_lat): np = ceil(units / SMs) units per block
// of 2 np warps, one wave
template <int FMT, bool OUT_F32>
int launch_lv(const dev_tables & T, const lnsb_mul_mat_args * a, void * dst, int64_t r2, int64_t r3, int64_t units,
              int dev, cudaStream_t stream, const peer_out_dev & peers) {
    static bool attr[k_max_devices] = {};
    auto kern = k_mat_vec_lat<FMT, OUT_F32>;
    constexpr int smem_max = k32f_words * 4 + LV_MAX_PAIRS * LV_RING_BYTES;
    if (!attr[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_max);
        if (e != cudaSuccess) return (int) e;
        attr[dev] = true;
    }
    const int64_t sms = sm_count(dev);
    const int np = (int) ((units + sms - 1) / sms);                    // 1 .. LV_MAX_PAIRS (checked by the caller)
    const int64_t grid = (units + np - 1) / np;
    const int smem = k32f_words * 4 + np * LV_RING_BYTES;
    using E = typename a32_fmt<FMT>::elem;
    launch_k(kern, (unsigned) grid, 64 * np, smem, stream, T, static_cast<const E *>(a->w), static_cast<const E *>(a->x),
             dst, a->K, a->M, a->N, a->ne02, a->ne12, r2, r3, units, peers);
    return launch_status();
}

// sum32-mode xlns16 and xlns32 mul_mat: one or two tokens per lane
int mul_mat_a32(int fmt, const dev_tables & T, const lnsb_mul_mat_args * a, void * dst, bool out_f32, int64_t r2,
                int64_t r3, cudaStream_t stream, const peer_out_dev & peers) {
    int dev = 0;
    const int ds = current_device(&dev);
    if (ds != 0) return ds;
    const int64_t nz = a->ne12 * a->ne13, RB = (a->M + 31) / 32;
    const int64_t es0 = fmt == LNSB_XLNS16 ? 2 : 4;
    const bool ring0 = (a->K * es0) % 16 == 0 && ((uintptr_t) a->x % 16) == 0 && (a->M * es0) % 16 == 0 &&
                       ((uintptr_t) a->w % 16) == 0;
    const int64_t warps = (int64_t) sm_count(dev) * (a32_threads(fmt == LNSB_XLNS16 ? 16 : 32, ring0) / 32);
    const bool tn2 = a->N >= 2 && 4 * nz * RB * ((a->N + 1) / 2) >= LNSB_A32_TN2_MIN_QUARTERS * warps;
    const int64_t units = nz * RB * (tn2 ? (a->N + 1) / 2 : a->N);
    const int64_t es = fmt == LNSB_XLNS16 ? 2 : 4;
    const bool vecx = (a->K * es) % 16 == 0 && ((uintptr_t) a->x % 16) == 0;
    const bool ring = vecx && (a->M * es) % 16 == 0 && ((uintptr_t) a->w % 16) == 0;
    // at most LNSB_A32_LV_PAIRS units of 32 rows x 1 token per SM, the flat adder: the latency mat-vec
    if (LNSB_A32_LV && (fmt == LNSB_XLNS32 || k_mode == M_SUM32) && a->K > 0 &&
        nz * RB * a->N <= (int64_t) sm_count(dev) * LNSB_A32_LV_PAIRS) {
        const int64_t lv_units = nz * RB * a->N;
        if (fmt == LNSB_XLNS16) return out_f32 ? launch_lv<16, true>(T, a, dst, r2, r3, lv_units, dev, stream, peers)
                                               : launch_lv<16, false>(T, a, dst, r2, r3, lv_units, dev, stream, peers);
        return out_f32 ? launch_lv<32, true>(T, a, dst, r2, r3, lv_units, dev, stream, peers)
                       : launch_lv<32, false>(T, a, dst, r2, r3, lv_units, dev, stream, peers);
    }
    if (fmt == LNSB_XLNS16) {
        if (tn2) return launch_a32_by<16, 2>(T, a, dst, out_f32, ring, r2, r3, units, dev, vecx, stream, peers);
        return launch_a32_by<16, 1>(T, a, dst, out_f32, ring, r2, r3, units, dev, vecx, stream, peers);
    }
    if (tn2) return launch_a32_by<32, 2>(T, a, dst, out_f32, ring, r2, r3, units, dev, vecx, stream, peers);
    return launch_a32_by<32, 1>(T, a, dst, out_f32, ring, r2, r3, units, dev, vecx, stream, peers);
}

int mul_mat_id_impl(int fmt, const lnsb_mul_mat_id_args * a, void * dst, bool out_f32, cudaStream_t stream) {
    if (!valid_fmt(fmt) || a == nullptr) return LNSB_E_INVALID;
    if (a->K < 0 || a->M < 0 || a->n_expert < 0 || a->ne11 <= 0 || a->n_used < 0 || a->n_tokens < 0 ||
        a->ids_stride < a->n_used)
        return LNSB_E_INVALID;
    if (a->n_used % a->ne11 != 0) return LNSB_E_INVALID;          // slot-based broadcast of the activation rows
    if (a->M == 0 || a->n_used == 0 || a->n_tokens == 0) return 0;
    if (dst == nullptr || a->ids == nullptr || (a->K > 0 && (a->w == nullptr || a->x == nullptr))) return LNSB_E_INVALID;
    int dev = 0;
    const int ds = current_device(&dev);
    if (ds != 0) return ds;
    const dev_tables * T = nullptr;
    const int st = tables_for(fmt, &T);
    if (st != 0) return st;
    const int64_t units = a->n_tokens * a->n_used * ((a->M + 31) / 32);
    const int64_t grid = imin64((units + 7) / 8, (int64_t) sm_count(dev) * 2);
    static bool attr[2][2][k_max_devices] = {};          // [xlns32][F32 out][device]
    auto go = [&](auto kern, int smem, auto * w, auto * x) -> int {
        bool & done = attr[fmt == LNSB_XLNS32][out_f32][dev];
        if (!done) {
            const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e != cudaSuccess) return (int) e;
            done = true;
        }
        launch_k(kern, (unsigned) grid, 256, smem, stream, *T, w, x, a->ids, dst, a->K, a->M, a->n_expert, a->ne11, a->n_used,
                                                     a->n_tokens, a->ids_stride, a->monte_seed);
        return launch_status();
    };
    if (fmt == LNSB_XLNS16) {
        const auto * w = static_cast<const uint16_t *>(a->w);
        const auto * x = static_cast<const uint16_t *>(a->x);
        return out_f32 ? go(k_mul_mat_id<16, true>, mmid_smem<16>(), w, x) : go(k_mul_mat_id<16, false>, mmid_smem<16>(), w, x);
    }
    const auto * w = static_cast<const uint32_t *>(a->w);
    const auto * x = static_cast<const uint32_t *>(a->x);
    return out_f32 ? go(k_mul_mat_id<32, true>, mmid_smem<32>(), w, x) : go(k_mul_mat_id<32, false>, mmid_smem<32>(), w, x);
}

// xf32: a->x holds F32 activations; the weight-resident latency kernel
// converts them as it stages its token rows, every other kernel reads codes
// converted into x_work (N x K per activation slice) first
int mul_mat_impl(int fmt, const lnsb_mul_mat_args * a, void * dst, bool out_f32, cudaStream_t stream,
                 const peer_out_dev * peers = nullptr, bool xf32 = false, void * x_work = nullptr) {
    if (!valid_fmt(fmt) || a == nullptr) return LNSB_E_INVALID;
    if (a->K < 0 || a->M < 0 || a->N < 0 || a->ne02 <= 0 || a->ne03 <= 0 || a->ne12 <= 0 || a->ne13 <= 0) return LNSB_E_INVALID;
    if (a->ne12 % a->ne02 != 0 || a->ne13 % a->ne03 != 0) return LNSB_E_INVALID;
    if (a->M == 0 || a->N == 0) return 0;
    if ((dst == nullptr && peers == nullptr) || (a->K > 0 && (a->w == nullptr || a->x == nullptr))) return LNSB_E_INVALID;
    if (xf32 && a->K > 0 && x_work == nullptr) return LNSB_E_INVALID;
    if (a->ne12 * a->ne13 > 65535) return LNSB_E_TOO_LARGE;
    const dev_tables * T = nullptr;
    const int st = tables_for(fmt, &T);
    if (st != 0) return st;
    const int64_t r2 = a->ne12 / a->ne02, r3 = a->ne13 / a->ne03;
    const int64_t tiles = ((a->M + FB_BM - 1) / FB_BM) * ((a->N + FB_BN - 1) / FB_BN) * a->ne12 * a->ne13;
    const peer_out_dev no_peers{ nullptr, 0, 0, 0 };
    if (peers != nullptr && out_f32) return LNSB_E_INVALID;   // the fused gather stores codes
    // few outputs, weight keys resident: the first lane layout (rows x token
    // slots per warp: 32 x 1, 16 x 1 with lanes repeated, 16 x 2) and the
    // fewest chain warps per CTA (1, 2, 3, then 4) that keep the grid within
    // one CTA per SM and the slice within shared memory
    int r2_R = 0, r2_tpw = 0, r2_cw = 0;
    if (fmt == LNSB_XLNS16 && k_mode == M_BASE && tiles < 2 * 148 && a->K <= (int64_t) LR_SEG * LR_MAXSEG &&
        (peers == nullptr || !out_f32)) {
        int dev = 0;
        const int ds = current_device(&dev);
        if (ds != 0) return ds;
        const int64_t sms = sm_count(dev);
        const int layouts[3][2] = { { 32, 1 }, { 16, 1 }, { 16, 2 } };
        for (const auto & L : layouts) {               // with at least one producer warp
            const int R = L[0], tpw = L[1];
            for (const int cw : { 1, 2, 3 }) {
                const int64_t tpc = (int64_t) cw * tpw;
                const int64_t ctas = ((a->M + R - 1) / R) * ((a->N + tpc - 1) / tpc) * a->ne12 * a->ne13;
                if (r2_smem(a->K, R, (int) tpc) > R2_SMEM_MAX || (a->N + tpc - 1) / tpc > 65535) break;
                if (ctas <= sms) { r2_R = R; r2_tpw = tpw; r2_cw = cw; break; }
            }
            if (r2_R != 0) break;
        }
        // more CTAs than SMs: 16 rows x 2 tokens, as many chain warps as fit
        for (const int cw : { 3, 2, 1 })
            if (r2_R == 0 && r2_smem(a->K, 16, 2 * cw) <= R2_SMEM_MAX && (a->N + 2 * cw - 1) / (2 * cw) <= 65535) {
                r2_R = 16; r2_tpw = 2; r2_cw = cw;
            }
    }
    lnsb_mul_mat_args xa;                                // the arguments over x_work's codes
    if (xf32 && r2_R == 0 && a->K > 0) {
        const int64_t n = a->N * a->K * a->ne12 * a->ne13;
        if (fmt == LNSB_XLNS16) launch_k(k_to_lns<16>, grid_for(n, 256), 256, 0, stream, *T, static_cast<const float *>(a->x), x_work, n);
        else                    launch_k(k_to_lns<32>, grid_for(n, 256), 256, 0, stream, *T, static_cast<const float *>(a->x), x_work, n);
        xa = *a;
        xa.x = x_work;
        a = &xa;
    }
    if (r2_R != 0) {
        const int tpc = r2_cw * r2_tpw;
        const dim3 grid((unsigned) ((a->M + r2_R - 1) / r2_R), (unsigned) ((a->N + tpc - 1) / tpc), (unsigned) (a->ne12 * a->ne13));
        const int smem = r2_smem(a->K, r2_R, tpc);
        const int li = r2_R == 32 ? 0 : r2_tpw == 1 ? 1 : 2;
        using r2_kern = void (*)(dev_tables, const uint16_t *, const void *, void *, int64_t, int64_t, int64_t, int64_t,
                                 int64_t, int64_t, int64_t, int, int, peer_out_dev);
        static const r2_kern kerns[2][2][3] = {          // [x F32][out F32][layout]
            { { k_mul_mat16_res2<false, 32, 1, false>, k_mul_mat16_res2<false, 16, 1, false>, k_mul_mat16_res2<false, 16, 2, false> },
              { k_mul_mat16_res2<true, 32, 1, false>,  k_mul_mat16_res2<true, 16, 1, false>,  k_mul_mat16_res2<true, 16, 2, false> } },
            { { k_mul_mat16_res2<false, 32, 1, true>,  k_mul_mat16_res2<false, 16, 1, true>,  k_mul_mat16_res2<false, 16, 2, true> },
              { k_mul_mat16_res2<true, 32, 1, true>,   k_mul_mat16_res2<true, 16, 1, true>,   k_mul_mat16_res2<true, 16, 2, true> } } };
        const r2_kern kern = kerns[xf32][out_f32][li];
        static bool r2attr[k_max_devices][2][2][3] = {};
        int dev = 0;
        const int ds = current_device(&dev);
        if (ds != 0) return ds;
        if (!r2attr[dev][xf32][out_f32][li]) {
            const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, R2_SMEM_MAX);
            if (e != cudaSuccess) return (int) e;
            r2attr[dev][xf32][out_f32][li] = true;
        }
        launch_k(kern, grid, R2_THREADS, smem, stream, *T, static_cast<const uint16_t *>(a->w), a->x,
                 dst, a->K, a->M, a->N, a->ne02, a->ne12, r2, r3, r2_cw,
                 a->M % 8 == 0 && ((uintptr_t) a->w % 16) == 0 ? 1 : 0, peers != nullptr ? *peers : no_peers);
    } else if (peers == nullptr && fmt == LNSB_XLNS16 && k_mode == M_BASE && tiles < 2 * 148 && a->K <= LT_MAX_K && a->N <= 65535) {
        // few outputs: latency form, two tokens per thread where they fit
#ifndef LNSB_LT_TN2
#define LNSB_LT_TN2 1
#endif
        // two tokens per thread share the weight work once there are enough CTAs to fill the
        // GPU (throughput); with few CTAs the single chain's latency is the time, and one
        // token per thread keeps it shortest
        const int64_t ctas1 = ((a->M + LT_ROWS - 1) / LT_ROWS) * a->N * a->ne12 * a->ne13;
        const int tn = LNSB_LT_TN2 && a->N >= 2 && a->K <= LT_MAX_K2 && ctas1 > 2 * 148 ? 2 : 1;
        const dim3 grid((unsigned) ((a->M + LT_ROWS - 1) / LT_ROWS), (unsigned) ((a->N + tn - 1) / tn),
                        (unsigned) (a->ne12 * a->ne13));
        const bool vec = a->M % 8 == 0 && ((uintptr_t) a->w % 16) == 0;
        const int smem = lt_smem(a->K, tn);
        auto kern = tn == 2 ? (out_f32 ? k_mul_mat16_lat<true, 2> : k_mul_mat16_lat<false, 2>)
                            : (out_f32 ? k_mul_mat16_lat<true, 1> : k_mul_mat16_lat<false, 1>);
        static int lattr[k_max_devices][2][2] = {};
        int dev = 0;
        const int ds = current_device(&dev);
        if (ds != 0) return ds;
        if (lattr[dev][out_f32][tn - 1] < smem) {
            const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e != cudaSuccess) return (int) e;
            lattr[dev][out_f32][tn - 1] = smem;
        }
        launch_k(kern, grid, LT_ROWS, smem, stream, *T, static_cast<const uint16_t *>(a->w), static_cast<const uint16_t *>(a->x),
                                              dst, a->K, a->M, a->N, a->ne02, a->ne12, r2, r3, vec ? 1 : 0);
    } else if (fmt == LNSB_XLNS16 && (k_mode == M_BASE || k_mode == M_MONTE)) {
        const int64_t gx = (a->M + FB_BM - 1) / FB_BM, gy = (a->N + FB_BN - 1) / FB_BN, nz = a->ne12 * a->ne13;
        int dev0 = 0;
        const int ds0 = current_device(&dev0);
        if (ds0 != 0) return ds0;
        // one slice: whole tiles in whole waves of SMs, the rest in quarter tiles
        const int64_t nt = gx * gy, sms = sm_count(dev0);
        const int64_t nfull = nz == 1 ? nt / sms * sms : nt;
        const int64_t nblk = nfull + 4 * (nt - nfull);
        if (nblk > 0x7FFFFFFF) return LNSB_E_TOO_LARGE;
        const dim3 grid((unsigned) nblk, 1u, (unsigned) nz);
        const bool vec = a->M % FB_BM == 0 && a->K % 8 == 0 && ((uintptr_t) a->w % 16) == 0 && ((uintptr_t) a->x % 16) == 0;
        if (!FB_MONTE) {
            // base: one CTA per SM over four table replicas, whole tiles only --
            // a quarter tile's four chains per thread hide the table latency
            // worse than the balance they buy is worth (measured).  The Monte
            // build measured slower on it (two groups: 1164 against 1188-1199
            // G-LNSadd/s on configs[1]) and keeps the two-replica kernel.
            const int64_t nfull4 = (FB_MONTE && nz == 1) ? nt / sms * sms : nt, nblk4 = nfull4 + 4 * (nt - nfull4);
            if (nblk4 > 0x7FFFFFFF) return LNSB_E_TOO_LARGE;
            static bool f4attr[k_max_devices][2] = {};
            auto kern4 = out_f32 ? k_mul_mat16_fast4<true> : k_mul_mat16_fast4<false>;
            if (!f4attr[dev0][out_f32]) {
                const cudaError_t e = cudaFuncSetAttribute(kern4, cudaFuncAttributeMaxDynamicSharedMemorySize, FB4_SMEM);
                if (e != cudaSuccess) return (int) e;
                f4attr[dev0][out_f32] = true;
            }
            launch_k(kern4, dim3((unsigned) imin64(sms, nblk4), 1u, (unsigned) nz), FB4_THREADS, FB4_SMEM, stream, *T,
                     static_cast<const uint16_t *>(a->w), static_cast<const uint16_t *>(a->x), dst, a->K, a->M, a->N,
                     a->ne02, a->ne12, r2, r3, a->monte_seed, vec ? 1 : 0, peers ? *peers : no_peers, gx, nfull4,
                     nblk4);
            return launch_status();
        }
        static bool fattr[k_max_devices][2] = {};
        auto kern = out_f32 ? k_mul_mat16_fast<true> : k_mul_mat16_fast<false>;
        int dev = 0;
        const int ds = current_device(&dev);
        if (ds != 0) return ds;
        if (!fattr[dev][out_f32]) {
            const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, FB_SMEM);
            if (e != cudaSuccess) return (int) e;
            fattr[dev][out_f32] = true;
        }
        launch_k(kern, grid, FB_THREADS, FB_SMEM, stream, *T, static_cast<const uint16_t *>(a->w),
                                                    static_cast<const uint16_t *>(a->x), dst, a->K, a->M, a->N, a->ne02,
                                                    a->ne12, r2, r3, a->monte_seed, vec ? 1 : 0, peers ? *peers : no_peers,
                                                    gx, nfull);
    } else if (fmt == LNSB_XLNS32 || k_mode == M_SUM32 || k_mode == M_LPVIP || k_mode == M_MONTE_BYLPVIP) {
        return mul_mat_a32(fmt, *T, a, dst, out_f32, r2, r3, stream, peers ? *peers : no_peers);
    } else {
        return LNSB_E_UNSUPPORTED;
    }
    return launch_status();
}

constexpr int NN_SMEM_MAX = 200 * 1024;      // dynamic shared memory of a normaliser block, at most

// raises a kernel's dynamic shared memory limit once per device and kernel
// (whenever it takes any: the default 48 KB covers static and dynamic together)
// resident blocks per SM of a kernel at a block size and dynamic shared
// memory (the occupancy query, cached per device; 0 if it fails)
int blocks_per_sm(const void * kern, int threads, int smem) {
    int dev = 0;
    if (current_device(&dev) != 0) return 0;
    struct entry { const void * k; int t, s, occ; };
    static std::mutex mu;
    static std::array<std::vector<entry>, k_max_devices> cache;
    std::lock_guard<std::mutex> lock(mu);
    for (const auto & e : cache[dev]) if (e.k == kern && e.t == threads && e.s == smem) return e.occ;
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, threads, (size_t) smem) != cudaSuccess) {
        cudaGetLastError();
        occ = 0;
    }
    cache[dev].push_back({ kern, threads, smem, occ });
    return occ;
}

int nn_smem_attr(const void * kern, int bytes) {
    if (bytes <= 0) return 0;
    int dev = 0;
    const int ds = current_device(&dev);
    if (ds != 0) return ds;
    static std::mutex mu;
    static std::array<std::vector<std::pair<const void *, int>>, k_max_devices> done;
    std::lock_guard<std::mutex> lock(mu);
    for (auto & e : done[dev]) if (e.first == kern && e.second >= bytes) return 0;
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, NN_SMEM_MAX);
    if (e != cudaSuccess) return (int) e;
    done[dev].push_back({ kern, NN_SMEM_MAX });
    return 0;
}

// true when the float -> xlns16 table is, for every normal float, the
// exponent-plus-mantissa split that conv16_split computes (G read off the
// entries at e = 127 and e = 126); checked once over all 131072 entries
bool conv16_splits() {
    static const bool ok = [] {
        const std::vector<uint16_t> & c = get_host_tables(false, false).conv16;
        for (uint32_t u = 0; u < 131072; u++) {
            const uint32_t e = (u >> 8) & 0xFFu, m = u & 0xFFu;
            if (e == 0 || e == 255) continue;
            const int gp = (int) c[(127u << 8) | m] - 0x4000, gn = (int) c[(126u << 8) | m] - 0x4000 + 128;
            if (gp < 0 || gp > 255 || gn < 0 || gn > 255) return false;
            int v = 128 * ((int) e - 127) + (e < 127 ? gn : gp) + 0x4000;
            v = v < 0 ? 0 : (v > 0x7FFF ? 0x7FFF : v);
            if (c[u] != (((u >> 1) & 0x8000u) | (uint32_t) v)) return false;
        }
        return true;
    }();
    return ok;
}

int rms_norm_impl(int fmt, const void * src, void * dst, int64_t ncols, int64_t nrows, float eps, uint16_t seed,
                  bool io_f32, cudaStream_t stream, bool fuse = false, const float * res = nullptr,
                  float * x_out = nullptr, const float * nw = nullptr) {
    if (!valid_fmt(fmt) || ncols < 0 || nrows < 0) return LNSB_E_INVALID;
    if (nrows == 0 || ncols == 0) return 0;
    if (src == nullptr || dst == nullptr) return LNSB_E_INVALID;
    const dev_tables * T = nullptr;
    const int st = tables_for(fmt, &T);
    if (st != 0) return st;
    const host_tables & H = get_host_tables(false, false);
    uint32_t eps_l, inv_n;
    const float invf = 1.0f / (float) ncols;
    if (fmt == LNSB_XLNS16) {
        uint32_t b;
        std::memcpy(&b, &eps, 4);  eps_l = H.conv16[b >> 15];
        std::memcpy(&b, &invf, 4); inv_n = H.conv16[b >> 15];
    } else {
        eps_l = host_from_f32_32(eps);
        inv_n = host_from_f32_32(invf);
    }
    // non-negative chains over shared memory (base, sum32): the block's squares must fit
    int rpb = 32, nn_ok = 0, dsmem = 0;
    if (fmt == LNSB_XLNS32 || NNCHAIN) {
        const int tabb = fmt == LNSB_XLNS32 ? nn_tab<32>() : nn_tab<16>();
        const int tb   = fmt == LNSB_XLNS32 ? 4 : 2;
        const int64_t fit = (NN_SMEM_MAX - tabb) / (nn_pitch(ncols, tb) * tb);
        if (fit >= 1) {
            rpb = (int) imin64(32, fit);
            nn_ok = 1;
            dsmem = tabb + (int) (((int64_t) rpb * nn_pitch(ncols, tb) * tb + 15) / 16 * 16);
        }
    }
    // rows over about two blocks per SM, 256 threads each: the element passes
    // (and the fused block's residual add, weight and conversions) are latency
    // bound, so more blocks with fewer rows each finish sooner
    rpb = (int) imin64(rpb, imin64(32, (nrows + 2 * 148 - 1) / (2 * 148)));
    if (rpb < 1) rpb = 1;
    if (nn_ok) {
        const int tb = fmt == LNSB_XLNS32 ? 4 : 2;
        dsmem = (fmt == LNSB_XLNS32 ? nn_tab<32>() : nn_tab<16>()) + (int) (((int64_t) rpb * nn_pitch(ncols, tb) * tb + 15) / 16 * 16);
    }
    const unsigned blocks = (unsigned) ((nrows + rpb - 1) / rpb);
    auto kern = fuse ? (fmt == LNSB_XLNS16 ? k_rms_norm<16, true, true> : k_rms_norm<32, true, true>)
                     : fmt == LNSB_XLNS16 ? (io_f32 ? k_rms_norm<16, true> : k_rms_norm<16, false>)
                                          : (io_f32 ? k_rms_norm<32, true> : k_rms_norm<32, false>);
    const int st2 = nn_smem_attr((const void *) kern, dsmem);
    if (st2 != 0) return st2;
    launch_k(kern, blocks, 256, dsmem, stream, *T, src, dst, ncols, nrows, eps_l, inv_n, seed, rpb, nn_ok, res,
             x_out, nw);
    return launch_status();
}

int soft_max_impl(int fmt, const void * src, lnsb_shape4 s, const void * mask, lnsb_shape4 ms, uint32_t scale_l,
                  void * dst, void * work, uint16_t seed, bool io_f32, cudaStream_t stream) {
    if (!valid_fmt(fmt)) return LNSB_E_INVALID;
    for (int i = 0; i < 4; i++) if (s.ne[i] < 0) return LNSB_E_INVALID;
    const int64_t nrows = s.ne[1] * s.ne[2] * s.ne[3];
    if (nrows == 0 || s.ne[0] == 0) return 0;
    if (src == nullptr || dst == nullptr || work == nullptr) return LNSB_E_INVALID;
    if (mask != nullptr) {
        if (ms.ne[0] != s.ne[0] || ms.ne[1] < s.ne[1] || ms.ne[2] <= 0 || ms.ne[3] <= 0) return LNSB_E_INVALID;
    } else {
        ms = lnsb_shape4{ { 1, 1, 1, 1 } };
    }
    const dev_tables * T = nullptr;
    const int st = tables_for(fmt, &T);
    if (st != 0) return st;
    int dev = 0;
    const int ds = current_device(&dev);
    if (ds != 0) return ds;
    auto kern = fmt == LNSB_XLNS16 ? (io_f32 ? k_soft_max<16, true> : k_soft_max<16, false>)
                                   : (io_f32 ? k_soft_max<32, true> : k_soft_max<32, false>);
    const int tabb = fmt == LNSB_XLNS32 ? nn_tab<32>() : nn_tab<16>();
    const int tb   = fmt == LNSB_XLNS32 ? 4 : 2;
    const int64_t pitch_b = nn_pitch(s.ne[0], tb) * tb;
    const int64_t fit = (NN_SMEM_MAX - tabb) / pitch_b;          // rows whose terms fit in shared memory
    const int nn_ok = fit >= 1 ? 1 : 0;
    auto smem_for = [&](int r) { return nn_ok ? tabb + (int) (((int64_t) r * pitch_b + 15) / 16 * 16) : 0; };
    // rows over about two blocks per SM, then as many more rows per block as it
    // takes for every block to be resident at once: a second wave would repeat
    // the whole chain time
    int rpb = (int) imin64(32, (nrows + 2 * sm_count(dev) - 1) / (2 * sm_count(dev)));
    if (nn_ok) rpb = (int) imin64(rpb, fit);
    const int st2 = nn_smem_attr((const void *) kern, smem_for(rpb));
    if (st2 != 0) return st2;
    for (int it = 0; it < 4; it++) {
        const int occ = blocks_per_sm((const void *) kern, SM_THREADS, smem_for(rpb));
        if (occ < 1) break;
        const int64_t resident = (int64_t) occ * sm_count(dev);
        if ((nrows + rpb - 1) / rpb <= resident) break;
        int want = (int) imin64(32, (nrows + resident - 1) / resident);
        if (nn_ok) want = (int) imin64(want, fit);
        if (want <= rpb) break;
        rpb = want;
    }
    const int dsmem = smem_for(rpb);
    const unsigned blocks = (unsigned) ((nrows + rpb - 1) / rpb);
    launch_k(kern, blocks, SM_THREADS, dsmem, stream, *T, src, s, mask, ms, scale_l, dst, work, seed, rpb, nn_ok);
    return launch_status();
}

// ============================ Monte state ==================================
std::mutex g_monte_mu;
uint16_t   g_monte_state = 7;

const char * mode_name() {
    switch (k_mode) {
        case M_MONTE:
        case M_MONTE_BYLPVIP: return "monte";
        case M_LPVIP:         return "lpvip";
        case M_SUM32:         return "sum32";
        default:              return "base";
    }
}

}  // namespace

// float -> xlns32 on the host, identical to the device conversion
uint32_t host_from_f32_32(float x) {
    const host_tables & H = get_host_tables(true, false);
    uint32_t b;
    std::memcpy(&b, &x, 4);
    const uint32_t sign = b & 0x80000000u;
    uint32_t ex = (b >> 23) & 0xFFu, man = b & 0x7FFFFFu;
    if (ex == 0xFFu) return man ? 0u : (sign | 0x7FFFFFFFu);
    if (ex == 0 && man == 0) return 0u;
    int e;
    if (ex == 0) {
        e = -126;
        while (!(man & 0x800000u)) { man <<= 1; e--; }
        man &= 0x7FFFFFu;
    } else {
        e = (int) ex - 127;
    }
    long long l = (long long) e * (long long) k32_one + (long long) H.logm32[man];
    if (e < 0 && man != 0) l += 1;
    return sign | (uint32_t) ((l + 0x40000000LL) & 0x7FFFFFFFLL);
}

}  // namespace lnsb

using namespace lnsb;

// The weight cache behind lnsb_weight_cache_* (lns-cuda-context.h:79-113):
// one map per cache from (data pointer, type, rows, cols) to a device
// buffer, a byte budget, and a device staging buffer for host-resident rows.
struct lnsb_weight_cache {
    struct key {
        const void * data;
        int          type;
        int64_t      rows, cols;
        bool operator<(const key & o) const {
            if (data != o.data) return data < o.data;
            if (type != o.type) return type < o.type;
            if (rows != o.rows) return rows < o.rows;
            return cols < o.cols;
        }
    };
    int                    fmt = 0, dev = 0;
    int64_t                budget = 0, used = 0;
    int64_t                fail_allocs = 0;      // host-side fault injection: allocations to refuse
    std::map<key, void *>  entries;
    void *                 staging = nullptr;
    size_t                 staging_bytes = 0;
    std::mutex             mu;
};

// Dependent latency of one addition, for the chain bounds of latency-bound
// ops: one warp runs `steps` dependent additions per lane over operands of a
// dot product's spread (logs -6 +- 2 octaves, mixed signs for the general
// addition, non-negative terms for the normalisers'), with the adder's table
// in shared memory as the kernels hold it; lanes past `lanes` repeat the
// first `lanes` (same addresses).  kind 0: the key-form general xlns16
// addition of the latency mul_mat kernels; 1: the non-negative xlns16
// addition (padd16); 2: the non-negative xlns32 addition (padd32f); 3: the
// general xlns32 addition of the latency mat-vecs (add32f_sel).  out[0]:
// SM cycles over the timed steps, out[1]: the final accumulator (keeps the
// chain live).
constexpr int AL_OPS = 256;                                      // operands per lane, cycled
constexpr int AL_TAB = k32f_words * 4 > k16s_bytes ? k32f_words * 4 : k16s_bytes;   // the largest table staged
__global__ void __launch_bounds__(32) k_add_latency(dev_tables T, int kind, int lanes, int steps, int64_t * out) {
    extern __shared__ __align__(16) unsigned char smem[];
    constexpr int TAB = AL_TAB;
    const int lane = threadIdx.x, me = lane % lanes;
    int32_t * ops = reinterpret_cast<int32_t *>(smem + TAB);     // [AL_OPS][32]
    if (kind == 0) stage_async(smem, T.key16s, k16s_bytes);
    else if (kind == 1) stage_async(smem, T.sbdb16, k16_tab_bytes16);
    else if (kind == 2) stage_async(smem, T.flat32, k32f_sb_bytes16);
    else stage_async(smem, T.flat32, k32f_words * 4);
    cp_async_commit();
    for (int i = 0; i < AL_OPS; i++) {
        uint32_t h = (uint32_t) (me * 7919 + i) * 2654435761u;
        h ^= h >> 15;
        h *= 2246822519u;
        h ^= h >> 13;
        const int lg = 0x4000 - 768 + (int) (h % 512u) - 256;    // -6 +- 2 octaves
        const uint32_t code = (uint32_t) lg | (kind == 0 || kind == 3 ? ((h >> 20) & 1u) << 15 : 0u);
        ops[i * 32 + lane] = kind == 0 ? key_of_product(key_of_code_w(code), key_of_code_x(0x4000u))
                           : kind == 1 ? (int32_t) code : (int32_t) (code << 16);
    }
    cp_async_wait<0>();
    __syncwarp();
    constexpr int KM = LT_KM;
    uint32_t a = (uint32_t) ops[lane];
    const long long t0 = clock64();
    if (kind == 0) {
        int ak = (int) a;
        for (int k = 1; k < steps; k++) {
            const int p = ops[(k & (AL_OPS - 1)) * 32 + lane];
            const uint32_t idx = __viaddmin_u32((uint32_t) ak, (uint32_t) (KM - p), 2u * KM);
            ak = __viaddmax_s32(max(ak, p), *reinterpret_cast<const int *>(smem + idx), 0);
        }
        a = (uint32_t) ak;
    } else if (kind == 1) {
        for (int k = 1; k < steps; k++) a = padd16(a, (uint32_t) ops[(k & (AL_OPS - 1)) * 32 + lane], reinterpret_cast<const int16_t *>(smem));
    } else if (kind == 2) {
        for (int k = 1; k < steps; k++) a = padd32f(reinterpret_cast<const int32_t *>(smem), a, (uint32_t) ops[(k & (AL_OPS - 1)) * 32 + lane]);
    } else {
        for (int k = 1; k < steps; k++) a = add32f_sel(reinterpret_cast<const int32_t *>(smem), a, (uint32_t) ops[(k & (AL_OPS - 1)) * 32 + lane]);
    }
    const long long t1 = clock64();
    if (lane == 0) { out[0] = t1 - t0; out[1] = (int64_t) a; }
}

// dst (packed [ne3][ne2][ne1][ne0]) = the strided view src (byte strides nb)
// of E elements: the gather of permuted views (KV-cache views and the like)
template <typename E>
__global__ void k_copy_strided(const unsigned char * __restrict__ src, lnsb_shape4 ne, lnsb_shape4 nb,
                               E * __restrict__ dst, int64_t n) {
    pdl_entry();
    LNSB_GRID_STRIDE(i, n) {
        const int64_t i0 = i % ne.ne[0], r = i / ne.ne[0];
        const int64_t i1 = r % ne.ne[1], r2 = r / ne.ne[1];
        const int64_t i2 = r2 % ne.ne[2], i3 = r2 / ne.ne[2];
        dst[i] = *reinterpret_cast<const E *>(src + i0 * nb.ne[0] + i1 * nb.ne[1] + i2 * nb.ne[2] + i3 * nb.ne[3]);
    }
}

// the glu kernels by format, output form and activation
template <int FMT, bool OUT_LNS>
void launch_glu(int op, unsigned g, cudaStream_t s, const dev_tables & T, const float * gate, const float * up,
                int64_t gs, int64_t us, void * dst, int64_t nc, int64_t nr) {
    if (op == LNSB_GLU_SWIGLU) launch_k(k_swiglu<FMT, OUT_LNS, LNSB_UNARY_SILU>, g, 256, 0, s, T, gate, up, gs, us, dst, nc, nr);
    else                       launch_k(k_swiglu<FMT, OUT_LNS, LNSB_UNARY_GELU>, g, 256, 0, s, T, gate, up, gs, us, dst, nc, nr);
}

// ================================ C ABI =====================================

extern "C" {

const char * lnsb_format_name(int fmt) {
    return fmt == LNSB_XLNS16 ? "xlns16" : fmt == LNSB_XLNS32 ? "xlns32" : nullptr;
}

size_t lnsb_value_size(int fmt) { return fmt == LNSB_XLNS16 ? 2 : fmt == LNSB_XLNS32 ? 4 : 0; }

const char * lnsb_sum_mode(int fmt) { return fmt == LNSB_XLNS16 ? mode_name() : nullptr; }

const char * lnsb_monte_impl(int fmt) {
    if (fmt != LNSB_XLNS16) return nullptr;
    if (k_mode == M_MONTE) return "pure16";
    if (k_mode == M_MONTE_BYLPVIP) return "bylpvip";
    return nullptr;
}

const char * lnsb_description(int fmt) {
    if (fmt == LNSB_XLNS32) return "Logarithmic Number System on B200 (xlns32)";
    if (fmt != LNSB_XLNS16) return nullptr;
    switch (k_mode) {
        case M_MONTE:         return "Logarithmic Number System on B200 (xlns16, sum=monte, monte=pure16)";
        case M_MONTE_BYLPVIP: return "Logarithmic Number System on B200 (xlns16, sum=monte, monte=bylpvip)";
        case M_LPVIP:         return "Logarithmic Number System on B200 (xlns16, sum=lpvip)";
        case M_SUM32:         return "Logarithmic Number System on B200 (xlns16, sum=sum32)";
        default:              return "Logarithmic Number System on B200 (xlns16, sum=base)";
    }
}

uint64_t lnsb_mul_mat_draws(int fmt, const lnsb_mul_mat_args * a) {
    if (fmt != LNSB_XLNS16 || !k_stochastic || a == nullptr || a->K <= 0) return 0;
    return (uint64_t) a->ne12 * (uint64_t) a->ne13 * (uint64_t) a->M * (uint64_t) a->N * (uint64_t) (a->K - 1);
}

uint64_t lnsb_mul_mat_id_draws(int fmt, const lnsb_mul_mat_id_args * a) {
    if (fmt != LNSB_XLNS16 || !k_stochastic || a == nullptr || a->K <= 0 || a->M < 0 || a->n_used < 0 || a->n_tokens < 0)
        return 0;
    return (uint64_t) a->n_tokens * (uint64_t) a->n_used * (uint64_t) a->M * (uint64_t) (a->K - 1);
}

uint64_t lnsb_soft_max_draws(int fmt, int64_t ncols, int64_t nrows) {
    return fmt == LNSB_XLNS16 && k_stochastic && ncols > 0 ? (uint64_t) nrows * (uint64_t) (ncols - 1) : 0;
}

uint64_t lnsb_rms_norm_draws(int fmt, int64_t ncols, int64_t nrows) {
    return fmt == LNSB_XLNS16 && k_stochastic ? (uint64_t) nrows * (uint64_t) ncols : 0;
}

int lnsb_upload_tables(int fmt) {
    if (!valid_fmt(fmt)) return LNSB_E_INVALID;
    int dev = 0;
    int st = current_device(&dev);
    if (st != 0) return st;
    const bool need32 = fmt == LNSB_XLNS32;
    const bool need_lpvip = k_mode == M_LPVIP || k_mode == M_MONTE_BYLPVIP;
    std::lock_guard<std::mutex> lock(g_mu);
    device_slot & s = g_slots[dev];
    if ((fmt == LNSB_XLNS16 && s.ready16) || (fmt == LNSB_XLNS32 && s.ready32)) return 0;
    const host_tables & H = get_host_tables(need32, need_lpvip);
    if (H.flat32.size() != (size_t) k32f_words) return LNSB_E_NO_TABLES;
    dev_tables & t = s.t;
    cudaError_t e = cudaSuccess;
    if (t.sbdb16 == nullptr) {
        if (e == cudaSuccess) e = upload(H.sbdb16, &t.sbdb16);
        if (e == cudaSuccess) e = upload(H.conv16, &t.conv16);
        if (e == cudaSuccess) e = upload(H.dec16, &t.dec16);
        if (e == cudaSuccess) e = upload(H.exp16, &t.exp16);
        if (e == cudaSuccess) e = upload(H.sig16, &t.sig16);
        if (e == cudaSuccess) e = upload(H.monte16, &t.monte16);
        if (e == cudaSuccess) e = upload(H.key16, &t.key16);
        if (e == cudaSuccess) e = upload(H.mkey16, &t.mkey16);
        if (e == cudaSuccess) e = upload(H.key16s, &t.key16s);
        if (e == cudaSuccess) e = upload(H.sb32, &t.sb32);
        if (e == cudaSuccess) e = upload(H.db32, &t.db32);
        if (e == cudaSuccess) e = upload(H.db32_hi, &t.db32_hi);
        if (e == cudaSuccess) e = upload(H.db32_lo, &t.db32_lo);
        if (e == cudaSuccess) e = upload(H.flat32, &t.flat32);
        if (e == cudaSuccess) e = upload(H.lfsr_log, &t.lfsr_log);
        if (e == cudaSuccess) e = upload(H.lfsr_alog, &t.lfsr_alog);
    }
    if (e == cudaSuccess && need_lpvip && t.lpvip_db == nullptr) e = upload(H.lpvip_db, &t.lpvip_db);
    if (e == cudaSuccess && need32 && t.logm32 == nullptr) {
        e = upload(H.logm32, &t.logm32);
        if (e == cudaSuccess) e = upload(H.expm32, &t.expm32);
    }
    if (e != cudaSuccess) return (int) e;
    if (fmt == LNSB_XLNS16) s.ready16 = true;
    else s.ready32 = true;
    return 0;
}

int lnsb_to_lns(int fmt, const float * src, void * dst, int64_t n, lnsb_stream_t stream) {
    if (!valid_fmt(fmt) || n < 0) return LNSB_E_INVALID;
    if (n == 0) return 0;
    if (src == nullptr || dst == nullptr) return LNSB_E_INVALID;
    const dev_tables * T = nullptr;
    const int st = tables_for(fmt, &T);
    if (st != 0) return st;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (fmt == LNSB_XLNS16) launch_k(k_to_lns<16>, grid_for(n, 256), 256, 0, s, *T, src, dst, n);
    else                    launch_k(k_to_lns<32>, grid_for(n, 256), 256, 0, s, *T, src, dst, n);
    return launch_status();
}

int lnsb_to_lns_transposed(int fmt, const float * src, void * dst, int64_t rows, int64_t cols, int64_t dst_ld,
                           lnsb_stream_t stream) {
    if (!valid_fmt(fmt) || rows < 0 || cols < 0 || dst_ld < rows) return LNSB_E_INVALID;
    if (rows == 0 || cols == 0) return 0;
    if (src == nullptr || dst == nullptr) return LNSB_E_INVALID;
    if ((cols + 31) / 32 > 0x7FFFFFFF || (rows + 31) / 32 > 65535) return LNSB_E_TOO_LARGE;
    const dev_tables * T = nullptr;
    const int st = tables_for(fmt, &T);
    if (st != 0) return st;
    const dim3 grid((unsigned) ((cols + 31) / 32), (unsigned) ((rows + 31) / 32));
    const dim3 block(32, 8);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (fmt == LNSB_XLNS16) launch_k(k_to_lns_transposed<16>, grid, block, 0, s, *T, src, dst, rows, cols, dst_ld);
    else                    launch_k(k_to_lns_transposed<32>, grid, block, 0, s, *T, src, dst, rows, cols, dst_ld);
    return launch_status();
}

static bool known_type(int type) {
    return type == LNSB_TYPE_F32 || type == LNSB_TYPE_F16 || type == LNSB_TYPE_BF16 || type == LNSB_TYPE_Q8_0 ||
           type == LNSB_TYPE_Q4_0 || type == LNSB_TYPE_Q4_K || type == LNSB_TYPE_Q6_K;
}

size_t lnsb_type_row_bytes(int type, int64_t cols) {
    if (cols < 0) return 0;
    switch (type) {
        case LNSB_TYPE_F32:  return (size_t) cols * 4;
        case LNSB_TYPE_F16:
        case LNSB_TYPE_BF16: return (size_t) cols * 2;
        case LNSB_TYPE_Q8_0: return cols % 32 ? 0 : (size_t) (cols / 32) * 34;
        case LNSB_TYPE_Q4_0: return cols % 32 ? 0 : (size_t) (cols / 32) * 18;
        case LNSB_TYPE_Q4_K: return cols % 256 ? 0 : (size_t) (cols / 256) * 144;
        case LNSB_TYPE_Q6_K: return cols % 256 ? 0 : (size_t) (cols / 256) * 210;
        default:             return 0;
    }
}

int lnsb_to_lns_transposed_typed(int fmt, int type, const void * src, void * dst, int64_t rows, int64_t cols,
                                 int64_t dst_ld, lnsb_stream_t stream) {
    if (!valid_fmt(fmt) || rows < 0 || cols < 0 || dst_ld < rows) return LNSB_E_INVALID;
    if (!known_type(type)) return LNSB_E_UNSUPPORTED;
    const size_t rb = lnsb_type_row_bytes(type, cols);
    if (cols > 0 && rb == 0) return LNSB_E_INVALID;          // cols not a whole number of blocks
    if (rows == 0 || cols == 0) return 0;
    if (src == nullptr || dst == nullptr) return LNSB_E_INVALID;
    if ((cols + 31) / 32 > 0x7FFFFFFF || (rows + 31) / 32 > 65535) return LNSB_E_TOO_LARGE;
    const dev_tables * T = nullptr;
    const int st = tables_for(fmt, &T);
    if (st != 0) return st;
    int dev = 0;
    const int ds = current_device(&dev);
    if (ds != 0) return ds;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const auto * p = static_cast<const unsigned char *>(src);
    if (fmt == LNSB_XLNS16 && conv16_splits() && ((rows + TW_ROWS - 1) / TW_ROWS) * ((cols + 127) / 128) < 0x7FFFFFFF) {
        auto tiled = [&](auto kern, int smem, int tcols) {
            const int as = nn_smem_attr(reinterpret_cast<const void *>(kern), smem);
            if (as != 0) return as;
            const int64_t ntiles = ((rows + TW_ROWS - 1) / TW_ROWS) * ((cols + tcols - 1) / tcols);
            const int vin = (uintptr_t) p % 16 == 0 && rb % 16 == 0;
            const int vout = (uintptr_t) dst % 16 == 0 && dst_ld % 8 == 0;
            launch_k(kern, dim3((unsigned) imin64(ntiles, (int64_t) sm_count(dev))), TW_THREADS, (size_t) smem, s, *T,
                     p, (int64_t) rb, static_cast<uint16_t *>(dst), rows, cols, dst_ld, vin, vout);
            return launch_status();
        };
#define LNSB_TW(TY) tiled(k_to_lns16_typed_tiled<TY>, tw_geom<TY>::smem, tw_geom<TY>::cols)
        switch (type) {
            case LNSB_TYPE_F32:  return LNSB_TW(LNSB_TYPE_F32);
            case LNSB_TYPE_F16:  return LNSB_TW(LNSB_TYPE_F16);
            case LNSB_TYPE_BF16: return LNSB_TW(LNSB_TYPE_BF16);
            case LNSB_TYPE_Q8_0: return LNSB_TW(LNSB_TYPE_Q8_0);
            case LNSB_TYPE_Q4_0: return LNSB_TW(LNSB_TYPE_Q4_0);
            case LNSB_TYPE_Q4_K: return LNSB_TW(LNSB_TYPE_Q4_K);
            default:             return LNSB_TW(LNSB_TYPE_Q6_K);
        }
#undef LNSB_TW
    }
    const int64_t ntiles = ((cols + 31) / 32) * ((rows + 31) / 32);
    const dim3 grid((unsigned) imin64(ntiles, (int64_t) sm_count(dev) * 16));
    const dim3 block(32, 8);
    auto go = [&](auto k16, auto k32) {
        if (fmt == LNSB_XLNS16) launch_k(k16, grid, block, 0, s, *T, type, p, (int64_t) rb, dst, rows, cols, dst_ld);
        else                    launch_k(k32, grid, block, 0, s, *T, type, p, (int64_t) rb, dst, rows, cols, dst_ld);
    };
    switch (type) {
        case LNSB_TYPE_F32:  go(k_to_lns_transposed_typed<16, LNSB_TYPE_F32>, k_to_lns_transposed_typed<32, LNSB_TYPE_F32>); break;
        case LNSB_TYPE_F16:  go(k_to_lns_transposed_typed<16, LNSB_TYPE_F16>, k_to_lns_transposed_typed<32, LNSB_TYPE_F16>); break;
        case LNSB_TYPE_BF16: go(k_to_lns_transposed_typed<16, LNSB_TYPE_BF16>, k_to_lns_transposed_typed<32, LNSB_TYPE_BF16>); break;
        case LNSB_TYPE_Q8_0: go(k_to_lns_transposed_typed<16, LNSB_TYPE_Q8_0>, k_to_lns_transposed_typed<32, LNSB_TYPE_Q8_0>); break;
        case LNSB_TYPE_Q4_0: go(k_to_lns_transposed_typed<16, LNSB_TYPE_Q4_0>, k_to_lns_transposed_typed<32, LNSB_TYPE_Q4_0>); break;
        case LNSB_TYPE_Q4_K: go(k_to_lns_transposed_typed<16, LNSB_TYPE_Q4_K>, k_to_lns_transposed_typed<32, LNSB_TYPE_Q4_K>); break;
        default:             go(k_to_lns_transposed_typed<16, LNSB_TYPE_Q6_K>, k_to_lns_transposed_typed<32, LNSB_TYPE_Q6_K>); break;
    }
    return launch_status();
}

int lnsb_dequantize(int type, const void * src, float * dst, int64_t rows, int64_t cols, lnsb_stream_t stream) {
    if (rows < 0 || cols < 0) return LNSB_E_INVALID;
    if (!known_type(type)) return LNSB_E_UNSUPPORTED;
    const size_t rb = lnsb_type_row_bytes(type, cols);
    if (cols > 0 && rb == 0) return LNSB_E_INVALID;
    if (rows == 0 || cols == 0) return 0;
    if (src == nullptr || dst == nullptr) return LNSB_E_INVALID;
    launch_k(k_dequantize, grid_for(rows * cols, 256), 256, 0, static_cast<cudaStream_t>(stream), 
        type, static_cast<const unsigned char *>(src), (int64_t) rb, dst, rows, cols);
    return launch_status();
}

int lnsb_to_f32(int fmt, const void * src, float * dst, int64_t n, lnsb_stream_t stream) {
    if (!valid_fmt(fmt) || n < 0) return LNSB_E_INVALID;
    if (n == 0) return 0;
    if (src == nullptr || dst == nullptr) return LNSB_E_INVALID;
    const dev_tables * T = nullptr;
    const int st = tables_for(fmt, &T);
    if (st != 0) return st;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (fmt == LNSB_XLNS16) launch_k(k_to_f32<16>, grid_for(n, 256), 256, 0, s, *T, src, dst, n);
    else                    launch_k(k_to_f32<32>, grid_for(n, 256), 256, 0, s, *T, src, dst, n);
    return launch_status();
}

int lnsb_mul_mat(int fmt, const lnsb_mul_mat_args * args, lnsb_stream_t stream) {
    return mul_mat_impl(fmt, args, args ? args->dst : nullptr, true, static_cast<cudaStream_t>(stream));
}

int lnsb_mul_mat_lns(int fmt, const lnsb_mul_mat_args * args, void * dst_lns, lnsb_stream_t stream) {
    return mul_mat_impl(fmt, args, dst_lns, false, static_cast<cudaStream_t>(stream));
}

int lnsb_mul_mat_xf32(int fmt, const lnsb_mul_mat_args * args, void * x_work, lnsb_stream_t stream) {
    return mul_mat_impl(fmt, args, args ? args->dst : nullptr, true, static_cast<cudaStream_t>(stream), nullptr, true, x_work);
}

int lnsb_mul_mat_lns_peers(int fmt, const lnsb_mul_mat_args * args, const lnsb_peer_out * peers, lnsb_stream_t stream) {
    if (peers == nullptr || peers->ptrs == nullptr || peers->n <= 0 || peers->offset < 0 || args == nullptr ||
        peers->ld < peers->offset + args->M)
        return LNSB_E_INVALID;
    const peer_out_dev p{ reinterpret_cast<uint16_t * const *>(peers->ptrs), peers->n, peers->ld, peers->offset };
    return mul_mat_impl(fmt, args, nullptr, false, static_cast<cudaStream_t>(stream), &p);
}

int lnsb_group_barrier(int32_t * const * flags, int world, int rank, int32_t epoch, int32_t * err, lnsb_stream_t stream) {
    if (flags == nullptr || err == nullptr || world <= 0 || world > 1024 || rank < 0 || rank >= world || epoch <= 0)
        return LNSB_E_INVALID;
    launch_k(k_group_barrier, dim3(1), dim3((unsigned) ((world + 31) / 32 * 32)), 0, static_cast<cudaStream_t>(stream),
             flags, world, rank, epoch, err, (long long) 1 << 21);
    return launch_status();
}

int lnsb_copy_strided(int elem_size, const void * src, const int64_t ne[4], const int64_t nb[4], void * dst,
                      lnsb_stream_t stream) {
    if ((elem_size != 2 && elem_size != 4) || ne == nullptr || nb == nullptr) return LNSB_E_INVALID;
    for (int i = 0; i < 4; i++) if (ne[i] < 0) return LNSB_E_INVALID;
    const int64_t n = ne[0] * ne[1] * ne[2] * ne[3];
    if (n == 0) return 0;
    if (src == nullptr || dst == nullptr) return LNSB_E_INVALID;
    const lnsb_shape4 e{ { ne[0], ne[1], ne[2], ne[3] } }, b{ { nb[0], nb[1], nb[2], nb[3] } };
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const auto * in = static_cast<const unsigned char *>(src);
    if (elem_size == 2) launch_k(k_copy_strided<uint16_t>, grid_for(n, 256), 256, 0, s, in, e, b, static_cast<uint16_t *>(dst), n);
    else                launch_k(k_copy_strided<uint32_t>, grid_for(n, 256), 256, 0, s, in, e, b, static_cast<uint32_t *>(dst), n);
    return launch_status();
}

int lnsb_add_latency(int kind, int lanes, int steps, int64_t * out, lnsb_stream_t stream) {
    if (kind < 0 || kind > 3 || lanes < 1 || lanes > 32 || steps < 2 || out == nullptr) return LNSB_E_INVALID;
    // every adder table here (key16s, sbdb16, the flat xlns32 image) is uploaded with either format's tables
    const dev_tables * T = nullptr;
    int st = tables_for(LNSB_XLNS16, &T);
    if (st == LNSB_E_NO_TABLES) st = tables_for(LNSB_XLNS32, &T);
    if (st != 0) return st;
    constexpr int smem = AL_TAB + AL_OPS * 32 * 4;
    static bool attr[k_max_devices] = {};
    int dev = 0;
    const int ds = current_device(&dev);
    if (ds != 0) return ds;
    if (!attr[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(k_add_latency, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return (int) e;
        attr[dev] = true;
    }
    k_add_latency<<<1, 32, smem, static_cast<cudaStream_t>(stream)>>>(*T, kind, lanes, steps, out);
    return launch_status();
}

int lnsb_mul_mat_id(int fmt, const lnsb_mul_mat_id_args * args, lnsb_stream_t stream) {
    return mul_mat_id_impl(fmt, args, args ? args->dst : nullptr, true, static_cast<cudaStream_t>(stream));
}

int lnsb_mul_mat_id_lns(int fmt, const lnsb_mul_mat_id_args * args, void * dst_lns, lnsb_stream_t stream) {
    return mul_mat_id_impl(fmt, args, dst_lns, false, static_cast<cudaStream_t>(stream));
}

int lnsb_mul_mat_id_bad_ids(int64_t * count) {
    if (count == nullptr) return LNSB_E_INVALID;
    unsigned long long v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_bad_ids, sizeof v);
    if (e == cudaSuccess) {
        const unsigned long long zero = 0;
        e = cudaMemcpyToSymbol(g_bad_ids, &zero, sizeof zero);
    }
    if (e != cudaSuccess) return (int) e;
    *count = (int64_t) v;
    return 0;
}

int lnsb_soft_max(int fmt, const lnsb_soft_max_args * a, lnsb_stream_t stream) {
    if (!valid_fmt(fmt) || a == nullptr) return LNSB_E_INVALID;
    uint32_t scale_l;
    if (fmt == LNSB_XLNS16) {
        const host_tables & H = get_host_tables(false, false);
        uint32_t b;
        std::memcpy(&b, &a->scale, 4);
        scale_l = H.conv16[b >> 15];
    } else {
        scale_l = host_from_f32_32(a->scale);
    }
    return soft_max_impl(fmt, a->src, a->src_shape, a->mask, a->mask_shape, scale_l, a->dst, a->work, a->monte_seed,
                         true, static_cast<cudaStream_t>(stream));
}

int lnsb_soft_max_lns(int fmt, const void * src, const int64_t ne[4], const void * mask, const int64_t mne[4],
                      uint32_t scale, void * dst, void * work, uint16_t monte_seed, lnsb_stream_t stream) {
    if (ne == nullptr || (mask != nullptr && mne == nullptr)) return LNSB_E_INVALID;
    lnsb_shape4 s{ { ne[0], ne[1], ne[2], ne[3] } };
    lnsb_shape4 ms{ { 1, 1, 1, 1 } };
    if (mask != nullptr) ms = lnsb_shape4{ { mne[0], mne[1], mne[2], mne[3] } };
    return soft_max_impl(fmt, src, s, mask, ms, scale, dst, work, monte_seed, false, static_cast<cudaStream_t>(stream));
}

int lnsb_soft_max_lns_noalloc(int fmt, const void * src, const int64_t ne[4], const void * mask,
                              const int64_t mne[4], uint32_t scale, void * dst, uint16_t monte_seed,
                              lnsb_stream_t stream) {
    static void * scratch_of[k_max_devices] = {};   // device address of g_noalloc_scratch, per device
    static std::mutex scratch_mu;
    if (!valid_fmt(fmt) || ne == nullptr || (mask != nullptr && mne == nullptr)) return LNSB_E_INVALID;
    for (int i = 0; i < 4; i++) if (ne[i] < 0) return LNSB_E_INVALID;
    for (int i = 0; i < 4; i++) if (ne[i] == 0) return 0;
    // the element count as a running product, refused as soon as it passes the
    // scratch's capacity, so that no product of huge dimensions can wrap
    const int64_t cap = (int64_t) (LNSB_NOALLOC_SCRATCH_BYTES / lnsb_value_size(fmt));
    int64_t nel = 1;
    for (int i = 0; i < 4; i++) {
        if (ne[i] > cap / nel) return LNSB_E_TOO_LARGE;
        nel *= ne[i];
    }
    int dev = 0;
    const int st = current_device(&dev);
    if (st != 0) return st;
    void * scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(scratch_mu);
        if (scratch_of[dev] == nullptr) {
            void * p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
            if (e != cudaSuccess) return (int) e;
            scratch_of[dev] = p;
        }
        scratch = scratch_of[dev];
    }
    // every element of the scratch is written (exp pass) before it is read
    // (normaliser and division passes), so nothing needs clearing between calls
    return lnsb_soft_max_lns(fmt, src, ne, mask, mne, scale, dst, scratch, monte_seed, stream);
}

int lnsb_rms_norm(int fmt, const float * src, float * dst, int64_t ncols, int64_t nrows, float eps, uint16_t monte_seed,
                  lnsb_stream_t stream) {
    return rms_norm_impl(fmt, src, dst, ncols, nrows, eps, monte_seed, true, static_cast<cudaStream_t>(stream));
}

int lnsb_rms_norm_lns(int fmt, const void * src, void * dst, int64_t ncols, int64_t nrows, float eps,
                      uint16_t monte_seed, lnsb_stream_t stream) {
    return rms_norm_impl(fmt, src, dst, ncols, nrows, eps, monte_seed, false, static_cast<cudaStream_t>(stream));
}

int lnsb_norm_block(int fmt, const lnsb_norm_block_args * a, lnsb_stream_t stream) {
    if (a == nullptr || a->src == nullptr || a->dst_lns == nullptr) return LNSB_E_INVALID;
    return rms_norm_impl(fmt, a->src, a->dst_lns, a->ncols, a->nrows, a->eps, a->monte_seed, true,
                         static_cast<cudaStream_t>(stream), true, a->residual, a->x_out, a->weight);
}

namespace {
bool shape_ok(const int64_t ne[4]) {
    if (ne == nullptr) return false;
    for (int i = 0; i < 4; i++) if (ne[i] < 0) return false;
    return true;
}
int64_t nel(const int64_t ne[4]) { return ne[0] * ne[1] * ne[2] * ne[3]; }
lnsb_shape4 shape_of(const int64_t ne[4]) { lnsb_shape4 s; for (int i = 0; i < 4; i++) s.ne[i] = ne[i]; return s; }
}  // namespace

int lnsb_binary(int fmt, int op, const float * a, const int64_t ane[4], const float * b, const int64_t bne[4],
                float * dst, lnsb_stream_t stream) {
    if (!valid_fmt(fmt) || op < LNSB_BINARY_ADD || op > LNSB_BINARY_DIV || !shape_ok(ane) || !shape_ok(bne)) return LNSB_E_INVALID;
    const int64_t n = nel(ane);
    if (n == 0) return 0;
    for (int i = 0; i < 4; i++) if (bne[i] <= 0 || ane[i] % bne[i] != 0) return LNSB_E_INVALID;   // b repeats to a
    if (a == nullptr || b == nullptr || dst == nullptr) return LNSB_E_INVALID;
    const dev_tables * T = nullptr;
    const int st = tables_for(fmt, &T);
    if (st != 0) return st;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const unsigned g = grid_for(n, 256);
    const lnsb_shape4 as = shape_of(ane), bs = shape_of(bne);
#define LNSB_BIN(F, O) launch_k(k_binary<F, O>, g, 256, 0, s, *T, a, as, b, bs, dst)
    if (fmt == LNSB_XLNS16) {
        if (op == LNSB_BINARY_ADD) LNSB_BIN(16, LNSB_BINARY_ADD); else if (op == LNSB_BINARY_MUL) LNSB_BIN(16, LNSB_BINARY_MUL); else LNSB_BIN(16, LNSB_BINARY_DIV);
    } else {
        if (op == LNSB_BINARY_ADD) LNSB_BIN(32, LNSB_BINARY_ADD); else if (op == LNSB_BINARY_MUL) LNSB_BIN(32, LNSB_BINARY_MUL); else LNSB_BIN(32, LNSB_BINARY_DIV);
    }
#undef LNSB_BIN
    return launch_status();
}

int lnsb_scale(int fmt, const float * src, float * dst, int64_t n, float sv, float bv, lnsb_stream_t stream) {
    if (!valid_fmt(fmt) || n < 0) return LNSB_E_INVALID;
    if (n == 0) return 0;
    if (src == nullptr || dst == nullptr) return LNSB_E_INVALID;
    const dev_tables * T = nullptr;
    const int st = tables_for(fmt, &T);
    if (st != 0) return st;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint32_t sl, bl;
    if (fmt == LNSB_XLNS16) {
        const host_tables & H = get_host_tables(false, false);
        uint32_t u;
        std::memcpy(&u, &sv, 4); sl = H.conv16[u >> 15];
        std::memcpy(&u, &bv, 4); bl = H.conv16[u >> 15];
        launch_k(k_scale<16>, grid_for(n, 256), 256, 0, s, *T, src, dst, n, sl, bl, bv != 0.0f ? 1 : 0);
    } else {
        sl = host_from_f32_32(sv);
        bl = host_from_f32_32(bv);
        launch_k(k_scale<32>, grid_for(n, 256), 256, 0, s, *T, src, dst, n, sl, bl, bv != 0.0f ? 1 : 0);
    }
    return launch_status();
}

int lnsb_unary(int fmt, int op, const float * src, float * dst, int64_t n, lnsb_stream_t stream) {
    if (!valid_fmt(fmt) || op < LNSB_UNARY_SILU || op > LNSB_UNARY_TANH || n < 0) return LNSB_E_INVALID;
    if (n == 0) return 0;
    if (src == nullptr || dst == nullptr) return LNSB_E_INVALID;
    const dev_tables * T = nullptr;
    const int st = tables_for(fmt, &T);
    if (st != 0) return st;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const unsigned g = grid_for(n, 256);
    if (fmt == LNSB_XLNS16) {
        switch (op) {
            case LNSB_UNARY_SILU: launch_k(k_unary<16, LNSB_UNARY_SILU>, g, 256, 0, s, *T, src, dst, n); break;
            case LNSB_UNARY_GELU: launch_k(k_unary<16, LNSB_UNARY_GELU>, g, 256, 0, s, *T, src, dst, n); break;
            case LNSB_UNARY_RELU: launch_k(k_unary<16, LNSB_UNARY_RELU>, g, 256, 0, s, *T, src, dst, n); break;
            default:              launch_k(k_unary<16, LNSB_UNARY_TANH>, g, 256, 0, s, *T, src, dst, n); break;
        }
    } else {
        switch (op) {
            case LNSB_UNARY_SILU: launch_k(k_unary<32, LNSB_UNARY_SILU>, g, 256, 0, s, *T, src, dst, n); break;
            case LNSB_UNARY_GELU: launch_k(k_unary<32, LNSB_UNARY_GELU>, g, 256, 0, s, *T, src, dst, n); break;
            case LNSB_UNARY_RELU: launch_k(k_unary<32, LNSB_UNARY_RELU>, g, 256, 0, s, *T, src, dst, n); break;
            default:              launch_k(k_unary<32, LNSB_UNARY_TANH>, g, 256, 0, s, *T, src, dst, n); break;
        }
    }
    return launch_status();
}

int lnsb_glu(int fmt, int op, const float * gate, const float * up, int64_t gate_stride, int64_t up_stride, float * dst,
             int64_t ncols, int64_t nrows, lnsb_stream_t stream) {
    if (!valid_fmt(fmt) || (op != LNSB_GLU_SWIGLU && op != LNSB_GLU_GEGLU) || ncols < 0 || nrows < 0) return LNSB_E_INVALID;
    if (ncols == 0 || nrows == 0) return 0;
    if (gate == nullptr || up == nullptr || dst == nullptr || gate_stride < ncols || up_stride < ncols) return LNSB_E_INVALID;
    const dev_tables * T = nullptr;
    const int st = tables_for(fmt, &T);
    if (st != 0) return st;
    const unsigned g = grid_for(ncols * nrows, 256);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (fmt == LNSB_XLNS16) launch_glu<16, false>(op, g, s, *T, gate, up, gate_stride, up_stride, dst, ncols, nrows);
    else                    launch_glu<32, false>(op, g, s, *T, gate, up, gate_stride, up_stride, dst, ncols, nrows);
    return launch_status();
}

int lnsb_glu_lns(int fmt, int op, const float * gate, const float * up, int64_t gate_stride, int64_t up_stride,
                 void * dst_lns, int64_t ncols, int64_t nrows, lnsb_stream_t stream) {
    if (!valid_fmt(fmt) || (op != LNSB_GLU_SWIGLU && op != LNSB_GLU_GEGLU) || ncols < 0 || nrows < 0) return LNSB_E_INVALID;
    if (ncols == 0 || nrows == 0) return 0;
    if (gate == nullptr || up == nullptr || dst_lns == nullptr || gate_stride < ncols || up_stride < ncols) return LNSB_E_INVALID;
    const dev_tables * T = nullptr;
    const int st = tables_for(fmt, &T);
    if (st != 0) return st;
    const unsigned g = grid_for(ncols * nrows, 256);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (fmt == LNSB_XLNS16) launch_glu<16, true>(op, g, s, *T, gate, up, gate_stride, up_stride, dst_lns, ncols, nrows);
    else                    launch_glu<32, true>(op, g, s, *T, gate, up, gate_stride, up_stride, dst_lns, ncols, nrows);
    return launch_status();
}

int lnsb_rope_qkv(int fmt, const lnsb_rope_qkv_args * a, lnsb_stream_t stream) {
    if (!valid_fmt(fmt) || a == nullptr) return LNSB_E_INVALID;
    if (a->n_tokens < 0 || a->n_head <= 0 || a->n_head_kv <= 0 || a->head_dim <= 0 || a->n_dims < 0 ||
        a->n_dims > a->head_dim || a->n_dims % 2 != 0 || a->ld < (int64_t) (a->n_head + 2 * a->n_head_kv) * a->head_dim ||
        a->kv_ld < (int64_t) a->n_head_kv * a->head_dim)
        return LNSB_E_INVALID;
    if (a->n_tokens == 0) return 0;
    if (a->qkv == nullptr || a->cos_sin == nullptr || a->q_out == nullptr || a->k_cache == nullptr || a->v_cache == nullptr)
        return LNSB_E_INVALID;
    const dev_tables * T = nullptr;
    const int st = tables_for(fmt, &T);
    if (st != 0) return st;
    const int64_t per = a->n_dims / 2 + (a->head_dim - a->n_dims);
    const int64_t n = a->n_tokens * ((int64_t) (a->n_head + a->n_head_kv) * per + (int64_t) a->n_head_kv * a->head_dim);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    auto kern = fmt == LNSB_XLNS16 ? k_rope_qkv<16> : k_rope_qkv<32>;
    launch_k(kern, grid_for(n, 256), 256, 0, s, *T, a->qkv, a->ld, a->cos_sin, a->n_dims, a->neox, a->n_head, a->n_head_kv,
             a->head_dim, a->n_tokens, a->q_out, reinterpret_cast<__half *>(a->k_cache), reinterpret_cast<__half *>(a->v_cache),
             a->kv_ld);
    return launch_status();
}

int lnsb_rope(int fmt, const lnsb_rope_args * a, lnsb_stream_t stream) {
    if (!valid_fmt(fmt) || a == nullptr || !shape_ok(a->shape.ne)) return LNSB_E_INVALID;
    if (a->n_dims <= 0 || a->n_dims % 2 != 0 || a->n_dims > a->shape.ne[0]) return LNSB_E_INVALID;
    const int64_t nrows = a->shape.ne[1] * a->shape.ne[2] * a->shape.ne[3];
    if (nrows == 0) return 0;
    if (a->src == nullptr || a->dst == nullptr || a->cos_sin == nullptr) return LNSB_E_INVALID;
    const dev_tables * T = nullptr;
    const int st = tables_for(fmt, &T);
    if (st != 0) return st;
    const int64_t per = a->n_dims / 2 + (a->shape.ne[0] - a->n_dims);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (fmt == LNSB_XLNS16) launch_k(k_rope<16>, grid_for(nrows * per, 256), 256, 0, s, *T, a->src, a->shape, a->cos_sin, a->n_dims, a->neox, a->dst);
    else                    launch_k(k_rope<32>, grid_for(nrows * per, 256), 256, 0, s, *T, a->src, a->shape, a->cos_sin, a->n_dims, a->neox, a->dst);
    return launch_status();
}

int64_t lnsb_attn_decode_max_keys(int fmt, int head_dim) {
    if (!valid_fmt(fmt) || head_dim <= 0) return 0;
    const int64_t fixed = (fmt == LNSB_XLNS16 ? attn_tab<16>() : attn_tab<32>()) + 4 * ((int64_t) head_dim * (ATTN_KT + 2));
    return fixed >= 220 * 1024 ? 0 : (220 * 1024 - fixed) / 8;
}

int lnsb_attn_decode(int fmt, const lnsb_attn_decode_args * a, lnsb_stream_t stream) {
    if (!valid_fmt(fmt) || a == nullptr) return LNSB_E_INVALID;
    if (a->nkv <= 0 || a->n_head <= 0 || a->n_head_kv <= 0 || a->head_dim <= 0 || a->n_head % a->n_head_kv != 0 ||
        a->kv_ld < (int64_t) a->n_head_kv * a->head_dim)
        return LNSB_E_INVALID;
    if (a->q == nullptr || a->k_cache == nullptr || a->v_cache == nullptr || (a->dst == nullptr && a->dst_lns == nullptr))
        return LNSB_E_INVALID;
    const int64_t bytes = (fmt == LNSB_XLNS16 ? attn_tab<16>() : attn_tab<32>()) +
                          4 * ((int64_t) a->head_dim * (ATTN_KT + 2) + 2 * a->nkv);
    if (a->nkv > lnsb_attn_decode_max_keys(fmt, a->head_dim) || a->n_head > 65535) return LNSB_E_TOO_LARGE;
    int dev = 0;
    const int ds = current_device(&dev);
    if (ds != 0) return ds;
    const dev_tables * T = nullptr;
    const int st = tables_for(fmt, &T);
    if (st != 0) return st;
    uint32_t scale_l;
    if (fmt == LNSB_XLNS16) {
        const host_tables & H = get_host_tables(false, false);
        uint32_t b;
        std::memcpy(&b, &a->scale, 4);
        scale_l = H.conv16[b >> 15];
    } else {
        scale_l = host_from_f32_32(a->scale);
    }
    static int attr[2][k_max_devices] = {};
    auto kern = fmt == LNSB_XLNS16 ? k_attn_decode<16> : k_attn_decode<32>;
    int & done = attr[fmt == LNSB_XLNS32][dev];
    if (done < bytes) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
        if (e != cudaSuccess) return (int) e;
        done = 220 * 1024;
    }
    launch_k(kern, dim3((unsigned) a->n_head), dim3(256), (size_t) bytes, static_cast<cudaStream_t>(stream), *T, a->q,
             reinterpret_cast<const __half *>(a->k_cache), reinterpret_cast<const __half *>(a->v_cache), a->kv_ld, a->nkv,
             a->n_head, a->n_head_kv, a->head_dim, scale_l, a->dst, (uint32_t) a->monte_seed, a->dst_lns);
    return launch_status();
}

int lnsb_f32_to_f16(const float * src, uint16_t * dst, int64_t n, lnsb_stream_t stream) {
    if (n < 0) return LNSB_E_INVALID;
    if (n == 0) return 0;
    if (src == nullptr || dst == nullptr) return LNSB_E_INVALID;
    launch_k(k_f32_to_f16, grid_for(n, 256), 256, 0, static_cast<cudaStream_t>(stream), src, reinterpret_cast<__half *>(dst), n);
    return launch_status();
}

int lnsb_f16_to_f32(const uint16_t * src, float * dst, int64_t n, lnsb_stream_t stream) {
    if (n < 0) return LNSB_E_INVALID;
    if (n == 0) return 0;
    if (src == nullptr || dst == nullptr) return LNSB_E_INVALID;
    launch_k(k_f16_to_f32, grid_for(n, 256), 256, 0, static_cast<cudaStream_t>(stream), reinterpret_cast<const __half *>(src), dst, n);
    return launch_status();
}

int lnsb_monte_get_state(uint16_t * state) {
    if (!k_stochastic) return LNSB_E_UNSUPPORTED;
    if (state == nullptr) return LNSB_E_INVALID;
    std::lock_guard<std::mutex> lock(g_monte_mu);
    *state = g_monte_state;
    return 0;
}

int lnsb_monte_set_state(uint16_t state) {
    if (!k_stochastic) return LNSB_E_UNSUPPORTED;
    if (state == 0) return LNSB_E_INVALID;
    std::lock_guard<std::mutex> lock(g_monte_mu);
    g_monte_state = state;
    return 0;
}

int lnsb_monte_reserve(uint64_t draws, uint16_t * start) {
    if (!k_stochastic) return LNSB_E_UNSUPPORTED;
    if (start == nullptr) return LNSB_E_INVALID;
    const host_tables & H = get_host_tables(false, false);
    std::lock_guard<std::mutex> lock(g_monte_mu);
    *start = g_monte_state;
    const uint64_t k = ((uint64_t) H.lfsr_log[g_monte_state] + draws % 65535u) % 65535u;
    g_monte_state = H.lfsr_alog[k];
    return 0;
}

const char * lnsb_error_string(int status) {
    switch (status) {
        case LNSB_OK:            return "success";
        case LNSB_E_INVALID:     return "invalid argument";
        case LNSB_E_NO_TABLES:   return "lnsb_upload_tables has not run on this device";
        case LNSB_E_UNSUPPORTED: return "not supported by this build";
        case LNSB_E_TOO_LARGE:   return "size beyond a documented limit";
        case LNSB_E_NO_DEVICE:   return "no usable CUDA device";
        default:                 return status > 0 ? cudaGetErrorString((cudaError_t) status) : "unknown error";
    }
}

lnsb_weight_cache * lnsb_weight_cache_create(int fmt, int64_t budget_bytes) {
    if (!valid_fmt(fmt)) return nullptr;
    int dev = 0;
    if (current_device(&dev) != 0) return nullptr;
    if (budget_bytes < 0) {
        constexpr int64_t MiB = 1 << 20, reserve = 1024 * MiB;      // scratch kept free beside the cache
        if (const char * env = std::getenv("GGML_LNS_CUDA_CACHE_MB")) {
            const long long mb = std::atoll(env);
            budget_bytes = (mb > 0 ? mb : 0) * MiB;
        } else {
            size_t fr = 0, tot = 0;
            if (cudaMemGetInfo(&fr, &tot) != cudaSuccess) return nullptr;
            budget_bytes = (int64_t) fr > reserve ? (int64_t) fr - reserve : 0;
        }
    }
    auto * c = new (std::nothrow) lnsb_weight_cache();
    if (c == nullptr) return nullptr;
    c->fmt = fmt;
    c->dev = dev;
    c->budget = budget_bytes;
    // LNSB_WEIGHT_CACHE_FAIL_ALLOCS=n: the cache's next n device allocations
    // report out-of-memory (failure handling is tested without exhausting
    // the device)
    if (const char * env = std::getenv("LNSB_WEIGHT_CACHE_FAIL_ALLOCS")) c->fail_allocs = std::atoll(env);
    return c;
}

void lnsb_weight_cache_destroy(lnsb_weight_cache * c) {
    if (c == nullptr) return;
    int cur = 0;
    const bool moved = cudaGetDevice(&cur) == cudaSuccess && cur != c->dev;
    if (moved) cudaSetDevice(c->dev);
    for (auto & e : c->entries) cudaFree(e.second);
    if (c->staging != nullptr) cudaFree(c->staging);
    if (moved) cudaSetDevice(cur);
    delete c;
}

int lnsb_weight_cache_get(lnsb_weight_cache * c, const void * src, int type, int64_t rows, int64_t cols,
                          void * scratch, const void ** out, lnsb_stream_t stream) {
    if (c == nullptr || out == nullptr || src == nullptr || rows <= 0 || cols <= 0) return LNSB_E_INVALID;
    if (!known_type(type)) return LNSB_E_UNSUPPORTED;
    const size_t rb = lnsb_type_row_bytes(type, cols);
    if (rb == 0) return LNSB_E_INVALID;
    int dev = 0;
    const int ds = current_device(&dev);
    if (ds != 0) return ds;
    if (dev != c->dev) return LNSB_E_INVALID;                        // a cache serves the device it was made on
    std::lock_guard<std::mutex> lock(c->mu);
    const lnsb_weight_cache::key k{ src, type, rows, cols };
    const auto it = c->entries.find(k);
    if (it != c->entries.end()) {
        *out = it->second;
        return 0;
    }
    const int64_t bytes = rows * cols * (int64_t) lnsb_value_size(c->fmt);
    void * dst = nullptr;
    if (c->used + bytes <= c->budget) {
        if (c->fail_allocs > 0) {
            c->fail_allocs--;                                        // injected out-of-memory
        } else if (cudaMalloc(&dst, (size_t) bytes) != cudaSuccess) {
            cudaGetLastError();                                      // out of memory: not sticky, fall back
            dst = nullptr;
        }
    }
    const bool cached = dst != nullptr;
    if (!cached) {
        if (scratch == nullptr) return LNSB_E_TOO_LARGE;
        dst = scratch;
    }
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaPointerAttributes at{};
    const bool on_device = cudaPointerGetAttributes(&at, src) == cudaSuccess &&
                           (at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged);
    cudaGetLastError();
    int st = 0;
    if (on_device) {
        st = lnsb_to_lns_transposed_typed(c->fmt, type, src, dst, rows, cols, rows, stream);
    } else {
        // host rows: staged through a bounded device buffer, chunk by chunk
        constexpr size_t k_chunk = (size_t) 64 << 20;
        const int64_t chunk_rows = rb >= k_chunk ? 1 : (int64_t) (k_chunk / rb);
        const size_t need = (size_t) (chunk_rows < rows ? chunk_rows : rows) * rb;
        if (c->staging_bytes < need) {
            if (c->staging != nullptr) cudaFree(c->staging);
            c->staging = nullptr;
            c->staging_bytes = 0;
            if (cudaMalloc(&c->staging, need) != cudaSuccess) st = LNSB_E_TOO_LARGE;
            else c->staging_bytes = need;
        }
        const size_t vs = lnsb_value_size(c->fmt);
        for (int64_t m0 = 0; st == 0 && m0 < rows; m0 += chunk_rows) {
            const int64_t n = rows - m0 < chunk_rows ? rows - m0 : chunk_rows;
            cudaError_t e = cudaMemcpyAsync(c->staging, static_cast<const unsigned char *>(src) + (size_t) m0 * rb,
                                            (size_t) n * rb, cudaMemcpyHostToDevice, s);
            if (e != cudaSuccess) { st = (int) e; break; }
            st = lnsb_to_lns_transposed_typed(c->fmt, type, c->staging, static_cast<unsigned char *>(dst) + (size_t) m0 * vs,
                                              n, cols, rows, stream);
            if (st == 0 && (e = cudaStreamSynchronize(s)) != cudaSuccess) st = (int) e;   // the staging buffer is reused
        }
    }
    if (st == 0) {
        const cudaError_t e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) st = (int) e;
    }
    if (st != 0) {
        if (cached) cudaFree(dst);
        return st;
    }
    if (cached) {
        c->entries.emplace(k, dst);
        c->used += bytes;
    }
    *out = dst;
    return 0;
}

int lnsb_weight_cache_stats(const lnsb_weight_cache * c, int64_t * entries, int64_t * used_bytes, int64_t * budget_bytes) {
    if (c == nullptr) return LNSB_E_INVALID;
    if (entries != nullptr) *entries = (int64_t) c->entries.size();
    if (used_bytes != nullptr) *used_bytes = c->used;
    if (budget_bytes != nullptr) *budget_bytes = c->budget;
    return 0;
}

}  // extern "C"
