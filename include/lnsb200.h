/*
 * lnsb200.h -- C ABI of the B200-native LNSCUDA16 / LNSCUDA32 hot path.
 *
 * The reference (xlnsresearch/xlns-ggml-backend) puts its GPU work behind one
 * C++ interface, lns_cuda::kernel_set (lns-backend/cuda/lns-cuda-kernels.h:85-139).
 * This header is that interface as a plain C ABI: one function per method,
 * the format as an argument (16 = xlns16 / LNSCUDA16, 32 = xlns32 / LNSCUDA32),
 * device pointers and sizes in, a status code out, every launch asynchronous
 * on the caller's stream.  A ctypes / cgo / JNI binding needs nothing else.
 *
 * Build mode.  Like the reference, the xlns16 summation mode is fixed when
 * the library is built (GGML_LNS16_SUM = base | monte | lpvip | sum32, plus
 * GGML_LNS16_MONTE_BYLPVIP): liblnsb200_<mode>.so.  lnsb_sum_mode() reports it.
 *
 * Conventions (lns-cuda-kernels.h:12-26):
 *   - tensors are contiguous arrays in ggml element order (ne[0] fastest);
 *   - reductions run in element order, one sequential chain per output;
 *   - Monte reductions start from monte_seed; reduction i starts i * draws
 *     LFSR steps later (CPU loop order);
 *   - xlns16 values are uint16 codes, xlns32 values uint32 codes.
 *
 * Status codes: 0 = success; > 0 = the cudaError_t of a failed CUDA call;
 * < 0 = LNSB_E_* below.  lnsb_error_string() names either kind.
 */
#ifndef LNSB200_H
#define LNSB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LNSB_XLNS16 16
#define LNSB_XLNS32 32

#define LNSB_OK             0
#define LNSB_E_INVALID    (-1)   /* bad format, null pointer, negative size, bad broadcast */
#define LNSB_E_NO_TABLES  (-2)   /* lnsb_upload_tables was not run on this device */
#define LNSB_E_UNSUPPORTED (-3)  /* argument combination this build does not implement */
#define LNSB_E_TOO_LARGE  (-4)   /* size beyond a documented limit */
#define LNSB_E_NO_DEVICE  (-5)   /* no usable CUDA device */

/* a cudaStream_t; NULL is the legacy default stream */
typedef void * lnsb_stream_t;

typedef struct { int64_t ne[4]; } lnsb_shape4;   /* lns-cuda-kernels.h:39-43 */

/*
 * dst = W^T x per activation slice, sequential over k
 * (mul_mat_args, lns-cuda-kernels.h:45-58):
 *   w   LNS, K x M per weight slice, k-major (element (k, m) at k*M + m),
 *       ne02 * ne03 slices
 *   x   LNS, N x K per activation slice, ne12 * ne13 slices
 *   dst F32, N x M per activation slice
 * Activation slice (i12, i13) uses weight slice (i12 / (ne12/ne02), i13 / (ne13/ne03)).
 */
typedef struct {
    const void * w;
    const void * x;
    float *      dst;
    int64_t      K, M, N;
    int64_t      ne02, ne03, ne12, ne13;
    uint16_t     monte_seed;
} lnsb_mul_mat_args;

/*
 * dst = softmax(src * scale + mask) over rows of src.ne[0]; mask (optional)
 * broadcasts over dims 2 and 3; work holds src.nelements() LNS values
 * (soft_max_args, lns-cuda-kernels.h:60-71).
 */
typedef struct {
    const float * src;
    lnsb_shape4   src_shape;
    const float * mask;
    lnsb_shape4   mask_shape;
    float         scale;
    float *       dst;
    void *        work;
    uint16_t      monte_seed;
} lnsb_soft_max_args;

/* ---- identity: kernel_set::format_name / value_size / sum_mode / monte_impl
 *      (lns-cuda-kernels.h:89-95) ---- */
const char * lnsb_format_name(int fmt);        /* "xlns16" | "xlns32" | NULL */
size_t       lnsb_value_size(int fmt);         /* 2 | 4 | 0 */
const char * lnsb_sum_mode(int fmt);           /* "base"|"monte"|"lpvip"|"sum32" for 16, NULL for 32 */
const char * lnsb_monte_impl(int fmt);         /* "pure16"|"bylpvip" in a monte build, else NULL */
/* device description with "sum=<mode>[, monte=<impl>]" (ggml-lns-cuda.cpp:21-31,61-74) */
const char * lnsb_description(int fmt);

/* ---- draw accounting: kernel_set::*_draws (lns-cuda-kernels.h:97-100) ---- */
uint64_t lnsb_mul_mat_draws(int fmt, const lnsb_mul_mat_args * args);
uint64_t lnsb_soft_max_draws(int fmt, int64_t ncols, int64_t nrows);
uint64_t lnsb_rms_norm_draws(int fmt, int64_t ncols, int64_t nrows);

/* ---- kernel_set::upload_tables (lns-cuda-kernels.h:102-104): builds the
 *      arithmetic tables once per process and uploads them to the current
 *      device once per device.  Must run before any other call on a device. ---- */
int lnsb_upload_tables(int fmt);

/* ---- conversions: kernel_set::to_lns / to_lns_transposed (lns-cuda-kernels.h:106-112) ---- */
int lnsb_to_lns(int fmt, const float * src, void * dst, int64_t n, lnsb_stream_t stream);
/* dst[c * dst_ld + r] = lns(src[r * cols + c]) */
int lnsb_to_lns_transposed(int fmt, const float * src, void * dst, int64_t rows, int64_t cols,
                           int64_t dst_ld, lnsb_stream_t stream);
/* ---- weights in ggml storage types.  The reference turns every weight into
 * F32 rows on the host with ggml's to_float and converts them with
 * to_lns_transposed (lns-cuda-context.cpp:163-195, 370-419); here one kernel
 * decodes the rows on the device and writes the k-major LNS image.  Type ids
 * are ggml's (ggml_type).  Rows are stored back to back, each
 * lnsb_type_row_bytes(type, cols) bytes; block types need cols to be a whole
 * number of blocks (32 values for Q8_0 / Q4_0, 256 for Q4_K / Q6_K). ---- */
#define LNSB_TYPE_F32   0
#define LNSB_TYPE_F16   1
#define LNSB_TYPE_Q4_0  2
#define LNSB_TYPE_Q8_0  8
#define LNSB_TYPE_Q4_K 12
#define LNSB_TYPE_Q6_K 14
#define LNSB_TYPE_BF16 30
/* bytes of one row of `cols` values; 0 for an unknown type or a partial block */
size_t lnsb_type_row_bytes(int type, int64_t cols);
/* dst[c * dst_ld + r] = lns(value c of row r of src), src and dst in device memory */
int lnsb_to_lns_transposed_typed(int fmt, int type, const void * src, void * dst, int64_t rows, int64_t cols,
                                 int64_t dst_ld, lnsb_stream_t stream);
/* the decoded F32 rows (ggml's to_float), rows x cols */
int lnsb_dequantize(int type, const void * src, float * dst, int64_t rows, int64_t cols, lnsb_stream_t stream);

/* ---- the weight cache (lns-cuda-context.h:79-113, lns-cuda-context.cpp:
 * 128-154, 290-300, 370-392): weights converted to LNS once and kept on the
 * device, keyed by (data pointer, type, rows, cols); a conversion that would
 * exceed the budget goes to the caller's scratch instead and is redone on
 * every use, as in the reference.  src may be host or device memory (host
 * rows are staged to the device in bounded chunks).  budget_bytes < 0 takes
 * the reference's rule: GGML_LNS_CUDA_CACHE_MB if set, else the device's free
 * memory less a 1 GiB reserve at creation.  A device allocation that fails
 * (out of memory) is not an error: the image goes to scratch as over budget.
 * LNSB_WEIGHT_CACHE_FAIL_ALLOCS=n, read at creation, makes the cache's next n
 * allocations fail that way (host-side fault injection for tests). ---- */
typedef struct lnsb_weight_cache lnsb_weight_cache;
lnsb_weight_cache * lnsb_weight_cache_create(int fmt, int64_t budget_bytes);
void lnsb_weight_cache_destroy(lnsb_weight_cache * cache);
/* *out = the k-major LNS image (K = cols, M = rows: element (k, m) at k * rows + m).
 * On a miss that does not fit, the image is written to `scratch` (rows * cols *
 * value_size bytes of device memory; NULL -> LNSB_E_TOO_LARGE).  The call
 * synchronises `stream` when it converts. */
int lnsb_weight_cache_get(lnsb_weight_cache * cache, const void * src, int type, int64_t rows, int64_t cols,
                          void * scratch, const void ** out, lnsb_stream_t stream);
int lnsb_weight_cache_stats(const lnsb_weight_cache * cache, int64_t * entries, int64_t * used_bytes,
                            int64_t * budget_bytes);

/* dst[i] = float(src[i]) -- the op-boundary decode the reference fuses into
 * every kernel's store (lns-cuda-kernels.cuh:155,249,324) */
int lnsb_to_f32(int fmt, const void * src, float * dst, int64_t n, lnsb_stream_t stream);

/* ---- the hot path ---- */

/* kernel_set::mul_mat (lns-cuda-kernels.h:114) */
int lnsb_mul_mat(int fmt, const lnsb_mul_mat_args * args, lnsb_stream_t stream);
/* same product with LNS codes out: dst_lns is N x M per activation slice
 * (args->dst is ignored).  The reference's LNS16-typed dst path,
 * lns-ops.cpp:374-379. */
int lnsb_mul_mat_lns(int fmt, const lnsb_mul_mat_args * args, void * dst_lns, lnsb_stream_t stream);
/* the MUL_MAT op over F32 activations: args->x holds F32 values (N x K per
 * activation slice) instead of codes.  Same result as lnsb_to_lns of x into
 * x_work followed by lnsb_mul_mat over x_work, which is the reference's
 * compute_mul_mat (lns-cuda-ops.cpp:57-75: to_lns of src1, then
 * kernel_set::mul_mat).  The weight-resident latency kernel (xlns16 base mode,
 * few outputs) converts the activations as it stages them, with no separate
 * launch and x_work untouched; every other case converts into x_work first.
 * x_work (N * K * ne12 * ne13 LNS values) is required whenever K > 0. */
int lnsb_mul_mat_xf32(int fmt, const lnsb_mul_mat_args * args, void * x_work, lnsb_stream_t stream);

/* mul_mat with the all-gather of output-row shards fused into the store (no
 * counterpart in the reference): the caller owns rows [offset, offset + M)
 * of a [slices][N][ld] codes result that lives on every GPU of the group; the
 * kernel stores each code into all `n` peer buffers (device pointers valid in
 * this process, e.g. a symmetric-memory allocation's buffer_ptrs_dev, own
 * buffer included) over NVLink, plain stores; codes of the format's width
 * (16 or 32 bits).  Every summation mode and both formats.
 * Ordering, both ways:
 *  - read after write: run lnsb_group_barrier after the call and before any
 *    read of the gathered result;
 *  - write after read: a peer may still be reading step e's result when this
 *    rank's step e+1 stores arrive.  Either alternate between two result
 *    buffers by step parity, with every read of step e issued on this rank's
 *    stream before its step e+1 call (passing barrier e+1 then means every
 *    peer has finished its step e reads), or run a second lnsb_group_barrier
 *    after the last read of step e, before the next call. */
typedef struct {
    void * const * ptrs;       /* device array of n buffer pointers */
    int            n;
    int64_t        ld, offset;
} lnsb_peer_out;
int lnsb_mul_mat_lns_peers(int fmt, const lnsb_mul_mat_args * args, const lnsb_peer_out * peers, lnsb_stream_t stream);
/* the barrier to follow it: flags is a device array of `world` pointers to
 * each GPU's int32[world] flag array (zeroed once; peer memory), epoch counts
 * the calls from 1.  Each GPU signals every peer and waits for every peer's
 * signal of this epoch.  The wait is bounded: after 2^21 polls, each followed
 * by a sleep of about 100 ns (in total about 0.2 s or more, depending on the
 * scheduler), it sets *err (device memory) to 1 and returns instead of
 * hanging. */
int lnsb_group_barrier(int32_t * const * flags, int world, int rank, int32_t epoch, int32_t * err, lnsb_stream_t stream);

/* Diagnostic, no counterpart in the reference: the dependent latency of one
 * LNS addition on the current device, for the chain bound T_chain = (n - 1)
 * L_add / f_sm of a latency-bound reduction.  One warp runs `steps` dependent
 * additions per lane (2 <= steps; lanes 1..32 distinct chains, the other lanes
 * repeating them) over operands of a dot product's spread, with the adder's
 * table in shared memory as the kernels hold it.  kind 0: the key-form xlns16
 * addition of the latency mul_mat kernels; 1: the non-negative xlns16
 * addition of the normalisers (base); 2: the non-negative xlns32 addition of
 * the normalisers (sum32, xlns32); 3: the general xlns32 addition of the
 * latency-bound mat-vecs (sum32, xlns32; both signs, the cotransformed db
 * beside the main result).  out: device memory, two int64 -- out[0] =
 * SM cycles over steps - 1 additions, out[1] = the final accumulator. */
int lnsb_add_latency(int kind, int lanes, int steps, int64_t * out, lnsb_stream_t stream);

/* kernel_set::soft_max (lns-cuda-kernels.h:136) */
int lnsb_soft_max(int fmt, const lnsb_soft_max_args * args, lnsb_stream_t stream);
/* codes in, codes out: src [ne3][ne2][ne1][ne0], mask (may be NULL) codes
 * [mne3][mne2][mne1][ne0] with ne0 == src ne0, mne1 >= ne1, dims 2/3
 * broadcast; scale is an LNS code; work holds nelements(src) LNS values.
 * The reference's LNS16-typed path, lns-ops.cpp:643-695. */
int lnsb_soft_max_lns(int fmt, const void * src, const int64_t ne[4], const void * mask,
                      const int64_t mne[4], uint32_t scale, void * dst, void * work,
                      uint16_t monte_seed, lnsb_stream_t stream);

/* Allocation-free variant of lnsb_soft_max_lns.  No counterpart in the
 * reference: it is for callers that must not call cudaMalloc (a host framework
 * whose own pool owns all device memory, a latency-critical loop that may not
 * take the driver allocator's implicit synchronisation).  The
 * per-element scratch the normaliser needs lives in one static device array
 * of LNSB_NOALLOC_SCRATCH_BYTES built into this library, so
 * nelements(src) * value_size must not exceed that (else LNSB_E_TOO_LARGE).
 * The array belongs to the loaded library, so every GPU that uses it holds
 * those bytes until the process exits.  The first call on a device looks up
 * the array's device address (cudaGetSymbolAddress) -- make that first call
 * before any stream capture.  The arithmetic tables still come from
 * lnsb_upload_tables, a one-time set-up call that does allocate.  All calls
 * share the one array: calls that can overlap on the GPU (different streams,
 * or different host threads, without ordering between them) race on it and
 * must be serialised by the caller. */
#define LNSB_NOALLOC_SCRATCH_BYTES ((size_t) 8 << 20)
int lnsb_soft_max_lns_noalloc(int fmt, const void * src, const int64_t ne[4], const void * mask,
                              const int64_t mne[4], uint32_t scale, void * dst, uint16_t monte_seed,
                              lnsb_stream_t stream);

/* kernel_set::rms_norm (lns-cuda-kernels.h:132-134) */
int lnsb_rms_norm(int fmt, const float * src, float * dst, int64_t ncols, int64_t nrows, float eps,
                  uint16_t monte_seed, lnsb_stream_t stream);
/* codes in, codes out (lns-ops.cpp:701-736 with LNS16 tensors) */
int lnsb_rms_norm_lns(int fmt, const void * src, void * dst, int64_t ncols, int64_t nrows, float eps,
                      uint16_t monte_seed, lnsb_stream_t stream);

/* ---- MUL_MAT_ID: the expert-selected product of mixture-of-experts FFNs
 * (lns-backend/src/lns-ops.cpp:394-462; the reference's GPU backend declines
 * the op and ggml runs it on the CPU backend).  For token t and slot s the
 * weight slice is expert e = ids[t * ids_stride + s] and the activation row is
 * x[t][s % ne11] (slot-based broadcast):
 *   dst[t][s][m] = sum_k w[e][k][m] * x[t][s % ne11][k], sequential over k
 *   w    LNS, n_expert slices of K x M, k-major: (e, k, m) at (e * K + k) * M + m
 *   x    LNS, [n_tokens][ne11][K], n_used % ne11 == 0
 *   ids  int32, device memory
 *   dst  F32 [n_tokens][n_used][M]
 * Monte: chain (t, s, m) starts ((t * n_used + s) * M + m) * (K - 1) draws
 * after monte_seed, the CPU loop order.  An id outside [0, n_expert) gives the
 * zero code for its slot's outputs and is counted (lnsb_mul_mat_id_bad_ids)
 * where the reference aborts. ---- */
typedef struct {
    const void *    w;
    const void *    x;
    const int32_t * ids;
    float *         dst;
    int64_t         K, M, n_expert, ne11, n_used, n_tokens, ids_stride;
    uint16_t        monte_seed;
} lnsb_mul_mat_id_args;
int lnsb_mul_mat_id(int fmt, const lnsb_mul_mat_id_args * args, lnsb_stream_t stream);
/* LNS codes out: dst_lns [n_tokens][n_used][M] (args->dst is ignored) */
int lnsb_mul_mat_id_lns(int fmt, const lnsb_mul_mat_id_args * args, void * dst_lns, lnsb_stream_t stream);
uint64_t lnsb_mul_mat_id_draws(int fmt, const lnsb_mul_mat_id_args * args);
/* out-of-range ids met on the current device since the last call; reads and
 * clears the count (synchronises with the device) */
int lnsb_mul_mat_id_bad_ids(int64_t * count);

/* ---- Elementwise ops of the model graph (kernel_set::binary / scale /
 * unary / glu / rope, lns-cuda-kernels.h:116-138; lns-backend/src/lns-ops.cpp:
 * 468-599, 786-868, 1199-1281).  F32 in and out, as at every ggml op
 * boundary: each operand is converted to LNS (lnsb_to_lns's table), the op
 * runs in LNS, the result is written back as F32.  Contiguous tensors.
 * An op code outside the lists below returns LNSB_E_INVALID. */
#define LNSB_BINARY_ADD 0
#define LNSB_BINARY_MUL 1
#define LNSB_BINARY_DIV 2
#define LNSB_UNARY_SILU 0
#define LNSB_UNARY_GELU 1
#define LNSB_UNARY_RELU 2
#define LNSB_UNARY_TANH 3
#define LNSB_GLU_SWIGLU 0
#define LNSB_GLU_GEGLU  1

/* dst = a op b, b repeated to a's shape (ggml_can_repeat(b, a)); ne[0] innermost */
int lnsb_binary(int fmt, int op, const float * a, const int64_t ane[4], const float * b, const int64_t bne[4],
                float * dst, lnsb_stream_t stream);
/* dst = src * s, plus b when b != 0 (ggml_scale_bias) */
int lnsb_scale(int fmt, const float * src, float * dst, int64_t n, float s, float b, lnsb_stream_t stream);
/* xlns16: silu(x) = x * sigmoid(x), sigmoid a 65536-entry table (the float
 * 1 / (1 + e^-x) of each code, converted); tanh(x) = (e^2x - 1) / (e^2x + 1)
 * and gelu(x) = 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))) in xlns16
 * arithmetic over the exp table (lns-backend/cuda/lns-cuda-kernels.cuh:191-206,
 * lns-ops.cpp:783-1000).  xlns32: silu in xlns32 arithmetic with exp through
 * float; tanh and gelu evaluated in double precision and converted.  relu. */
int lnsb_unary(int fmt, int op, const float * src, float * dst, int64_t n, lnsb_stream_t stream);
/* dst[r][c] = act(gate[r * gate_stride + c]) * up[r * up_stride + c], act =
 * silu (LNSB_GLU_SWIGLU) or gelu (LNSB_GLU_GEGLU) as in lnsb_unary */
int lnsb_glu(int fmt, int op, const float * gate, const float * up, int64_t gate_stride, int64_t up_stride,
             float * dst, int64_t ncols, int64_t nrows, lnsb_stream_t stream);

/* rope_args, lns-cuda-kernels.h:73-80: rows of shape.ne[0]; row (i1, i2, i3)
 * has position index i2 and cos_sin[(i2 * n_dims/2 + j) * 2 + {0, 1}] =
 * (cos, sin) of its pair j, computed by the caller on the host */
typedef struct {
    const float * src;
    lnsb_shape4   shape;
    const float * cos_sin;
    int           n_dims;
    int           neox;        /* pairs (j, j + n_dims/2) instead of (2j, 2j+1) */
    float *       dst;
} lnsb_rope_args;
int lnsb_rope(int fmt, const lnsb_rope_args * args, lnsb_stream_t stream);

/* One decode step's attention (a query at the last cache position, every
 * cached key visible), fused: for each query head h (kv head h / (n_head /
 * n_head_kv)), the ops the graph runs as F16 -> F32 of the caches, to_lns,
 * mul_mat kq, soft_max (scale, the all-zero causal mask row), to_lns and
 * mul_mat kqv, with every op-boundary conversion kept, so the output is
 * bit-identical to those ops run one by one (monte_seed for each of the
 * three, as in lnsb_mul_mat / lnsb_soft_max).
 *   q        F32 [n_head][head_dim]
 *   k_cache  F16 [nkv][kv_ld], kv head j at columns [j * head_dim, (j+1) * head_dim)
 *   v_cache  F16, same layout
 *   dst      F32 [n_head][head_dim] (may be NULL when dst_lns is given)
 *   dst_lns  optional: the codes of dst (to_lns of it, the next mat-vec's input)
 * LNSB_E_TOO_LARGE when nkv exceeds lnsb_attn_decode_max_keys (the
 * kernel's shared memory: about 5,700 keys at head_dim 64 beside the 101 KB
 * flat xlns32 image of sum32 and xlns32, about 19,000 in the other modes). */
typedef struct {
    const float *    q;
    const uint16_t * k_cache;
    const uint16_t * v_cache;
    int64_t          kv_ld, nkv;
    int              n_head, n_head_kv, head_dim;
    float            scale;
    float *          dst;
    uint16_t         monte_seed;
    void *           dst_lns;
} lnsb_attn_decode_args;
int lnsb_attn_decode(int fmt, const lnsb_attn_decode_args * args, lnsb_stream_t stream);
int64_t lnsb_attn_decode_max_keys(int fmt, int head_dim);

/* ---- The decode graph's other steps fused, each op boundary kept (the
 * results are bit-identical to the ops run one by one):
 * lnsb_norm_block: x = src (+ residual: the residual add), rms_norm(x), times
 *   the norm weight (if given), to_lns -> dst_lns; x_out (if given) gets x (F32)
 * lnsb_glu_lns: lnsb_glu followed by to_lns of its output
 * lnsb_rope_qkv: from the q/k/v mat-vec's output rows [n_tokens][ld] (q heads,
 *   k heads, v heads): rope of q (F32 -> q_out [n_tokens][n_head * head_dim])
 *   and of k, k and v into the F16 caches (rows [n_tokens][kv_ld]); cos_sin
 *   as lnsb_rope's, one position per token ---- */
typedef struct {
    const float * src;
    const float * residual;
    float *       x_out;
    const float * weight;
    void *        dst_lns;
    int64_t       ncols, nrows;
    float         eps;
    uint16_t      monte_seed;
} lnsb_norm_block_args;
int lnsb_norm_block(int fmt, const lnsb_norm_block_args * args, lnsb_stream_t stream);
int lnsb_glu_lns(int fmt, int op, const float * gate, const float * up, int64_t gate_stride, int64_t up_stride,
                 void * dst_lns, int64_t ncols, int64_t nrows, lnsb_stream_t stream);
typedef struct {
    const float * qkv;
    int64_t       ld;
    const float * cos_sin;
    int           n_dims, neox, n_head, n_head_kv, head_dim;
    int64_t       n_tokens;
    float *       q_out;
    uint16_t *    k_cache;
    uint16_t *    v_cache;
    int64_t       kv_ld;
} lnsb_rope_qkv_args;
int lnsb_rope_qkv(int fmt, const lnsb_rope_qkv_args * args, lnsb_stream_t stream);

/* F16 storage of F32 values (KV caches): IEEE binary16, round to nearest
 * even, and back (exact).  No LNS involved; not part of kernel_set. */
int lnsb_f32_to_f16(const float * src, uint16_t * dst, int64_t n, lnsb_stream_t stream);
int lnsb_f16_to_f32(const uint16_t * src, float * dst, int64_t n, lnsb_stream_t stream);

/* ---- Monte state: one LFSR per process, seed 7 (ggml-lns.h:13-24).  All
 *      return 0 on success, LNSB_E_UNSUPPORTED outside a monte build;
 *      set_state rejects 0 (absorbing). ---- */
int lnsb_monte_get_state(uint16_t * state);
int lnsb_monte_set_state(uint16_t state);
/* *start = current state, then advance it by `draws` steps (lns-ops.cpp:178-195) */
int lnsb_monte_reserve(uint64_t draws, uint16_t * start);

const char * lnsb_error_string(int status);

#ifdef __cplusplus
}
#endif
#endif
