/*
 * lnsb200_graph.h -- the ggml backend's host layer, over the C ABI of
 * lnsb200.h and compiled into the same library.
 *
 * It restates, against this library's own tensor descriptor (so it builds and
 * is tested without ggml), what the reference's ggml layer decides and runs:
 *   - the op-support predicates (lns-backend/common/lns-op-support.h:33-202,
 *     lns-backend/cuda/lns-cuda-ops.cpp:25-230, lns-backend-framework.h:
 *     176-190: views and no-ops are accepted, ops without a kernel refused);
 *   - backend selection, GGML_LNS_BACKEND (lns-backend-config.h:55-136);
 *   - op bisection, LNS_DISABLE_OPS / LNS_ENABLE_OPS (lns-backend-config.h:
 *     138-199);
 *   - the supports_op audit, LNS_OP_AUDIT (lns-backend-config.h:201-239);
 *   - supports_op = selection AND predicate AND NOT disabled
 *     (lns-backend-framework.h:287-295);
 *   - the device description with "sum=<mode>[, monte=<impl>]"
 *     (lns-backend/cuda/ggml-lns-cuda.cpp:21-31, 61-74);
 *   - graph_compute's node walk (lns-backend-framework.h:207-221) and each
 *     op's compute (lns-cuda-ops.cpp:57-250), including the weight cache for
 *     weight tensors (lns-cuda-context.cpp:370-392) and the gather of strided
 *     views (lns-cuda-context.cpp:158-195, 338-346) -- on the device here.
 * A ggml adapter fills one lnsb_tensor per ggml_tensor (ggml's type ids; the
 * op and sub-op ids below) and forwards supports_op / graph_compute to these
 * calls; include/lnsb200_ggml.hpp is that adapter, compiled where ggml's
 * ggml-backend-impl.h is available.
 */
#ifndef LNSB200_GRAPH_H
#define LNSB200_GRAPH_H

#include "lnsb200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ops, named as ggml_op_name prints them */
enum {
    LNSB_OP_NONE = 0,
    LNSB_OP_RESHAPE,
    LNSB_OP_VIEW,
    LNSB_OP_PERMUTE,
    LNSB_OP_TRANSPOSE,
    LNSB_OP_MUL_MAT,
    LNSB_OP_MUL_MAT_ID,
    LNSB_OP_ADD,
    LNSB_OP_MUL,
    LNSB_OP_DIV,
    LNSB_OP_SCALE,
    LNSB_OP_RMS_NORM,
    LNSB_OP_SOFT_MAX,
    LNSB_OP_ROPE,
    LNSB_OP_UNARY,
    LNSB_OP_GLU,
    LNSB_OP_GET_ROWS,
    LNSB_OP_CPY,
    LNSB_OP_CONT,
    LNSB_OP_COUNT
};

#define LNSB_TYPE_I32 26                 /* ggml's GGML_TYPE_I32 (ids, positions) */
#define LNSB_TENSOR_FLAG_COMPUTE 1       /* a node the graph computes */
#define LNSB_TENSOR_FLAG_WEIGHTS 2       /* data in a weight buffer: converted once, cached */
#define LNSB_ROPE_TYPE_NEOX 2

/*
 * One node or leaf.  op_params holds ggml's op parameter words:
 *   SOFT_MAX  f32 [0] scale, [1] max_bias
 *   RMS_NORM  f32 [0] eps
 *   SCALE     f32 [0] s, [1] b
 *   ROPE      i32 [1] n_dims, [2] mode; f32 [5] freq_base, [6] freq_scale,
 *             [7] ext_factor, [8] attn_factor
 *   UNARY     i32 [0] LNSB_UNARY_*
 *   GLU       i32 [0] LNSB_GLU_*, [1] swapped (fused layout: up first)
 * src: MUL_MAT (weights, activations), MUL_MAT_ID (weights, activations,
 * ids), SOFT_MAX (logits, mask or NULL), ROPE (x, positions, frequency
 * factors or NULL), GLU (gate, up) or (fused rows).  data: device or host
 * memory (host data goes through the reference's per-op upload and
 * download).
 */
typedef struct lnsb_tensor lnsb_tensor;
struct lnsb_tensor {
    int32_t             type;           /* ggml type id: LNSB_TYPE_* */
    int32_t             op;             /* LNSB_OP_* */
    int64_t             ne[4];          /* elements per dimension, ne[0] innermost */
    int64_t             nb[4];          /* byte strides */
    int32_t             op_params[16];
    int32_t             flags;          /* LNSB_TENSOR_FLAG_* */
    const lnsb_tensor * src[4];
    void *              data;
    char                name[64];
};

/* ggml_op_name; ggml_op_desc (the unary / glu op's name for those) */
const char * lnsb_op_name(int op);
const char * lnsb_op_desc(const lnsb_tensor * node);

/* The predicate alone (the kernels can run the node exactly as ggml defines
 * it): 1 or 0, *reason (a static string, may be NULL) the audit's reason. */
int lnsb_check_op(int fmt, const lnsb_tensor * node, const char ** reason);

/* GGML_LNS_BACKEND: the device names a selection value names (aliases 16, 32,
 * cuda, cuda16, cuda32, or device names; case-insensitive; NULL or empty =
 * the default "16"; unknown tokens reported on stderr and ignored; nothing
 * valid = the default), comma-separated into out.  Returns the count. */
int lnsb_resolve_backend_selection(const char * selection, char * out, size_t cap);
int lnsb_backend_selected_by(const char * device_name, const char * selection);

/* LNS_DISABLE_OPS / LNS_ENABLE_OPS tokens: the op name or desc
 * (case-insensitive), OP:pattern, a pattern over the tensor name, or
 * <pattern over its second input's name; a pattern with *?[ is a whole-name
 * wildcard, otherwise a case-sensitive substring.  enable_list NULL = unset;
 * set but empty: no op runs in LNS.  1 = the node falls back. */
int lnsb_op_matches(const lnsb_tensor * node, const char * token);
int lnsb_op_disabled_by(const lnsb_tensor * node, const char * disable_list, const char * enable_list);

/* the LNS_OP_AUDIT line (JSON, no newline) into out; returns its length */
int lnsb_audit_line(const char * backend, int fmt, const lnsb_tensor * node, int supported, const char * reason,
                    char * out, size_t cap);

/* supports_op as the registered device answers it: GGML_LNS_BACKEND selects
 * device_name, the predicate holds, and LNS_DISABLE_OPS / LNS_ENABLE_OPS do not
 * exclude the node (the environment is read once per process); with
 * LNS_OP_AUDIT set, one audit line on stderr per query. */
int lnsb_supports_op(const char * device_name, int fmt, const lnsb_tensor * node);

/* "Logarithmic Number System on CUDA (<format>[, sum=<mode>[, monte=<impl>]])
 * on <GPU name>" for the current device */
const char * lnsb_device_description(int fmt);

/* graph_compute.  A context holds the stream, the weight cache (budget as
 * lnsb_weight_cache_create) and device scratch.  Each node with the COMPUTE
 * flag, other than views, no-ops and empty tensors, runs its kernel in graph
 * order; Monte draws are reserved from the library's LFSR state per op.
 * Returns 0, or the first failing status with *failed (may be NULL) its node
 * index: LNSB_E_UNSUPPORTED for a node the predicate refuses (the reference
 * aborts there). */
typedef struct lnsb_graph_ctx lnsb_graph_ctx;
lnsb_graph_ctx * lnsb_graph_ctx_create(int fmt, int64_t cache_budget_bytes, lnsb_stream_t stream);
void lnsb_graph_ctx_destroy(lnsb_graph_ctx * ctx);
int lnsb_graph_compute(lnsb_graph_ctx * ctx, lnsb_tensor * const * nodes, int n_nodes, int * failed);

/* dst (contiguous, [ne3][ne2][ne1][ne0]) = the strided view (src, ne, nb
 * byte strides) of elem_size-byte elements (2 or 4), device memory -- the
 * gather of permuted views the reference does on the host */
int lnsb_copy_strided(int elem_size, const void * src, const int64_t ne[4], const int64_t nb[4], void * dst,
                      lnsb_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif
