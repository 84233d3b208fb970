// The ggml backend's host layer (include/lnsb200_graph.h): op-support
// predicates, backend selection, op bisection, the supports_op audit, the
// device description and graph_compute over this library's C ABI.
#include "lnsb200_graph.h"

#include <cuda_runtime.h>
#include <fnmatch.h>
#include <strings.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

namespace {

// ------------------------------------------------------------------ names

const char * const k_op_names[LNSB_OP_COUNT] = {
    "NONE", "RESHAPE", "VIEW", "PERMUTE", "TRANSPOSE", "MUL_MAT", "MUL_MAT_ID", "ADD", "MUL", "DIV", "SCALE",
    "RMS_NORM", "SOFT_MAX", "ROPE", "UNARY", "GLU", "GET_ROWS", "CPY", "CONT",
};
const char * const k_unary_names[] = { "SILU", "GELU", "RELU", "TANH" };   // LNSB_UNARY_* order
const char * const k_glu_names[]   = { "SWIGLU", "GEGLU" };                // LNSB_GLU_* order

// ------------------------------------------------------------------ tensor facts (ggml's definitions)

int64_t blck_size(int type) {
    switch (type) {
        case LNSB_TYPE_Q4_0: case LNSB_TYPE_Q8_0: return 32;
        case LNSB_TYPE_Q4_K: case LNSB_TYPE_Q6_K: return 256;
        default: return 1;
    }
}
// bytes of one block (one element for the plain types); 0 for a type this library does not know
int64_t type_size(int type) {
    switch (type) {
        case LNSB_TYPE_F32: case LNSB_TYPE_I32: return 4;
        case LNSB_TYPE_F16: case LNSB_TYPE_BF16: return 2;
        default: return (int64_t) lnsb_type_row_bytes(type, blck_size(type));
    }
}
bool known_type(int type) { return type_size(type) > 0; }
// the types a matrix operand may have: F32 or one the device decodes (ggml's to_float)
bool convertible_to_f32(int type) {
    return type == LNSB_TYPE_F32 || type == LNSB_TYPE_F16 || type == LNSB_TYPE_BF16 || type == LNSB_TYPE_Q4_0 ||
           type == LNSB_TYPE_Q8_0 || type == LNSB_TYPE_Q4_K || type == LNSB_TYPE_Q6_K;
}
int64_t nelements(const lnsb_tensor * t) { return t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3]; }
int64_t nrows(const lnsb_tensor * t) { return t->ne[1] * t->ne[2] * t->ne[3]; }
int64_t row_bytes(const lnsb_tensor * t) { return t->ne[0] / blck_size(t->type) * type_size(t->type); }
bool rows_contiguous(const lnsb_tensor * t) { return t->nb[0] == type_size(t->type); }
// dims > n packed, dim 0 contiguous; dims 1..n may have any stride
bool contiguous_n(const lnsb_tensor * t, int n) {
    int64_t next = type_size(t->type);
    if (t->ne[0] != blck_size(t->type) && t->nb[0] != next) return false;
    next *= t->ne[0] / blck_size(t->type);
    for (int i = 1; i < 4; i++) {
        if (t->ne[i] == 1) continue;
        if (i > n) {
            if (t->nb[i] != next) return false;
            next *= t->ne[i];
        } else {
            next = t->ne[i] * t->nb[i];
        }
    }
    return true;
}
bool contiguous(const lnsb_tensor * t) { return contiguous_n(t, 0); }
bool same_shape(const lnsb_tensor * a, const lnsb_tensor * b) {
    return a->ne[0] == b->ne[0] && a->ne[1] == b->ne[1] && a->ne[2] == b->ne[2] && a->ne[3] == b->ne[3];
}
bool can_repeat(const lnsb_tensor * b, const lnsb_tensor * a) {        // b repeats to a's shape
    for (int i = 0; i < 4; i++)
        if (b->ne[i] <= 0 || a->ne[i] % b->ne[i] != 0) return false;
    return true;
}
float param_f32(const lnsb_tensor * t, int i) {
    float v;
    std::memcpy(&v, &t->op_params[i], sizeof v);
    return v;
}
bool is_view_or_noop(int op) {
    return op == LNSB_OP_NONE || op == LNSB_OP_RESHAPE || op == LNSB_OP_VIEW || op == LNSB_OP_PERMUTE ||
           op == LNSB_OP_TRANSPOSE;
}
const char * type_name(const lnsb_tensor * t) {
    if (t == nullptr) return "null";
    switch (t->type) {
        case LNSB_TYPE_F32: return "f32";
        case LNSB_TYPE_F16: return "f16";
        case LNSB_TYPE_BF16: return "bf16";
        case LNSB_TYPE_Q4_0: return "q4_0";
        case LNSB_TYPE_Q8_0: return "q8_0";
        case LNSB_TYPE_Q4_K: return "q4_K";
        case LNSB_TYPE_Q6_K: return "q6_K";
        case LNSB_TYPE_I32: return "i32";
        default: return "unknown";
    }
}

// ------------------------------------------------------------------ predicates

struct support {
    bool         ok;
    const char * reason;
};

// every handler writes an F32 result of its first input's shape
support f32_result(const lnsb_tensor * op, support base) {
    if (!base.ok) return base;
    if (op->type != LNSB_TYPE_F32 || op->src[0] == nullptr || !same_shape(op, op->src[0]))
        return { false, "lns_cuda_requires_f32_dst_of_src0_shape" };
    return base;
}

support check_mul_mat(const lnsb_tensor * op) {
    const lnsb_tensor * s0 = op->src[0];
    const lnsb_tensor * s1 = op->src[1];
    if (s0 == nullptr || s1 == nullptr || s1->type != LNSB_TYPE_F32 || !convertible_to_f32(s0->type))
        return { false, "mul_mat_requires_src1_f32_and_convertible_src0" };
    if (!rows_contiguous(s0) || !rows_contiguous(s1)) return { false, "mul_mat_requires_contiguous_rows" };
    if (op->type != LNSB_TYPE_F32) return { false, "lns_cuda_mul_mat_requires_f32_dst" };
    if (s1->ne[2] * s1->ne[3] > 65535) return { false, "lns_cuda_mul_mat_grid_too_large" };
    if (s0->ne[2] <= 0 || s0->ne[3] <= 0 || s1->ne[2] % s0->ne[2] != 0 || s1->ne[3] % s0->ne[3] != 0)
        return { false, "lns_cuda_mul_mat_requires_whole_broadcast" };
    if (s0->ne[0] != s1->ne[0] || op->ne[0] != s0->ne[1] || op->ne[1] != s1->ne[1] || op->ne[2] != s1->ne[2] ||
        op->ne[3] != s1->ne[3])
        return { false, "mul_mat_shape_mismatch" };
    // a quantised matrix is converted row block by row block: its rows must be packed within a slice
    if (blck_size(s0->type) > 1 && s0->ne[1] > 1 && s0->nb[1] != row_bytes(s0))
        return { false, "lns_cuda_mul_mat_requires_packed_quantized_rows" };
    return { true, "lns_cuda_mul_mat" };
}

support check_mul_mat_id(const lnsb_tensor * op) {
    const lnsb_tensor * s0 = op->src[0];
    const lnsb_tensor * s1 = op->src[1];
    const lnsb_tensor * ids = op->src[2];
    if (s0 == nullptr || s1 == nullptr || ids == nullptr || s1->type != LNSB_TYPE_F32 || ids->type != LNSB_TYPE_I32 ||
        !convertible_to_f32(s0->type))
        return { false, "mul_mat_id_requires_src1_f32_and_i32_ids_and_convertible_src0" };
    if (op->type != LNSB_TYPE_F32) return { false, "lns_cuda_mul_mat_id_requires_f32_dst" };
    if (!rows_contiguous(s0) || !contiguous(s1) || !contiguous(ids) || s0->ne[3] != 1 || s1->ne[3] != 1 ||
        s0->ne[0] != s1->ne[0] || op->ne[0] != s0->ne[1] || op->ne[1] != ids->ne[0] || op->ne[2] != ids->ne[1] ||
        s1->ne[2] != ids->ne[1] || ids->ne[0] % s1->ne[1] != 0)
        return { false, "lns_cuda_mul_mat_id_layout_unsupported" };
    if (blck_size(s0->type) > 1 && s0->ne[1] > 1 && s0->nb[1] != row_bytes(s0))
        return { false, "lns_cuda_mul_mat_requires_packed_quantized_rows" };
    return { true, "lns_cuda_mul_mat_id" };
}

support check_binary(const lnsb_tensor * op) {
    if (op->src[0] == nullptr || op->src[1] == nullptr || op->src[0]->type != LNSB_TYPE_F32 ||
        op->src[1]->type != LNSB_TYPE_F32)
        return { false, "binary_requires_f32_srcs" };
    const support base = f32_result(op, { true, "lns_cuda_binary" });
    if (base.ok && !can_repeat(op->src[1], op->src[0])) return { false, "lns_cuda_binary_requires_repeatable_src1" };
    return base;
}

support check_contiguous_f32(const lnsb_tensor * op, const char * reason_bad) {
    if (op->src[0] == nullptr || op->src[0]->type != LNSB_TYPE_F32 || !contiguous(op->src[0]) || !contiguous(op))
        return { false, reason_bad };
    return { true, nullptr };
}

support check_scale(const lnsb_tensor * op) {
    support s = check_contiguous_f32(op, "requires_contiguous_f32_src0_and_dst");
    if (s.ok) s.reason = "lns_cuda_scale";
    return f32_result(op, s);
}

support check_unary(const lnsb_tensor * op) {
    const int u = op->op_params[0];
    if (u < LNSB_UNARY_SILU || u > LNSB_UNARY_TANH) return { false, "unsupported_unary_op" };
    support s = check_contiguous_f32(op, "unary_activation_requires_contiguous_f32_src0_and_dst");
    if (s.ok) s.reason = "lns_cuda_unary";
    return f32_result(op, s);
}

support check_glu(const lnsb_tensor * op) {
    const int g = op->op_params[0];
    if (g != LNSB_GLU_SWIGLU && g != LNSB_GLU_GEGLU) return { false, "unsupported_glu_op" };
    const lnsb_tensor * s0 = op->src[0];
    const lnsb_tensor * s1 = op->src[1];
    if (s0 == nullptr || s0->type != LNSB_TYPE_F32 || op->type != LNSB_TYPE_F32)
        return { false, "glu_requires_f32_src0_and_dst" };
    if (!contiguous_n(s0, 1) || !contiguous_n(op, 1)) return { false, "glu_requires_contiguous_rows" };
    if (s1 != nullptr) {
        const bool ok = s1->type == LNSB_TYPE_F32 && contiguous_n(s1, 1) && s1->ne[0] == s0->ne[0] &&
                        nrows(s1) == nrows(s0) && op->ne[0] == s0->ne[0] && nrows(op) == nrows(s0);
        return { ok, "glu_split_requires_matching_f32_contiguous_inputs" };
    }
    const bool ok = s0->ne[0] % 2 == 0 && op->ne[0] == s0->ne[0] / 2 && nrows(op) == nrows(s0);
    return { ok, "glu_fused_requires_even_src0_and_half_width_dst" };
}

support check_rms_norm(const lnsb_tensor * op) {
    if (op->src[0] == nullptr || op->src[0]->type != LNSB_TYPE_F32) return { false, "unary_like_requires_src0_f32" };
    return f32_result(op, { true, "lns_cuda_rms_norm" });
}

support check_soft_max(const lnsb_tensor * op) {
    const lnsb_tensor * mask = op->src[1];
    if (op->src[0] == nullptr || op->src[0]->type != LNSB_TYPE_F32 || (mask != nullptr && mask->type != LNSB_TYPE_F32))
        return { false, "soft_max_requires_f32_src0_and_f32_mask" };
    if (op->src[2] != nullptr) return { false, "soft_max_sinks_unsupported" };
    if (param_f32(op, 1) != 0.0f) return { false, "soft_max_alibi_unsupported" };
    const support base = f32_result(op, { true, "soft_max_f32" });
    if (base.ok && mask != nullptr && (mask->ne[0] < op->ne[0] || mask->ne[1] < op->ne[1] || !rows_contiguous(mask)))
        return { false, "lns_cuda_soft_max_mask_smaller_than_src0" };
    return base;
}

support check_rope(const lnsb_tensor * op) {
    if (op->src[0] == nullptr || op->src[0]->type != LNSB_TYPE_F32) return { false, "rope_requires_src0_f32" };
    const int mode = op->op_params[2];
    if (mode != 0 && mode != LNSB_ROPE_TYPE_NEOX) return { false, "rope_mode_unsupported" };
    if (param_f32(op, 6) != 1.0f || param_f32(op, 7) != 0.0f || param_f32(op, 8) != 1.0f)
        return { false, "rope_scaling_unsupported" };
    const int n_dims = op->op_params[1];
    const lnsb_tensor * ff = op->src[2];
    if (ff != nullptr && (ff->type != LNSB_TYPE_F32 || !contiguous(ff) || ff->ne[0] < n_dims / 2))
        return { false, "rope_freq_factors_require_contiguous_f32" };
    const support base = f32_result(op, { true, "rope_normal_or_neox" });
    if (!base.ok) return base;
    const lnsb_tensor * pos = op->src[1];
    if (pos == nullptr || pos->type != LNSB_TYPE_I32 || !contiguous(pos) || pos->ne[0] < op->src[0]->ne[2])
        return { false, "lns_cuda_rope_requires_i32_positions" };
    if (n_dims <= 0 || n_dims % 2 != 0 || n_dims > op->src[0]->ne[0]) return { false, "lns_cuda_rope_requires_even_n_dims" };
    return { true, "lns_cuda_rope" };
}

support check(const lnsb_tensor * n) {
    if (is_view_or_noop(n->op)) return { true, "supported_view_or_noop" };
    for (int i = 0; i < 4; i++)
        if (n->src[i] != nullptr && !known_type(n->src[i]->type)) return { false, "unsupported_type" };
    switch (n->op) {
        case LNSB_OP_MUL_MAT:    return check_mul_mat(n);
        case LNSB_OP_MUL_MAT_ID: return check_mul_mat_id(n);
        case LNSB_OP_ADD: case LNSB_OP_MUL: case LNSB_OP_DIV: return check_binary(n);
        case LNSB_OP_SCALE:      return check_scale(n);
        case LNSB_OP_RMS_NORM:   return check_rms_norm(n);
        case LNSB_OP_SOFT_MAX:   return check_soft_max(n);
        case LNSB_OP_ROPE:       return check_rope(n);
        case LNSB_OP_UNARY:      return check_unary(n);
        case LNSB_OP_GLU:        return check_glu(n);
        default:                 return { false, "unsupported_op" };
    }
}

// ------------------------------------------------------------------ selection, bisection, audit

std::vector<std::string> split_list(const char * list) {
    std::vector<std::string> out;
    if (list == nullptr) return out;
    const std::string s(list);
    size_t pos = 0;
    while (pos <= s.size()) {
        const size_t comma = s.find(',', pos);
        std::string tok = s.substr(pos, comma == std::string::npos ? std::string::npos : comma - pos);
        const size_t a = tok.find_first_not_of(" \t");
        if (a != std::string::npos) out.push_back(tok.substr(a, tok.find_last_not_of(" \t") - a + 1));
        if (comma == std::string::npos) break;
        pos = comma + 1;
    }
    return out;
}

struct alias {
    const char * token;
    const char * devices;
};
// The LNS devices of the reference (LNS16, LNS32 on the CPU; LNSCUDA16,
// LNSCUDA32 on the GPU, which this library serves); a GPU alias also selects
// the matching CPU backend, which takes the ops the GPU backend declines
const alias k_aliases[] = {
    { "16", "LNS16" }, { "32", "LNS32" }, { "cuda", "LNSCUDA16,LNS16" }, { "cuda16", "LNSCUDA16,LNS16" },
    { "cuda32", "LNSCUDA32,LNS32" },
};
const char * const k_default_selection = "16";

bool known_device(const std::string & name) {
    for (const alias & a : k_aliases)
        for (const std::string & d : split_list(a.devices))
            if (strcasecmp(d.c_str(), name.c_str()) == 0) return true;
    return false;
}

std::vector<std::string> resolve(const char * value) {
    std::vector<std::string> devs;
    const char * spec = (value != nullptr && value[0] != '\0') ? value : k_default_selection;
    for (const std::string & tok : split_list(spec)) {
        bool matched = false;
        for (const alias & a : k_aliases) {
            if (strcasecmp(a.token, tok.c_str()) == 0) {
                for (const std::string & d : split_list(a.devices)) devs.push_back(d);
                matched = true;
                break;
            }
        }
        if (!matched && known_device(tok)) {
            devs.push_back(tok);
            matched = true;
        }
        if (!matched) std::fprintf(stderr, "ggml-lns: ignoring unknown GGML_LNS_BACKEND token '%s'\n", tok.c_str());
    }
    if (devs.empty()) return resolve(k_default_selection);
    return devs;
}

bool selected_in(const char * device, const std::vector<std::string> & sel) {
    for (const std::string & d : sel)
        if (device != nullptr && strcasecmp(d.c_str(), device) == 0) return true;
    return false;
}

bool name_matches(const char * name, const std::string & pattern) {
    if (name == nullptr || name[0] == '\0') return false;
    if (pattern.find_first_of("*?[") != std::string::npos) return fnmatch(pattern.c_str(), name, 0) == 0;
    return std::strstr(name, pattern.c_str()) != nullptr;
}

bool op_matches(const lnsb_tensor * op, const std::string & tok) {
    const char * op_name = lnsb_op_name(op->op);
    const char * desc = lnsb_op_desc(op);
    if (strcasecmp(tok.c_str(), op_name) == 0 || strcasecmp(tok.c_str(), desc) == 0) return true;
    std::string pattern = tok;
    const size_t colon = tok.find(':');
    if (colon != std::string::npos) {
        const std::string want = tok.substr(0, colon);
        if (strcasecmp(want.c_str(), op_name) != 0 && strcasecmp(want.c_str(), desc) != 0) return false;
        pattern = tok.substr(colon + 1);
    }
    if (!pattern.empty() && pattern[0] == '<')
        return op->src[1] != nullptr && name_matches(op->src[1]->name, pattern.substr(1));
    return name_matches(op->name, pattern);
}

bool matches_any(const lnsb_tensor * op, const std::vector<std::string> & toks) {
    for (const std::string & t : toks)
        if (op_matches(op, t)) return true;
    return false;
}

bool env_flag(const char * name) {
    const char * v = std::getenv(name);
    return v != nullptr && v[0] != '\0' && std::strcmp(v, "0") != 0;
}

const char * sum_mode_fields(int fmt) {
    static std::string f[2];
    static std::once_flag once;
    std::call_once(once, [] {
        const char * m = lnsb_sum_mode(LNSB_XLNS16);
        f[0] = m ? std::string("\"sum_mode\":\"") + m + "\"," : std::string();
    });
    return fmt == LNSB_XLNS16 ? f[0].c_str() : f[1].c_str();
}

// ------------------------------------------------------------------ graph compute

enum role : int { R_SRC0, R_SRC1, R_SRC2, R_LNS0, R_LNS1, R_DST, R_WORK, R_AUX, R_GATHER, R_COUNT };

}  // namespace

struct lnsb_graph_ctx {
    int                 fmt = LNSB_XLNS16;
    int                 device = 0;
    cudaStream_t        stream = nullptr;
    lnsb_weight_cache * cache = nullptr;
    void *              scratch[R_COUNT] = {};
    size_t              bytes[R_COUNT] = {};
    std::vector<char>   host[R_COUNT];

    ~lnsb_graph_ctx() {
        if (cache != nullptr) lnsb_weight_cache_destroy(cache);
        for (int i = 0; i < R_COUNT; i++)
            if (scratch[i] != nullptr) cudaFree(scratch[i]);
    }
    void * dev(role r, size_t n) {
        n = std::max<size_t>(n, 16);
        if (bytes[r] < n) {
            if (scratch[r] != nullptr) {
                cudaStreamSynchronize(stream);
                cudaFree(scratch[r]);
                scratch[r] = nullptr;
                bytes[r] = 0;
            }
            if (cudaMalloc(&scratch[r], n) != cudaSuccess) {
                cudaGetLastError();                      // not sticky: clear it, report the failure
                return nullptr;
            }
            bytes[r] = n;
        }
        return scratch[r];
    }
};

namespace {

bool on_device(const void * p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// the strided view of t as a packed host array of elem-sized elements
void gather_host(const lnsb_tensor * t, int64_t elem, char * out) {
    int64_t o = 0;
    for (int64_t i3 = 0; i3 < t->ne[3]; i3++)
        for (int64_t i2 = 0; i2 < t->ne[2]; i2++)
            for (int64_t i1 = 0; i1 < t->ne[1]; i1++) {
                const char * row = static_cast<const char *>(t->data) + i1 * t->nb[1] + i2 * t->nb[2] + i3 * t->nb[3];
                if (t->nb[0] == elem) {
                    std::memcpy(out + o, row, (size_t) (t->ne[0] * elem));
                    o += t->ne[0] * elem;
                } else {
                    for (int64_t i0 = 0; i0 < t->ne[0]; i0++, o += elem) std::memcpy(out + o, row + i0 * t->nb[0], (size_t) elem);
                }
            }
}
void scatter_host(const char * in, int64_t elem, lnsb_tensor * t) {
    int64_t o = 0;
    for (int64_t i3 = 0; i3 < t->ne[3]; i3++)
        for (int64_t i2 = 0; i2 < t->ne[2]; i2++)
            for (int64_t i1 = 0; i1 < t->ne[1]; i1++) {
                char * row = static_cast<char *>(t->data) + i1 * t->nb[1] + i2 * t->nb[2] + i3 * t->nb[3];
                for (int64_t i0 = 0; i0 < t->ne[0]; i0++, o += elem) std::memcpy(row + i0 * t->nb[0], in + o, (size_t) elem);
            }
}

// A packed device copy of t's elements (plain types: F32, F16, BF16, I32):
// t's own memory when it is on the device and contiguous, else a gather into
// the role's scratch (on the device for device views, on the host and then
// uploaded for host memory).  nullptr on an allocation failure.
const void * packed(lnsb_graph_ctx & c, const lnsb_tensor * t, role r, int * st) {
    const int64_t elem = type_size(t->type);
    const int64_t n = nelements(t);
    if (on_device(t->data)) {
        if (contiguous(t)) return t->data;
        void * d = c.dev(r, (size_t) (n * elem));
        if (d == nullptr) { *st = LNSB_E_TOO_LARGE; return nullptr; }
        const int s = lnsb_copy_strided((int) elem, t->data, t->ne, t->nb, d, c.stream);
        if (s != 0) { *st = s; return nullptr; }
        return d;
    }
    void * d = c.dev(r, (size_t) (n * elem));
    if (d == nullptr) { *st = LNSB_E_TOO_LARGE; return nullptr; }
    const void * src = t->data;
    if (!contiguous(t)) {
        c.host[r].resize((size_t) (n * elem));
        gather_host(t, elem, c.host[r].data());
        src = c.host[r].data();
    }
    cudaError_t e = cudaMemcpyAsync(d, src, (size_t) (n * elem), cudaMemcpyHostToDevice, c.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c.stream);
    if (e != cudaSuccess) { *st = (int) e; return nullptr; }
    return d;
}

// where a node's F32 result is computed: its own memory when it is on the
// device and contiguous, else the DST scratch (finish() copies it out)
float * result(lnsb_graph_ctx & c, lnsb_tensor * t, int * st) {
    if (on_device(t->data) && contiguous(t)) return static_cast<float *>(t->data);
    float * d = static_cast<float *>(c.dev(R_DST, (size_t) (nelements(t) * 4)));
    if (d == nullptr) *st = LNSB_E_TOO_LARGE;
    return d;
}
int finish(lnsb_graph_ctx & c, lnsb_tensor * t, const float * d) {
    if (d == t->data) return 0;
    const int64_t n = nelements(t);
    if (on_device(t->data)) {                           // a strided device result: not produced by any node here
        return LNSB_E_UNSUPPORTED;
    }
    cudaError_t e;
    if (contiguous(t)) {
        e = cudaMemcpyAsync(t->data, d, (size_t) (n * 4), cudaMemcpyDeviceToHost, c.stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(c.stream);
        return (int) e;
    }
    c.host[R_DST].resize((size_t) (n * 4));
    e = cudaMemcpyAsync(c.host[R_DST].data(), d, (size_t) (n * 4), cudaMemcpyDeviceToHost, c.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c.stream);
    if (e != cudaSuccess) return (int) e;
    scatter_host(c.host[R_DST].data(), 4, t);
    return 0;
}

uint16_t reserve_monte(uint64_t draws) {
    uint16_t s = 0;
    if (draws > 0 && lnsb_monte_reserve(draws, &s) != 0) s = 0;
    return s;
}

// The k-major LNS image of a matrix operand [slices][K][M] (K = ne0, M = ne1),
// slice by slice: from the weight cache for a 2-D weight tensor with packed
// rows (converted once, kept), else converted into the LNS0 scratch; a
// strided F32 / F16 / BF16 view is gathered first, host rows are uploaded.
const void * lns_matrix(lnsb_graph_ctx & c, const lnsb_tensor * t, int * st) {
    const int64_t K = t->ne[0], M = t->ne[1], S = t->ne[2] * t->ne[3];
    const int64_t rb = row_bytes(t);
    const bool packed_rows = M <= 1 || t->nb[1] == rb;
    const size_t vs = lnsb_value_size(c.fmt);
    if ((t->flags & LNSB_TENSOR_FLAG_WEIGHTS) && S == 1 && packed_rows) {
        void * spill = c.dev(R_LNS0, (size_t) (K * M) * vs);
        const void * out = nullptr;
        const int s = lnsb_weight_cache_get(c.cache, t->data, t->type, M, K, spill, &out, c.stream);
        if (s != 0) { *st = s; return nullptr; }
        return out;
    }
    char * img = static_cast<char *>(c.dev(R_LNS0, (size_t) (S * K * M) * vs));
    if (img == nullptr) { *st = LNSB_E_TOO_LARGE; return nullptr; }
    const bool dev_src = on_device(t->data);
    for (int64_t i3 = 0; i3 < t->ne[3]; i3++)
        for (int64_t i2 = 0; i2 < t->ne[2]; i2++) {
            const char * slice = static_cast<const char *>(t->data) + i2 * t->nb[2] + i3 * t->nb[3];
            const void * src = slice;
            if (!dev_src || !packed_rows || !rows_contiguous(t)) {
                // one slice, packed on the device (gathered or uploaded)
                lnsb_tensor v = *t;
                v.data = const_cast<char *>(slice);
                v.ne[2] = v.ne[3] = 1;
                v.nb[2] = v.nb[3] = v.nb[1] * v.ne[1];
                if (blck_size(t->type) > 1) {            // packed quantised rows: upload as bytes
                    void * d = c.dev(R_GATHER, (size_t) (M * rb));
                    if (d == nullptr) { *st = LNSB_E_TOO_LARGE; return nullptr; }
                    cudaError_t e = cudaMemcpyAsync(d, slice, (size_t) (M * rb), dev_src ? cudaMemcpyDeviceToDevice
                                                                                           : cudaMemcpyHostToDevice, c.stream);
                    if (e == cudaSuccess && !dev_src) e = cudaStreamSynchronize(c.stream);
                    if (e != cudaSuccess) { *st = (int) e; return nullptr; }
                    src = d;
                } else {
                    src = packed(c, &v, R_GATHER, st);
                    if (src == nullptr) return nullptr;
                }
            }
            const int s = lnsb_to_lns_transposed_typed(c.fmt, t->type, src, img + (size_t) ((i3 * t->ne[2] + i2) * K * M) * vs,
                                                      M, K, M, c.stream);
            if (s != 0) { *st = s; return nullptr; }
        }
    return img;
}

// the LNS codes of an F32 activation operand
const void * lns_operand(lnsb_graph_ctx & c, const lnsb_tensor * t, role staged, role r, int * st) {
    const float * f = static_cast<const float *>(packed(c, t, staged, st));
    if (f == nullptr) return nullptr;
    void * d = c.dev(r, (size_t) nelements(t) * lnsb_value_size(c.fmt));
    if (d == nullptr) { *st = LNSB_E_TOO_LARGE; return nullptr; }
    const int s = lnsb_to_lns(c.fmt, f, d, nelements(t), c.stream);
    if (s != 0) { *st = s; return nullptr; }
    return d;
}

int compute_mul_mat(lnsb_graph_ctx & c, lnsb_tensor * n) {
    int st = 0;
    const lnsb_tensor * s0 = n->src[0];
    const lnsb_tensor * s1 = n->src[1];
    const void * w = lns_matrix(c, s0, &st);
    if (w == nullptr) return st;
    // the F32 activations go to lnsb_mul_mat_xf32, which converts them while
    // staging where its kernel can (else into x_work first): the reference's
    // to_lns + mul_mat pair in one call
    const float * xf = static_cast<const float *>(packed(c, s1, R_SRC1, &st));
    if (xf == nullptr) return st;
    void * x_work = c.dev(R_LNS1, (size_t) nelements(s1) * lnsb_value_size(c.fmt));
    if (x_work == nullptr) return LNSB_E_TOO_LARGE;
    float * out = result(c, n, &st);
    if (out == nullptr) return st;
    lnsb_mul_mat_args a{ w, xf, out, s0->ne[0], s0->ne[1], s1->ne[1], s0->ne[2], s0->ne[3], s1->ne[2], s1->ne[3], 0 };
    a.monte_seed = reserve_monte(lnsb_mul_mat_draws(c.fmt, &a));
    st = lnsb_mul_mat_xf32(c.fmt, &a, x_work, c.stream);
    return st != 0 ? st : finish(c, n, out);
}

int compute_mul_mat_id(lnsb_graph_ctx & c, lnsb_tensor * n) {
    int st = 0;
    const lnsb_tensor * s0 = n->src[0];
    const lnsb_tensor * s1 = n->src[1];
    const lnsb_tensor * ids = n->src[2];
    const void * w = lns_matrix(c, s0, &st);
    if (w == nullptr) return st;
    const void * x = lns_operand(c, s1, R_SRC1, R_LNS1, &st);
    if (x == nullptr) return st;
    const int32_t * id = static_cast<const int32_t *>(packed(c, ids, R_AUX, &st));
    if (id == nullptr) return st;
    float * out = result(c, n, &st);
    if (out == nullptr) return st;
    lnsb_mul_mat_id_args a{ w, x, id, out, s0->ne[0], s0->ne[1], s0->ne[2], s1->ne[1], ids->ne[0], ids->ne[1],
                            ids->ne[0], 0 };
    a.monte_seed = reserve_monte(lnsb_mul_mat_id_draws(c.fmt, &a));
    st = lnsb_mul_mat_id(c.fmt, &a, c.stream);
    return st != 0 ? st : finish(c, n, out);
}

int compute_binary(lnsb_graph_ctx & c, lnsb_tensor * n) {
    int st = 0;
    const float * a = static_cast<const float *>(packed(c, n->src[0], R_SRC0, &st));
    if (a == nullptr) return st;
    const float * b = static_cast<const float *>(packed(c, n->src[1], R_SRC1, &st));
    if (b == nullptr) return st;
    float * out = result(c, n, &st);
    if (out == nullptr) return st;
    const int op = n->op == LNSB_OP_ADD ? LNSB_BINARY_ADD : n->op == LNSB_OP_MUL ? LNSB_BINARY_MUL : LNSB_BINARY_DIV;
    st = lnsb_binary(c.fmt, op, a, n->src[0]->ne, b, n->src[1]->ne, out, c.stream);
    return st != 0 ? st : finish(c, n, out);
}

int compute_scale(lnsb_graph_ctx & c, lnsb_tensor * n) {
    int st = 0;
    const float * a = static_cast<const float *>(packed(c, n->src[0], R_SRC0, &st));
    if (a == nullptr) return st;
    float * out = result(c, n, &st);
    if (out == nullptr) return st;
    st = lnsb_scale(c.fmt, a, out, nelements(n), param_f32(n, 0), param_f32(n, 1), c.stream);
    return st != 0 ? st : finish(c, n, out);
}

int compute_unary(lnsb_graph_ctx & c, lnsb_tensor * n) {
    int st = 0;
    const float * a = static_cast<const float *>(packed(c, n->src[0], R_SRC0, &st));
    if (a == nullptr) return st;
    float * out = result(c, n, &st);
    if (out == nullptr) return st;
    st = lnsb_unary(c.fmt, n->op_params[0], a, out, nelements(n), c.stream);
    return st != 0 ? st : finish(c, n, out);
}

int compute_glu(lnsb_graph_ctx & c, lnsb_tensor * n) {
    int st = 0;
    const lnsb_tensor * s0 = n->src[0];
    const lnsb_tensor * s1 = n->src[1];
    const int64_t nc = n->ne[0], nr = nrows(n);
    const float * gate;
    const float * up;
    int64_t gs, us;
    if (s1 != nullptr) {
        gate = static_cast<const float *>(packed(c, s0, R_SRC0, &st));
        if (gate == nullptr) return st;
        up = static_cast<const float *>(packed(c, s1, R_SRC1, &st));
        if (up == nullptr) return st;
        gs = us = nc;
    } else {
        const float * f = static_cast<const float *>(packed(c, s0, R_SRC0, &st));
        if (f == nullptr) return st;
        const bool swapped = n->op_params[1] != 0;
        gate = swapped ? f + nc : f;
        up = swapped ? f : f + nc;
        gs = us = 2 * nc;
    }
    float * out = result(c, n, &st);
    if (out == nullptr) return st;
    st = lnsb_glu(c.fmt, n->op_params[0], gate, up, gs, us, out, nc, nr, c.stream);
    return st != 0 ? st : finish(c, n, out);
}

int compute_rms_norm(lnsb_graph_ctx & c, lnsb_tensor * n) {
    int st = 0;
    const lnsb_tensor * s0 = n->src[0];
    const float * a = static_cast<const float *>(packed(c, s0, R_SRC0, &st));
    if (a == nullptr) return st;
    float * out = result(c, n, &st);
    if (out == nullptr) return st;
    const uint16_t seed = reserve_monte(lnsb_rms_norm_draws(c.fmt, s0->ne[0], nrows(s0)));
    st = lnsb_rms_norm(c.fmt, a, out, s0->ne[0], nrows(s0), param_f32(n, 0), seed, c.stream);
    return st != 0 ? st : finish(c, n, out);
}

int compute_soft_max(lnsb_graph_ctx & c, lnsb_tensor * n) {
    int st = 0;
    const lnsb_tensor * s0 = n->src[0];
    const lnsb_tensor * mask = n->src[1];
    lnsb_soft_max_args a{};
    a.src = static_cast<const float *>(packed(c, s0, R_SRC0, &st));
    if (a.src == nullptr) return st;
    a.src_shape = lnsb_shape4{ { s0->ne[0], s0->ne[1], s0->ne[2], s0->ne[3] } };
    a.mask_shape = lnsb_shape4{ { 1, 1, 1, 1 } };
    if (mask != nullptr) {
        // the mask's rows as wide as the logits' (a padded mask is gathered to ne0 columns)
        lnsb_tensor m = *mask;
        m.ne[0] = s0->ne[0];
        a.mask = static_cast<const float *>(packed(c, &m, R_SRC1, &st));
        if (a.mask == nullptr) return st;
        a.mask_shape = lnsb_shape4{ { m.ne[0], m.ne[1], m.ne[2], m.ne[3] } };
    }
    a.scale = param_f32(n, 0);
    a.dst = result(c, n, &st);
    if (a.dst == nullptr) return st;
    a.work = c.dev(R_WORK, (size_t) nelements(s0) * lnsb_value_size(c.fmt));
    if (a.work == nullptr) return LNSB_E_TOO_LARGE;
    a.monte_seed = reserve_monte(lnsb_soft_max_draws(c.fmt, s0->ne[0], nrows(s0)));
    st = lnsb_soft_max(c.fmt, &a, c.stream);
    return st != 0 ? st : finish(c, n, a.dst);
}

int compute_rope(lnsb_graph_ctx & c, lnsb_tensor * n) {
    int st = 0;
    const lnsb_tensor * s0 = n->src[0];
    const lnsb_tensor * pos_t = n->src[1];
    const lnsb_tensor * ff_t = n->src[2];
    const int n_dims = n->op_params[1];
    const int64_t np = s0->ne[2], half = n_dims / 2;
    // positions (and frequency factors) on the host
    std::vector<int32_t> pos((size_t) np);
    std::vector<float> ff;
    cudaError_t e = cudaMemcpyAsync(pos.data(), pos_t->data, (size_t) np * 4, cudaMemcpyDefault, c.stream);
    if (ff_t != nullptr && e == cudaSuccess) {
        ff.resize((size_t) half);
        e = cudaMemcpyAsync(ff.data(), ff_t->data, (size_t) half * 4, cudaMemcpyDefault, c.stream);
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(c.stream);
    if (e != cudaSuccess) return (int) e;
    // (cos, sin) per position and pair in lns_rope's float recurrence
    // (lns-backend/src/lns-ops.cpp:1231-1262, lns-cuda-ops.cpp:222-234)
    const float theta_scale = powf(param_f32(n, 5), -2.0f / (float) n_dims);
    std::vector<float> table((size_t) (np * half * 2));
    for (int64_t i2 = 0; i2 < np; i2++) {
        float t = (float) pos[(size_t) i2];
        for (int64_t p = 0; p < half; p++) {
            const float theta = ff.empty() ? t : t / ff[(size_t) p];
            table[(size_t) ((i2 * half + p) * 2 + 0)] = cosf(theta);
            table[(size_t) ((i2 * half + p) * 2 + 1)] = sinf(theta);
            t *= theta_scale;
        }
    }
    float * dcs = static_cast<float *>(c.dev(R_AUX, table.size() * 4));
    if (dcs == nullptr) return LNSB_E_TOO_LARGE;
    e = cudaMemcpyAsync(dcs, table.data(), table.size() * 4, cudaMemcpyHostToDevice, c.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c.stream);
    if (e != cudaSuccess) return (int) e;
    lnsb_rope_args a{};
    a.src = static_cast<const float *>(packed(c, s0, R_SRC0, &st));
    if (a.src == nullptr) return st;
    a.shape = lnsb_shape4{ { s0->ne[0], s0->ne[1], s0->ne[2], s0->ne[3] } };
    a.cos_sin = dcs;
    a.n_dims = n_dims;
    a.neox = (n->op_params[2] & LNSB_ROPE_TYPE_NEOX) != 0;
    a.dst = result(c, n, &st);
    if (a.dst == nullptr) return st;
    st = lnsb_rope(c.fmt, &a, c.stream);
    return st != 0 ? st : finish(c, n, a.dst);
}

int compute(lnsb_graph_ctx & c, lnsb_tensor * n) {
    switch (n->op) {
        case LNSB_OP_MUL_MAT:    return compute_mul_mat(c, n);
        case LNSB_OP_MUL_MAT_ID: return compute_mul_mat_id(c, n);
        case LNSB_OP_ADD: case LNSB_OP_MUL: case LNSB_OP_DIV: return compute_binary(c, n);
        case LNSB_OP_SCALE:      return compute_scale(c, n);
        case LNSB_OP_RMS_NORM:   return compute_rms_norm(c, n);
        case LNSB_OP_SOFT_MAX:   return compute_soft_max(c, n);
        case LNSB_OP_ROPE:       return compute_rope(c, n);
        case LNSB_OP_UNARY:      return compute_unary(c, n);
        case LNSB_OP_GLU:        return compute_glu(c, n);
        default:                 return LNSB_E_UNSUPPORTED;
    }
}

}  // namespace

extern "C" {

const char * lnsb_op_name(int op) { return op >= 0 && op < LNSB_OP_COUNT ? k_op_names[op] : "UNKNOWN"; }

const char * lnsb_op_desc(const lnsb_tensor * n) {
    if (n == nullptr) return "UNKNOWN";
    if (n->op == LNSB_OP_UNARY && n->op_params[0] >= 0 && n->op_params[0] < 4) return k_unary_names[n->op_params[0]];
    if (n->op == LNSB_OP_GLU && n->op_params[0] >= 0 && n->op_params[0] < 2) return k_glu_names[n->op_params[0]];
    return lnsb_op_name(n->op);
}

int lnsb_check_op(int fmt, const lnsb_tensor * node, const char ** reason) {
    if (node == nullptr || (fmt != LNSB_XLNS16 && fmt != LNSB_XLNS32)) {
        if (reason) *reason = "invalid";
        return 0;
    }
    const support s = check(node);
    if (reason) *reason = s.reason;
    return s.ok ? 1 : 0;
}

int lnsb_resolve_backend_selection(const char * selection, char * out, size_t cap) {
    const std::vector<std::string> devs = resolve(selection);
    std::string joined;
    for (size_t i = 0; i < devs.size(); i++) joined += (i ? "," : "") + devs[i];
    if (out != nullptr && cap > 0) std::snprintf(out, cap, "%s", joined.c_str());
    return (int) devs.size();
}

int lnsb_backend_selected_by(const char * device_name, const char * selection) {
    return selected_in(device_name, resolve(selection)) ? 1 : 0;
}

int lnsb_op_matches(const lnsb_tensor * node, const char * token) {
    return node != nullptr && token != nullptr && op_matches(node, token) ? 1 : 0;
}

int lnsb_op_disabled_by(const lnsb_tensor * node, const char * disable_list, const char * enable_list) {
    if (node == nullptr) return 1;
    if (enable_list != nullptr && !matches_any(node, split_list(enable_list))) return 1;
    return matches_any(node, split_list(disable_list)) ? 1 : 0;
}

int lnsb_audit_line(const char * backend, int fmt, const lnsb_tensor * op, int supported, const char * reason,
                    char * out, size_t cap) {
    if (op == nullptr) return 0;
    return std::snprintf(out, cap,
        "{\"event\":\"lns_supports_op\",\"backend\":\"%s\",%s\"op\":\"%s\",\"desc\":\"%s\",\"supported\":%s,"
        "\"dst_type\":\"%s\",\"src_types\":[\"%s\",\"%s\",\"%s\",\"%s\"],\"shape\":[%lld,%lld,%lld,%lld],"
        "\"reason\":\"%s\"}",
        backend ? backend : "", sum_mode_fields(fmt), lnsb_op_name(op->op), lnsb_op_desc(op),
        supported ? "true" : "false", type_name(op), type_name(op->src[0]), type_name(op->src[1]),
        type_name(op->src[2]), type_name(op->src[3]), (long long) op->ne[0], (long long) op->ne[1],
        (long long) op->ne[2], (long long) op->ne[3], reason ? reason : "");
}

int lnsb_supports_op(const char * device_name, int fmt, const lnsb_tensor * node) {
    static const std::vector<std::string> selection = resolve(std::getenv("GGML_LNS_BACKEND"));
    static const char * enable_env = std::getenv("LNS_ENABLE_OPS");
    static const std::string disable = std::getenv("LNS_DISABLE_OPS") ? std::getenv("LNS_DISABLE_OPS") : "";
    static const std::string enable = enable_env ? enable_env : "";
    static const bool audit = env_flag("LNS_OP_AUDIT");
    if (node == nullptr) return 0;
    auto log = [&](bool ok, const char * reason) {
        if (!audit) return;
        char line[1024];
        lnsb_audit_line(device_name, fmt, node, ok ? 1 : 0, reason, line, sizeof line);
        std::fprintf(stderr, "%s\n", line);
    };
    if (!selected_in(device_name, selection)) {
        log(false, "disabled_by_env");
        return 0;
    }
    const char * reason = nullptr;
    const int ok = lnsb_check_op(fmt, node, &reason);
    log(ok != 0, reason);
    return ok && !lnsb_op_disabled_by(node, disable.c_str(), enable_env ? enable.c_str() : nullptr) ? 1 : 0;
}

const char * lnsb_device_description(int fmt) {
    static std::string desc[2];
    static std::mutex mu;
    if (fmt != LNSB_XLNS16 && fmt != LNSB_XLNS32) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    std::string & d = desc[fmt == LNSB_XLNS32];
    if (d.empty()) {
        d = std::string("Logarithmic Number System on CUDA (") + lnsb_format_name(fmt);
        const char * sm = lnsb_sum_mode(fmt);
        if (sm != nullptr) {
            d += std::string(", sum=") + sm;
            const char * mi = lnsb_monte_impl(fmt);
            if (mi != nullptr) d += std::string(", monte=") + mi;
        }
        d += ")";
        int dev = -1;
        cudaDeviceProp prop;
        if (cudaGetDevice(&dev) == cudaSuccess && cudaGetDeviceProperties(&prop, dev) == cudaSuccess)
            d += std::string(" on ") + prop.name;
        else
            cudaGetLastError();
    }
    return d.c_str();
}

lnsb_graph_ctx * lnsb_graph_ctx_create(int fmt, int64_t cache_budget_bytes, lnsb_stream_t stream) {
    if (fmt != LNSB_XLNS16 && fmt != LNSB_XLNS32) return nullptr;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    if (lnsb_upload_tables(fmt) != 0) return nullptr;
    lnsb_graph_ctx * c = new lnsb_graph_ctx();
    c->fmt = fmt;
    c->device = dev;
    c->stream = static_cast<cudaStream_t>(stream);
    c->cache = lnsb_weight_cache_create(fmt, cache_budget_bytes);
    if (c->cache == nullptr) {
        delete c;
        return nullptr;
    }
    return c;
}

void lnsb_graph_ctx_destroy(lnsb_graph_ctx * ctx) {
    if (ctx == nullptr) return;
    int cur = -1;
    const bool known = cudaGetDevice(&cur) == cudaSuccess;
    if (!known) cudaGetLastError();
    if (known && cur != ctx->device) cudaSetDevice(ctx->device);   // the scratch belongs to the context's device
    delete ctx;
    if (known && cur != ctx->device) cudaSetDevice(cur);
}

int lnsb_graph_compute(lnsb_graph_ctx * ctx, lnsb_tensor * const * nodes, int n_nodes, int * failed) {
    if (failed) *failed = -1;
    if (ctx == nullptr || (nodes == nullptr && n_nodes > 0) || n_nodes < 0) return LNSB_E_INVALID;
    // calls may come from any host thread: bind the context's device first
    if (cudaSetDevice(ctx->device) != cudaSuccess) {
        cudaGetLastError();
        return LNSB_E_NO_DEVICE;
    }
    for (int i = 0; i < n_nodes; i++) {
        lnsb_tensor * n = nodes[i];
        if (n == nullptr) {
            if (failed) *failed = i;
            return LNSB_E_INVALID;
        }
        if ((n->flags & LNSB_TENSOR_FLAG_COMPUTE) == 0 || is_view_or_noop(n->op) || nelements(n) == 0) continue;
        const char * reason = nullptr;
        int st = lnsb_check_op(ctx->fmt, n, &reason) ? compute(*ctx, n) : LNSB_E_UNSUPPORTED;
        if (st != 0) {
            if (failed) *failed = i;
            return st;
        }
    }
    return 0;
}

}  // extern "C"
