// lnsb200_ggml.hpp -- the ggml registration of this library's backends
// (LNSCUDA16 / LNSCUDA32): the vtables of lns-backend/common/
// lns-backend-framework.h:118-350 and lns-backend/cuda/ggml-lns-cuda.cpp,
// forwarding supports_op and graph_compute to include/lnsb200_graph.h.
//
// Compiled only where ggml's ggml-backend-impl.h is on the include path (a
// llama.cpp / ggml build tree); elsewhere this header is empty.  Include it in
// exactly one translation unit of the program that registers the backends,
// and link one liblnsb200_<mode>.so (the build-time summation mode).  The
// vtables are filled member by member on zero-initialised structs, so fields
// a newer ggml adds stay null (optional) instead of shifting the order.
#pragma once

#if defined(__has_include)
#if __has_include("ggml-backend-impl.h")
#define LNSB200_HAVE_GGML 1
#endif
#endif

#ifdef LNSB200_HAVE_GGML

#include "ggml-backend-impl.h"
#include "ggml-impl.h"
#include "lnsb200_graph.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <vector>

namespace lnsb200_ggml {

inline int op_of(ggml_op op) {
    switch (op) {
        case GGML_OP_NONE:       return LNSB_OP_NONE;
        case GGML_OP_RESHAPE:    return LNSB_OP_RESHAPE;
        case GGML_OP_VIEW:       return LNSB_OP_VIEW;
        case GGML_OP_PERMUTE:    return LNSB_OP_PERMUTE;
        case GGML_OP_TRANSPOSE:  return LNSB_OP_TRANSPOSE;
        case GGML_OP_MUL_MAT:    return LNSB_OP_MUL_MAT;
        case GGML_OP_MUL_MAT_ID: return LNSB_OP_MUL_MAT_ID;
        case GGML_OP_ADD:        return LNSB_OP_ADD;
        case GGML_OP_MUL:        return LNSB_OP_MUL;
        case GGML_OP_DIV:        return LNSB_OP_DIV;
        case GGML_OP_SCALE:      return LNSB_OP_SCALE;
        case GGML_OP_RMS_NORM:   return LNSB_OP_RMS_NORM;
        case GGML_OP_SOFT_MAX:   return LNSB_OP_SOFT_MAX;
        case GGML_OP_ROPE:       return LNSB_OP_ROPE;
        case GGML_OP_UNARY:      return LNSB_OP_UNARY;
        case GGML_OP_GLU:        return LNSB_OP_GLU;
        case GGML_OP_GET_ROWS:   return LNSB_OP_GET_ROWS;
        case GGML_OP_CPY:        return LNSB_OP_CPY;
        case GGML_OP_CONT:       return LNSB_OP_CONT;
        default:                 return LNSB_OP_COUNT;        // no kernel: the predicate refuses it
    }
}

inline int unary_of(ggml_unary_op u) {
    switch (u) {
        case GGML_UNARY_OP_SILU: return LNSB_UNARY_SILU;
        case GGML_UNARY_OP_GELU: return LNSB_UNARY_GELU;
        case GGML_UNARY_OP_RELU: return LNSB_UNARY_RELU;
        case GGML_UNARY_OP_TANH: return LNSB_UNARY_TANH;
        default:                 return -1;
    }
}

inline int glu_of(ggml_glu_op g) {
    switch (g) {
        case GGML_GLU_OP_SWIGLU: return LNSB_GLU_SWIGLU;
        case GGML_GLU_OP_GEGLU:  return LNSB_GLU_GEGLU;
        default:                 return -1;
    }
}

// A node and its sources as descriptors (storage owned by the object).
struct node_desc {
    lnsb_tensor node;
    lnsb_tensor src[4];

    explicit node_desc(const ggml_tensor * t) {
        fill(t, &node);
        for (int i = 0; i < 4; i++) {
            if (t->src[i] != nullptr) {
                fill(t->src[i], &src[i]);
                node.src[i] = &src[i];
            }
        }
    }

    static void fill(const ggml_tensor * t, lnsb_tensor * d) {
        std::memset(d, 0, sizeof *d);
        d->type = (int32_t) t->type;
        d->op   = op_of(t->op);
        for (int i = 0; i < 4; i++) {
            d->ne[i] = t->ne[i];
            d->nb[i] = (int64_t) t->nb[i];
        }
        static_assert(sizeof(t->op_params) >= sizeof(d->op_params), "op_params words");
        std::memcpy(d->op_params, t->op_params, sizeof d->op_params);
        if (t->op == GGML_OP_UNARY) d->op_params[0] = unary_of(ggml_get_unary_op(t));
        if (t->op == GGML_OP_GLU)   d->op_params[0] = glu_of(ggml_get_glu_op(t));
        d->flags = ((t->flags & GGML_TENSOR_FLAG_COMPUTE) ? LNSB_TENSOR_FLAG_COMPUTE : 0) |
                   (t->buffer != nullptr && ggml_backend_buffer_get_usage(t->buffer) == GGML_BACKEND_BUFFER_USAGE_WEIGHTS
                        ? LNSB_TENSOR_FLAG_WEIGHTS : 0);
        d->data = t->data;
        std::snprintf(d->name, sizeof d->name, "%s", t->name);
    }
};

// One registered device per format: LNSCUDA16 (xlns16, this build's
// summation mode) and LNSCUDA32 (xlns32), ACCEL devices on host buffers
// (lns-backend-framework.h:257-281), GUIDs ASCII "LNSCUDA16-bkend-" /
// "LNSCUDA32-bkend-" (ggml-lns-cuda.cpp:36-52).
template <int FMT>
struct backend {
    static const char * name() { return FMT == LNSB_XLNS16 ? "LNSCUDA16" : "LNSCUDA32"; }

    static ggml_guid_t guid() {
        static ggml_guid g = { 0x4c, 0x4e, 0x53, 0x43, 0x55, 0x44, 0x41, FMT == LNSB_XLNS16 ? 0x31 : 0x33,
                               FMT == LNSB_XLNS16 ? 0x36 : 0x32, 0x2d, 0x62, 0x6b, 0x65, 0x6e, 0x64, 0x2d };
        return &g;
    }

    static size_t device_count() {
        int n = 0;
        return cudaGetDeviceCount(&n) == cudaSuccess && n > 0 ? 1 : 0;
    }

    // ---- backend

    static const char * get_name(ggml_backend_t) { return name(); }
    static void free_backend(ggml_backend_t b) {
        lnsb_graph_ctx_destroy(static_cast<lnsb_graph_ctx *>(b->context));
        delete b;
    }
    static ggml_status graph_compute(ggml_backend_t b, ggml_cgraph * g) {
        std::vector<node_desc> descs;
        descs.reserve((size_t) g->n_nodes);
        for (int i = 0; i < g->n_nodes; i++) descs.emplace_back(g->nodes[i]);
        std::vector<lnsb_tensor *> nodes;
        for (node_desc & d : descs) nodes.push_back(&d.node);
        int failed = -1;
        const int st = lnsb_graph_compute(static_cast<lnsb_graph_ctx *>(b->context), nodes.data(), (int) nodes.size(), &failed);
        if (st != 0) {
            GGML_ABORT("%s: %s at node %d (%s): %s\n", name(), lnsb_error_string(st), failed,
                       failed >= 0 ? ggml_op_desc(g->nodes[failed]) : "-", failed >= 0 ? g->nodes[failed]->name : "");
        }
        return GGML_STATUS_SUCCESS;
    }
    static ggml_backend_i backend_iface() {
        ggml_backend_i i;
        std::memset(&i, 0, sizeof i);
        i.get_name      = get_name;
        i.free          = free_backend;
        i.graph_compute = graph_compute;
        return i;
    }

    // ---- device

    static const char * dev_name(ggml_backend_dev_t) { return name(); }
    static const char * dev_description(ggml_backend_dev_t) { return lnsb_device_description(FMT); }
    static void dev_memory(ggml_backend_dev_t, size_t * free_b, size_t * total_b) {
        if (cudaMemGetInfo(free_b, total_b) != cudaSuccess) { *free_b = 0; *total_b = 0; }
    }
    static enum ggml_backend_dev_type dev_type(ggml_backend_dev_t) { return GGML_BACKEND_DEVICE_TYPE_ACCEL; }
    static void dev_props(ggml_backend_dev_t d, ggml_backend_dev_props * p) {
        p->name        = dev_name(d);
        p->description = dev_description(d);
        p->type        = dev_type(d);
        p->device_id   = nullptr;
        dev_memory(d, &p->memory_free, &p->memory_total);
        p->caps.async                = false;
        p->caps.host_buffer          = false;
        p->caps.buffer_from_host_ptr = true;
        p->caps.events               = false;
    }
    static ggml_backend_t init() {
        if (device_count() == 0) return nullptr;
        lnsb_graph_ctx * ctx = lnsb_graph_ctx_create(FMT, -1, nullptr);
        if (ctx == nullptr) return nullptr;
        static ggml_backend_i iface = backend_iface();
        return new ggml_backend{ guid(), iface, device(), ctx };
    }
    static ggml_backend_t dev_init(ggml_backend_dev_t, const char *) { return init(); }
    static ggml_backend_buffer_type_t dev_buft(ggml_backend_dev_t) { return ggml_backend_cpu_buffer_type(); }
    static ggml_backend_buffer_t dev_from_host_ptr(ggml_backend_dev_t, void * ptr, size_t size, size_t) {
        return ggml_backend_cpu_buffer_from_ptr(ptr, size);
    }
    static bool dev_supports_op(ggml_backend_dev_t, const ggml_tensor * t) {
        node_desc d(t);
        return lnsb_supports_op(name(), FMT, &d.node) != 0;
    }
    static bool dev_supports_buft(ggml_backend_dev_t, ggml_backend_buffer_type_t b) { return ggml_backend_buft_is_host(b); }
    static bool dev_offload_op(ggml_backend_dev_t d, const ggml_tensor * t) { return dev_supports_op(d, t); }
    static ggml_backend_dev_t device() {
        static ggml_backend_device_i iface = [] {
            ggml_backend_device_i i;
            std::memset(&i, 0, sizeof i);
            i.get_name             = dev_name;
            i.get_description      = dev_description;
            i.get_memory           = dev_memory;
            i.get_type             = dev_type;
            i.get_props            = dev_props;
            i.init_backend         = dev_init;
            i.get_buffer_type      = dev_buft;
            i.buffer_from_host_ptr = dev_from_host_ptr;
            i.supports_op          = dev_supports_op;
            i.supports_buft        = dev_supports_buft;
            i.offload_op           = dev_offload_op;
            return i;
        }();
        static ggml_backend_device dev = { iface, reg(), nullptr };
        return &dev;
    }

    // ---- registry

    static const char * reg_name(ggml_backend_reg_t) { return name(); }
    static size_t reg_count(ggml_backend_reg_t) { return device_count(); }
    static ggml_backend_dev_t reg_device(ggml_backend_reg_t, size_t index) {
        GGML_ASSERT(index < device_count());
        return device();
    }
    static void * reg_proc(ggml_backend_reg_t, const char *) { return nullptr; }
    static ggml_backend_reg_t reg() {
        static ggml_backend_reg_i iface = [] {
            ggml_backend_reg_i i;
            std::memset(&i, 0, sizeof i);
            i.get_name         = reg_name;
            i.get_device_count = reg_count;
            i.get_device       = reg_device;
            i.get_proc_address = reg_proc;
            return i;
        }();
        static ggml_backend_reg r = { GGML_BACKEND_API_VERSION, iface, nullptr };
        return &r;
    }
    static bool is(ggml_backend_t b) { return b != nullptr && ggml_guid_matches(b->guid, guid()); }
};

}  // namespace lnsb200_ggml

// The registration entry points of include/ggml-lns-cuda.h (reference
// lns-backend/include/ggml-lns-cuda.h:19-23), defined in the one translation
// unit that includes this header.
inline ggml_backend_t ggml_backend_lns_cuda16_init(void) { return lnsb200_ggml::backend<LNSB_XLNS16>::init(); }
inline ggml_backend_t ggml_backend_lns_cuda32_init(void) { return lnsb200_ggml::backend<LNSB_XLNS32>::init(); }
inline ggml_backend_reg_t ggml_backend_lns_cuda16_reg(void) { return lnsb200_ggml::backend<LNSB_XLNS16>::reg(); }
inline ggml_backend_reg_t ggml_backend_lns_cuda32_reg(void) { return lnsb200_ggml::backend<LNSB_XLNS32>::reg(); }
inline bool ggml_backend_is_lns_cuda(ggml_backend_t b) {
    return lnsb200_ggml::backend<LNSB_XLNS16>::is(b) || lnsb200_ggml::backend<LNSB_XLNS32>::is(b);
}

#endif  // LNSB200_HAVE_GGML
