// Minimal stand-in for the reference's internal header, just enough to compile its
// gt_flash_attention (csrc/gt_ops_nn.cpp:2423-2525) on its own as a CPU checker -- TEST
// INFRASTRUCTURE ONLY, used by oracle/build_ref.py to build oracle/_ref/.
//
// The reference's header (csrc/gt_internal.h) pulls in ggml from a llama.cpp tree that its build
// downloads; the attention loop itself needs none of ggml. It needs a tensor record with ndim /
// shape / dtype / device fields (gt_internal.h:60-70), the error setter, an allocator for the
// output, the host-view and contiguous-owner helpers (gt_internal.h:330-351; here every tensor is
// already a contiguous host array, so they hand back its pointer) and the element readers and
// writers (gt_internal.h:243-300: float64 in and out, f16 / bf16 stored with round-to-nearest-even).
// The field and helper names are the reference's so that its function compiles unchanged; the
// bodies are written for this shim.
#pragma once

#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <string>
#include <vector>

enum { GT_F32 = 0, GT_F16 = 1, GT_BF16 = 2, GT_F64 = 3, GT_I32 = 7, GT_BOOL = 9 };
enum { GT_DEV_CPU = 0 };
#define GT_MAX_DIMS 12

struct gt_tensor {
    int ndim = 0;
    int64_t shape[GT_MAX_DIMS] = {};
    int64_t strides[GT_MAX_DIMS] = {};
    int64_t offset = 0;
    int64_t numel = 1;
    int dtype = GT_F32;
    int device_type = GT_DEV_CPU;
    int device_index = 0;
    void* data = nullptr;  // contiguous host elements
    bool owns = false;
};

// the message of the last failure on this thread
inline std::string& shim_error() {
    thread_local std::string e;
    return e;
}
inline void gt_set_error(const std::string& m) { shim_error() = m; }

inline size_t shim_elem_size(int dt) {
    switch (dt) {
        case GT_F64: return 8;
        case GT_F32: case GT_I32: return 4;
        case GT_F16: case GT_BF16: return 2;
        case GT_BOOL: return 1;
        default: return 0;
    }
}

inline gt_tensor* gt_tensor_empty(int ndim, const int64_t* shape, int dtype, int device_type, int device_index) {
    gt_tensor* t = new gt_tensor();
    t->ndim = ndim;
    t->dtype = dtype;
    t->device_type = device_type;
    t->device_index = device_index;
    t->numel = 1;
    for (int i = ndim - 1; i >= 0; --i) {
        t->shape[i] = shape[i];
        t->strides[i] = t->numel;
        t->numel *= shape[i];
    }
    t->data = std::calloc((size_t)(t->numel > 0 ? t->numel : 1), shim_elem_size(dtype));
    t->owns = true;
    return t;
}

inline void gt_tensor_free(gt_tensor* t) {
    if (!t) return;
    if (t->owns) std::free(t->data);
    delete t;
}

struct gt_contig_owner {
    const gt_tensor* ptr = nullptr;
    explicit gt_contig_owner(const gt_tensor* t) : ptr(t) {}
};

struct gt_host_view {
    const void* read(const gt_tensor* t) { return t->data; }
    void* write_empty(gt_tensor* t) { return t->data; }
    void commit(gt_tensor*) {}
};

// IEEE binary16 / bfloat16 <-> float, round to nearest even (the storage rules of the
// reference's element writers)
inline float shim_f16_to_f32(uint16_t h) {
    _Float16 v;
    std::memcpy(&v, &h, 2);
    return (float)v;
}
inline uint16_t shim_f32_to_f16(float f) {
    _Float16 v = (_Float16)f;
    uint16_t h;
    std::memcpy(&h, &v, 2);
    return h;
}
inline float shim_bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}
inline uint16_t shim_f32_to_bf16(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 64);  // quiet NaN
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

inline double gt_read_f64_at(const void* p, int dt, int64_t i) {
    switch (dt) {
        case GT_F64: return ((const double*)p)[i];
        case GT_F32: return (double)((const float*)p)[i];
        case GT_F16: return (double)shim_f16_to_f32(((const uint16_t*)p)[i]);
        case GT_BF16: return (double)shim_bf16_to_f32(((const uint16_t*)p)[i]);
        case GT_I32: return (double)((const int32_t*)p)[i];
        case GT_BOOL: return ((const uint8_t*)p)[i] ? 1.0 : 0.0;
        default: return 0.0;
    }
}

inline int64_t gt_read_i64_at(const void* p, int dt, int64_t i) {
    if (dt == GT_BOOL) return ((const uint8_t*)p)[i] ? 1 : 0;
    if (dt == GT_I32) return ((const int32_t*)p)[i];
    return (int64_t)gt_read_f64_at(p, dt, i);
}

inline void gt_write_f64_at(void* p, int dt, int64_t i, double v) {
    switch (dt) {
        case GT_F64: ((double*)p)[i] = v; break;
        case GT_F32: ((float*)p)[i] = (float)v; break;
        case GT_F16: ((uint16_t*)p)[i] = shim_f32_to_f16((float)v); break;
        case GT_BF16: ((uint16_t*)p)[i] = shim_f32_to_bf16((float)v); break;
        default: break;
    }
}
