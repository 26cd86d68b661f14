// Handle runtime of the attention engine (include/gguf_train_attn.h): gt_tensor storage on the host
// or on a CUDA device, views, copies, seeded fills, and the reference-shaped attention exports.
//
// Layout semantics follow the reference's gt_tensor (csrc/gt_internal.h:60-70): shape, element
// strides and an element offset over a shared storage; views share the storage. Storage here is
// plain malloc / cudaMalloc memory instead of ggml backend buffers (gt_core.cpp:457-518).

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <random>
#include <string>
#include <vector>

#include "../../include/gguf_train_attn.h"
#include "../../include/gtb_attn.h"
#include "gt_copy.h"
#include "q8_0_internal.h"

namespace gtb {
void set_error(const std::string& msg);
void set_errorf(const char* fmt, ...);
const char* last_error();
void clear_error();
bool cuda_failed(cudaError_t e, const char* what);
}  // namespace gtb

using gtb::set_error;
using gtb::set_errorf;

struct gt_storage {
    void* ptr = nullptr;
    size_t nbytes = 0;
    int device_type = GT_DEV_CPU;
    int device_index = 0;
    bool owned = true;
    ~gt_storage() {
        if (!owned || !ptr) return;
        if (device_type == GT_DEV_CUDA) {
            int prev = 0;
            cudaGetDevice(&prev);
            cudaSetDevice(device_index);
            cudaFree(ptr);
            cudaSetDevice(prev);
        } else {
            std::free(ptr);
        }
    }
};

struct gt_tensor {
    int ndim = 0;
    int64_t shape[GT_MAX_DIMS] = {};
    int64_t strides[GT_MAX_DIMS] = {};
    int64_t offset = 0;
    int64_t numel = 1;
    int dtype = GT_F32;
    int device_type = GT_DEV_CPU;
    int device_index = 0;
    std::shared_ptr<gt_storage> storage;
};

namespace {

std::mutex g_rng_mtx;
std::mt19937_64 g_rng;

bool is_q8(int dt) { return dt == GT_Q8_0; }

size_t elem_size(int dt) {
    switch (dt) {
        case GT_F32: return 4;
        case GT_F16: return 2;
        case GT_BF16: return 2;
        case GT_F64: return 8;
        case GT_I8: return 1;
        case GT_U8: return 1;
        case GT_I16: return 2;
        case GT_I32: return 4;
        case GT_I64: return 8;
        case GT_BOOL: return 1;
        default: return 0;
    }
}

// bytes of n elements of dtype (Q8_0: 34 bytes per 32 values)
size_t bytes_for(int dt, int64_t n) {
    if (is_q8(dt)) return (size_t)(n / 32) * 34;
    return elem_size(dt) * (size_t)n;
}

bool valid_dtype(int dt) { return elem_size(dt) > 0 || is_q8(dt); }

bool fill_meta(gt_tensor* t, int ndim, const int64_t* shape, int dtype) {
    if (ndim < 0 || ndim > GT_MAX_DIMS) {
        set_errorf("tensor: ndim %d outside [0, %d]", ndim, GT_MAX_DIMS);
        return false;
    }
    if (!valid_dtype(dtype)) {
        set_errorf("tensor: unsupported dtype %d", dtype);
        return false;
    }
    t->ndim = ndim;
    t->dtype = dtype;
    t->numel = 1;
    for (int i = 0; i < ndim; ++i) {
        if (shape[i] < 0) {
            set_error("tensor: negative dimension");
            return false;
        }
        t->shape[i] = shape[i];
        t->numel *= shape[i];
    }
    int64_t st = 1;
    for (int i = ndim - 1; i >= 0; --i) {
        t->strides[i] = st;
        st *= std::max<int64_t>(shape[i], 1);
    }
    if (is_q8(dtype) && (t->numel % 32 != 0)) {
        set_error("Tensor size must be a multiple of ggml quantization block size");
        return false;
    }
    return true;
}

bool contiguous(const gt_tensor* t) {
    int64_t st = 1;
    for (int i = t->ndim - 1; i >= 0; --i) {
        if (t->shape[i] != 1 && t->strides[i] != st) return false;
        st *= t->shape[i];
    }
    return true;
}

char* data_of(const gt_tensor* t) {
    if (!t->storage || !t->storage->ptr) return nullptr;
    return (char*)t->storage->ptr + bytes_for(t->dtype, t->offset);
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

gt_tensor* alloc_tensor(int ndim, const int64_t* shape, int dtype, int device_type, int device_index) {
    auto* t = new gt_tensor();
    if (!fill_meta(t, ndim, shape, dtype)) {
        delete t;
        return nullptr;
    }
    if (device_type != GT_DEV_CPU && device_type != GT_DEV_CUDA) {
        set_errorf("tensor: unsupported device type %d", device_type);
        delete t;
        return nullptr;
    }
    t->device_type = device_type;
    t->device_index = device_type == GT_DEV_CUDA ? device_index : 0;
    auto st = std::make_shared<gt_storage>();
    st->device_type = t->device_type;
    st->device_index = t->device_index;
    st->nbytes = bytes_for(dtype, t->numel);
    const size_t alloc = std::max<size_t>(st->nbytes, 16);
    if (device_type == GT_DEV_CUDA) {
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess || device_index < 0 || device_index >= n) {
            cudaGetLastError();
            set_errorf("tensor: cuda:%d is not available", device_index);
            delete t;
            return nullptr;
        }
        DeviceGuard g(device_index);
        if (gtb::cuda_failed(cudaMalloc(&st->ptr, alloc), "tensor: cudaMalloc")) {
            delete t;
            return nullptr;
        }
    } else {
        st->ptr = std::aligned_alloc(64, (alloc + 63) / 64 * 64);
        if (!st->ptr) {
            set_error("tensor: out of host memory");
            delete t;
            return nullptr;
        }
    }
    t->storage = st;
    return t;
}

// copy the logical elements of t into contiguous host memory
bool read_contiguous(const gt_tensor* t, void* dst) {
    const size_t nb = bytes_for(t->dtype, t->numel);
    if (nb == 0) return true;
    if (t->device_type == GT_DEV_CUDA) {
        DeviceGuard g(t->device_index);
        if (contiguous(t)) {
            if (gtb::cuda_failed(cudaMemcpy(dst, data_of(t), nb, cudaMemcpyDeviceToHost), "copy_to_host")) return false;
            return true;
        }
        if (is_q8(t->dtype)) {
            set_error("copy_to_host: a Q8_0 tensor must be contiguous");
            return false;
        }
        void* tmp = nullptr;
        if (gtb::cuda_failed(cudaMalloc(&tmp, nb), "copy_to_host: cudaMalloc")) return false;
        int rc = gtb::launch_gather(tmp, data_of(t), t->ndim, t->shape, t->strides, elem_size(t->dtype), t->numel, 0);
        if (rc == 0 && gtb::cuda_failed(cudaMemcpy(dst, tmp, nb, cudaMemcpyDeviceToHost), "copy_to_host")) rc = -1;
        cudaFree(tmp);
        return rc == 0;
    }
    if (contiguous(t)) {
        std::memcpy(dst, data_of(t), nb);
        return true;
    }
    const size_t es = elem_size(t->dtype);
    const char* src = data_of(t);
    for (int64_t i = 0; i < t->numel; ++i) {
        int64_t rem = i, off = 0;
        for (int d = t->ndim - 1; d >= 0; --d) {
            off += (rem % t->shape[d]) * t->strides[d];
            rem /= t->shape[d];
        }
        std::memcpy((char*)dst + i * es, src + off * es, es);
    }
    return true;
}

// host value conversions for seeded fills (the reference stores through float: gt_internal.h:261-277)
uint16_t f32_to_bf16_bits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

uint16_t f32_to_f16_bits(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);
    if (ax < 0x38800000u) {
        float a;
        std::memcpy(&a, &ax, 4);
        return (uint16_t)(sign | (uint32_t)std::nearbyint((double)a * 16777216.0));
    }
    uint32_t h = ((((ax >> 23) - 112u)) << 10) | ((ax & 0x7fffffu) >> 13);
    const uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1;
    return (uint16_t)(sign | h);
}

bool store_values(int dtype, const std::vector<double>& v, std::vector<unsigned char>& out) {
    const size_t es = elem_size(dtype);
    out.resize(es * v.size());
    for (size_t i = 0; i < v.size(); ++i) {
        unsigned char* p = out.data() + i * es;
        switch (dtype) {
            case GT_F32: { float f = (float)v[i]; std::memcpy(p, &f, 4); break; }
            case GT_F64: std::memcpy(p, &v[i], 8); break;
            case GT_F16: { uint16_t h = f32_to_f16_bits((float)v[i]); std::memcpy(p, &h, 2); break; }
            case GT_BF16: { uint16_t h = f32_to_bf16_bits((float)v[i]); std::memcpy(p, &h, 2); break; }
            case GT_BOOL: *p = v[i] != 0.0; break;
            case GT_I32: { int32_t x = (int32_t)v[i]; std::memcpy(p, &x, 4); break; }
            case GT_I64: { int64_t x = (int64_t)v[i]; std::memcpy(p, &x, 8); break; }
            default: set_error("fill: unsupported dtype"); return false;
        }
    }
    return true;
}

// write contiguous values (row-major over the logical shape) into t, strided or not
bool write_values(gt_tensor* t, const void* src) {
    const size_t nb = bytes_for(t->dtype, t->numel);
    if (nb == 0) return true;
    if (!contiguous(t)) {
        set_error("fill: the tensor must be contiguous");
        return false;
    }
    if (t->device_type == GT_DEV_CUDA) {
        DeviceGuard g(t->device_index);
        return !gtb::cuda_failed(cudaMemcpy(data_of(t), src, nb, cudaMemcpyHostToDevice), "copy_from_host");
    }
    std::memcpy(data_of(t), src, nb);
    return true;
}

template <typename Dist>
int fill_with(gt_tensor* t, Dist&& draw) {
    if (!t) return -1;
    if (t->numel == 0) return 0;
    std::vector<double> v((size_t)t->numel);
    {
        std::lock_guard<std::mutex> lk(g_rng_mtx);
        for (auto& x : v) x = draw();
    }
    std::vector<unsigned char> bytes;
    if (!store_values(t->dtype, v, bytes)) return -1;
    return write_values(t, bytes.data()) ? 0 : -1;
}

// ---- attention plumbing

bool as_t4(const gt_tensor* t, const char* ctx, const char* name, gtb_tensor4& out) {
    if (!t) {
        set_errorf("%s: %s is NULL", ctx, name);
        return false;
    }
    if (t->ndim != 4) {
        set_errorf("%s expects 4D q, k, v tensors (B, H, L, D)", ctx);
        return false;
    }
    if (t->device_type != GT_DEV_CUDA) {
        set_errorf("%s: %s is a CPU tensor; this engine runs CUDA tensors only (move it with .to('cuda'))", ctx, name);
        return false;
    }
    out.data = data_of(t);
    for (int i = 0; i < 4; ++i) {
        out.shape[i] = t->shape[i];
        out.stride[i] = t->strides[i];
    }
    out.dtype = t->dtype;
    return true;
}

// mask of the reference: 2-D (L|1, S|1) or 4-D (B|1, H|1, L|1, S|1) (gt_ops_nn.cpp:2437-2454)
bool mask_t4(const gt_tensor* m, const int64_t want[4], const char* ctx, gtb_tensor4& out) {
    bool fits = m->ndim == 2 || m->ndim == 4;
    for (int i = 0; fits && i < m->ndim; ++i) {
        const int64_t s = m->shape[i];
        fits = (s == 1 || s == want[4 - m->ndim + i]);
    }
    if (!fits) {
        std::string shape = "[";
        for (int i = 0; i < m->ndim; ++i) shape += (i ? ", " : "") + std::to_string(m->shape[i]);
        set_errorf("%s: attn_mask of shape %s] cannot be broadcast to the attention weights [%lld, %lld, %lld, %lld]",
                   ctx, shape.c_str(), (long long)want[0], (long long)want[1], (long long)want[2], (long long)want[3]);
        return false;
    }
    if (m->device_type != GT_DEV_CUDA) {
        set_errorf("%s: attn_mask is a CPU tensor; this engine runs CUDA tensors only", ctx);
        return false;
    }
    out.data = data_of(m);
    out.dtype = m->dtype;
    const int lead = 4 - m->ndim;
    for (int i = 0; i < 4; ++i) {
        out.shape[i] = i < lead ? 1 : m->shape[i - lead];
        out.stride[i] = i < lead ? 0 : m->strides[i - lead];
    }
    return true;
}

bool same_device(const gt_tensor* a, const gt_tensor* b, const char* ctx) {
    if (a && b && (a->device_type != b->device_type || a->device_index != b->device_index)) {
        set_errorf("%s: all tensors must be on the same device", ctx);
        return false;
    }
    return true;
}

gtb_tensor4 t4_of(gt_tensor* t) {
    gtb_tensor4 r;
    r.data = data_of(t);
    for (int i = 0; i < 4; ++i) {
        r.shape[i] = t->shape[i];
        r.stride[i] = t->strides[i];
    }
    r.dtype = t->dtype;
    return r;
}

gt_tensor* attention_forward(const gt_tensor* q, const gt_tensor* k, const gt_tensor* v, const gt_tensor* mask,
                             float scale, int is_causal, gt_tensor** lse_out) {
    const char* ctx = "flash_attention";
    gtb_tensor4 tq, tk, tv, tm;
    if (!as_t4(q, ctx, "q", tq) || !as_t4(k, ctx, "k", tk) || !as_t4(v, ctx, "v", tv)) return nullptr;
    if (!same_device(q, k, ctx) || !same_device(q, v, ctx) || !same_device(q, mask, ctx)) return nullptr;
    const int64_t want[4] = {q->shape[0], q->shape[1], q->shape[2], k->shape[2]};
    if (mask && !mask_t4(mask, want, ctx, tm)) return nullptr;
    DeviceGuard g(q->device_index);
    const int64_t osh[4] = {q->shape[0], q->shape[1], q->shape[2], v->shape[3]};
    gt_tensor* out = alloc_tensor(4, osh, q->dtype, GT_DEV_CUDA, q->device_index);
    if (!out) return nullptr;
    gt_tensor* lse = nullptr;
    if (lse_out) {
        lse = alloc_tensor(3, osh, q->dtype == GT_F64 ? GT_F64 : GT_F32, GT_DEV_CUDA, q->device_index);
        if (!lse) {
            gt_tensor_free(out);
            return nullptr;
        }
    }
    gtb_tensor4 to = t4_of(out);
    if (gtb_sdpa_fwd(&tq, &tk, &tv, mask ? &tm : nullptr, scale, is_causal, &to, lse ? (void*)data_of(lse) : nullptr,
                     nullptr) != 0) {
        gt_tensor_free(out);
        if (lse) gt_tensor_free(lse);
        return nullptr;
    }
    if (lse_out) *lse_out = lse;
    return out;
}

}  // namespace

extern "C" {

GT_API const char* gt_last_error(void) { return gtb::last_error(); }
GT_API void gt_clear_error(void) { gtb::clear_error(); }

GT_API void gt_manual_seed(uint64_t seed) {
    std::lock_guard<std::mutex> lk(g_rng_mtx);
    g_rng.seed(seed);
}

GT_API int gt_device_count(int device_type) {
    if (device_type == GT_DEV_CPU) return 1;
    if (device_type != GT_DEV_CUDA) return 0;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

GT_API void gt_device_name(int device_type, int idx, char* buf, int buf_len) {
    if (!buf || buf_len <= 0) return;
    buf[0] = 0;
    if (device_type == GT_DEV_CPU) {
        std::snprintf(buf, (size_t)buf_len, "cpu");
        return;
    }
    cudaDeviceProp prop;
    if (device_type == GT_DEV_CUDA && cudaGetDeviceProperties(&prop, idx) == cudaSuccess)
        std::snprintf(buf, (size_t)buf_len, "%s", prop.name);
    else
        cudaGetLastError();
}

GT_API void gt_device_memory(int device_type, int idx, size_t* free_bytes, size_t* total_bytes) {
    size_t f = 0, t = 0;
    if (device_type == GT_DEV_CUDA) {
        DeviceGuard g(idx);
        if (cudaMemGetInfo(&f, &t) != cudaSuccess) cudaGetLastError();
    }
    if (free_bytes) *free_bytes = f;
    if (total_bytes) *total_bytes = t;
}

GT_API void gt_synchronize(int device_type, int idx) {
    if (device_type != GT_DEV_CUDA) return;
    DeviceGuard g(idx);
    gtb::cuda_failed(cudaDeviceSynchronize(), "synchronize");
}

GT_API gt_tensor* gt_tensor_empty(int ndim, const int64_t* shape, int dtype, int device_type, int device_index) {
    return alloc_tensor(ndim, shape, dtype, device_type, device_index);
}

GT_API gt_tensor* gt_tensor_from_data(int ndim, const int64_t* shape, int dtype, int device_type, int device_index,
                                      const void* data, size_t nbytes) {
    gt_tensor* t = alloc_tensor(ndim, shape, dtype, device_type, device_index);
    if (!t) return nullptr;
    const size_t need = bytes_for(dtype, t->numel);
    if (need && (!data || nbytes < need)) {
        set_errorf("from_data: %zu bytes given, %zu needed", nbytes, need);
        gt_tensor_free(t);
        return nullptr;
    }
    if (need && !write_values(t, data)) {
        gt_tensor_free(t);
        return nullptr;
    }
    return t;
}

GT_API gt_tensor* gt_tensor_from_external(int ndim, const int64_t* shape, const int64_t* strides, int dtype, void* data,
                                          uint64_t token) {
    (void)token;
    auto* t = new gt_tensor();
    if (!fill_meta(t, ndim, shape, dtype)) {
        delete t;
        return nullptr;
    }
    if (strides) {
        for (int i = 0; i < ndim; ++i) {
            if (strides[i] < 0) {
                set_error("from_external: negative strides are not supported");
                delete t;
                return nullptr;
            }
            t->strides[i] = strides[i];
        }
    }
    auto st = std::make_shared<gt_storage>();
    st->ptr = data;
    st->owned = false;
    cudaPointerAttributes attr;
    if (data && cudaPointerGetAttributes(&attr, data) == cudaSuccess && attr.type == cudaMemoryTypeDevice) {
        st->device_type = GT_DEV_CUDA;
        st->device_index = attr.device;
    } else {
        cudaGetLastError();
    }
    t->device_type = st->device_type;
    t->device_index = st->device_index;
    t->storage = st;
    return t;
}

GT_API gt_tensor* gt_tensor_view(const gt_tensor* t, int ndim, const int64_t* shape, const int64_t* strides,
                                 int64_t offset) {
    if (!t) return nullptr;
    if (ndim < 0 || ndim > GT_MAX_DIMS) {
        set_error("view: bad ndim");
        return nullptr;
    }
    auto* r = new gt_tensor(*t);
    r->ndim = ndim;
    r->numel = 1;
    for (int i = 0; i < ndim; ++i) {
        r->shape[i] = shape[i];
        r->strides[i] = strides[i];
        r->numel *= shape[i];
    }
    r->offset = offset;
    return r;
}

GT_API gt_tensor* gt_tensor_contiguous(const gt_tensor* t) {
    if (!t) return nullptr;
    gt_tensor* r = alloc_tensor(t->ndim, t->shape, t->dtype, t->device_type, t->device_index);
    if (!r) return nullptr;
    const size_t nb = bytes_for(t->dtype, t->numel);
    if (nb == 0) return r;
    if (t->device_type == GT_DEV_CUDA) {
        DeviceGuard g(t->device_index);
        int rc;
        if (contiguous(t))
            rc = gtb::cuda_failed(cudaMemcpy(data_of(r), data_of(t), nb, cudaMemcpyDeviceToDevice), "contiguous") ? -1 : 0;
        else if (is_q8(t->dtype)) {
            set_error("contiguous: a Q8_0 tensor cannot be a strided view");
            rc = -1;
        } else
            rc = gtb::launch_gather(data_of(r), data_of(t), t->ndim, t->shape, t->strides, elem_size(t->dtype), t->numel, 0);
        if (rc != 0) {
            gt_tensor_free(r);
            return nullptr;
        }
        return r;
    }
    if (!read_contiguous(t, data_of(r))) {
        gt_tensor_free(r);
        return nullptr;
    }
    return r;
}

GT_API gt_tensor* gt_tensor_clone(const gt_tensor* t) { return gt_tensor_contiguous(t); }

GT_API gt_tensor* gt_tensor_to_device(const gt_tensor* t, int device_type, int device_index) {
    if (!t) return nullptr;
    gt_tensor* r = alloc_tensor(t->ndim, t->shape, t->dtype, device_type, device_index);
    if (!r) return nullptr;
    const size_t nb = bytes_for(t->dtype, t->numel);
    if (nb == 0) return r;
    std::vector<unsigned char> host(nb);
    bool ok = read_contiguous(t, host.data());
    if (ok) ok = write_values(r, host.data());
    if (!ok) {
        gt_tensor_free(r);
        return nullptr;
    }
    return r;
}

GT_API gt_tensor* gt_quantize(const gt_tensor* t, int quant_dtype) {
    if (!t) return nullptr;
    if (!is_q8(quant_dtype)) {
        set_errorf("quantize: only Q8_0 (%d) is supported by this engine", GT_Q8_0);
        return nullptr;
    }
    if (t->device_type != GT_DEV_CUDA) {
        set_error("quantize: this engine quantises CUDA tensors only");
        return nullptr;
    }
    gt_tensor* c = contiguous(t) ? nullptr : gt_tensor_contiguous(t);
    const gt_tensor* src = c ? c : t;
    gt_tensor* r = alloc_tensor(t->ndim, t->shape, quant_dtype, GT_DEV_CUDA, t->device_index);
    int rc = -1;
    if (r) {
        DeviceGuard g(t->device_index);
        const int64_t row = t->ndim ? std::max<int64_t>(t->shape[t->ndim - 1], 1) : 1;
        rc = gtb_q8_0_quantize(data_of(src), src->dtype, t->numel / row, row, data_of(r), nullptr);
    }
    if (c) gt_tensor_free(c);
    if (rc != 0 && r) {
        gt_tensor_free(r);
        r = nullptr;
    }
    return r;
}

GT_API gt_tensor* gt_dequantize(const gt_tensor* t, int target_dtype) {
    if (!t) return nullptr;
    if (!is_q8(t->dtype)) {
        set_error("dequantize: the tensor is not Q8_0");
        return nullptr;
    }
    if (t->device_type != GT_DEV_CUDA) {
        set_error("dequantize: this engine dequantises CUDA tensors only");
        return nullptr;
    }
    gt_tensor* r = alloc_tensor(t->ndim, t->shape, target_dtype, GT_DEV_CUDA, t->device_index);
    if (!r) return nullptr;
    DeviceGuard g(t->device_index);
    const int64_t row = t->ndim ? std::max<int64_t>(t->shape[t->ndim - 1], 1) : 1;
    if (gtb_q8_0_dequantize(data_of(t), t->numel / row, row, data_of(r), target_dtype, nullptr) != 0) {
        gt_tensor_free(r);
        return nullptr;
    }
    return r;
}

GT_API gt_tensor* gt_tensor_to_dtype(const gt_tensor* t, int dtype) {
    if (!t) return nullptr;
    if (t->dtype == dtype) return gt_tensor_contiguous(t);
    if (is_q8(dtype)) return gt_quantize(t, dtype);
    if (is_q8(t->dtype)) return gt_dequantize(t, dtype);
    if (t->device_type != GT_DEV_CUDA) {
        set_error("to_dtype: this engine converts CUDA tensors only");
        return nullptr;
    }
    gt_tensor* c = contiguous(t) ? nullptr : gt_tensor_contiguous(t);
    const gt_tensor* src = c ? c : t;
    gt_tensor* r = alloc_tensor(t->ndim, t->shape, dtype, GT_DEV_CUDA, t->device_index);
    int rc = -1;
    if (r) {
        DeviceGuard g(t->device_index);
        rc = gtb::launch_convert(data_of(r), dtype, data_of(src), src->dtype, t->numel, 0);
    }
    if (c) gt_tensor_free(c);
    if (rc != 0 && r) {
        gt_tensor_free(r);
        r = nullptr;
    }
    return r;
}

GT_API void gt_tensor_free(gt_tensor* t) { delete t; }

GT_API int gt_tensor_ndim(const gt_tensor* t) { return t ? t->ndim : -1; }
GT_API void gt_tensor_shape(const gt_tensor* t, int64_t* out) {
    if (t && out) std::memcpy(out, t->shape, sizeof(int64_t) * t->ndim);
}
GT_API void gt_tensor_strides(const gt_tensor* t, int64_t* out) {
    if (t && out) std::memcpy(out, t->strides, sizeof(int64_t) * t->ndim);
}
GT_API int64_t gt_tensor_offset(const gt_tensor* t) { return t ? t->offset : 0; }
GT_API int64_t gt_tensor_numel(const gt_tensor* t) { return t ? t->numel : 0; }
GT_API int gt_tensor_dtype(const gt_tensor* t) { return t ? t->dtype : -1; }
GT_API int gt_tensor_device_type(const gt_tensor* t) { return t ? t->device_type : -1; }
GT_API int gt_tensor_device_index(const gt_tensor* t) { return t ? t->device_index : -1; }
GT_API int gt_tensor_is_contiguous(const gt_tensor* t) { return t && contiguous(t) ? 1 : 0; }
GT_API uint64_t gt_tensor_data_ptr(const gt_tensor* t) { return t ? (uint64_t)(uintptr_t)data_of(t) : 0; }
GT_API size_t gt_tensor_nbytes(const gt_tensor* t) { return t ? bytes_for(t->dtype, t->numel) : 0; }
GT_API size_t gt_tensor_elem_size(int dtype) { return is_q8(dtype) ? 34 : elem_size(dtype); }

GT_API int gt_tensor_copy_to_host(const gt_tensor* t, void* dst, size_t dst_bytes) {
    if (!t || !dst) return -1;
    const size_t nb = bytes_for(t->dtype, t->numel);
    if (dst_bytes < nb) {
        set_errorf("copy_to_host: %zu bytes needed, %zu given", nb, dst_bytes);
        return -1;
    }
    return read_contiguous(t, dst) ? 0 : -1;
}

GT_API int gt_tensor_copy_from_host(gt_tensor* t, const void* src, size_t src_bytes) {
    if (!t || !src) return -1;
    const size_t nb = bytes_for(t->dtype, t->numel);
    if (src_bytes < nb) {
        set_errorf("copy_from_host: %zu bytes needed, %zu given", nb, src_bytes);
        return -1;
    }
    return write_values(t, src) ? 0 : -1;
}

GT_API int gt_fill_uniform(gt_tensor* t, double low, double high) {
    std::uniform_real_distribution<double> dist(low, high);
    return fill_with(t, [&] { return dist(g_rng); });
}

GT_API int gt_fill_normal(gt_tensor* t, double mean, double stdv) {
    std::normal_distribution<double> dist(mean, stdv > 0.0 ? stdv : 1e-30);
    return fill_with(t, [&] { return stdv == 0.0 ? mean : dist(g_rng); });
}

GT_API int gt_fill_bernoulli_prob(gt_tensor* t, double p) {
    std::bernoulli_distribution dist(std::min(1.0, std::max(0.0, p)));
    return fill_with(t, [&] { return dist(g_rng) ? 1.0 : 0.0; });
}

GT_API gt_tensor* gt_flash_attention(const gt_tensor* q, const gt_tensor* k, const gt_tensor* v, const gt_tensor* mask,
                                     float scale, int is_causal) {
    return attention_forward(q, k, v, mask, scale, is_causal, nullptr);
}

GT_API gt_tensor* gt_flash_attention_fwd_lse(const gt_tensor* q, const gt_tensor* k, const gt_tensor* v,
                                             const gt_tensor* mask, float scale, int is_causal, gt_tensor** lse_out) {
    if (!lse_out) {
        set_error("flash_attention_fwd_lse: lse_out is NULL");
        return nullptr;
    }
    return attention_forward(q, k, v, mask, scale, is_causal, lse_out);
}

GT_API int gt_flash_attention_backward(const gt_tensor* grad_out, const gt_tensor* q, const gt_tensor* k,
                                       const gt_tensor* v, const gt_tensor* mask, const gt_tensor* out,
                                       const gt_tensor* lse, float scale, int is_causal, gt_tensor** dq,
                                       gt_tensor** dk, gt_tensor** dv) {
    const char* ctx = "flash_attention_backward";
    gtb_tensor4 tg, tq, tk, tv, to, tm;
    if (!as_t4(grad_out, ctx, "grad_out", tg) || !as_t4(q, ctx, "q", tq) || !as_t4(k, ctx, "k", tk) ||
        !as_t4(v, ctx, "v", tv) || !as_t4(out, ctx, "out", to))
        return -1;
    if (!lse || lse->device_type != GT_DEV_CUDA || lse->dtype != (q->dtype == GT_F64 ? GT_F64 : GT_F32) || !contiguous(lse) ||
        lse->numel != q->shape[0] * q->shape[1] * q->shape[2]) {
        set_errorf("%s: lse must be the contiguous (B, H, L) CUDA tensor of the forward (f64 for f64 inputs, else f32)", ctx);
        return -1;
    }
    if (!dq || !dk || !dv) {
        set_errorf("%s: output pointers are NULL", ctx);
        return -1;
    }
    const int64_t want[4] = {q->shape[0], q->shape[1], q->shape[2], k->shape[2]};
    if (mask && !mask_t4(mask, want, ctx, tm)) return -1;
    DeviceGuard g(q->device_index);
    gt_tensor* gq = alloc_tensor(4, q->shape, q->dtype, GT_DEV_CUDA, q->device_index);
    gt_tensor* gk = alloc_tensor(4, k->shape, k->dtype, GT_DEV_CUDA, q->device_index);
    gt_tensor* gv = alloc_tensor(4, v->shape, v->dtype, GT_DEV_CUDA, q->device_index);
    if (!gq || !gk || !gv) {
        gt_tensor_free(gq); gt_tensor_free(gk); gt_tensor_free(gv);
        return -1;
    }
    gtb_tensor4 tdq = t4_of(gq), tdk = t4_of(gk), tdv = t4_of(gv);
    if (gtb_sdpa_bwd(&tg, &tq, &tk, &tv, mask ? &tm : nullptr, &to, (const void*)data_of(lse), scale, is_causal, &tdq,
                     &tdk, &tdv, nullptr) != 0) {
        gt_tensor_free(gq); gt_tensor_free(gk); gt_tensor_free(gv);
        return -1;
    }
    *dq = gq;
    *dk = gk;
    *dv = gv;
    return 0;
}

// a 1-D CUDA tensor of positions as contiguous int32 (values truncated toward zero), through the host:
// positions are one per sequence element, so this is a few KB at most
static gt_tensor* positions_i32(const gt_tensor* pos) {
    const int64_t n = pos->numel;
    std::vector<unsigned char> raw(bytes_for(pos->dtype, n));
    std::vector<int32_t> v((size_t)n);
    if (!raw.empty() && !read_contiguous(pos, raw.data())) return nullptr;
    for (int64_t i = 0; i < n; ++i) {
        const unsigned char* e = raw.data() + (size_t)i * elem_size(pos->dtype);
        double x;
        switch (pos->dtype) {
            case GT_F32: { float f; std::memcpy(&f, e, 4); x = f; break; }
            case GT_F64: std::memcpy(&x, e, 8); break;
            case GT_I32: { int32_t k; std::memcpy(&k, e, 4); x = k; break; }
            case GT_I64: { int64_t k; std::memcpy(&k, e, 8); x = (double)k; break; }
            default:
                set_error("rope: pos must be an integer or float32/float64 tensor");
                return nullptr;
        }
        v[(size_t)i] = (int32_t)x;
    }
    gt_tensor* r = alloc_tensor(1, &n, GT_I32, GT_DEV_CUDA, pos->device_index);
    if (r && n > 0 && gt_tensor_copy_from_host(r, v.data(), v.size() * 4) != 0) {
        gt_tensor_free(r);
        return nullptr;
    }
    return r;
}

// gt_rope / gt_rope_backward on CUDA tensors: x (B, H, S, D) or (H, S, D), pos 1-D with a position per
// sequence element (converted to int32 as the reference does, gt_ops_nn.cpp:2367-2371)
static gt_tensor* rope_handle(const gt_tensor* x, const gt_tensor* pos, int n_dims, int mode, float freq_base,
                              float freq_scale, int backward) {
    if (!x || !pos) {
        set_error("rope: x and pos are required");
        return nullptr;
    }
    if (x->ndim < 3 || x->ndim > 4) {
        std::string sh = "[";
        for (int i = 0; i < x->ndim; ++i) sh += (i ? ", " : "") + std::to_string(x->shape[i]);
        set_errorf("rope: expected x of shape (batch, heads, seq_len, head_dim) or (heads, seq_len, head_dim), got %s]",
                   sh.c_str());
        return nullptr;
    }
    if (x->device_type != GT_DEV_CUDA || pos->device_type != GT_DEV_CUDA) {
        set_error("rope: this engine runs CUDA tensors only (move x and pos with .to('cuda'))");
        return nullptr;
    }
    if (pos->ndim != 1) {
        set_errorf("rope: pos must be a 1-D tensor with a position for each of the %lld sequence elements",
                   (long long)x->shape[x->ndim - 2]);
        return nullptr;
    }
    const bool four = x->ndim == 4;
    const int64_t B = four ? x->shape[0] : 1, H = x->shape[four ? 1 : 0], S = x->shape[four ? 2 : 1],
                  D = x->shape[four ? 3 : 2];
    gt_tensor* xc = contiguous(x) ? nullptr : gt_tensor_contiguous(x);
    gt_tensor* pc = (pos->dtype == GT_I32 && contiguous(pos)) ? nullptr : positions_i32(pos);
    const gt_tensor* xs = xc ? xc : x;
    const gt_tensor* ps = pc ? pc : pos;
    gt_tensor* out = (xs && ps) ? alloc_tensor(x->ndim, x->shape, x->dtype, GT_DEV_CUDA, x->device_index) : nullptr;
    int rc = -1;
    if (out) {
        DeviceGuard g(x->device_index);
        rc = gtb_rope(data_of(xs), xs->dtype, B, H, S, D, (const int32_t*)data_of(ps), ps->shape[0], n_dims, mode,
                      freq_base, freq_scale, backward, data_of(out), nullptr);
    }
    if (xc) gt_tensor_free(xc);
    if (pc) gt_tensor_free(pc);
    if (rc != 0) {
        if (out) gt_tensor_free(out);
        return nullptr;
    }
    return out;
}

GT_API gt_tensor* gt_rope(const gt_tensor* x, const gt_tensor* pos, int n_dims, int mode, int n_ctx_orig, float freq_base,
                          float freq_scale) {
    (void)n_ctx_orig;  // only read by ggml when ext_factor != 0, which the reference never passes
    return rope_handle(x, pos, n_dims, mode, freq_base, freq_scale, 0);
}

GT_API gt_tensor* gt_rope_backward(const gt_tensor* grad_out, const gt_tensor* pos, int n_dims, int mode, int n_ctx_orig,
                                   float freq_base, float freq_scale) {
    (void)n_ctx_orig;
    return rope_handle(grad_out, pos, n_dims, mode, freq_base, freq_scale, 1);
}

GT_API gt_tensor* gt_flash_decode_q8_0(const gt_tensor* q, const gt_tensor* k_q8, const gt_tensor* v_q8,
                                       const gt_tensor* seq_lens, float scale) {
    const char* ctx = "flash_decode_q8_0";
    if (!q || !k_q8 || !v_q8 || !seq_lens) {
        set_errorf("%s: q, k, v and seq_lens are required", ctx);
        return nullptr;
    }
    if (q->device_type != GT_DEV_CUDA || k_q8->device_type != GT_DEV_CUDA || v_q8->device_type != GT_DEV_CUDA ||
        seq_lens->device_type != GT_DEV_CUDA) {
        set_errorf("%s: this engine runs CUDA tensors only", ctx);
        return nullptr;
    }
    if (!is_q8(k_q8->dtype) || !is_q8(v_q8->dtype) || k_q8->ndim != 4 || v_q8->ndim != 4) {
        set_errorf("%s: k and v must be 4-D Q8_0 tensors (B, Hkv, Smax, D)", ctx);
        return nullptr;
    }
    if (seq_lens->dtype != GT_I32 || seq_lens->ndim != 1 || !contiguous(seq_lens)) {
        set_errorf("%s: seq_lens must be a contiguous int32 (B) tensor", ctx);
        return nullptr;
    }
    const int64_t B = k_q8->shape[0], Hkv = k_q8->shape[1], Smax = k_q8->shape[2], D = k_q8->shape[3];
    if ((q->ndim != 4 && q->ndim != 3) || q->shape[0] != B || (q->ndim == 4 && q->shape[2] != 1) ||
        q->shape[q->ndim - 1] != D || seq_lens->shape[0] != B) {
        set_errorf("%s: q must be (B, H, 1, D) matching the cache", ctx);
        return nullptr;
    }
    for (int i = 0; i < 4; ++i) {
        if (v_q8->shape[i] != k_q8->shape[i]) {
            set_errorf("%s: k and v caches differ in shape", ctx);
            return nullptr;
        }
    }
    const int64_t H = q->shape[1];
    gt_tensor* qc = contiguous(q) ? nullptr : gt_tensor_contiguous(q);
    const gt_tensor* qs = qc ? qc : q;
    const int64_t osh[4] = {B, H, 1, D};
    gt_tensor* out = alloc_tensor(4, osh, q->dtype, GT_DEV_CUDA, q->device_index);
    int rc = -1;
    if (out) {
        DeviceGuard g(q->device_index);
        rc = gtb_decode_q8_0(data_of(qs), qs->dtype, data_of(k_q8), data_of(v_q8), (const int32_t*)data_of(seq_lens), B,
                             H, Hkv, Smax, D, scale, data_of(out), nullptr);
    }
    if (qc) gt_tensor_free(qc);
    if (rc != 0 && out) {
        gt_tensor_free(out);
        out = nullptr;
    }
    return out;
}

}  // extern "C"
