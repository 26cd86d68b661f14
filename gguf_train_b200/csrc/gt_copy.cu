// Data-movement kernels behind the handle ABI: strided -> contiguous gather and dtype conversion.
#include "gtb_common.cuh"
#include "gt_copy.h"

namespace gtb {
namespace {

struct Layout {
    int ndim;
    int64_t shape[kMaxDims];
    int64_t stride[kMaxDims];
};

template <typename E>
__global__ void gather_kernel(E* __restrict__ dst, const E* __restrict__ src, Layout lay, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t rem = i, off = 0;
        for (int d = lay.ndim - 1; d >= 0; --d) {
            const int64_t c = rem % lay.shape[d];
            rem /= lay.shape[d];
            off += c * lay.stride[d];
        }
        dst[i] = src[off];
    }
}

template <typename S, typename D>
__global__ void convert_kernel(D* __restrict__ dst, const S* __restrict__ src, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        if constexpr (sizeof(S) == 8 || sizeof(D) == 8) {
            double x;
            if constexpr (std::is_same<S, double>::value) x = src[i];
            else x = (double)Elem<S>::load(src + i);
            if constexpr (std::is_same<D, double>::value) dst[i] = x;
            else Elem<D>::store(dst + i, (float)x);  // through float, as the reference stores values
        } else {
            Elem<D>::store(dst + i, Elem<S>::load(src + i));
        }
    }
}

unsigned grid_for(int64_t n) {
    int64_t g = (n + 255) / 256;
    if (g > 148 * 32) g = 148 * 32;
    return (unsigned)(g < 1 ? 1 : g);
}

template <typename S>
int convert_from(void* dst, int dst_dt, const S* src, int64_t n, cudaStream_t st) {
    const unsigned g = grid_for(n);
    switch (dst_dt) {
        case F32: convert_kernel<S, float><<<g, 256, 0, st>>>((float*)dst, src, n); break;
        case F64: convert_kernel<S, double><<<g, 256, 0, st>>>((double*)dst, src, n); break;
        case F16: convert_kernel<S, __half><<<g, 256, 0, st>>>((__half*)dst, src, n); break;
        case BF16: convert_kernel<S, __nv_bfloat16><<<g, 256, 0, st>>>((__nv_bfloat16*)dst, src, n); break;
        default: set_error("to_dtype: unsupported target dtype on CUDA"); return -1;
    }
    return cuda_failed(cudaGetLastError(), "to_dtype launch") ? -1 : 0;
}

}  // namespace

int launch_gather(void* dst, const void* src, int ndim, const int64_t* shape, const int64_t* strides, size_t esize,
                  int64_t n, cudaStream_t st) {
    if (n == 0) return 0;
    Layout lay;
    lay.ndim = ndim;
    for (int i = 0; i < ndim; ++i) { lay.shape[i] = shape[i]; lay.stride[i] = strides[i]; }
    const unsigned g = grid_for(n);
    switch (esize) {
        case 1: gather_kernel<uint8_t><<<g, 256, 0, st>>>((uint8_t*)dst, (const uint8_t*)src, lay, n); break;
        case 2: gather_kernel<uint16_t><<<g, 256, 0, st>>>((uint16_t*)dst, (const uint16_t*)src, lay, n); break;
        case 4: gather_kernel<uint32_t><<<g, 256, 0, st>>>((uint32_t*)dst, (const uint32_t*)src, lay, n); break;
        case 8: gather_kernel<uint64_t><<<g, 256, 0, st>>>((uint64_t*)dst, (const uint64_t*)src, lay, n); break;
        default: set_error("contiguous: unsupported element size"); return -1;
    }
    return cuda_failed(cudaGetLastError(), "contiguous launch") ? -1 : 0;
}

int launch_convert(void* dst, int dst_dt, const void* src, int src_dt, int64_t n, cudaStream_t st) {
    if (n == 0) return 0;
    switch (src_dt) {
        case F32: return convert_from<float>(dst, dst_dt, (const float*)src, n, st);
        case F64: return convert_from<double>(dst, dst_dt, (const double*)src, n, st);
        case F16: return convert_from<__half>(dst, dst_dt, (const __half*)src, n, st);
        case BF16: return convert_from<__nv_bfloat16>(dst, dst_dt, (const __nv_bfloat16*)src, n, st);
        default: set_error("to_dtype: unsupported source dtype on CUDA"); return -1;
    }
}

}  // namespace gtb
