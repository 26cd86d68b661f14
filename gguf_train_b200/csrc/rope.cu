// Device RoPE (gt_rope / gt_rope_backward of the reference, csrc/gt_ops_nn.cpp:2298-2421): x (B, H, S, D)
// contiguous f32/f16/bf16, pos int32 (>= S entries, one per sequence element), out of x's type
// computed in f32. One thread per pair of values; pairs past n_dims / 2 are copied.

#include <cmath>

#include "gtb_common.cuh"
#include "q8_0_internal.h"
#include "rope.cuh"
#include "sdpa_args.h"

namespace gtb {
namespace {

template <typename T>
__global__ void rope_kernel(const T* __restrict__ x, T* __restrict__ out, const int32_t* __restrict__ pos, int64_t S,
                            int64_t D, int64_t rows, RopeArgs r) {
    const int64_t npair = D / 2;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * npair) return;
    const int64_t row = idx / npair;
    const int i = (int)(idx - row * npair);
    const T* xr = x + row * D;
    T* orow = out + row * D;
    if (i < r.n_dims / 2) {
        int c0, c1;
        rope_pair_index(r, i, c0, c1);
        float x0 = Elem<T>::load(xr + c0), x1 = Elem<T>::load(xr + c1);
        rope_rotate(r, pos[row % S], i, x0, x1);
        Elem<T>::store(orow + c0, x0);
        Elem<T>::store(orow + c1, x1);
    } else {
        // the copied tail: pair i covers dims 2i, 2i+1 (which are >= n_dims in both modes)
        orow[2 * i] = xr[2 * i];
        orow[2 * i + 1] = xr[2 * i + 1];
    }
    if ((D & 1) && i == npair - 1) orow[D - 1] = xr[D - 1];  // an odd head dimension's last value
}

}  // namespace

int launch_rope(const void* x, int dtype, int64_t rows, int64_t S, int64_t D, const int32_t* pos, const RopeArgs& r,
                void* out, cudaStream_t st) {
    const int64_t n = rows * (D / 2);
    if (n == 0) return 0;
    const unsigned grid = (unsigned)((n + 255) / 256);
    switch (dtype) {
        case F32: rope_kernel<float><<<grid, 256, 0, st>>>((const float*)x, (float*)out, pos, S, D, rows, r); break;
        case F16: rope_kernel<__half><<<grid, 256, 0, st>>>((const __half*)x, (__half*)out, pos, S, D, rows, r); break;
        case BF16: rope_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)x, (__nv_bfloat16*)out, pos, S, D, rows, r); break;
        default: set_error("rope: x must be f32, f16 or bf16"); return -1;
    }
    return cuda_failed(cudaGetLastError(), "rope launch") ? -1 : 0;
}

}  // namespace gtb
