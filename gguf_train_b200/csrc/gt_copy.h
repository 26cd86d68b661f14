// Data-movement launchers used by the handle runtime.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace gtb {

constexpr int kMaxDims = 12;

// dst (contiguous, n elements) <- src viewed with shape/strides (elements)
int launch_gather(void* dst, const void* src, int ndim, const int64_t* shape, const int64_t* strides, size_t esize,
                  int64_t n, cudaStream_t st);
// contiguous dtype conversion between f32/f64/f16/bf16
int launch_convert(void* dst, int dst_dt, const void* src, int src_dt, int64_t n, cudaStream_t st);

}  // namespace gtb
