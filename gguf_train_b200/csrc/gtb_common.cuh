// Shared helpers of the B200 attention library: dtype codes, element load/store, error state.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <string>

#include "../../include/gtb_attn.h"

namespace gtb {

// gt_dtype codes of the reference C-ABI (csrc/gguf_train.h:22-36)
enum Dtype : int { F32 = 0, F16 = 1, BF16 = 2, F64 = 3, I32 = 7, BOOL = 9, Q8_0 = 108 };

inline size_t dtype_size(int dt) {
    switch (dt) {
        case F32: return 4;
        case F16: return 2;
        case BF16: return 2;
        case F64: return 8;
        case I32: return 4;
        case BOOL: return 1;
        default: return 0;
    }
}

inline bool is_float_dtype(int dt) { return dt == F32 || dt == F16 || dt == BF16 || dt == F64; }

// thread-local error message, same convention as gt_last_error (csrc/gt_core.cpp:7-23)
void set_error(const std::string& msg);
void set_errorf(const char* fmt, ...);
const char* last_error();
void clear_error();

// Map a CUDA error to the thread-local message; returns true if there was one.
bool cuda_failed(cudaError_t e, const char* what);

// Per-device status word that kernels set when a bounded wait runs out (never trap, never hang).
// Allocated on first use.
int* device_status_word(int device);
// A further status word of `device` that gtb_device_status() reads and clears with the main one
// (the no-allocation decode entry point keeps its own, a file-scope device variable).
void register_status_word(int device, int* word);

// Keep freed memory in the device's stream-ordered pool (per-call scratch stays allocation-free).
void retain_pool_memory(int dev);

template <typename T> struct Elem;
template <> struct Elem<float> {
    __device__ static float load(const float* p) { return *p; }
    __device__ static void store(float* p, float v) { *p = v; }
};
template <> struct Elem<double> {
    __device__ static double load(const double* p) { return *p; }
    __device__ static void store(double* p, double v) { *p = v; }
};
template <> struct Elem<__half> {
    __device__ static float load(const __half* p) { return __half2float(*p); }
    __device__ static void store(__half* p, float v) { *p = __float2half_rn(v); }
};
template <> struct Elem<__nv_bfloat16> {
    __device__ static float load(const __nv_bfloat16* p) { return __bfloat162float(*p); }
    __device__ static void store(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
};

// Load one element of a runtime-typed buffer as Acc (mask values)
template <typename Acc>
__device__ inline Acc load_any(const void* base, int64_t idx, int dtype) {
    switch (dtype) {
        case F32: return (Acc)((const float*)base)[idx];
        case F64: return (Acc)((const double*)base)[idx];
        case F16: return (Acc)__half2float(((const __half*)base)[idx]);
        case BF16: return (Acc)__bfloat162float(((const __nv_bfloat16*)base)[idx]);
        case BOOL: return ((const uint8_t*)base)[idx] ? (Acc)1 : (Acc)0;
        default: return (Acc)0;
    }
}

}  // namespace gtb
