// Attention masks on the tensor-core kernels: a per-tile class table and the per-element adjustment.
//
// The reference applies its mask inside the attention loop (gt_flash_attention, csrc/gt_ops_nn.cpp:
// 2488-2500): a bool mask entry 0 masks the key (score -inf), a float entry is added to the scaled
// score. The tcgen05 kernels hold raw scores x = q.k (unscaled) and exponentiate x * scale * log2(e)
// - m, so a float entry m_ls enters as x + m_ls / scale, and a masked bool entry as -inf.
//
// Most masks leave most tiles alone (a key-padding mask touches the last key block of a row; a causal
// or windowed bool mask only the blocks its edge crosses). mask_class_kernel therefore classifies each
// (mask batch, mask head, 128-row tile, 128-key block) region once per call:
//   MASK_NONE  every entry allows its key and adds 0: the block is computed as if unmasked;
//   MASK_MIXED the entries are read and applied one by one;
//   MASK_ALL   no entry allows its key: every score of the block is -inf.
// A size-1 (broadcast) mask dimension has one class entry for all its indices.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gtb_common.cuh"

namespace gtb {

enum : uint8_t { MASK_NONE = 0, MASK_MIXED = 1, MASK_ALL = 2 };
constexpr int MASK_TILE = 128;  // rows of a class region (query tile) and keys (key block)

// What the tcgen05 kernels need of a mask (element strides 0 on broadcast dimensions).
struct MaskView {
    const unsigned char* data = nullptr;  // nullptr: no mask
    int dtype = 0;                        // BOOL, F32, F16 or BF16
    int esize = 1;
    int vec = 0;                          // rows 16-byte aligned and contiguous along keys: vector loads
    int64_t s0 = 0, s1 = 0, s2 = 0, s3 = 0;  // element strides of (b, h, l, s)
    const uint8_t* cls = nullptr;         // class table
    int64_t c0 = 0, c1 = 0, c2 = 0;       // its strides of (b, h, row tile); key block stride 1
    float inv_scale = 1.0f;               // float entries are added to raw scores as m * inv_scale

    __device__ __forceinline__ uint8_t tile_class(int64_t b, int64_t h, int row_tile, int key_block) const {
        return cls[b * c0 + h * c1 + (int64_t)row_tile * c2 + key_block];
    }
    // byte address of entry (b, h, l, 0)
    __device__ __forceinline__ const unsigned char* row(int64_t b, int64_t h, int64_t l) const {
        return data + (b * s0 + h * s1 + l * s2) * esize;
    }
};

__device__ __forceinline__ float mask_entry_add(const unsigned char* p, int dtype, float inv_scale) {
    switch (dtype) {
        case BOOL: return *p ? 0.0f : -INFINITY;
        case F32: return *(const float*)p * inv_scale;
        case F16: return __half2float(*(const __half*)p) * inv_scale;
        default: return __bfloat162float(*(const __nv_bfloat16*)p) * inv_scale;
    }
}

// Adds the mask entries of keys s0 .. s0+31 of one query row (mrow = m.row(b, h, l)) to 32 raw
// scores: -inf where a bool entry is 0, m * inv_scale for float entries. Keys at or past S are left
// alone (the caller masks them).
__device__ __forceinline__ void mask_apply32(float* x, const MaskView& m, const unsigned char* mrow, int s0, int64_t S) {
    if (m.vec && (int64_t)s0 + 32 <= S) {
        if (m.dtype == BOOL) {
            const uint4* src = (const uint4*)(mrow + s0);
            const uint4 a = src[0], b = src[1];
            const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (((w[i >> 2] >> ((i & 3) * 8)) & 0xffu) == 0u) x[i] = -INFINITY;
        } else if (m.dtype == F32) {
            const float4* src = (const float4*)(mrow + (int64_t)s0 * 4);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float4 v = src[k];
                x[4 * k] = fmaf(v.x, m.inv_scale, x[4 * k]);
                x[4 * k + 1] = fmaf(v.y, m.inv_scale, x[4 * k + 1]);
                x[4 * k + 2] = fmaf(v.z, m.inv_scale, x[4 * k + 2]);
                x[4 * k + 3] = fmaf(v.w, m.inv_scale, x[4 * k + 3]);
            }
        } else {
            const uint4* src = (const uint4*)(mrow + (int64_t)s0 * 2);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint4 v = src[k];
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float lo, hi;
                    if (m.dtype == F16) {
                        const __half2 h2 = *(const __half2*)&w[j];
                        lo = __low2float(h2);
                        hi = __high2float(h2);
                    } else {
                        const __nv_bfloat162 h2 = *(const __nv_bfloat162*)&w[j];
                        lo = __low2float(h2);
                        hi = __high2float(h2);
                    }
                    x[8 * k + 2 * j] = fmaf(lo, m.inv_scale, x[8 * k + 2 * j]);
                    x[8 * k + 2 * j + 1] = fmaf(hi, m.inv_scale, x[8 * k + 2 * j + 1]);
                }
            }
        }
        return;
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) {  // fully unrolled: x stays in registers
        const int64_t s = (int64_t)s0 + i;
        if (s < S) x[i] += mask_entry_add(mrow + s * m.s3 * m.esize, m.dtype, m.inv_scale);
    }
}

// The same for 32 consecutive query rows l0 .. l0+31 of one key (a column of the mask, as the
// dK/dV kernel holds its transposed scores: one key per thread). Rows at or past L read row L - 1
// (their probabilities are 0 whatever the entry).
__device__ __forceinline__ void mask_apply_col32(float* x, const MaskView& m, int64_t b, int64_t h, int l0, int64_t L,
                                                 int64_t key) {
    const unsigned char* base = m.row(b, h, 0) + key * m.s3 * m.esize;
    const int64_t rs = m.s2 * m.esize;
#define GTB_MASK_COL_LOOP(EXPR)                                         \
    _Pragma("unroll") for (int i = 0; i < 32; ++i) {                    \
        const unsigned char* p = base + min((int64_t)l0 + i, L - 1) * rs; \
        x[i] += (EXPR);                                                  \
    }
    switch (m.dtype) {
        case BOOL: GTB_MASK_COL_LOOP(*p ? 0.0f : -INFINITY) break;
        case F32: GTB_MASK_COL_LOOP(*(const float*)p * m.inv_scale) break;
        case F16: GTB_MASK_COL_LOOP(__half2float(*(const __half*)p) * m.inv_scale) break;
        default: GTB_MASK_COL_LOOP(__bfloat162float(*(const __nv_bfloat16*)p) * m.inv_scale) break;
    }
#undef GTB_MASK_COL_LOOP
}

// Host side (mask_tiles.cu): checks whether the tensor-core kernels can read this mask and, if so,
// builds the class table in `table` (stream-ordered memory the caller frees on `st` after the
// attention kernels) and fills `mv`. row_tiles = the query tiles the table covers (ceil(L / 128)).
bool mask_supported(const gtb_tensor4& mask);
int build_mask_view(const gtb_tensor4& mask, int64_t B, int64_t H, int64_t L, int64_t S, float scale, MaskView& mv,
                    void** table, cudaStream_t st);

}  // namespace gtb
