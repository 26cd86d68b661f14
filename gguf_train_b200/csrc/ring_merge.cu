// Log-sum-exp merge of partial attention results, the combine step of the long-context K/V ring.
//
// A query row attended over two disjoint key sets gives outputs o1, o2 (each normalised over its
// own keys) and log-sum-exps l1, l2; over the union the output is
//   o = (e^(l1 - m) o1 + e^(l2 - m) o2) / (e^(l1 - m) + e^(l2 - m)),  l = m + log(e^(l1 - m) + e^(l2 - m)),
// m = max(l1, l2). A row with no allowed key has l = -inf and contributes nothing. The reference has
// no multi-device path; this is the exchange-free half of splitting one causal attention over GPUs.

#include <cmath>

#include "gtb_common.cuh"

namespace gtb {
namespace {

template <typename T>
__global__ void attn_merge_kernel(float* __restrict__ o_acc, float* __restrict__ lse_acc, const T* __restrict__ o_part,
                                  const float* __restrict__ lse_part, int64_t groups, int64_t rows, int64_t D,
                                  int64_t part_gstride, int64_t lse_gstride) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t row = warp; row < groups * rows; row += nwarps) {
        const int64_t g = row / rows, r = row % rows;
        const float la = lse_acc[row];
        const float lp = lse_part[g * lse_gstride + r];
        const float m = fmaxf(la, lp);
        if (m == -INFINITY) continue;  // neither part saw an allowed key
        const float wa = la == -INFINITY ? 0.0f : expf(la - m);
        const float wp = lp == -INFINITY ? 0.0f : expf(lp - m);
        const float inv = 1.0f / (wa + wp);
        float* oa = o_acc + row * D;
        const T* op = o_part + g * part_gstride + r * D;
        for (int64_t d = lane; d < D; d += 32) oa[d] = (oa[d] * wa + Elem<T>::load(op + d) * wp) * inv;
        if (lane == 0) lse_acc[row] = m + logf(wa + wp);
    }
}

}  // namespace
}  // namespace gtb

using namespace gtb;

extern "C" GTB_API int gtb_attn_merge(float* o_acc, float* lse_acc, const void* o_part, const float* lse_part,
                                      int part_dtype, int64_t groups, int64_t rows, int64_t D, int64_t part_gstride,
                                      int64_t lse_gstride, void* stream) {
    if (groups < 0 || rows < 0 || D <= 0 || part_gstride < rows * D || lse_gstride < rows) {
        set_error("attn_merge: bad sizes");
        return -1;
    }
    if (groups == 0 || rows == 0) return 0;
    const int64_t total_rows = groups * rows;
    const int threads = 256;
    const int64_t blocks = std::min<int64_t>((total_rows * 32 + threads - 1) / threads, 148 * 16);
    cudaStream_t st = (cudaStream_t)stream;
    switch (part_dtype) {
        case F32:
            attn_merge_kernel<float><<<(unsigned)blocks, threads, 0, st>>>(o_acc, lse_acc, (const float*)o_part, lse_part,
                                                                          groups, rows, D, part_gstride, lse_gstride);
            break;
        case F16:
            attn_merge_kernel<__half><<<(unsigned)blocks, threads, 0, st>>>(o_acc, lse_acc, (const __half*)o_part,
                                                                           lse_part, groups, rows, D, part_gstride,
                                                                           lse_gstride);
            break;
        case BF16:
            attn_merge_kernel<__nv_bfloat16><<<(unsigned)blocks, threads, 0, st>>>(
                o_acc, lse_acc, (const __nv_bfloat16*)o_part, lse_part, groups, rows, D, part_gstride, lse_gstride);
            break;
        default:
            set_error("attn_merge: the partial output must be f32, f16 or bf16");
            return -1;
    }
    return cuda_failed(cudaGetLastError(), "attn_merge launch") ? -1 : 0;
}
