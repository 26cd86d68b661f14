// Validated argument bundles passed from the C-ABI layer to the kernel launchers.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/gtb_attn.h"

namespace gtb {

struct AttnShape {
    int64_t B, H, Hkv, L, S, D, Dv;
};

struct FwdArgs {
    AttnShape sh;
    gtb_tensor4 q, k, v, o;
    bool has_mask;
    gtb_tensor4 mask;  // broadcast dims carry stride 0
    float scale;       // already resolved (> 0)
    int causal;
    void* lse;         // nullable, (B,H,L) contiguous; double for f64 inputs, else float
    float drop_p = 0.0f;         // dropout probability of the attention weights (0: none)
    uint32_t drop_thr = 0;       // keep threshold of dropout.cuh
    uint64_t drop_seed = 0;
    // RoPE of q inside the tcgen05 forward (no mask, no dropout, n_dims % 16 == 0): (cos, sin) of query
    // row l, pair i at rope_q_tab[2 (l n_dims/2 + i)], 16-byte aligned; null: q is used as given
    const float* rope_q_tab = nullptr;
    int rope_n_dims = 0;
    int rope_mode = 0;
};

struct BwdArgs {
    AttnShape sh;
    gtb_tensor4 q, k, v, o, dout, dq, dk, dv;
    bool has_mask;
    gtb_tensor4 mask;
    float scale;
    int causal;
    const void* lse;   // (B,H,L) contiguous, from the forward (double for f64 inputs)
    void* scratch;     // B*H*L accumulators (float or double) for rowsum(dout * out)
    bool deterministic = false;  // the separate dQ kernel instead of f32 reductions in global memory
    float drop_p = 0.0f;         // dropout of the forward this backward belongs to (same seed)
    uint32_t drop_thr = 0;
    uint64_t drop_seed = 0;
};

// C (M, N) = A (M, K) B (N, K)^T (+ bias) on the tensor cores (linear_sm100.cu): bf16/f16, row-major
// with leading dimensions lda, ldb, ldc (elements), 16-byte aligned rows, K > 0.
int launch_linear_sm100(const void* a, const void* b, const void* bias, void* c, int64_t M, int64_t N, int64_t K,
                        int64_t lda, int64_t ldb, int64_t ldc, int dtype, cudaStream_t st);

// Attention weights from a finished forward's lse (attn_weights.cu): out (B, L, S) when `average`
// (mean over heads) else (B, H, L, S), contiguous, in q's dtype.
int launch_attn_weights(const FwdArgs& a, const void* lse, void* out, bool average, cudaStream_t st);
// ... on the tensor cores for bf16/f16 q/k with D in {64, 128} (attn_weights_sm100.cu)
bool weights_sm100_supported(const FwdArgs& a, const void* out);
int launch_weights_sm100(const FwdArgs& a, const void* lse, void* out, bool average, cudaStream_t st);

// fp32 kernels register-blocked on 64 x 64 tiles (sdpa_f32_tiled.cu): f32 with D = Dv = 64, masks,
// dropout, any strides. The backward takes rowsum(dout * out) per row in `delta` (B, H, L).
bool f32_tiled_supported(const AttnShape& sh, int dtype);
int launch_fwd_f32_tiled(const FwdArgs& a, cudaStream_t st);
bool attn_weights_f32_tiled_supported(const FwdArgs& a, const void* out);
int launch_attn_weights_f32_tiled(const FwdArgs& a, const void* lse, void* out, bool average, cudaStream_t st);
int launch_bwd_f32_tiled(const BwdArgs& a, const float* delta, cudaStream_t st);

// SIMT kernels: any float dtype, any D/Dv <= 256, masks, any strides.
int launch_fwd_simt(const FwdArgs& a, cudaStream_t st);
int launch_bwd_simt(const BwdArgs& a, cudaStream_t st);
size_t bwd_simt_scratch_bytes(const BwdArgs& a);

// TMA: the driver's tensor-map encoder (nullptr if unavailable) and a 4-D (d, row, head, batch) map of
// a 16-bit tensor with a 64 x box_rows box and 128-byte swizzle.
PFN_cuTensorMapEncodeTiled_v12000 encode_fn();
bool make_tma_map_4d(CUtensorMap* tm, const gtb_tensor4& t, int64_t d_extent, bool bf16, int box_rows);

// tcgen05/TMA forward: bf16/f16, D == Dv in {64,128}, unit inner stride, no mask.
bool fwd_sm100_supported(const FwdArgs& a);
int launch_fwd_sm100(const FwdArgs& a, cudaStream_t st);

// tcgen05/TMA backward (dK/dV kernel + dQ kernel): same conditions as the forward, plus dq/dk/dv
// with unit inner stride and 16-byte aligned rows; scratch = bwd_sm100_scratch_bytes().
bool bwd_sm100_supported(const BwdArgs& a);
size_t bwd_sm100_scratch_bytes(const BwdArgs& a);
int launch_bwd_sm100(const BwdArgs& a, cudaStream_t st);

}  // namespace gtb
