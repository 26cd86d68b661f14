// Rotary position embedding as the reference applies it (gt_rope, csrc/gt_ops_nn.cpp:2298-2421): it
// calls ggml_rope_ext(x, pos, n_dims, mode, n_ctx_orig, freq_base, freq_scale, ext_factor = 0,
// attn_factor = 1, beta_fast = 0, beta_slow = 0) on x permuted to (D, H, S, B), so one position per
// sequence element, shared by batch and heads. The rotation restated from ggml's published rope
// (llama.cpp b12283, ggml CPU ops: the rope cache and rope_yarn); with ext_factor = 0 there is no
// YaRN ramp and the magnitude scale is attn_factor = 1:
//   theta_scale = freq_base^(-2 / n_dims); angle of pair i = freq_scale * (p * theta_scale * ... * theta_scale)
//   (p multiplied by theta_scale i times in float, as the cache loop does);
//   normal mode (0): pairs (2i, 2i+1); NeoX mode (2): pairs (i, i + n_dims/2);
//   x0' = x0 cos - x1 sin, x1' = x0 sin + x1 cos; dims >= n_dims pass through;
//   the backward is the same with sin negated.
#pragma once

#include "gtb_common.cuh"

namespace gtb {

struct RopeArgs {
    int n_dims;         // even, <= D
    int mode;           // 0 normal, 2 NeoX
    float theta_scale;  // freq_base^(-2 / n_dims), computed on the host with powf as ggml does
    float freq_scale;
    float sin_sign;     // +1 forward, -1 backward
};

__device__ __forceinline__ float rope_theta(int p, int i, float theta_scale, float freq_scale) {
    float t = (float)p;
    for (int k = 0; k < i; ++k) t = __fmul_rn(t, theta_scale);
    return __fmul_rn(freq_scale, t);
}

// the two elements (c0, c1) of pair i of a row
__device__ __forceinline__ void rope_pair_index(const RopeArgs& r, int i, int& c0, int& c1) {
    if (r.mode == 2) {
        c0 = i;
        c1 = i + r.n_dims / 2;
    } else {
        c0 = 2 * i;
        c1 = 2 * i + 1;
    }
}

// rotate one pair (x0, x1) at position p
__device__ __forceinline__ void rope_rotate(const RopeArgs& r, int p, int i, float& x0, float& x1) {
    float s, c;
    sincosf(rope_theta(p, i, r.theta_scale, r.freq_scale), &s, &c);
    s *= r.sin_sign;
    const float a = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    const float b = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    x0 = a;
    x1 = b;
}

}  // namespace gtb
