// Attention weights of a forward that has already run: MultiheadAttention's need_weights=True output.
//
// The reference forms them explicitly (gguf_train/nn/modules/transformer.py:153-166): scores =
// q k^T * scale, -1e9 above the diagonal when causal, plus the mask, softmax over keys, dropout in
// training, then the mean over heads (average_attn_weights) or all heads. Here the forward kernels
// have produced each row's log-sum-exp, so a weight is one exponential: P[b,h,l,s] =
// exp(q.k * scale + mask - lse[b,h,l]) (0 where masked), times keep / (1 - p) under dropout (the
// decisions of dropout.cuh, so the weights are exactly those the forward multiplied v by). No
// (B, H, L, S) buffer exists: the head mean accumulates in registers.
//
// One CTA per (batch, 32-row tile, 32-key tile): for each head the CTA stages the 32 query rows and
// the 32 keys in shared memory, each warp owns 8 rows and each lane one key, and the lane's dot
// products run over D from shared memory (row broadcast, padded key rows). f32/f16/bf16 inputs
// accumulate in f32, f64 in f64; any head size up to 256, any strides, masks as gtb_sdpa_fwd takes them.

#include <cmath>

#include "dropout.cuh"
#include "gtb_common.cuh"
#include "sdpa_args.h"

namespace gtb {
namespace {

constexpr int WT = 32;        // rows and keys per CTA tile
constexpr int WARPS = 4;      // 8 rows per warp
constexpr int RPW = WT / WARPS;

struct W4 {
    const void* p;
    int64_t s0, s1, s2, s3;
};

struct WeightsP {
    W4 q, k, m;
    int mask_dtype;  // -1: no mask
    const void* lse;  // (B, H, L) Acc
    void* out;        // (B, L, S) or (B, H, L, S) contiguous, q's dtype
    int64_t B, H, Hkv, L, S, D;
    float scale;
    int causal, average;
    int drop;
    uint32_t drop_thr;
    uint64_t drop_seed;
    float inv_keep;
};

template <typename T, typename Acc>
__global__ void __launch_bounds__(WARPS * 32) attn_weights_kernel(WeightsP p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Acc* q_s = (Acc*)smem_raw;          // [WT][D]
    Acc* k_s = q_s + WT * p.D;          // [WT][D + 1]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t b = blockIdx.z, l0 = (int64_t)blockIdx.y * WT, s0 = (int64_t)blockIdx.x * WT;
    const int64_t s = s0 + lane;
    const int64_t group = p.H / p.Hkv;
    Acc acc[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) acc[r] = 0;
    // causal: the whole tile lies above the diagonal (every key after every row) -> weights 0
    const bool dead_tile = p.causal && s0 > l0 + WT - 1;
    for (int64_t h = 0; h < p.H && !dead_tile; ++h) {
        const int64_t hk = h / group;
        __syncthreads();
        for (int64_t i = threadIdx.x; i < WT * p.D; i += blockDim.x) {
            const int64_t r = i / p.D, d = i % p.D, l = l0 + r;
            q_s[i] = l < p.L ? (Acc)Elem<T>::load((const T*)p.q.p + b * p.q.s0 + h * p.q.s1 + l * p.q.s2 + d * p.q.s3) : (Acc)0;
        }
        for (int64_t i = threadIdx.x; i < WT * p.D; i += blockDim.x) {
            const int64_t j = i / p.D, d = i % p.D, ss = s0 + j;
            k_s[j * (p.D + 1) + d] =
                ss < p.S ? (Acc)Elem<T>::load((const T*)p.k.p + b * p.k.s0 + hk * p.k.s1 + ss * p.k.s2 + d * p.k.s3) : (Acc)0;
        }
        __syncthreads();
        const uint32_t hkey = p.drop ? drop_head_key(p.drop_seed, (uint32_t)(b * p.H + h)) : 0u;
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
            const int64_t l = l0 + warp * RPW + r;
            Acc w = 0;
            if (l < p.L && s < p.S && !(p.causal && s > l)) {
                const Acc lse = ((const Acc*)p.lse)[(b * p.H + h) * p.L + l];
                Acc x = 0;
                const Acc* qr = q_s + (warp * RPW + r) * p.D;
                const Acc* kr = k_s + lane * (p.D + 1);
                for (int64_t d = 0; d < p.D; ++d) x += qr[d] * kr[d];
                x *= (Acc)p.scale;
                bool allowed = lse != -(Acc)INFINITY;
                if (allowed && p.mask_dtype >= 0) {
                    const int64_t mi = b * p.m.s0 + h * p.m.s1 + l * p.m.s2 + s * p.m.s3;
                    if (p.mask_dtype == BOOL) allowed = ((const uint8_t*)p.m.p)[mi] != 0;
                    else x += load_any<Acc>(p.m.p, mi, p.mask_dtype);
                }
                if (allowed) {
                    w = exp(x - lse);
                    if (p.drop)
                        w = drop_keep(drop_row_key(hkey, (uint32_t)l), (uint32_t)s, p.drop_thr) ? w * (Acc)p.inv_keep : (Acc)0;
                }
            }
            if (p.average) {
                acc[r] += w;
            } else if (l < p.L && s < p.S) {
                T* o = (T*)p.out + ((b * p.H + h) * p.L + l) * p.S + s;
                Elem<T>::store(o, (decltype(Elem<T>::load(o)))w);
            }
        }
    }
    if (!p.average && !dead_tile) return;
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
        const int64_t l = l0 + warp * RPW + r;
        if (l >= p.L || s >= p.S) continue;
        if (p.average) {
            T* o = (T*)p.out + (b * p.L + l) * p.S + s;
            Elem<T>::store(o, (decltype(Elem<T>::load(o)))(acc[r] / (Acc)p.H));
        } else {  // a dead tile of the per-head output: zeros for every head
            for (int64_t h = 0; h < p.H; ++h) {
                T* o = (T*)p.out + ((b * p.H + h) * p.L + l) * p.S + s;
                Elem<T>::store(o, (decltype(Elem<T>::load(o)))0.0f);
            }
        }
    }
}

template <typename T, typename Acc>
int run_weights(const WeightsP& p, cudaStream_t st) {
    const size_t smem = sizeof(Acc) * (size_t)(WT * p.D + WT * (p.D + 1));
    if (smem > 48 * 1024 &&
        cuda_failed(cudaFuncSetAttribute(attn_weights_kernel<T, Acc>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                    "attention weights: shared memory"))
        return -1;
    dim3 grid((unsigned)((p.S + WT - 1) / WT), (unsigned)((p.L + WT - 1) / WT), (unsigned)p.B);
    attn_weights_kernel<T, Acc><<<grid, WARPS * 32, smem, st>>>(p);
    return cuda_failed(cudaGetLastError(), "attention weights launch") ? -1 : 0;
}

}  // namespace

int launch_attn_weights(const FwdArgs& a, const void* lse, void* out, bool average, cudaStream_t st) {
    if (a.sh.D > 256) {
        set_error("attention weights: head sizes above 256 are not supported");
        return -1;
    }
    if (a.sh.L >= (1ll << 31) / WT || a.sh.S >= (1ll << 31) || a.sh.B > 65535) {
        set_error("attention weights: sizes out of range");
        return -1;
    }
    WeightsP p;
    p.q = W4{a.q.data, a.q.stride[0], a.q.stride[1], a.q.stride[2], a.q.stride[3]};
    p.k = W4{a.k.data, a.k.stride[0], a.k.stride[1], a.k.stride[2], a.k.stride[3]};
    p.m = a.has_mask ? W4{a.mask.data, a.mask.stride[0], a.mask.stride[1], a.mask.stride[2], a.mask.stride[3]}
                     : W4{nullptr, 0, 0, 0, 0};
    p.mask_dtype = a.has_mask ? a.mask.dtype : -1;
    p.lse = lse;
    p.out = out;
    p.B = a.sh.B; p.H = a.sh.H; p.Hkv = a.sh.Hkv; p.L = a.sh.L; p.S = a.sh.S; p.D = a.sh.D;
    p.scale = a.scale;
    p.causal = a.causal;
    p.average = average ? 1 : 0;
    p.drop = a.drop_p > 0.0f;
    p.drop_thr = a.drop_thr;
    p.drop_seed = a.drop_seed;
    p.inv_keep = 1.0f / (1.0f - a.drop_p);
    // bf16/f16 with D in {64, 128}: the tensor-core kernel of attn_weights_sm100.cu
    if (weights_sm100_supported(a, out)) return launch_weights_sm100(a, lse, out, average, st);
    // fp32, head size 64, 16-byte rows: the register-blocked kernel of sdpa_f32_tiled.cu
    if (attn_weights_f32_tiled_supported(a, out)) return launch_attn_weights_f32_tiled(a, lse, out, average, st);
    switch (a.q.dtype) {
        case F32: return run_weights<float, float>(p, st);
        case F64: return run_weights<double, double>(p, st);
        case F16: return run_weights<__half, float>(p, st);
        case BF16: return run_weights<__nv_bfloat16, float>(p, st);
        default: set_error("attention weights: unsupported dtype"); return -1;
    }
}

}  // namespace gtb
