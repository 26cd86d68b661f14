// SIMT attention kernels: the general path for every dtype, head size <= 256, mask and stride.
//
// Semantics follow gt_flash_attention (reference csrc/gt_ops_nn.cpp:2423-2525): causal s > l is
// masked (top-left), a bool mask value 0 masks, a float mask is added, GQA maps query head h to
// kv head h / (H/Hkv), and a row with no allowed key gives 0. The reference accumulates in double;
// these kernels accumulate in float for f32/f16/bf16 inputs and in double for f64 inputs, with an
// online (streaming) softmax over key tiles so no (L, S) buffer exists.
//
// The backward follows FlashAttentionFn.backward (gguf_train/_functions.py:1934-1965) analytically:
// p = exp(s - lse), dv = p^T dO, dp = dO v^T, ds = p (dp - rowsum(dO * O)), dq = ds k * scale,
// dk = ds^T q * scale. dk/dv of a kv head sum over its query heads. It runs as three kernels
// (rowsum, dq by query rows, dk/dv by key rows) that recompute p, so no atomics are needed and the
// result is deterministic.

#include <cfloat>
#include <cmath>
#include <type_traits>

#include "dropout.cuh"
#include "gtb_common.cuh"
#include "sdpa_args.h"

namespace gtb {
namespace {

constexpr int ROWS = 4;   // warps per CTA = query (or key) rows per CTA
constexpr int KT = 32;    // keys (or queries) per staged tile = lanes
constexpr int MAXD = 256; // largest head size of the SIMT path
constexpr int MAXI = MAXD / 32;

template <typename Acc> __device__ inline Acc neg_inf();
template <> __device__ inline float neg_inf<float>() { return -INFINITY; }
template <> __device__ inline double neg_inf<double>() { return -(double)INFINITY; }

__device__ inline float acc_exp(float x) { return expf(x); }
__device__ inline double acc_exp(double x) { return exp(x); }
__device__ inline float acc_log(float x) { return logf(x); }
__device__ inline double acc_log(double x) { return log(x); }

template <typename Acc> __device__ inline Acc warp_max(Acc v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
template <typename Acc> __device__ inline Acc warp_sum(Acc v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

struct T4 {  // device-side copy of a strided 4-D view
    const void* p;
    int64_t s0, s1, s2, s3;
};

inline T4 t4(const gtb_tensor4& t) { return T4{t.data, t.stride[0], t.stride[1], t.stride[2], t.stride[3]}; }

struct FwdP {
    T4 q, k, v, o, m;
    int mask_dtype;  // -1 = no mask
    int64_t H, Hkv, L, S, D, Dv, group;
    float scale;
    int causal;
    void* lse;  // Acc[B*H*L]
    int drop;   // dropout of the attention probabilities (dropout.cuh)
    uint32_t drop_thr;
    uint64_t drop_seed;
    float inv_keep;  // 1 / (1 - p)
};

struct BwdP {
    T4 q, k, v, o, dout, dq, dk, dv, m;
    int mask_dtype;
    int64_t H, Hkv, L, S, D, Dv, group;
    float scale;
    int causal;
    const void* lse;  // Acc[B*H*L]
    void* rowsum;     // Acc[B*H*L]
    int drop;
    uint32_t drop_thr;
    uint64_t drop_seed;
    float inv_keep;
};

// score modifier: returns false if (b,h,l,s) may not be attended, else adds a float mask value
template <typename Acc>
__device__ inline bool apply_mask(const T4& m, int mask_dtype, int64_t b, int64_t h, int64_t l, int64_t s, Acc& x) {
    if (mask_dtype < 0) return true;
    const int64_t idx = b * m.s0 + h * m.s1 + l * m.s2 + s * m.s3;
    if (mask_dtype == BOOL) return ((const uint8_t*)m.p)[idx] != 0;
    x += load_any<Acc>(m.p, idx, mask_dtype);
    return true;
}

// ------------------------------------------------------------------ forward

template <typename T, typename Acc>
__global__ void __launch_bounds__(ROWS * 32) fwd_simt_kernel(FwdP p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Acc* q_s = (Acc*)smem_raw;                 // [ROWS][D]
    Acc* k_s = q_s + ROWS * p.D;               // [KT][D+1]
    Acc* v_s = k_s + KT * (p.D + 1);           // [KT][Dv]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t b = blockIdx.z, h = blockIdx.y, hk = h / p.group;
    const int64_t l0 = (int64_t)blockIdx.x * ROWS, l = l0 + warp;
    const bool row_ok = l < p.L;
    const T* qg = (const T*)p.q.p;
    const T* kg = (const T*)p.k.p;
    const T* vg = (const T*)p.v.p;

    for (int64_t i = threadIdx.x; i < ROWS * p.D; i += blockDim.x) {
        const int64_t r = i / p.D, d = i % p.D, ll = l0 + r;
        q_s[i] = ll < p.L ? (Acc)Elem<T>::load(qg + b * p.q.s0 + h * p.q.s1 + ll * p.q.s2 + d * p.q.s3) : (Acc)0;
    }
    int64_t s_end = p.S;
    if (p.causal) s_end = min(p.S, min(l0 + ROWS, p.L));  // keys 0 .. last row of the CTA
    const uint32_t rkey = p.drop ? drop_row_key(drop_head_key(p.drop_seed, (uint32_t)(b * p.H + h)), (uint32_t)l) : 0u;
    Acc m = neg_inf<Acc>(), lsum = 0;
    Acc o[MAXI];
#pragma unroll
    for (int i = 0; i < MAXI; ++i) o[i] = 0;

    for (int64_t s0 = 0; s0 < s_end; s0 += KT) {
        __syncthreads();
        for (int64_t i = threadIdx.x; i < KT * p.D; i += blockDim.x) {
            const int64_t j = i / p.D, d = i % p.D, s = s0 + j;
            k_s[j * (p.D + 1) + d] = s < p.S ? (Acc)Elem<T>::load(kg + b * p.k.s0 + hk * p.k.s1 + s * p.k.s2 + d * p.k.s3) : (Acc)0;
        }
        for (int64_t i = threadIdx.x; i < KT * p.Dv; i += blockDim.x) {
            const int64_t j = i / p.Dv, d = i % p.Dv, s = s0 + j;
            v_s[i] = s < p.S ? (Acc)Elem<T>::load(vg + b * p.v.s0 + hk * p.v.s1 + s * p.v.s2 + d * p.v.s3) : (Acc)0;
        }
        __syncthreads();
        if (!row_ok) continue;
        const int64_t s = s0 + lane;
        Acc sc = neg_inf<Acc>();
        if (s < p.S && !(p.causal && s > l)) {
            Acc dot = 0;
            const Acc* qr = q_s + warp * p.D;
            const Acc* kr = k_s + lane * (p.D + 1);
            for (int64_t d = 0; d < p.D; ++d) dot += qr[d] * kr[d];
            dot *= (Acc)p.scale;
            if (apply_mask<Acc>(p.m, p.mask_dtype, b, h, l, s, dot)) sc = dot;
        }
        const Acc m_new = fmax(m, warp_max(sc));
        if (m_new == neg_inf<Acc>()) continue;  // nothing allowed so far in this row
        const Acc alpha = (m == neg_inf<Acc>()) ? (Acc)0 : acc_exp(m - m_new);
        const Acc pj = (sc == neg_inf<Acc>()) ? (Acc)0 : acc_exp(sc - m_new);
        lsum = lsum * alpha + warp_sum(pj);  // the normaliser sums the undropped probabilities
        const Acc pv = (p.drop && !drop_keep(rkey, (uint32_t)s, p.drop_thr)) ? (Acc)0 : pj;
#pragma unroll
        for (int i = 0; i < MAXI; ++i) o[i] *= alpha;
        for (int j = 0; j < KT; ++j) {
            const Acc pb = __shfl_sync(0xffffffffu, pv, j);
            if (pb == (Acc)0) continue;
            const Acc* vr = v_s + j * p.Dv;
#pragma unroll
            for (int i = 0; i < MAXI; ++i) {
                const int64_t d = lane + 32 * i;
                if (d < p.Dv) o[i] += pb * vr[d];
            }
        }
        m = m_new;
    }
    if (!row_ok) return;
    const Acc inv = lsum > (Acc)0 ? (p.drop ? (Acc)p.inv_keep : (Acc)1) / lsum : (Acc)0;
    T* og = (T*)p.o.p;
#pragma unroll
    for (int i = 0; i < MAXI; ++i) {
        const int64_t d = lane + 32 * i;
        if (d < p.Dv) Elem<T>::store(og + b * p.o.s0 + h * p.o.s1 + l * p.o.s2 + d * p.o.s3, (decltype(Elem<T>::load(og)))(o[i] * inv));
    }
    if (p.lse && lane == 0) {
        ((Acc*)p.lse)[(b * p.H + h) * p.L + l] = lsum > (Acc)0 ? m + acc_log(lsum) : neg_inf<Acc>();
    }
}

// ------------------------------------------------------------------ backward

template <typename T, typename Acc>
__global__ void __launch_bounds__(ROWS * 32) bwd_rowsum_kernel(BwdP p, int64_t B) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * ROWS + warp;  // over B*H*L
    if (row >= B * p.H * p.L) return;
    const int64_t l = row % p.L, bh = row / p.L, h = bh % p.H, b = bh / p.H;
    const T* og = (const T*)p.o.p;
    const T* gg = (const T*)p.dout.p;
    Acc acc = 0;
    for (int64_t d = lane; d < p.Dv; d += 32) {
        acc += (Acc)Elem<T>::load(og + b * p.o.s0 + h * p.o.s1 + l * p.o.s2 + d * p.o.s3) *
               (Acc)Elem<T>::load(gg + b * p.dout.s0 + h * p.dout.s1 + l * p.dout.s2 + d * p.dout.s3);
    }
    acc = warp_sum(acc);
    if (lane == 0) ((Acc*)p.rowsum)[row] = acc;
}

template <typename T, typename Acc>
__global__ void __launch_bounds__(ROWS * 32) bwd_dq_kernel(BwdP p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Acc* q_s = (Acc*)smem_raw;              // [ROWS][D]
    Acc* g_s = q_s + ROWS * p.D;            // [ROWS][Dv]
    Acc* k_s = g_s + ROWS * p.Dv;           // [KT][D+1]
    Acc* v_s = k_s + KT * (p.D + 1);        // [KT][Dv+1]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t b = blockIdx.z, h = blockIdx.y, hk = h / p.group;
    const int64_t l0 = (int64_t)blockIdx.x * ROWS, l = l0 + warp;
    const bool row_ok = l < p.L;
    const T* qg = (const T*)p.q.p;
    const T* kg = (const T*)p.k.p;
    const T* vg = (const T*)p.v.p;
    const T* gg = (const T*)p.dout.p;
    for (int64_t i = threadIdx.x; i < ROWS * p.D; i += blockDim.x) {
        const int64_t r = i / p.D, d = i % p.D, ll = l0 + r;
        q_s[i] = ll < p.L ? (Acc)Elem<T>::load(qg + b * p.q.s0 + h * p.q.s1 + ll * p.q.s2 + d * p.q.s3) : (Acc)0;
    }
    for (int64_t i = threadIdx.x; i < ROWS * p.Dv; i += blockDim.x) {
        const int64_t r = i / p.Dv, d = i % p.Dv, ll = l0 + r;
        g_s[i] = ll < p.L ? (Acc)Elem<T>::load(gg + b * p.dout.s0 + h * p.dout.s1 + ll * p.dout.s2 + d * p.dout.s3) : (Acc)0;
    }
    const int64_t row = (b * p.H + h) * p.L + l;
    const Acc lse = row_ok ? ((const Acc*)p.lse)[row] : neg_inf<Acc>();
    const Acc di = row_ok ? ((const Acc*)p.rowsum)[row] : (Acc)0;
    int64_t s_end = p.S;
    if (p.causal) s_end = min(p.S, min(l0 + ROWS, p.L));
    const uint32_t rkey = p.drop ? drop_row_key(drop_head_key(p.drop_seed, (uint32_t)(b * p.H + h)), (uint32_t)l) : 0u;
    Acc dq[MAXI];
#pragma unroll
    for (int i = 0; i < MAXI; ++i) dq[i] = 0;

    for (int64_t s0 = 0; s0 < s_end; s0 += KT) {
        __syncthreads();
        for (int64_t i = threadIdx.x; i < KT * p.D; i += blockDim.x) {
            const int64_t j = i / p.D, d = i % p.D, s = s0 + j;
            k_s[j * (p.D + 1) + d] = s < p.S ? (Acc)Elem<T>::load(kg + b * p.k.s0 + hk * p.k.s1 + s * p.k.s2 + d * p.k.s3) : (Acc)0;
        }
        for (int64_t i = threadIdx.x; i < KT * p.Dv; i += blockDim.x) {
            const int64_t j = i / p.Dv, d = i % p.Dv, s = s0 + j;
            v_s[j * (p.Dv + 1) + d] = s < p.S ? (Acc)Elem<T>::load(vg + b * p.v.s0 + hk * p.v.s1 + s * p.v.s2 + d * p.v.s3) : (Acc)0;
        }
        __syncthreads();
        if (!row_ok || lse == neg_inf<Acc>()) continue;
        const int64_t s = s0 + lane;
        Acc ds = 0;
        if (s < p.S && !(p.causal && s > l)) {
            Acc dot = 0;
            const Acc* qr = q_s + warp * p.D;
            const Acc* kr = k_s + lane * (p.D + 1);
            for (int64_t d = 0; d < p.D; ++d) dot += qr[d] * kr[d];
            dot *= (Acc)p.scale;
            if (apply_mask<Acc>(p.m, p.mask_dtype, b, h, l, s, dot) && dot != neg_inf<Acc>()) {
                const Acc pr = acc_exp(dot - lse);
                Acc dp = 0;
                const Acc* gr = g_s + warp * p.Dv;
                const Acc* vr = v_s + lane * (p.Dv + 1);
                for (int64_t d = 0; d < p.Dv; ++d) dp += gr[d] * vr[d];
                if (p.drop) dp = drop_keep(rkey, (uint32_t)s, p.drop_thr) ? dp * (Acc)p.inv_keep : (Acc)0;
                ds = pr * (dp - di);
            }
        }
        for (int j = 0; j < KT; ++j) {
            const Acc db = __shfl_sync(0xffffffffu, ds, j);
            if (db == (Acc)0) continue;
            const Acc* kr = k_s + j * (p.D + 1);
#pragma unroll
            for (int i = 0; i < MAXI; ++i) {
                const int64_t d = lane + 32 * i;
                if (d < p.D) dq[i] += db * kr[d];
            }
        }
    }
    if (!row_ok) return;
    T* out = (T*)p.dq.p;
#pragma unroll
    for (int i = 0; i < MAXI; ++i) {
        const int64_t d = lane + 32 * i;
        if (d < p.D) Elem<T>::store(out + b * p.dq.s0 + h * p.dq.s1 + l * p.dq.s2 + d * p.dq.s3, (decltype(Elem<T>::load(out)))(dq[i] * (Acc)p.scale));
    }
}

template <typename T, typename Acc>
__global__ void __launch_bounds__(ROWS * 32) bwd_dkdv_kernel(BwdP p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Acc* k_s = (Acc*)smem_raw;              // [ROWS][D]
    Acc* v_s = k_s + ROWS * p.D;            // [ROWS][Dv]
    Acc* q_s = v_s + ROWS * p.Dv;           // [KT][D+1]
    Acc* g_s = q_s + KT * (p.D + 1);        // [KT][Dv+1]
    Acc* lse_s = g_s + KT * (p.Dv + 1);     // [KT]
    Acc* di_s = lse_s + KT;                 // [KT]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t b = blockIdx.z, hk = blockIdx.y;
    const int64_t s0 = (int64_t)blockIdx.x * ROWS, s = s0 + warp;
    const bool key_ok = s < p.S;
    const T* qg = (const T*)p.q.p;
    const T* kg = (const T*)p.k.p;
    const T* vg = (const T*)p.v.p;
    const T* gg = (const T*)p.dout.p;
    for (int64_t i = threadIdx.x; i < ROWS * p.D; i += blockDim.x) {
        const int64_t r = i / p.D, d = i % p.D, ss = s0 + r;
        k_s[i] = ss < p.S ? (Acc)Elem<T>::load(kg + b * p.k.s0 + hk * p.k.s1 + ss * p.k.s2 + d * p.k.s3) : (Acc)0;
    }
    for (int64_t i = threadIdx.x; i < ROWS * p.Dv; i += blockDim.x) {
        const int64_t r = i / p.Dv, d = i % p.Dv, ss = s0 + r;
        v_s[i] = ss < p.S ? (Acc)Elem<T>::load(vg + b * p.v.s0 + hk * p.v.s1 + ss * p.v.s2 + d * p.v.s3) : (Acc)0;
    }
    Acc dk[MAXI], dv[MAXI];
#pragma unroll
    for (int i = 0; i < MAXI; ++i) { dk[i] = 0; dv[i] = 0; }
    // causal: key s is seen by rows l >= s; start at the tile holding the CTA's first key
    const int64_t l_begin = p.causal ? (s0 / KT) * KT : 0;

    for (int64_t h = hk * p.group; h < (hk + 1) * p.group; ++h) {
        for (int64_t l0 = l_begin; l0 < p.L; l0 += KT) {
            __syncthreads();
            for (int64_t i = threadIdx.x; i < KT * p.D; i += blockDim.x) {
                const int64_t j = i / p.D, d = i % p.D, l = l0 + j;
                q_s[j * (p.D + 1) + d] = l < p.L ? (Acc)Elem<T>::load(qg + b * p.q.s0 + h * p.q.s1 + l * p.q.s2 + d * p.q.s3) : (Acc)0;
            }
            for (int64_t i = threadIdx.x; i < KT * p.Dv; i += blockDim.x) {
                const int64_t j = i / p.Dv, d = i % p.Dv, l = l0 + j;
                g_s[j * (p.Dv + 1) + d] = l < p.L ? (Acc)Elem<T>::load(gg + b * p.dout.s0 + h * p.dout.s1 + l * p.dout.s2 + d * p.dout.s3) : (Acc)0;
            }
            for (int i = threadIdx.x; i < KT; i += blockDim.x) {
                const int64_t l = l0 + i;
                const int64_t row = (b * p.H + h) * p.L + l;
                lse_s[i] = l < p.L ? ((const Acc*)p.lse)[row] : neg_inf<Acc>();
                di_s[i] = l < p.L ? ((const Acc*)p.rowsum)[row] : (Acc)0;
            }
            __syncthreads();
            if (!key_ok) continue;
            const int64_t l = l0 + lane;
            Acc pr = 0, ds = 0;
            const Acc lse = lse_s[lane];
            if (l < p.L && !(p.causal && s > l) && lse != neg_inf<Acc>()) {
                Acc dot = 0;
                const Acc* qr = q_s + lane * (p.D + 1);
                const Acc* kr = k_s + warp * p.D;
                for (int64_t d = 0; d < p.D; ++d) dot += qr[d] * kr[d];
                dot *= (Acc)p.scale;
                if (apply_mask<Acc>(p.m, p.mask_dtype, b, h, l, s, dot) && dot != neg_inf<Acc>()) {
                    pr = acc_exp(dot - lse);
                    Acc dp = 0;
                    const Acc* gr = g_s + lane * (p.Dv + 1);
                    const Acc* vr = v_s + warp * p.Dv;
                    for (int64_t d = 0; d < p.Dv; ++d) dp += gr[d] * vr[d];
                    Acc pv = pr;  // the probability the forward multiplied v by
                    if (p.drop) {
                        const bool kept = drop_keep(drop_row_key(drop_head_key(p.drop_seed, (uint32_t)(b * p.H + h)),
                                                                 (uint32_t)l), (uint32_t)s, p.drop_thr);
                        dp = kept ? dp * (Acc)p.inv_keep : (Acc)0;
                        pv = kept ? pr * (Acc)p.inv_keep : (Acc)0;
                    }
                    ds = pr * (dp - di_s[lane]);
                    pr = pv;
                }
            }
            for (int j = 0; j < KT; ++j) {
                const Acc pb = __shfl_sync(0xffffffffu, pr, j);
                const Acc db = __shfl_sync(0xffffffffu, ds, j);
                if (pb == (Acc)0 && db == (Acc)0) continue;
                const Acc* gr = g_s + j * (p.Dv + 1);
                const Acc* qr = q_s + j * (p.D + 1);
#pragma unroll
                for (int i = 0; i < MAXI; ++i) {
                    const int64_t d = lane + 32 * i;
                    if (d < p.Dv) dv[i] += pb * gr[d];
                    if (d < p.D) dk[i] += db * qr[d];
                }
            }
        }
    }
    if (!key_ok) return;
    T* dko = (T*)p.dk.p;
    T* dvo = (T*)p.dv.p;
#pragma unroll
    for (int i = 0; i < MAXI; ++i) {
        const int64_t d = lane + 32 * i;
        if (d < p.D) Elem<T>::store(dko + b * p.dk.s0 + hk * p.dk.s1 + s * p.dk.s2 + d * p.dk.s3, (decltype(Elem<T>::load(dko)))(dk[i] * (Acc)p.scale));
        if (d < p.Dv) Elem<T>::store(dvo + b * p.dv.s0 + hk * p.dv.s1 + s * p.dv.s2 + d * p.dv.s3, (decltype(Elem<T>::load(dvo)))dv[i]);
    }
}

template <typename Acc> size_t fwd_smem(int64_t D, int64_t Dv) {
    return sizeof(Acc) * (ROWS * D + KT * (D + 1) + KT * Dv);
}
template <typename Acc> size_t dq_smem(int64_t D, int64_t Dv) {
    return sizeof(Acc) * (ROWS * D + ROWS * Dv + KT * (D + 1) + KT * (Dv + 1));
}
template <typename Acc> size_t dkdv_smem(int64_t D, int64_t Dv) {
    return sizeof(Acc) * (ROWS * D + ROWS * Dv + KT * (D + 1) + KT * (Dv + 1) + 2 * KT);
}

template <typename K>
bool set_smem(K kernel, size_t bytes) {
    if (bytes <= 48 * 1024) return true;
    return !cuda_failed(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes),
                        "cudaFuncSetAttribute");
}

template <typename T, typename Acc>
int run_fwd(const FwdArgs& a, cudaStream_t st) {
    FwdP p;
    p.q = t4(a.q); p.k = t4(a.k); p.v = t4(a.v); p.o = t4(a.o);
    p.m = a.has_mask ? t4(a.mask) : T4{nullptr, 0, 0, 0, 0};
    p.mask_dtype = a.has_mask ? a.mask.dtype : -1;
    p.H = a.sh.H; p.Hkv = a.sh.Hkv; p.L = a.sh.L; p.S = a.sh.S; p.D = a.sh.D; p.Dv = a.sh.Dv;
    p.group = a.sh.H / a.sh.Hkv;
    p.scale = a.scale; p.causal = a.causal; p.lse = a.lse;
    p.drop = a.drop_p > 0.0f; p.drop_thr = a.drop_thr; p.drop_seed = a.drop_seed;
    p.inv_keep = 1.0f / (1.0f - a.drop_p);
    const size_t smem = fwd_smem<Acc>(p.D, p.Dv);
    if (!set_smem(fwd_simt_kernel<T, Acc>, smem)) return -1;
    dim3 grid((unsigned)((p.L + ROWS - 1) / ROWS), (unsigned)p.H, (unsigned)a.sh.B);
    fwd_simt_kernel<T, Acc><<<grid, ROWS * 32, smem, st>>>(p);
    return cuda_failed(cudaGetLastError(), "sdpa forward (SIMT) launch") ? -1 : 0;
}

template <typename T, typename Acc>
int run_bwd(const BwdArgs& a, cudaStream_t st) {
    BwdP p;
    p.q = t4(a.q); p.k = t4(a.k); p.v = t4(a.v); p.o = t4(a.o); p.dout = t4(a.dout);
    p.dq = t4(a.dq); p.dk = t4(a.dk); p.dv = t4(a.dv);
    p.m = a.has_mask ? t4(a.mask) : T4{nullptr, 0, 0, 0, 0};
    p.mask_dtype = a.has_mask ? a.mask.dtype : -1;
    p.H = a.sh.H; p.Hkv = a.sh.Hkv; p.L = a.sh.L; p.S = a.sh.S; p.D = a.sh.D; p.Dv = a.sh.Dv;
    p.group = a.sh.H / a.sh.Hkv;
    p.scale = a.scale; p.causal = a.causal; p.lse = a.lse; p.rowsum = a.scratch;
    p.drop = a.drop_p > 0.0f; p.drop_thr = a.drop_thr; p.drop_seed = a.drop_seed;
    p.inv_keep = 1.0f / (1.0f - a.drop_p);
    const int64_t B = a.sh.B;
    const int64_t rows = B * p.H * p.L;
    if (rows > 0) {
        bwd_rowsum_kernel<T, Acc><<<(unsigned)((rows + ROWS - 1) / ROWS), ROWS * 32, 0, st>>>(p, B);
        if (cuda_failed(cudaGetLastError(), "sdpa backward rowsum launch")) return -1;
    }
    if (std::is_same<T, float>::value && f32_tiled_supported(a.sh, a.q.dtype))  // fp32, D = 64: blocked kernels
        return launch_bwd_f32_tiled(a, (const float*)a.scratch, st);
    if (rows > 0) {
        const size_t s1 = dq_smem<Acc>(p.D, p.Dv);
        if (!set_smem(bwd_dq_kernel<T, Acc>, s1)) return -1;
        dim3 g1((unsigned)((p.L + ROWS - 1) / ROWS), (unsigned)p.H, (unsigned)B);
        bwd_dq_kernel<T, Acc><<<g1, ROWS * 32, s1, st>>>(p);
        if (cuda_failed(cudaGetLastError(), "sdpa backward dq launch")) return -1;
    }
    if (p.S > 0) {
        const size_t s2 = dkdv_smem<Acc>(p.D, p.Dv);
        if (!set_smem(bwd_dkdv_kernel<T, Acc>, s2)) return -1;
        dim3 g2((unsigned)((p.S + ROWS - 1) / ROWS), (unsigned)p.Hkv, (unsigned)B);
        bwd_dkdv_kernel<T, Acc><<<g2, ROWS * 32, s2, st>>>(p);
        if (cuda_failed(cudaGetLastError(), "sdpa backward dk/dv launch")) return -1;
    }
    return 0;
}

}  // namespace

int launch_fwd_simt(const FwdArgs& a, cudaStream_t st) {
    if (a.sh.D > MAXD || a.sh.Dv > MAXD) {
        set_errorf("flash_attention: head sizes above %d are not supported (D=%lld, Dv=%lld)", MAXD,
                   (long long)a.sh.D, (long long)a.sh.Dv);
        return -1;
    }
    if (f32_tiled_supported(a.sh, a.q.dtype)) return launch_fwd_f32_tiled(a, st);
    switch (a.q.dtype) {
        case F32: return run_fwd<float, float>(a, st);
        case F64: return run_fwd<double, double>(a, st);
        case F16: return run_fwd<__half, float>(a, st);
        case BF16: return run_fwd<__nv_bfloat16, float>(a, st);
        default: set_error("flash_attention: unsupported dtype"); return -1;
    }
}

size_t bwd_simt_scratch_bytes(const BwdArgs& a) {
    const size_t per = a.q.dtype == F64 ? sizeof(double) : sizeof(float);
    return per * (size_t)(a.sh.B * a.sh.H * a.sh.L);
}

int launch_bwd_simt(const BwdArgs& a, cudaStream_t st) {
    if (a.sh.D > MAXD || a.sh.Dv > MAXD) {
        set_errorf("flash_attention_backward: head sizes above %d are not supported", MAXD);
        return -1;
    }
    switch (a.q.dtype) {
        case F32: return run_bwd<float, float>(a, st);
        case F64: return run_bwd<double, double>(a, st);
        case F16: return run_bwd<__half, float>(a, st);
        case BF16: return run_bwd<__nv_bfloat16, float>(a, st);
        default: set_error("flash_attention_backward: unsupported dtype"); return -1;
    }
}

}  // namespace gtb
