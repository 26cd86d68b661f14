// fp32 attention on the CUDA cores, register-blocked: the path of f32 inputs with head size 64 (the
// tensor-core kernels take 16-bit inputs; a single-pass tf32 product would miss the 1e-3 tolerance of
// fp32 attention). Other fp32 head sizes run on the one-warp-per-row kernels of sdpa_simt.cu.
//
// Every kernel works on 64 x 64 tiles with 256 threads: thread t owns a 4 x 4 block (rows 4*(t/16)..,
// columns 4*(t%16)..), so the 16 threads of one half-warp hold one row group and a row's reductions are
// four shuffles. The inner loops issue two 16-byte shared loads per 16 FMAs. With 16-byte rows (the
// VEC instances) the tiles a kernel streams are copied with cp.async as row-major tiles whose 16-byte
// chunks are XOR-swizzled by (row / 4) % 8, which the products read either as the transposed operand
// (block_dot_rb, block_dot_rr) or row-major (block_pv_swz) without bank conflicts, so one copy serves
// both roles and no transposing store is needed; otherwise tiles are loaded transposed and row-major.
// An f32 or bool mask with contiguous, aligned key rows is read four keys per load.
//
//   forward     one CTA per 64 query rows of one (batch, head), key tiles of 64 (K and V double-
//               buffered a tile ahead): S = Q K^T, online softmax (running max and sum per row), P to
//               shared memory, O += P V; out = O / sum, lse = max + log(sum).
//   dq          one CTA per 64 query rows: S and dP = dO V^T recomputed per key tile, P = exp(S - lse),
//               dS = P (dP - delta), dQ += dS K.
//   dk / dv     one CTA per 64 keys of one (batch, kv head), looping over the query tiles of every query
//               head of the kv head: S^T = K Q^T, dP^T = V dO^T, P^T, dS^T; dV += P^T dO, dK += dS^T Q.
//   weights     MultiheadAttention's need_weights output from the forward's lse: one CTA per (batch, 64
//               rows, 64 keys), the heads' Q and K tiles double-buffered, exp(S - lse) averaged over
//               heads in registers or stored per head.
//
// Semantics are those of the SIMT kernels (sdpa_simt.cu) and of gt_flash_attention (reference
// csrc/gt_ops_nn.cpp:2423-2525): top-left causal, bool mask 0 = masked, float mask added to the scaled
// score, GQA head map h / (H/Hkv), a row with no allowed key gives 0 (and zero gradients), dropout with
// the decisions of dropout.cuh. delta = rowsum(dO * O) comes from the SIMT rowsum kernel.

#include <cmath>

#include "dropout.cuh"
#include "gtb_common.cuh"
#include "sdpa_args.h"

namespace gtb {
namespace {

constexpr int T = 64;          // rows and columns of a tile
constexpr int NT = 256;        // threads per CTA
constexpr int PAD = 4;         // float padding of transposed tiles (keeps 16-byte alignment)

struct V4 {
    const float* p;
    int64_t s0, s1, s2, s3;
};

struct TiledP {
    V4 q, k, v, o, g, dq, dk, dv, m;
    int mask_dtype;  // -1: none
    int vec;         // q, k, v, dO rows contiguous and 16-byte aligned: 16-byte row-major tile loads
    int mvec;        // f32 or bool mask with contiguous, aligned key rows and S % 4 == 0: mask_row4
    int64_t B, H, Hkv, L, S, group;
    float scale;
    int causal;
    float* lse;            // (B, H, L) forward output / backward input
    const float* delta;    // (B, H, L) rowsum(dO * O), backward
    int drop;
    uint32_t drop_thr;
    uint64_t drop_seed;
    float inv_keep;
    int average;           // attention weights: the mean over heads (B, L, S), else every head (B, H, L, S)
};

__device__ __forceinline__ float half_warp_max(float v) {
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float half_warp_sum(float v) {
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// mask adjustment of one scaled score: false if (b, h, l, s) may not be attended, else adds a float
// mask entry
__device__ __forceinline__ bool mask_score(const TiledP& p, int64_t b, int64_t h, int64_t l, int64_t s, float& x) {
    if (p.mask_dtype < 0) return true;
    const int64_t idx = b * p.m.s0 + h * p.m.s1 + l * p.m.s2 + s * p.m.s3;
    if (p.mask_dtype == BOOL) return ((const uint8_t*)p.m.p)[idx] != 0;
    x += load_any<float>(p.m.p, idx, p.mask_dtype);
    return true;
}

// The mask's additive values for keys s .. s+3 of row (b, h, l) in one load (p.mvec; s % 4 == 0 and
// s < S): an f32 mask's entries (16 bytes), or 0 / -inf for a bool mask's allowed / masked keys (4 bytes)
__device__ __forceinline__ float4 mask_row4(const TiledP& p, int64_t b, int64_t h, int64_t l, int64_t s) {
    const int64_t idx = b * p.m.s0 + h * p.m.s1 + l * p.m.s2 + s;
    if (p.mask_dtype == BOOL) {
        const uint32_t w = *(const uint32_t*)((const uint8_t*)p.m.p + idx);
        return make_float4((w & 0xffu) ? 0.0f : -INFINITY, (w & 0xff00u) ? 0.0f : -INFINITY,
                           (w & 0xff0000u) ? 0.0f : -INFINITY, (w >> 24) ? 0.0f : -INFINITY);
    }
    return *(const float4*)(p.m.p + idx);
}

// Load a 64 x D tile of a (B, heads, rows, D) tensor transposed into sm[d][r] (row stride T + PAD);
// rows at or past `rows` read 0. With 16-byte rows (vec) a thread reads four consecutive d of one row
// and consecutive threads take consecutive rows, so that a warp's four scalar stores per load each
// cover 32 consecutive words of sm (no bank conflict); all of a thread's loads are issued first.
template <int D>
__device__ __forceinline__ void load_t(float* sm, const V4& t, int64_t b, int64_t h, int64_t r0, int64_t rows,
                                       bool vec = false) {
    if (vec) {
        constexpr int PER = T * D / 4 / NT;  // float4 loads per thread
        constexpr int G = 1;                 // loads in flight per thread
#pragma unroll
        for (int u0 = 0; u0 < PER; u0 += G) {
            float4 v[G];
#pragma unroll
            for (int u = 0; u < G; ++u) {
                const int i = threadIdx.x + (u0 + u) * NT;
                const int r = i % T, d = 4 * (i / T);
                const int64_t row = r0 + r;
                v[u] = row < rows ? *(const float4*)(t.p + b * t.s0 + h * t.s1 + row * t.s2 + d)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < G; ++u) {
                const int i = threadIdx.x + (u0 + u) * NT;
                const int r = i % T, d = 4 * (i / T);
                sm[(d + 0) * (T + PAD) + r] = v[u].x;
                sm[(d + 1) * (T + PAD) + r] = v[u].y;
                sm[(d + 2) * (T + PAD) + r] = v[u].z;
                sm[(d + 3) * (T + PAD) + r] = v[u].w;
            }
        }
        return;
    }
    for (int i = threadIdx.x; i < T * D; i += NT) {
        const int r = i / D, d = i % D;
        const int64_t row = r0 + r;
        sm[d * (T + PAD) + r] = row < rows ? t.p[b * t.s0 + h * t.s1 + row * t.s2 + d * t.s3] : 0.0f;
    }
}
// The same tile row-major: sm[r][d] (row stride D + PAD); 16-byte loads and stores when the rows are
// contiguous and 16-byte aligned (vec)
template <int D>
__device__ __forceinline__ void load_r(float* sm, const V4& t, int64_t b, int64_t h, int64_t r0, int64_t rows, bool vec) {
    if (vec) {
        for (int i = threadIdx.x; i < T * D / 4; i += NT) {
            const int r = i / (D / 4), d = 4 * (i % (D / 4));
            const int64_t row = r0 + r;
            *(float4*)(sm + r * (D + PAD) + d) =
                row < rows ? *(const float4*)(t.p + b * t.s0 + h * t.s1 + row * t.s2 + d) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        return;
    }
    for (int i = threadIdx.x; i < T * D; i += NT) {
        const int r = i / D, d = i % D;
        const int64_t row = r0 + r;
        sm[r * (D + PAD) + d] = row < rows ? t.p[b * t.s0 + h * t.s1 + row * t.s2 + d * t.s3] : 0.0f;
    }
}

// The same row-major tile with asynchronous 16-byte copies (cp.async, rows past `rows` zero-filled), for
// 16-byte rows (vec): the copies run while the kernel computes with other tiles; cp_async_wait() and a
// barrier before the tile is read.
template <int D>
__device__ __forceinline__ void load_r_async(float* sm, const V4& t, int64_t b, int64_t h, int64_t r0, int64_t rows) {
    for (int i = threadIdx.x; i < T * D / 4; i += NT) {
        const int r = i / (D / 4), d = 4 * (i % (D / 4));
        const int64_t row = r0 + r;
        const bool in = row < rows;
        const float* src = t.p + b * t.s0 + h * t.s1 + (in ? row : r0) * t.s2 + d;  // a valid address either way
        const uint32_t dst = (uint32_t)__cvta_generic_to_shared(sm + r * (D + PAD) + d);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(in ? 16 : 0) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

// A 64 x D tile row-major without padding, its 16-byte chunks XOR-swizzled by (row / 4) % 8 (chunk c
// of row r at r * D + 4 * (c ^ ((r >> 2) & 7))), loaded with cp.async (16-byte rows; rows past `rows`
// zero-filled; the caller commits): block_dot_rb reads it as the transposed operand without bank
// conflicts, so no transposing store is needed and the copy can run behind other work.
template <int D>
__device__ __forceinline__ void load_swz_async(float* sm, const V4& t, int64_t b, int64_t h, int64_t r0, int64_t rows) {
    static_assert(D / 4 >= 8, "the swizzle spans eight 16-byte chunks");
    for (int i = threadIdx.x; i < T * D / 4; i += NT) {
        const int r = i / (D / 4), c = i % (D / 4);
        const int64_t row = r0 + r;
        const bool in = row < rows;
        const float* src = t.p + b * t.s0 + h * t.s1 + (in ? row : r0) * t.s2 + 4 * c;
        const uint32_t dst = (uint32_t)__cvta_generic_to_shared(sm + r * D + 4 * (c ^ ((r >> 2) & 7)));
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(in ? 16 : 0) : "memory");
    }
}

// acc[i][j] += sum_d A[d][ra + i] * Br[cb + j][d] over d < D: A transposed (as block_dot), Br a
// swizzled row-major tile (load_swz_async). Rows cb..cb+3 share one swizzle (cb is a multiple of 4), and
// the eight threads of a quarter warp (cb/4 = 0..7 or 8..15) read eight different bank groups.
template <int D>
__device__ __forceinline__ void block_dot_rb(float (&acc)[4][4], const float* A, const float* Br, int ra, int cb) {
    const int sw = (cb >> 2) & 7;
#pragma unroll 2
    for (int c = 0; c < D / 4; ++c) {
        float bv[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float4 t = *(const float4*)(Br + (cb + j) * D + 4 * (c ^ sw));
            bv[j][0] = t.x; bv[j][1] = t.y; bv[j][2] = t.z; bv[j][3] = t.w;
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float4 a = *(const float4*)(A + (4 * c + k) * (T + PAD) + ra);
            const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j][k], acc[i][j]);
        }
    }
}

// acc[i][j] += sum_d A[d][ra + i] * B[d][cb + j] over d < D (A, B transposed tiles)
template <int D>
__device__ __forceinline__ void block_dot(float (&acc)[4][4], const float* A, const float* B, int ra, int cb) {
#pragma unroll 8
    for (int d = 0; d < D; ++d) {
        const float4 a = *(const float4*)(A + d * (T + PAD) + ra);
        const float4 c = *(const float4*)(B + d * (T + PAD) + cb);
        const float av[4] = {a.x, a.y, a.z, a.w}, cv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], cv[j], acc[i][j]);
    }
}

// out[i][j] += sum_s P[s][ra + i] * V[s][cb + j] over the 64 rows s of P (transposed) and V (row-major)
template <int D>
__device__ __forceinline__ void block_pv(float (&out)[4][D / 16], const float* P, const float* V, int ra, int cb) {
#pragma unroll 4
    for (int s = 0; s < T; ++s) {
        const float4 a = *(const float4*)(P + s * (T + PAD) + ra);
        const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int q = 0; q < D / 64; ++q) {
            const float4 c = *(const float4*)(V + s * (D + PAD) + cb + 64 * q);
            const float cv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) out[i][4 * q + j] = fmaf(av[i], cv[j], out[i][4 * q + j]);
        }
    }
}

// The same with V a swizzled row-major tile (load_swz_async): row s, chunk c at 4 * (c ^ ((s >> 2) & 7)).
// The threads of a quarter warp read one row s at eight different chunks: no bank conflict.
template <int D>
__device__ __forceinline__ void block_pv_swz(float (&out)[4][D / 16], const float* P, const float* Vz, int ra, int cb) {
#pragma unroll 4
    for (int s = 0; s < T; ++s) {
        const float4 a = *(const float4*)(P + s * (T + PAD) + ra);
        const float av[4] = {a.x, a.y, a.z, a.w};
        const int sw = (s >> 2) & 7;
#pragma unroll
        for (int q = 0; q < D / 64; ++q) {
            const float4 c = *(const float4*)(Vz + s * D + 4 * (((cb >> 2) + 16 * q) ^ sw));
            const float cv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) out[i][4 * q + j] = fmaf(av[i], cv[j], out[i][4 * q + j]);
        }
    }
}

// ------------------------------------------------------------------ forward

// VEC (16-byte rows): K as a swizzled row-major tile and V row-major, both double-buffered and copied
// with cp.async one key tile ahead, so that the loads run behind the products; otherwise K transposed
// and V row-major, loaded synchronously per key tile.
template <int D, bool VEC>
__global__ void __launch_bounds__(NT, 2) fwd_f32_tiled_kernel(TiledP p) {
    extern __shared__ __align__(16) float smem[];
    float* Qs = smem;                        // [D][T + PAD]
    float* Ps = Qs + D * (T + PAD);          // [T keys][T + PAD rows]
    float* Kb = Ps + T * (T + PAD);          // VEC: 2 x [T][D] swizzled; else [D][T + PAD]
    float* Vb = Kb + (VEC ? 2 * T * D : D * (T + PAD));  // VEC: 2 x [T][D + PAD]; else [T][D + PAD]
    const int tid = threadIdx.x, rg = tid / 16, cg = tid % 16;
    const int ra = 4 * rg, cb = 4 * cg;
    const int64_t b = blockIdx.z, h = blockIdx.y, hk = h / p.group, l0 = (int64_t)blockIdx.x * T;
    load_t<D>(Qs, p.q, b, h, l0, p.L, p.vec);
    float m[4], lsum[4], o[4][D / 16];
    uint32_t rkey[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -INFINITY;
        lsum[i] = 0.0f;
        rkey[i] = p.drop ? drop_row_key(drop_head_key(p.drop_seed, (uint32_t)(b * p.H + h)), (uint32_t)(l0 + ra + i)) : 0u;
#pragma unroll
        for (int j = 0; j < D / 16; ++j) o[i][j] = 0.0f;
    }
    int64_t s_end = p.S;
    if (p.causal) s_end = min(p.S, min(l0 + T, p.L));
    if constexpr (VEC) {
        if (s_end > 0) {
            load_swz_async<D>(Kb, p.k, b, hk, 0, p.S);
            load_r_async<D>(Vb, p.v, b, hk, 0, p.S);  // commits the group
        }
    }
    for (int64_t s0 = 0, it = 0; s0 < s_end; s0 += T, ++it) {
        const int buf = VEC ? (int)(it & 1) : 0;
        float* Ks = Kb + buf * T * D;
        float* Vs = Vb + buf * T * (D + PAD);
        if constexpr (VEC) {
            cp_async_wait();  // this tile's K and V
            __syncthreads();  // ... visible to all; the other buffers are free (the last tile is done)
            if (s0 + T < s_end) {
                load_swz_async<D>(Kb + (buf ^ 1) * T * D, p.k, b, hk, s0 + T, p.S);
                load_r_async<D>(Vb + (buf ^ 1) * T * (D + PAD), p.v, b, hk, s0 + T, p.S);
            }
        } else {
            __syncthreads();
            load_r<D>(Vs, p.v, b, hk, s0, p.S, false);
            load_t<D>(Ks, p.k, b, hk, s0, p.S);
            __syncthreads();
        }
        float x[4][4] = {};
        if constexpr (VEC) block_dot_rb<D>(x, Qs, Ks, ra, cb);
        else block_dot<D>(x, Qs, Ks, ra, cb);
        float pv[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int64_t l = l0 + ra + i;
            float rmax = -INFINITY;
            const float4 mv4 = p.mvec && l < p.L && s0 + cb < p.S ? mask_row4(p, b, h, l, s0 + cb) : make_float4(0.f, 0.f, 0.f, 0.f);
            const float mv[4] = {mv4.x, mv4.y, mv4.z, mv4.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int64_t s = s0 + cb + j;
                float v = x[i][j] * p.scale + mv[j];
                const bool ok = l < p.L && s < p.S && !(p.causal && s > l) && (p.mvec || mask_score(p, b, h, l, s, v));
                x[i][j] = ok ? v : -INFINITY;
                rmax = fmaxf(rmax, x[i][j]);
            }
            const float m_new = fmaxf(m[i], half_warp_max(rmax));
            const float alpha = m_new == -INFINITY ? 1.0f : __expf(m[i] - m_new);
            float rs = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float e = x[i][j] == -INFINITY ? 0.0f : __expf(x[i][j] - m_new);
                rs += e;
                pv[i][j] = (p.drop && !drop_keep(rkey[i], (uint32_t)(s0 + cb + j), p.drop_thr)) ? 0.0f : e;
            }
            lsum[i] = lsum[i] * alpha + half_warp_sum(rs);
#pragma unroll
            for (int j = 0; j < D / 16; ++j) o[i][j] *= alpha;
            m[i] = m_new;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
            *(float4*)(Ps + (cb + j) * (T + PAD) + ra) = make_float4(pv[0][j], pv[1][j], pv[2][j], pv[3][j]);
        __syncthreads();
        block_pv<D>(o, Ps, Vs, ra, cb);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t l = l0 + ra + i;
        if (l >= p.L) continue;
        const float inv = lsum[i] > 0.0f ? (p.drop ? p.inv_keep : 1.0f) / lsum[i] : 0.0f;
        float* orow = (float*)p.o.p + b * p.o.s0 + h * p.o.s1 + l * p.o.s2;
#pragma unroll
        for (int q = 0; q < D / 64; ++q)
#pragma unroll
            for (int j = 0; j < 4; ++j) orow[(cb + 64 * q + j) * p.o.s3] = o[i][4 * q + j] * inv;
        if (p.lse && cg == 0) p.lse[(b * p.H + h) * p.L + l] = lsum[i] > 0.0f ? m[i] + __logf(lsum[i]) : -INFINITY;
    }
}

// ------------------------------------------------------------------ dq

// VEC (16-byte rows): per key tile one swizzled row-major copy of K (the operand of S = Q K^T and of
// dQ += dS K) and of V (the operand of dP = dO V^T), copied with cp.async; the next tile's V is copied
// while dQ += dS K runs. Otherwise K is loaded transposed and row-major and V transposed.
template <int D, bool VEC>
__global__ void __launch_bounds__(NT, 2) bwd_dq_f32_tiled_kernel(TiledP p) {
    extern __shared__ __align__(16) float smem[];
    float* Qs = smem;                        // [D][T + PAD]
    float* Gs = Qs + D * (T + PAD);          // dO [D][T + PAD]
    float* Ks = Gs + D * (T + PAD);          // [D][T + PAD]  (K transposed, for S; VEC: K swizzled [T][D])
    float* Vs = Ks + D * (T + PAD);          // [D][T + PAD]  (V transposed, for dP; VEC: V swizzled [T][D])
    float* Kr = Vs + D * (T + PAD);          // [T][D + PAD]  (K row-major, for dQ += dS K; VEC: unused)
    float* Ds = Kr + T * (D + PAD);          // dS [T keys][T + PAD rows]
    const int tid = threadIdx.x, rg = tid / 16, cg = tid % 16;
    const int ra = 4 * rg, cb = 4 * cg;
    const int64_t b = blockIdx.z, h = blockIdx.y, hk = h / p.group, l0 = (int64_t)blockIdx.x * T;
    load_t<D>(Qs, p.q, b, h, l0, p.L, p.vec);
    load_t<D>(Gs, p.g, b, h, l0, p.L, p.vec);
    float lse[4], dl[4], dq[4][D / 16];
    uint32_t rkey[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t l = l0 + ra + i;
        lse[i] = l < p.L ? p.lse[(b * p.H + h) * p.L + l] : -INFINITY;
        dl[i] = l < p.L ? p.delta[(b * p.H + h) * p.L + l] : 0.0f;
        rkey[i] = p.drop ? drop_row_key(drop_head_key(p.drop_seed, (uint32_t)(b * p.H + h)), (uint32_t)l) : 0u;
#pragma unroll
        for (int j = 0; j < D / 16; ++j) dq[i][j] = 0.0f;
    }
    int64_t s_end = p.S;
    if (p.causal) s_end = min(p.S, min(l0 + T, p.L));
    if constexpr (VEC) {
        if (s_end > 0) {
            load_swz_async<D>(Vs, p.v, b, hk, 0, p.S);
            cp_async_commit();
        }
    }
    for (int64_t s0 = 0; s0 < s_end; s0 += T) {
        __syncthreads();  // the last tile's dQ += dS K is done with K and dS
        if constexpr (VEC) {
            load_swz_async<D>(Ks, p.k, b, hk, s0, p.S);
            cp_async_commit();
            cp_async_wait();  // this tile's K and V
        } else {
            load_r<D>(Kr, p.k, b, hk, s0, p.S, false);
            load_t<D>(Ks, p.k, b, hk, s0, p.S);  // the scalar loads keep this loop within 128 registers
            load_t<D>(Vs, p.v, b, hk, s0, p.S);
        }
        __syncthreads();
        float x[4][4] = {}, dp[4][4] = {};
        if constexpr (VEC) {
            block_dot_rb<D>(x, Qs, Ks, ra, cb);
            block_dot_rb<D>(dp, Gs, Vs, ra, cb);
        } else {
            block_dot<D>(x, Qs, Ks, ra, cb);
            block_dot<D>(dp, Gs, Vs, ra, cb);
        }
        float ds[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int64_t l = l0 + ra + i;
            const float4 mv4 = p.mvec && l < p.L && s0 + cb < p.S ? mask_row4(p, b, h, l, s0 + cb) : make_float4(0.f, 0.f, 0.f, 0.f);
            const float mv[4] = {mv4.x, mv4.y, mv4.z, mv4.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int64_t s = s0 + cb + j;
                float v = x[i][j] * p.scale + mv[j];
                const bool ok = l < p.L && s < p.S && !(p.causal && s > l) && lse[i] != -INFINITY &&
                                (p.mvec || mask_score(p, b, h, l, s, v)) && v != -INFINITY;
                const float pr = ok ? __expf(v - lse[i]) : 0.0f;
                float d = dp[i][j];
                if (p.drop) d = drop_keep(rkey[i], (uint32_t)s, p.drop_thr) ? d * p.inv_keep : 0.0f;
                ds[i][j] = pr * (d - dl[i]);
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
            *(float4*)(Ds + (cb + j) * (T + PAD) + ra) = make_float4(ds[0][j], ds[1][j], ds[2][j], ds[3][j]);
        __syncthreads();  // dS is written and every thread is done with V
        if constexpr (VEC) {
            if (s0 + T < s_end) {  // the next tile's V, behind dQ += dS K
                load_swz_async<D>(Vs, p.v, b, hk, s0 + T, p.S);
                cp_async_commit();
            }
            block_pv_swz<D>(dq, Ds, Ks, ra, cb);
        } else {
            block_pv<D>(dq, Ds, Kr, ra, cb);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t l = l0 + ra + i;
        if (l >= p.L) continue;
        float* row = (float*)p.dq.p + b * p.dq.s0 + h * p.dq.s1 + l * p.dq.s2;
#pragma unroll
        for (int q = 0; q < D / 64; ++q)
#pragma unroll
            for (int j = 0; j < 4; ++j) row[(cb + 64 * q + j) * p.dq.s3] = dq[i][4 * q + j] * p.scale;
    }
}

// ------------------------------------------------------------------ dk / dv

// VEC (16-byte rows): each query tile's Q and dO are copied once (cp.async) as swizzled row-major tiles
// that serve both as the operand of S^T = K Q^T / dP^T = V dO^T and as the row-major operand of
// dK += dS^T Q / dV += P^T dO. Otherwise Q and dO are loaded transposed and row-major, and P^T / dS^T
// take the place of the transposed tiles once S^T and dP^T are formed. Either way 102.5 KB of shared
// memory: two CTAs per SM.
template <int D, bool VEC>
__global__ void __launch_bounds__(NT, 2) bwd_dkdv_f32_tiled_kernel(TiledP p) {
    extern __shared__ __align__(16) float smem[];
    float* Ks = smem;                        // K^T [D][T + PAD]  (rows = this CTA's keys)
    float* Vs = Ks + D * (T + PAD);          // V^T [D][T + PAD]
    float* Qs = Vs + D * (T + PAD);          // Q^T [D][T + PAD] (VEC: P^T only)
    float* Gs = Qs + D * (T + PAD);          // dO^T [D][T + PAD] (VEC: dS^T only)
    float* Qr = Gs + D * (T + PAD);          // Q row-major [T][D + PAD] (VEC: swizzled [T][D])
    float* Gr = Qr + T * (D + PAD);          // dO row-major [T][D + PAD] (VEC: swizzled [T][D])
    // P^T and dS^T as [query][key + PAD] (for dV += P^T dO, dK += dS^T Q)
    static_assert(D == T, "P^T / dS^T take the place of the transposed Q / dO tiles");
    float* Ps = Qs;
    float* Ds = Gs;
    float* LD = Gr + T * (D + PAD);          // lse[T], delta[T] of the query tile
    const int tid = threadIdx.x, rg = tid / 16, cg = tid % 16;
    const int ra = 4 * rg, cb = 4 * cg;      // ra: this thread's keys, cb: queries (S^T) or dims (dK/dV)
    const int64_t b = blockIdx.z, hk = blockIdx.y, s0 = (int64_t)blockIdx.x * T;
    load_t<D>(Ks, p.k, b, hk, s0, p.S, p.vec);
    load_t<D>(Vs, p.v, b, hk, s0, p.S, p.vec);
    float dk[4][D / 16], dv[4][D / 16];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < D / 16; ++j) { dk[i][j] = 0.0f; dv[i][j] = 0.0f; }
    // causal: keys s0.. are seen by queries l >= s0
    const int64_t l_begin = p.causal ? (s0 / T) * T : 0;
    for (int64_t h = hk * p.group; h < (hk + 1) * p.group; ++h) {
        const uint32_t hkey = p.drop ? drop_head_key(p.drop_seed, (uint32_t)(b * p.H + h)) : 0u;
        for (int64_t l0 = l_begin; l0 < p.L; l0 += T) {
            __syncthreads();
            if constexpr (VEC) {
                load_swz_async<D>(Qr, p.q, b, h, l0, p.L);
                load_swz_async<D>(Gr, p.g, b, h, l0, p.L);
                cp_async_commit();
            } else {
                load_r<D>(Qr, p.q, b, h, l0, p.L, false);
                load_r<D>(Gr, p.g, b, h, l0, p.L, false);
                load_t<D>(Qs, p.q, b, h, l0, p.L);  // the scalar loads keep this loop within 128 registers
                load_t<D>(Gs, p.g, b, h, l0, p.L);
            }
            for (int i = tid; i < T; i += NT) {
                const int64_t l = l0 + i;
                LD[i] = l < p.L ? p.lse[(b * p.H + h) * p.L + l] : -INFINITY;
                LD[T + i] = l < p.L ? p.delta[(b * p.H + h) * p.L + l] : 0.0f;
            }
            if constexpr (VEC) cp_async_wait();
            __syncthreads();
            float x[4][4] = {}, dp[4][4] = {};
            if constexpr (VEC) {
                block_dot_rb<D>(x, Ks, Qr, ra, cb);  // S^T[key][query]
                block_dot_rb<D>(dp, Vs, Gr, ra, cb); // dP^T
            } else {
                block_dot<D>(x, Ks, Qs, ra, cb);
                block_dot<D>(dp, Vs, Gs, ra, cb);
            }
            float pt[4][4], dst[4][4];
            // queries outer: the mask entries of query l for this thread's four keys are one load
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int64_t l = l0 + cb + j;
                const float lse = LD[cb + j];
                const float4 mv4 =
                    p.mvec && l < p.L && s0 + ra < p.S ? mask_row4(p, b, h, l, s0 + ra) : make_float4(0.f, 0.f, 0.f, 0.f);
                const float mv[4] = {mv4.x, mv4.y, mv4.z, mv4.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int64_t s = s0 + ra + i;
                    float v = x[i][j] * p.scale + mv[i];
                    const bool ok = l < p.L && s < p.S && !(p.causal && s > l) && lse != -INFINITY &&
                                    (p.mvec || mask_score(p, b, h, l, s, v)) && v != -INFINITY;
                    const float pr = ok ? __expf(v - lse) : 0.0f;
                    float d = dp[i][j], pk = pr;
                    if (p.drop) {
                        const bool kept = drop_keep(drop_row_key(hkey, (uint32_t)l), (uint32_t)s, p.drop_thr);
                        d = kept ? d * p.inv_keep : 0.0f;
                        pk = kept ? pr * p.inv_keep : 0.0f;
                    }
                    pt[i][j] = pk;
                    dst[i][j] = pr * (d - LD[T + cb + j]);
                }
            }
            __syncthreads();  // every thread has read the transposed Q / dO tiles that P^T / dS^T replace
            // P^T, dS^T stored [query][key]: rows of the "A" operand of block_pv are queries
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                *(float4*)(Ps + (cb + j) * (T + PAD) + ra) = make_float4(pt[0][j], pt[1][j], pt[2][j], pt[3][j]);
                *(float4*)(Ds + (cb + j) * (T + PAD) + ra) = make_float4(dst[0][j], dst[1][j], dst[2][j], dst[3][j]);
            }
            __syncthreads();
            if constexpr (VEC) {
                block_pv_swz<D>(dv, Ps, Gr, ra, cb);  // dV[key][d] += sum_l P^T[key][l] dO[l][d]
                block_pv_swz<D>(dk, Ds, Qr, ra, cb);  // dK[key][d] += sum_l dS^T[key][l] Q[l][d]
            } else {
                block_pv<D>(dv, Ps, Gr, ra, cb);
                block_pv<D>(dk, Ds, Qr, ra, cb);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t s = s0 + ra + i;
        if (s >= p.S) continue;
        float* krow = (float*)p.dk.p + b * p.dk.s0 + hk * p.dk.s1 + s * p.dk.s2;
        float* vrow = (float*)p.dv.p + b * p.dv.s0 + hk * p.dv.s1 + s * p.dv.s2;
#pragma unroll
        for (int q = 0; q < D / 64; ++q)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                krow[(cb + 64 * q + j) * p.dk.s3] = dk[i][4 * q + j] * p.scale;
                vrow[(cb + 64 * q + j) * p.dv.s3] = dv[i][4 * q + j];
            }
    }
}

// ------------------------------------------------------------------ attention weights

// acc[i][j] += sum_d Ar[ra + i][d] * Br[cb + j][d]: both operands swizzled row-major tiles
// (load_swz_async). Rows ra..ra+3 share one swizzle and the threads of a quarter warp share ra (one
// broadcast address for A); for B they read eight different bank groups, as in block_dot_rb.
template <int D>
__device__ __forceinline__ void block_dot_rr(float (&acc)[4][4], const float* Ar, const float* Br, int ra, int cb) {
    const int swa = (ra >> 2) & 7, swb = (cb >> 2) & 7;
#pragma unroll 2
    for (int c = 0; c < D / 4; ++c) {
        float av[4][4], bv[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 t = *(const float4*)(Ar + (ra + i) * D + 4 * (c ^ swa));
            av[i][0] = t.x; av[i][1] = t.y; av[i][2] = t.z; av[i][3] = t.w;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float4 t = *(const float4*)(Br + (cb + j) * D + 4 * (c ^ swb));
            bv[j][0] = t.x; bv[j][1] = t.y; bv[j][2] = t.z; bv[j][3] = t.w;
        }
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i][k], bv[j][k], acc[i][j]);
    }
}

// MultiheadAttention's need_weights output for fp32 q/k with head size 64 and 16-byte rows, from the
// forward's lse: P[b,h,l,s] = exp(q.k * scale + mask - lse[b,h,l]) (0 where masked or causal-masked;
// under dropout times keep / (1 - p), the forward's decisions). One CTA per (batch, 64 rows, 64 keys):
// per head, the Q rows and the K rows are copied with cp.async as swizzled row-major tiles, double-
// buffered so that the next head's copies run behind this head's products; each thread forms a 4 x 4
// block of scores, and the head mean accumulates in registers (or every head's weights are stored).
template <int D>
__global__ void __launch_bounds__(NT, 2) attn_weights_f32_tiled_kernel(TiledP p) {
    extern __shared__ __align__(16) float smem[];  // 2 x (Q [T][D], K [T][D]) swizzled
    const int tid = threadIdx.x, rg = tid / 16, cg = tid % 16;
    const int ra = 4 * rg, cb = 4 * cg;  // rows ra.., keys cb.. of the tile
    const int64_t b = blockIdx.z, l0 = (int64_t)blockIdx.y * T, s0 = (int64_t)blockIdx.x * T;
    const bool dead = p.causal && s0 > l0 + T - 1;  // every key after every row of the tile
    float acc[4][4] = {};
    auto issue = [&](int64_t h, int buf) {
        float* qb = smem + buf * 2 * T * D;
        load_swz_async<D>(qb, p.q, b, h, l0, p.L);
        load_swz_async<D>(qb + T * D, p.k, b, h / p.group, s0, p.S);
        cp_async_commit();
    };
    if (!dead) issue(0, 0);
    for (int64_t h = 0; h < p.H; ++h) {
        const int buf = (int)(h & 1);
        float w[4][4] = {};
        if (!dead) {
            cp_async_wait();  // this head's Q and K
            __syncthreads();  // ... visible to all; the other buffer is free (the last head is done)
            if (h + 1 < p.H) issue(h + 1, buf ^ 1);
            const float* qb = smem + buf * 2 * T * D;
            float x[4][4] = {};
            block_dot_rr<D>(x, qb, qb + T * D, ra, cb);
            const uint32_t hkey = p.drop ? drop_head_key(p.drop_seed, (uint32_t)(b * p.H + h)) : 0u;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int64_t l = l0 + ra + i;
                if (l >= p.L) continue;
                const float lse = p.lse[(b * p.H + h) * p.L + l];
                const float4 mv4 = p.mvec && s0 + cb < p.S ? mask_row4(p, b, h, l, s0 + cb) : make_float4(0.f, 0.f, 0.f, 0.f);
                const float mv[4] = {mv4.x, mv4.y, mv4.z, mv4.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int64_t s = s0 + cb + j;
                    float v = x[i][j] * p.scale + mv[j];
                    const bool ok = s < p.S && !(p.causal && s > l) && lse != -INFINITY &&
                                    (p.mvec || mask_score(p, b, h, l, s, v)) && v != -INFINITY;
                    float e = ok ? __expf(v - lse) : 0.0f;
                    if (p.drop && e != 0.0f)
                        e = drop_keep(drop_row_key(hkey, (uint32_t)l), (uint32_t)s, p.drop_thr) ? e * p.inv_keep : 0.0f;
                    w[i][j] = e;
                }
            }
        }
        if (p.average) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] += w[i][j];
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int64_t l = l0 + ra + i;
                if (l >= p.L) continue;
                float* o = (float*)p.o.p + ((b * p.H + h) * p.L + l) * p.S + s0 + cb;
                if (s0 + cb + 3 < p.S && (p.S & 3) == 0) *(float4*)o = make_float4(w[i][0], w[i][1], w[i][2], w[i][3]);
                else
                    for (int j = 0; j < 4; ++j)
                        if (s0 + cb + j < p.S) o[j] = w[i][j];
            }
        }
    }
    if (!p.average) return;
    const float inv_h = 1.0f / (float)p.H;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t l = l0 + ra + i;
        if (l >= p.L) continue;
        float* o = (float*)p.o.p + (b * p.L + l) * p.S + s0 + cb;
        if (s0 + cb + 3 < p.S && (p.S & 3) == 0)
            *(float4*)o = make_float4(acc[i][0] * inv_h, acc[i][1] * inv_h, acc[i][2] * inv_h, acc[i][3] * inv_h);
        else
            for (int j = 0; j < 4; ++j)
                if (s0 + cb + j < p.S) o[j] = acc[i][j] * inv_h;
    }
}

template <typename K>
bool smem_attr(K kern, size_t bytes) {
    return !cuda_failed(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes),
                        "fp32 tiled attention: shared memory");
}

V4 v4(const gtb_tensor4& t) { return V4{(const float*)t.data, t.stride[0], t.stride[1], t.stride[2], t.stride[3]}; }

// rows of 16-byte-aligned, contiguous floats: the tile loads may use 16-byte accesses
bool rows16(const gtb_tensor4& t) {
    if (((uintptr_t)t.data & 15) != 0 || t.stride[3] != 1) return false;
    for (int i = 0; i < 3; ++i)
        if (t.shape[i] > 1 && t.stride[i] % 4 != 0) return false;
    return true;
}

template <int D, bool VEC>
int fwd_dv(const TiledP& p, cudaStream_t st) {
    const size_t smem = sizeof(float) * (D * (T + PAD) + T * (T + PAD) +
                                         (VEC ? 2 * T * D + 2 * T * (D + PAD) : D * (T + PAD) + T * (D + PAD)));
    if (!smem_attr(fwd_f32_tiled_kernel<D, VEC>, smem)) return -1;
    dim3 grid((unsigned)((p.L + T - 1) / T), (unsigned)p.H, (unsigned)p.B);
    fwd_f32_tiled_kernel<D, VEC><<<grid, NT, smem, st>>>(p);
    return cuda_failed(cudaGetLastError(), "fp32 tiled attention forward launch") ? -1 : 0;
}

template <int D>
int fwd_d(const TiledP& p, cudaStream_t st) {
    return p.vec ? fwd_dv<D, true>(p, st) : fwd_dv<D, false>(p, st);
}

template <int D>
int bwd_d(const TiledP& p, cudaStream_t st) {
    const size_t s_dq = sizeof(float) * (4 * D * (T + PAD) + T * (D + PAD) + T * (T + PAD));
    const size_t s_kv = sizeof(float) * (4 * D * (T + PAD) + 2 * T * (D + PAD) + 2 * T);
    auto kv_kern = p.vec ? bwd_dkdv_f32_tiled_kernel<D, true> : bwd_dkdv_f32_tiled_kernel<D, false>;
    auto dq_kern = p.vec ? bwd_dq_f32_tiled_kernel<D, true> : bwd_dq_f32_tiled_kernel<D, false>;
    if (!smem_attr(dq_kern, s_dq) || !smem_attr(kv_kern, s_kv)) return -1;
    if (p.L > 0) {
        dq_kern<<<dim3((unsigned)((p.L + T - 1) / T), (unsigned)p.H, (unsigned)p.B), NT, s_dq, st>>>(p);
        if (cuda_failed(cudaGetLastError(), "fp32 tiled attention dq launch")) return -1;
    }
    if (p.S > 0) {
        kv_kern<<<dim3((unsigned)((p.S + T - 1) / T), (unsigned)p.Hkv, (unsigned)p.B), NT, s_kv, st>>>(p);
        if (cuda_failed(cudaGetLastError(), "fp32 tiled attention dk/dv launch")) return -1;
    }
    return 0;
}

TiledP common(const gtb_tensor4& q, const gtb_tensor4& k, const gtb_tensor4& v, bool has_mask, const gtb_tensor4& mask,
              const AttnShape& sh, float scale, int causal, float drop_p, uint32_t drop_thr, uint64_t drop_seed) {
    TiledP p{};
    p.q = v4(q); p.k = v4(k); p.v = v4(v);
    p.m = has_mask ? V4{(const float*)mask.data, mask.stride[0], mask.stride[1], mask.stride[2], mask.stride[3]}
                   : V4{nullptr, 0, 0, 0, 0};
    p.mask_dtype = has_mask ? mask.dtype : -1;
    p.vec = rows16(q) && rows16(k) && rows16(v);
    // the mask's key rows read four entries at a time: f32 or bool, contiguous along the keys, every
    // stride a multiple of four entries and S a multiple of four (a 4-key group never straddles S)
    p.mvec = 0;
    if (has_mask && (mask.dtype == F32 || mask.dtype == BOOL) && mask.stride[3] == 1 && sh.S % 4 == 0) {
        bool ok = ((uintptr_t)mask.data & (mask.dtype == F32 ? 15 : 3)) == 0;
        for (int i = 0; i < 3; ++i) ok = ok && mask.stride[i] % 4 == 0;
        p.mvec = ok ? 1 : 0;
    }
    p.B = sh.B; p.H = sh.H; p.Hkv = sh.Hkv; p.L = sh.L; p.S = sh.S; p.group = sh.H / sh.Hkv;
    p.scale = scale;
    p.causal = causal;
    p.drop = drop_p > 0.0f;
    p.drop_thr = drop_thr;
    p.drop_seed = drop_seed;
    p.inv_keep = 1.0f / (1.0f - drop_p);
    return p;
}

}  // namespace

bool f32_tiled_supported(const AttnShape& sh, int dtype) {
    return dtype == F32 && sh.D == 64 && sh.Dv == 64 && sh.B <= 65535 && sh.H <= 65535 && sh.L < (1ll << 31) &&
           sh.S < (1ll << 31);
}

bool attn_weights_f32_tiled_supported(const FwdArgs& a, const void* out) {
    return a.q.dtype == F32 && a.k.dtype == F32 && a.sh.D == 64 && a.sh.B <= 65535 && a.sh.L < (1ll << 31) &&
           a.sh.S < (1ll << 31) && ((uintptr_t)out & 15) == 0 && rows16(a.q) && rows16(a.k);
}

int launch_attn_weights_f32_tiled(const FwdArgs& a, const void* lse, void* out, bool average, cudaStream_t st) {
    TiledP p = common(a.q, a.k, a.v, a.has_mask, a.mask, a.sh, a.scale, a.causal, a.drop_p, a.drop_thr, a.drop_seed);
    p.o = V4{(const float*)out, 0, 0, 0, 1};
    p.lse = (float*)lse;
    p.average = average ? 1 : 0;
    constexpr int D = 64;
    const size_t smem = sizeof(float) * 4 * T * D;
    if (!smem_attr(attn_weights_f32_tiled_kernel<D>, smem)) return -1;
    dim3 grid((unsigned)((a.sh.S + T - 1) / T), (unsigned)((a.sh.L + T - 1) / T), (unsigned)a.sh.B);
    attn_weights_f32_tiled_kernel<D><<<grid, NT, smem, st>>>(p);
    return cuda_failed(cudaGetLastError(), "attention weights (fp32 tiled) launch") ? -1 : 0;
}

int launch_fwd_f32_tiled(const FwdArgs& a, cudaStream_t st) {
    TiledP p = common(a.q, a.k, a.v, a.has_mask, a.mask, a.sh, a.scale, a.causal, a.drop_p, a.drop_thr, a.drop_seed);
    p.o = v4(a.o);
    p.lse = (float*)a.lse;
    return fwd_d<64>(p, st);
}

int launch_bwd_f32_tiled(const BwdArgs& a, const float* delta, cudaStream_t st) {
    TiledP p = common(a.q, a.k, a.v, a.has_mask, a.mask, a.sh, a.scale, a.causal, a.drop_p, a.drop_thr, a.drop_seed);
    p.o = v4(a.o);
    p.g = v4(a.dout);
    p.vec = p.vec && rows16(a.dout);
    p.dq = v4(a.dq);
    p.dk = v4(a.dk);
    p.dv = v4(a.dv);
    p.lse = (float*)a.lse;
    p.delta = delta;
    return bwd_d<64>(p, st);
}

}  // namespace gtb
