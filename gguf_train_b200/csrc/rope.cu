// Device RoPE (gt_rope / gt_rope_backward of the reference, csrc/gt_ops_nn.cpp:2298-2421): x (B, H, S, D)
// contiguous f32/f16/bf16, pos int32 (>= S entries, one per sequence element), out of x's type
// computed in f32. 16-bit rows of 16 bytes take rope_rows_kernel (a per-position angle table shared by
// every plane, 16-byte accesses); otherwise one thread per pair of values, pairs past n_dims / 2 copied.

#include <algorithm>
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

// The same rotation for 16-bit x with 16-byte rows: a CTA takes 16 sequence positions, computes their
// (cos, sin) table once into shared memory (the angles exactly as rope_theta forms them, so the
// results equal rope_kernel's), then streams the rows of those positions in every (batch, head)
// plane it is given with 16-byte loads and stores: 8 values per thread, 4 pairs in normal mode; in
// NeoX mode a thread takes 8 values of the first half and their partners n_dims / 2 further on.
// Requires D % 8 == 0, n_dims % 16 == 0, 16-byte-aligned x and out.
constexpr int RB = 16;  // sequence positions per CTA

template <typename T>
__global__ void __launch_bounds__(256) rope_rows_kernel(const T* __restrict__ x, T* __restrict__ out,
                                                        const int32_t* __restrict__ pos, int64_t S, int64_t D,
                                                        int64_t planes, int planes_per_cta, RopeArgs r) {
    extern __shared__ float2 tab[];  // [RB][n_dims / 2]: (cos, sin with the direction's sign)
    const int np = r.n_dims / 2;
    const int64_t s0 = (int64_t)blockIdx.x * RB;
    for (int t = threadIdx.x; t < RB * np; t += blockDim.x) {
        const int sl = t / np, i = t - sl * np;
        float c = 1.0f, sn = 0.0f;
        if (s0 + sl < S) {
            sincosf(rope_theta(pos[s0 + sl], i, r.theta_scale, r.freq_scale), &sn, &c);
            sn *= r.sin_sign;
        }
        tab[t] = make_float2(c, sn);
    }
    __syncthreads();
    const int cpr = (int)(D / 8);  // 16-byte chunks per row
    const int64_t p0 = (int64_t)blockIdx.y * planes_per_cta, p1 = min(planes, p0 + planes_per_cta);
    constexpr int U = 4;  // planes in flight per thread
    // a thread keeps one (position, chunk) for every plane: its angles come out of the table once
    for (int t = threadIdx.x; t < RB * cpr; t += blockDim.x) {
        const int sl = t / cpr, d0 = 8 * (t - sl * cpr);
        const int64_t s = s0 + sl;
        if (s >= S) continue;
        const int64_t off = s * D + d0, pstride = S * D;
        if (d0 >= r.n_dims) {  // dims past n_dims pass through
            for (int64_t pl = p0; pl < p1; ++pl) *(uint4*)(out + pl * pstride + off) = *(const uint4*)(x + pl * pstride + off);
            continue;
        }
        const bool neox = r.mode == 2;
        if (neox && d0 >= np) continue;  // the second half: rotated with its partners
        float2 cs[8];
        const float2* tr = tab + sl * np + (neox ? d0 : d0 / 2);
#pragma unroll
        for (int k = 0; k < 8; ++k) cs[k] = (neox || k < 4) ? tr[k] : make_float2(1.0f, 0.0f);
        for (int64_t pl = p0; pl < p1; pl += U) {
            const int n = (int)min((int64_t)U, p1 - pl);
            uint4 ua[U], ub[U];
#pragma unroll
            for (int u = 0; u < U; ++u)
                if (u < n) {
                    ua[u] = *(const uint4*)(x + (pl + u) * pstride + off);
                    if (neox) ub[u] = *(const uint4*)(x + (pl + u) * pstride + off + np);
                }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (u >= n) break;
                const T* a = (const T*)&ua[u];
                T ra[8];
                if (neox) {
                    const T* b = (const T*)&ub[u];
                    T rb[8];
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const float x0 = Elem<T>::load(a + k), x1 = Elem<T>::load(b + k);
                        Elem<T>::store(ra + k, __fsub_rn(__fmul_rn(x0, cs[k].x), __fmul_rn(x1, cs[k].y)));
                        Elem<T>::store(rb + k, __fadd_rn(__fmul_rn(x0, cs[k].y), __fmul_rn(x1, cs[k].x)));
                    }
                    *(uint4*)(out + (pl + u) * pstride + off + np) = *(const uint4*)rb;
                } else {
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const float x0 = Elem<T>::load(a + 2 * k), x1 = Elem<T>::load(a + 2 * k + 1);
                        Elem<T>::store(ra + 2 * k, __fsub_rn(__fmul_rn(x0, cs[k].x), __fmul_rn(x1, cs[k].y)));
                        Elem<T>::store(ra + 2 * k + 1, __fadd_rn(__fmul_rn(x0, cs[k].y), __fmul_rn(x1, cs[k].x)));
                    }
                }
                *(uint4*)(out + (pl + u) * pstride + off) = *(const uint4*)ra;
            }
        }
    }
}

template <typename T>
int launch_rope_rows(const void* x, int64_t rows, int64_t S, int64_t D, const int32_t* pos, const RopeArgs& r, void* out,
                     cudaStream_t st) {
    const int64_t planes = rows / S;
    const int64_t sblocks = (S + RB - 1) / RB;
    // enough planes per CTA to amortise the table, enough CTAs to fill the GPU (~8 per SM)
    int ppc = (int)std::max<int64_t>(1, std::min<int64_t>(planes, (planes * sblocks + 1183) / 1184));
    const int64_t gy = (planes + ppc - 1) / ppc;
    const size_t smem = sizeof(float2) * RB * (r.n_dims / 2);
    rope_rows_kernel<T><<<dim3((unsigned)sblocks, (unsigned)gy), 256, smem, st>>>((const T*)x, (T*)out, pos, S, D, planes,
                                                                                  ppc, r);
    return cuda_failed(cudaGetLastError(), "rope launch") ? -1 : 0;
}

}  // namespace

int launch_rope(const void* x, int dtype, int64_t rows, int64_t S, int64_t D, const int32_t* pos, const RopeArgs& r,
                void* out, cudaStream_t st) {
    const int64_t n = rows * (D / 2);
    if (n == 0) return 0;
    const bool rows16 = (dtype == F16 || dtype == BF16) && D % 8 == 0 && r.n_dims % 16 == 0 && r.n_dims <= D &&
                        S > 0 && rows % S == 0 && S <= INT32_MAX && ((uintptr_t)x & 15) == 0 && ((uintptr_t)out & 15) == 0 &&
                        (int64_t)RB * (r.n_dims / 2) * 8 <= 48 * 1024;
    if (rows16)
        return dtype == F16 ? launch_rope_rows<__half>(x, rows, S, D, pos, r, out, st)
                            : launch_rope_rows<__nv_bfloat16>(x, rows, S, D, pos, r, out, st);
    const unsigned grid = (unsigned)((n + 255) / 256);
    switch (dtype) {
        case F32: rope_kernel<float><<<grid, 256, 0, st>>>((const float*)x, (float*)out, pos, S, D, rows, r); break;
        case F16: rope_kernel<__half><<<grid, 256, 0, st>>>((const __half*)x, (__half*)out, pos, S, D, rows, r); break;
        case BF16: rope_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)x, (__nv_bfloat16*)out, pos, S, D, rows, r); break;
        default: set_error("rope: x must be f32, f16 or bf16"); return -1;
    }
    return cuda_failed(cudaGetLastError(), "rope launch") ? -1 : 0;
}

namespace {

// one (position, pair) per thread: the angle as rope_theta forms it, sin times the direction's sign,
// exactly the entries rope_rows_kernel builds in shared memory
__global__ void rope_table_kernel(const int32_t* __restrict__ pos, int64_t n, RopeArgs r, float2* __restrict__ tab) {
    const int np = r.n_dims / 2;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n * np) return;
    const int64_t s = t / np;
    const int i = (int)(t - s * np);
    float c, sn;
    sincosf(rope_theta(pos[s], i, r.theta_scale, r.freq_scale), &sn, &c);
    tab[t] = make_float2(c, sn * r.sin_sign);
}

}  // namespace

int launch_rope_table(const int32_t* pos, int64_t n, const RopeArgs& r, float* tab, cudaStream_t st) {
    const int64_t total = n * (r.n_dims / 2);
    if (total == 0) return 0;
    rope_table_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(pos, n, r, (float2*)tab);
    return cuda_failed(cudaGetLastError(), "rope table launch") ? -1 : 0;
}

}  // namespace gtb
