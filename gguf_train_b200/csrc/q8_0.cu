// GGUF Q8_0 on the device: quantise / dequantise, and a split-KV decode step over a Q8_0 cache.
//
// Q8_0 block (ggml block_q8_0): fp16 scale d, then 32 int8 quants; 34 bytes per 32 values.
// Quantisation is bit-exact with ggml's reference row quantiser, which the reference reaches
// through gt_quantize -> gt_tensor_to_dtype -> ggml_quantize_chunk (csrc/gt_ops_extra.cpp:2002,
// csrc/gt_core.cpp:792-840): amax = max|x|, d = amax/127, id = d ? 1/d : 0,
// q = round-half-away(x*id), d stored as fp16 (round to nearest even). Every step uses an
// explicitly rounded intrinsic so no FMA contraction or fast-math changes a bit.
//
// Decode: the reference has no fused path; a user dequantises K/V and calls
// F.scaled_dot_product_attention with a single query row per sequence. Here one CTA takes one
// (sequence, kv head, chunk of GTB_DECODE_CHUNK rows); all H/Hkv query heads of that kv head are
// served from one read of the cache. The 34-byte blocks are not 16-byte aligned, so whole tiles of
// rows (an even number of 136-byte rows = a multiple of 16 bytes) are staged into shared memory
// with cp.async.bulk and dequantised in registers from there. Partial (max, sum, out) triples per
// chunk go to scratch and a second kernel merges them.

#include <cfloat>
#include <cmath>

#include "gtb_common.cuh"
#include "q8_0_internal.h"
#include "rope.cuh"

namespace gtb {
namespace {

constexpr int QK = 32;
constexpr int QBYTES = 34;

// ------------------------------------------------------------------ quantise / dequantise

// 32 values into the 34-byte block at `dst` (2-byte aligned)
__device__ __forceinline__ void quantize_floats(const float* v, uint8_t* __restrict__ dst) {
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < QK; ++j) amax = fmaxf(amax, fabsf(v[j]));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __frcp_rn(d) : 0.0f;
    // the 34-byte block as 17 little-endian 16-bit words (blocks start 2-byte aligned)
    uint16_t* ob = (uint16_t*)dst;
    ob[0] = __half_as_ushort(__float2half_rn(d));
#pragma unroll
    for (int j = 0; j < QK; j += 2) {
        const uint32_t lo = (uint32_t)(uint8_t)(int8_t)roundf(__fmul_rn(v[j], id));
        const uint32_t hi = (uint32_t)(uint8_t)(int8_t)roundf(__fmul_rn(v[j + 1], id));
        ob[1 + j / 2] = (uint16_t)(lo | (hi << 8));
    }
}

// one 32-value block of x into the 34-byte block at `dst`
template <typename T>
__device__ __forceinline__ void quantize_block(const T* __restrict__ xb, uint8_t* __restrict__ dst) {
    float v[QK];
#pragma unroll
    for (int j = 0; j < QK; ++j) v[j] = (float)Elem<T>::load(xb + j);
    quantize_floats(v, dst);
}

template <typename T>
__global__ void q8_0_quantize_kernel(const T* __restrict__ x, int64_t nblocks, uint8_t* __restrict__ out) {
    const int64_t blk = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (blk >= nblocks) return;
    quantize_block(x + blk * QK, out + blk * QBYTES);
}

// KV-cache append: block j of row t of (sequence b, kv head hk) of x (B, Hkv, n_new, D) goes to
// cache row pos[b] + t of (B, Hkv, Smax, D/32 blocks). A row outside [0, Smax) is not written and
// records status 60.
// With ROPE, each new row is first rotated for its cache position pos[b] + t (rope.cuh), in f32,
// so the cache holds the quantised rotated keys without an intermediate rounding.
template <typename T, bool ROPE>
__global__ void q8_0_append_kernel(const T* __restrict__ x, int64_t Hkv, int64_t n_new, int64_t nb_row,
                                   uint8_t* __restrict__ cache, int64_t Smax, const int32_t* __restrict__ pos,
                                   int64_t nblocks, int* status, RopeArgs ra) {
    const int64_t blk = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (blk >= nblocks) return;
    const int64_t j = blk % nb_row, r = blk / nb_row;  // r over (b, hk, t)
    const int64_t t = r % n_new, bh = r / n_new, b = bh / Hkv;
    const int64_t row = (int64_t)pos[b] + t;
    if (row < 0 || row >= Smax) {
        if (status) atomicCAS(status, 0, 60);
        return;
    }
    uint8_t* dst = cache + ((bh * Smax + row) * nb_row + j) * QBYTES;
    if constexpr (!ROPE) {
        quantize_block(x + blk * QK, dst);
    } else {
        const T* xr = x + r * nb_row * QK;  // the whole row: a NeoX partner can sit in another block
        float v[QK];
#pragma unroll  // constant indices: v stays in registers
        for (int e = 0; e < QK; ++e) {
            const int c = (int)(j * QK) + e;
            float xc = (float)Elem<T>::load(xr + c);
            if (c < ra.n_dims) {
                const int half = ra.n_dims / 2;
                const bool first = ra.mode == 2 ? c < half : (c & 1) == 0;
                const int i = ra.mode == 2 ? (first ? c : c - half) : c >> 1;
                const int partner = ra.mode == 2 ? (first ? c + half : c - half) : (c ^ 1);
                const float xp = (float)Elem<T>::load(xr + partner);
                float x0 = first ? xc : xp, x1 = first ? xp : xc;
                rope_rotate(ra, (int)row, i, x0, x1);
                xc = first ? x0 : x1;
            }
            v[e] = xc;
        }
        quantize_floats(v, dst);
    }
}

__global__ void q8_0_advance_kernel(int32_t* pos, int64_t B, int32_t n_new) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B) pos[b] += n_new;
}

template <typename T>
__global__ void q8_0_dequantize_kernel(const uint8_t* __restrict__ in, int64_t nblocks, T* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // one value per thread
    if (i >= nblocks * QK) return;
    const int64_t blk = i / QK;
    const int j = (int)(i % QK);
    const uint8_t* ib = in + blk * QBYTES;
    const uint16_t dbits = (uint16_t)ib[0] | ((uint16_t)ib[1] << 8);
    const float d = __half2float(__ushort_as_half(dbits));
    Elem<T>::store(out + i, __fmul_rn((float)(int8_t)ib[2 + j], d));
}

// ------------------------------------------------------------------ decode

constexpr int DEC_WARPS = 4;
constexpr int DEC_TILE = 64;    // rows per staged tile (even: 64 * 136 B is a multiple of 16)
constexpr int DEC_STAGES = 3;

__device__ inline uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ inline void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ inline void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// Bounded wait on an mbarrier phase. Returns false (and records a status code) if the phase
// has not completed within ~2^31 cycles; the caller then skips its remaining work.
__device__ inline bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* status, int code) {
    const uint32_t addr = smem_u32(bar);
    const long long t0 = clock64();
    while (true) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
        if (clock64() - t0 > (1ll << 31)) {
            if (status) atomicExch(status, code);
            return false;
        }
    }
}

__device__ inline void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ inline float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Read 16 quants (half of a Q8_0 block) and the block scale from a staged row.
// o = byte offset of the block in shared memory, half = 0/1. Returns the scale; q[0..15] as floats.
__device__ inline float read_half_block(const uint8_t* base, uint32_t o, int half, float q[16]) {
    const uint16_t dbits = *(const uint16_t*)(base + o);  // o is even
    const uint32_t start = o + 2 + 16 * half;              // first quant byte, even
    const uint32_t a = start & ~3u;
    const uint32_t sh = (start & 3u) * 8;                  // 0 or 16
    const uint32_t* w = (const uint32_t*)(base + a);
    uint32_t ww[5];
#pragma unroll
    for (int i = 0; i < 5; ++i) ww[i] = w[i];
    // int8 -> float without the (slow) integer-to-float conversion unit: flip the sign bit so the
    // byte reads as u = s + 128, place it in the low mantissa byte of a float with exponent 2^23
    // (value 2^23 + u), and subtract 2^23 + 128. Exact for every int8.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t x = __funnelshift_r(ww[i], ww[i + 1], sh) ^ 0x80808080u;
#pragma unroll
        for (int b = 0; b < 4; ++b)
            q[4 * i + b] = __int_as_float((int)__byte_perm(x, 0x4B000000u, 0x7440u | (uint32_t)b)) - 8388736.0f;
    }
    return __half2float(__ushort_as_half(dbits));
}

struct DecP {
    const void* q;
    int q_dtype;
    const uint8_t* k;
    const uint8_t* v;
    const int32_t* lens;
    void* out;
    float* part;        // [B][Hkv][nchunks][G][D + 2]
    int64_t B, H, Hkv, Smax, D, G, nchunks, chunk;
    int64_t nhg;        // head groups per kv head (G / GH)
    float scale_log2;   // softmax scale * log2(e)
    int bulk;           // 1: tiles start 16-byte aligned -> cp.async.bulk staging
    int rows_align;     // rows per 16 bytes of cache (tile row counts are rounded up to this)
    int* status;
};

template <int D, int GH>
__global__ void __launch_bounds__(DEC_WARPS * 32)
decode_q8_0_kernel(DecP p) {
    constexpr int NB = D / QK;                // blocks per row
    constexpr int LANES_PER_ROW = NB * 2;     // half a block per lane
    constexpr int ROWS_PER_STEP = 32 / LANES_PER_ROW;
    constexpr int ROWB = NB * QBYTES;         // bytes per cached row
    constexpr int TILE_BYTES = DEC_TILE * ROWB;
    extern __shared__ __align__(128) unsigned char smem[];
    uint8_t* kt = smem;                                        // [STAGES][TILE_BYTES + 16]
    uint8_t* vt = kt + DEC_STAGES * (TILE_BYTES + 16);
    uint64_t* bars = (uint64_t*)(vt + DEC_STAGES * (TILE_BYTES + 16));
    float* red = (float*)(bars + DEC_STAGES);                  // [DEC_WARPS][GH][D + 2]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t chunk = blockIdx.x, hk = blockIdx.y / p.nhg, hg = blockIdx.y % p.nhg, b = blockIdx.z;
    int64_t len = p.lens[b];
    len = len < 0 ? 0 : (len > p.Smax ? p.Smax : len);
    const int64_t c0 = chunk * p.chunk;
    if (c0 >= len && !(chunk == 0)) return;  // chunk past the end (chunk 0 always reports)
    const int64_t c1 = min(len, c0 + p.chunk);
    const int64_t h0 = hk * p.G + hg * GH;   // first query head of this CTA

    const int slot = lane / LANES_PER_ROW;       // which row of the step
    const int sub = lane % LANES_PER_ROW;
    const int blk = sub >> 1, half = sub & 1;
    const int d0 = blk * QK + half * 16;

    // query values of this lane's 16 dims for every head of the group, pre-scaled to log2 units
    float qv[GH][16];
#pragma unroll
    for (int g = 0; g < GH; ++g) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int64_t idx = ((b * p.H + h0 + g) * p.D) + d0 + i;
            float x;
            if (p.q_dtype == F16) x = __half2float(((const __half*)p.q)[idx]);
            else if (p.q_dtype == BF16) x = __bfloat162float(((const __nv_bfloat16*)p.q)[idx]);
            else x = ((const float*)p.q)[idx];
            qv[g][i] = x * p.scale_log2;
        }
    }
    float m[GH], l[GH], o[GH][16];
#pragma unroll
    for (int g = 0; g < GH; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i) o[g][i] = 0.0f;
    }

    const uint8_t* kbase = p.k + ((b * p.Hkv + hk) * p.Smax) * (int64_t)ROWB;
    const uint8_t* vbase = p.v + ((b * p.Hkv + hk) * p.Smax) * (int64_t)ROWB;
    const int64_t ntiles = (c1 - c0 + DEC_TILE - 1) / DEC_TILE;

    if (p.bulk && threadIdx.x == 0) {
        for (int s = 0; s < DEC_STAGES; ++s) mbar_init(&bars[s], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    auto issue = [&](int64_t t) {  // thread 0 only
        const int s = (int)(t % DEC_STAGES);
        const int64_t r0 = c0 + t * DEC_TILE;
        int64_t n = min((int64_t)DEC_TILE, c1 - r0);
        // whole 16-byte units: Smax is a multiple of rows_align on this path, so the rows exist
        n = (n + p.rows_align - 1) / p.rows_align * p.rows_align;
        const uint32_t bytes = (uint32_t)(n * ROWB);
        const uint8_t* ksrc = kbase + r0 * ROWB;
        const uint8_t* vsrc = vbase + r0 * ROWB;
        uint8_t* kdst = kt + s * (TILE_BYTES + 16);
        uint8_t* vdst = vt + s * (TILE_BYTES + 16);
        // a bulk copy needs 16-byte aligned addresses and size: check, and on a violation record
        // status 2 and complete the stage without data instead of issuing the copy
        if ((((uintptr_t)ksrc | (uintptr_t)vsrc | (uintptr_t)smem_u32(kdst) | (uintptr_t)smem_u32(vdst) | bytes) & 15) != 0 ||
            n > DEC_TILE) {
            if (p.status) atomicExch(p.status, 2);
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&bars[s])) : "memory");
            return;
        }
        mbar_expect_tx(&bars[s], 2 * bytes);
        bulk_g2s(kdst, ksrc, bytes, &bars[s]);
        bulk_g2s(vdst, vsrc, bytes, &bars[s]);
    };

    if (p.bulk && threadIdx.x == 0) {
        for (int64_t t = 0; t < ntiles && t < DEC_STAGES; ++t) issue(t);
    }

    bool ok = true;
    for (int64_t t = 0; t < ntiles; ++t) {
        const int s = (int)(t % DEC_STAGES);
        uint8_t* ks = kt + s * (TILE_BYTES + 16);
        uint8_t* vs = vt + s * (TILE_BYTES + 16);
        const int64_t r0 = c0 + t * DEC_TILE;
        const int nrows = (int)min((int64_t)DEC_TILE, c1 - r0);
        if (p.bulk) {
            if (ok) ok = mbar_wait_bounded(&bars[s], (uint32_t)((t / DEC_STAGES) & 1), p.status, 1);
        } else {
            // rows are 4-byte aligned (34 * D/32 bytes, D % 64 == 0): word-wise cooperative loads
            const int nwords = nrows * ROWB / 4;
            const uint32_t* ksrc = (const uint32_t*)(kbase + r0 * ROWB);
            const uint32_t* vsrc = (const uint32_t*)(vbase + r0 * ROWB);
            for (int i = threadIdx.x; i < nwords; i += blockDim.x) {
                ((uint32_t*)ks)[i] = ksrc[i];
                ((uint32_t*)vs)[i] = vsrc[i];
            }
            __syncthreads();
        }
        if (ok) {
            for (int rr = warp * ROWS_PER_STEP; rr < nrows; rr += DEC_WARPS * ROWS_PER_STEP) {
                const int r = rr + slot;
                const bool valid = r < nrows;
                const int rs = valid ? r : 0;
                float kq[16];
                const float dk = read_half_block(ks, (uint32_t)(rs * ROWB + blk * QBYTES), half, kq);
                float sc[GH];
#pragma unroll
                for (int g = 0; g < GH; ++g) {
                    float acc = 0.0f;
#pragma unroll
                    for (int i = 0; i < 16; ++i) acc = fmaf(qv[g][i], kq[i], acc);
                    sc[g] = acc * dk;
                }
#pragma unroll
                for (int off = 1; off < LANES_PER_ROW; off <<= 1) {
#pragma unroll
                    for (int g = 0; g < GH; ++g) sc[g] += __shfl_xor_sync(0xffffffffu, sc[g], off);
                }
                float vq[16];
                const float dv = read_half_block(vs, (uint32_t)(rs * ROWB + blk * QBYTES), half, vq);
#pragma unroll
                for (int g = 0; g < GH; ++g) {
                    if (!valid) continue;
                    const float x = sc[g];
                    if (x > m[g] + 8.0f) {  // lazy rescale: only when the max grows by 2^8
                        const float alpha = fast_exp2(m[g] - x);  // m = -inf -> 0
                        l[g] *= alpha;
#pragma unroll
                        for (int i = 0; i < 16; ++i) o[g][i] *= alpha;
                        m[g] = x;
                    }
                    const float pr = fast_exp2(x - m[g]);
                    l[g] += pr;
                    const float pv = pr * dv;
#pragma unroll
                    for (int i = 0; i < 16; ++i) o[g][i] = fmaf(pv, vq[i], o[g][i]);
                }
            }
        }
        __syncthreads();  // every warp is done with stage s
        if (p.bulk && ok && threadIdx.x == 0 && t + DEC_STAGES < ntiles) issue(t + DEC_STAGES);
    }

    // merge the row slots of a warp (lanes with the same sub), then the warps through shared memory
#pragma unroll
    for (int off = LANES_PER_ROW; off < 32; off <<= 1) {
#pragma unroll
        for (int g = 0; g < GH; ++g) {
            const float mo = __shfl_xor_sync(0xffffffffu, m[g], off);
            const float lo = __shfl_xor_sync(0xffffffffu, l[g], off);
            const float mn = fmaxf(m[g], mo);
            const float a = (m[g] == -INFINITY) ? 0.0f : fast_exp2(m[g] - mn);
            const float c = (mo == -INFINITY) ? 0.0f : fast_exp2(mo - mn);
            l[g] = l[g] * a + lo * c;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float oo = __shfl_xor_sync(0xffffffffu, o[g][i], off);
                o[g][i] = o[g][i] * a + oo * c;
            }
            m[g] = mn;
        }
    }
    const int stride = (int)p.D + 2;
    if (slot == 0) {
#pragma unroll
        for (int g = 0; g < GH; ++g) {
            float* rw = red + (warp * GH + g) * stride;
#pragma unroll
            for (int i = 0; i < 16; ++i) rw[d0 + i] = o[g][i];
            if (sub == 0) { rw[p.D] = m[g]; rw[p.D + 1] = l[g]; }
        }
    }
    __syncthreads();
    // each thread finishes (head, dim) pairs
    for (int idx = threadIdx.x; idx < GH * D; idx += blockDim.x) {
        const int g = idx / D, d = idx % D;
        float mm = -INFINITY;
        for (int w = 0; w < DEC_WARPS; ++w) mm = fmaxf(mm, red[(w * GH + g) * stride + D]);
        float ll = 0.0f, oo = 0.0f;
        for (int w = 0; w < DEC_WARPS; ++w) {
            const float* rw = red + (w * GH + g) * stride;
            const float a = (rw[D] == -INFINITY) ? 0.0f : fast_exp2(rw[D] - mm);
            ll += rw[D + 1] * a;
            oo += rw[d] * a;
        }
        if (p.nchunks == 1) {
            const float r = ll > 0.0f ? oo / ll : 0.0f;
            const int64_t oi = (b * p.H + h0 + g) * p.D + d;
            if (p.q_dtype == F16) ((__half*)p.out)[oi] = __float2half_rn(r);
            else if (p.q_dtype == BF16) ((__nv_bfloat16*)p.out)[oi] = __float2bfloat16_rn(r);
            else ((float*)p.out)[oi] = r;
        } else {
            float* pp = p.part + ((((b * p.Hkv + hk) * p.nchunks + chunk) * p.G + hg * GH + g) * stride);
            pp[d] = oo;
            if (d == 0) { pp[D] = mm; pp[D + 1] = ll; }
        }
    }
}

// Merge the chunk partials of one (b, query head): one CTA of D threads per (b, h).
__global__ void decode_combine_kernel(DecP p) {
    const int64_t h = blockIdx.x, b = blockIdx.y;
    const int64_t hk = h / p.G, g = h % p.G;
    const int d = threadIdx.x;
    if (d >= p.D) return;
    int64_t len = p.lens[b];
    len = len < 0 ? 0 : (len > p.Smax ? p.Smax : len);
    const int64_t nch = max((int64_t)1, (len + p.chunk - 1) / p.chunk);
    const int stride = (int)p.D + 2;
    const float* base = p.part + (((b * p.Hkv + hk) * p.nchunks) * p.G + g) * stride;
    float mm = -INFINITY;
    for (int64_t c = 0; c < nch; ++c) mm = fmaxf(mm, base[c * p.G * stride + p.D]);
    float ll = 0.0f, oo = 0.0f;
    for (int64_t c = 0; c < nch; ++c) {
        const float* pc = base + c * p.G * stride;
        const float a = (pc[p.D] == -INFINITY) ? 0.0f : fast_exp2(pc[p.D] - mm);
        ll += pc[p.D + 1] * a;
        oo += pc[d] * a;
    }
    const float r = ll > 0.0f ? oo / ll : 0.0f;
    const int64_t oi = (b * p.H + h) * p.D + d;
    if (p.q_dtype == F16) ((__half*)p.out)[oi] = __float2half_rn(r);
    else if (p.q_dtype == BF16) ((__nv_bfloat16*)p.out)[oi] = __float2bfloat16_rn(r);
    else ((float*)p.out)[oi] = r;
}

// The same merge for D = 128, one warp per (b, query head): the lanes first take one chunk each for
// the maximum and the weights 2^(m_c - M), then every lane accumulates its d pairs (2 lane, 2 lane + 1)
// and (64 + 2 lane, 65 + 2 lane) over the chunks with independent loads (the weight of chunk j comes
// from lane j by shuffle). Latency-bound work, so many loads in flight per lane.
__global__ void __launch_bounds__(256) decode_combine128_kernel(DecP p) {
    constexpr int D = 128, ST = D + 2;
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= p.B * p.H) return;
    const int64_t b = row / p.H, h = row % p.H, hk = h / p.G, g = h % p.G;
    int64_t len = p.lens[b];
    len = len < 0 ? 0 : (len > p.Smax ? p.Smax : len);
    const int nch = (int)max((int64_t)1, (len + p.chunk - 1) / p.chunk);
    const float* base = p.part + (((b * p.Hkv + hk) * p.nchunks) * p.G + g) * ST;
    const int64_t cst = p.G * ST;  // floats between consecutive chunks of one head
    float mm = -INFINITY;
    for (int c = lane; c < nch; c += 32) mm = fmaxf(mm, base[c * cst + D]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, off));
    float ll = 0.0f, o0 = 0.0f, o1 = 0.0f, o2 = 0.0f, o3 = 0.0f;
    for (int c0 = 0; c0 < nch; c0 += 32) {
        const int c = c0 + lane;
        float w = 0.0f;
        if (c < nch) {
            const float mc = base[c * cst + D];
            w = mc == -INFINITY ? 0.0f : fast_exp2(mc - mm);
            ll = fmaf(w, base[c * cst + D + 1], ll);
        }
        const int n = min(32, nch - c0);
#pragma unroll 4
        for (int j = 0; j < n; ++j) {
            const float wj = __shfl_sync(0xffffffffu, w, j);
            const float* e = base + (c0 + j) * cst;
            const float2 x0 = *(const float2*)(e + 2 * lane);
            const float2 x1 = *(const float2*)(e + 64 + 2 * lane);
            o0 = fmaf(wj, x0.x, o0);
            o1 = fmaf(wj, x0.y, o1);
            o2 = fmaf(wj, x1.x, o2);
            o3 = fmaf(wj, x1.y, o3);
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ll += __shfl_xor_sync(0xffffffffu, ll, off);
    const float inv = ll > 0.0f ? 1.0f / ll : 0.0f;
    const float r[4] = {o0 * inv, o1 * inv, o2 * inv, o3 * inv};
    const int dd[4] = {2 * lane, 2 * lane + 1, 64 + 2 * lane, 65 + 2 * lane};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t oi = row * D + dd[i];
        if (p.q_dtype == F16) ((__half*)p.out)[oi] = __float2half_rn(r[i]);
        else if (p.q_dtype == BF16) ((__nv_bfloat16*)p.out)[oi] = __float2bfloat16_rn(r[i]);
        else ((float*)p.out)[oi] = r[i];
    }
}

int launch_decode_combine(const DecP& p, cudaStream_t st) {
    if (p.D == 128) {
        const int64_t rows = p.B * p.H;
        decode_combine128_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(p);
    } else {
        dim3 g2((unsigned)p.H, (unsigned)p.B);
        decode_combine_kernel<<<g2, (unsigned)p.D, 0, st>>>(p);
    }
    return cuda_failed(cudaGetLastError(), "decode_q8_0 combine launch") ? -1 : 0;
}

template <int D, int GH>
size_t decode_smem() {
    constexpr int ROWB = D / QK * QBYTES;
    return 2 * DEC_STAGES * (size_t)(DEC_TILE * ROWB + 16) + DEC_STAGES * sizeof(uint64_t) +
           (size_t)DEC_WARPS * GH * (D + 2) * sizeof(float);
}

template <int D, int GH>
int run_decode_gh(DecP p, cudaStream_t st) {
    const size_t smem = decode_smem<D, GH>();
    if (cuda_failed(cudaFuncSetAttribute(decode_q8_0_kernel<D, GH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                    "cudaFuncSetAttribute(decode)"))
        return -1;
    // all of the unified L1/shared storage as shared memory: more resident CTAs, more bytes in flight
    if (cuda_failed(cudaFuncSetAttribute(decode_q8_0_kernel<D, GH>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                         (int)cudaSharedmemCarveoutMaxShared),
                    "cudaFuncSetAttribute(decode carveout)"))
        return -1;
    p.nhg = p.G / GH;
    dim3 grid((unsigned)p.nchunks, (unsigned)(p.Hkv * p.nhg), (unsigned)p.B);
    decode_q8_0_kernel<D, GH><<<grid, DEC_WARPS * 32, smem, st>>>(p);
    if (cuda_failed(cudaGetLastError(), "decode_q8_0 launch")) return -1;
    if (p.nchunks > 1 && launch_decode_combine(p, st) != 0) return -1;
    return 0;
}

// Query heads per CTA: the largest of 4, 3, 2, 1 dividing the group (GTB_DECODE_GH caps it, for tuning:
// fewer heads per CTA means fewer registers and more resident CTAs, but K/V are dequantised once
// per head group).
int max_gh() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("GTB_DECODE_GH");
        v = e ? atoi(e) : 4;
        if (v < 1 || v > 4) v = 4;
    }
    return v;
}

template <int D>
int run_decode(DecP p, cudaStream_t st) {
    const int cap = max_gh();
    if (cap >= 4 && p.G % 4 == 0) return run_decode_gh<D, 4>(p, st);
    if (cap >= 3 && p.G % 3 == 0) return run_decode_gh<D, 3>(p, st);
    if (cap >= 2 && p.G % 2 == 0) return run_decode_gh<D, 2>(p, st);
    return run_decode_gh<D, 1>(p, st);
}


}  // namespace

int launch_q8_0_quantize(const void* x, int x_dtype, int64_t nblocks, void* out, cudaStream_t st) {
    if (nblocks == 0) return 0;
    const unsigned grid = (unsigned)((nblocks + 127) / 128);
    switch (x_dtype) {
        case F32: q8_0_quantize_kernel<float><<<grid, 128, 0, st>>>((const float*)x, nblocks, (uint8_t*)out); break;
        case F16: q8_0_quantize_kernel<__half><<<grid, 128, 0, st>>>((const __half*)x, nblocks, (uint8_t*)out); break;
        case BF16: q8_0_quantize_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>((const __nv_bfloat16*)x, nblocks, (uint8_t*)out); break;
        default: set_error("quantize: Q8_0 input must be f32, f16 or bf16"); return -1;
    }
    return cuda_failed(cudaGetLastError(), "q8_0 quantize launch") ? -1 : 0;
}

template <bool ROPE>
void append_launch(const void* x, int x_dtype, unsigned grid, int64_t Hkv, int64_t n_new, int64_t nb_row, uint8_t* c,
                   int64_t Smax, const int32_t* pos, int64_t nblocks, int* status, const RopeArgs& ra, cudaStream_t st) {
    switch (x_dtype) {
        case F32: q8_0_append_kernel<float, ROPE><<<grid, 128, 0, st>>>((const float*)x, Hkv, n_new, nb_row, c, Smax, pos, nblocks, status, ra); break;
        case F16: q8_0_append_kernel<__half, ROPE><<<grid, 128, 0, st>>>((const __half*)x, Hkv, n_new, nb_row, c, Smax, pos, nblocks, status, ra); break;
        default: q8_0_append_kernel<__nv_bfloat16, ROPE><<<grid, 128, 0, st>>>((const __nv_bfloat16*)x, Hkv, n_new, nb_row, c, Smax, pos, nblocks, status, ra); break;
    }
}

int launch_q8_0_append(const void* x, int x_dtype, int64_t B, int64_t Hkv, int64_t n_new, int64_t D, void* cache,
                       int64_t Smax, int32_t* pos, bool advance, const RopeArgs* rope, cudaStream_t st) {
    const int64_t nb_row = D / QK, nblocks = B * Hkv * n_new * nb_row;
    if (x_dtype != F32 && x_dtype != F16 && x_dtype != BF16) {
        set_error("q8_0_append: the new rows must be f32, f16 or bf16");
        return -1;
    }
    int dev = 0;
    cudaGetDevice(&dev);
    int* status = device_status_word(dev);
    if (nblocks > 0) {
        const unsigned grid = (unsigned)((nblocks + 127) / 128);
        uint8_t* c = (uint8_t*)cache;
        if (rope) append_launch<true>(x, x_dtype, grid, Hkv, n_new, nb_row, c, Smax, pos, nblocks, status, *rope, st);
        else append_launch<false>(x, x_dtype, grid, Hkv, n_new, nb_row, c, Smax, pos, nblocks, status, RopeArgs{}, st);
        if (cuda_failed(cudaGetLastError(), "q8_0 append launch")) return -1;
    }
    if (advance && n_new > 0 && B > 0) {
        q8_0_advance_kernel<<<(unsigned)((B + 255) / 256), 256, 0, st>>>(pos, B, (int32_t)n_new);
        if (cuda_failed(cudaGetLastError(), "q8_0 append: length update launch")) return -1;
    }
    return 0;
}

int launch_q8_0_dequantize(const void* blocks, int64_t nblocks, void* out, int out_dtype, cudaStream_t st) {
    const int64_t n = nblocks * QK;
    if (n == 0) return 0;
    const unsigned grid = (unsigned)((n + 255) / 256);
    switch (out_dtype) {
        case F32: q8_0_dequantize_kernel<float><<<grid, 256, 0, st>>>((const uint8_t*)blocks, nblocks, (float*)out); break;
        case F16: q8_0_dequantize_kernel<__half><<<grid, 256, 0, st>>>((const uint8_t*)blocks, nblocks, (__half*)out); break;
        case BF16: q8_0_dequantize_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const uint8_t*)blocks, nblocks, (__nv_bfloat16*)out); break;
        default: set_error("dequantize: output dtype must be f32, f16 or bf16"); return -1;
    }
    return cuda_failed(cudaGetLastError(), "q8_0 dequantize launch") ? -1 : 0;
}

int64_t decode_num_chunks(int64_t Smax) {
    return Smax <= 0 ? 1 : (Smax + GTB_DECODE_CHUNK - 1) / GTB_DECODE_CHUNK;
}

int64_t decode_list_offset(int64_t B) { return 2 * B + 4; }  // in ints, 8-byte aligned: counter, 2 prefixes

size_t decode_work_bytes(int64_t B, int64_t Hkv, int64_t Smax) {
    const int64_t items = B * Hkv * decode_num_chunks(Smax);
    return (size_t)(decode_list_offset(B) * sizeof(int) + items * 2 * sizeof(int) + 255) / 256 * 256;
}

size_t decode_scratch_bytes(int64_t B, int64_t H, int64_t Hkv, int64_t Smax, int64_t D) {
    const int64_t nch = decode_num_chunks(Smax);
    const size_t part = nch <= 1 ? 0 : (size_t)B * Hkv * nch * (H / Hkv) * (D + 2) * sizeof(float);
    return decode_work_bytes(B, Hkv, Smax) + part;
}

int launch_decode_q8_0(const DecodeArgs& a, void* scratch, cudaStream_t st) {
    DecP p;
    p.q = a.q; p.q_dtype = a.q_dtype; p.k = (const uint8_t*)a.k; p.v = (const uint8_t*)a.v;
    p.lens = a.lens; p.out = a.out;
    p.B = a.B; p.H = a.H; p.Hkv = a.Hkv; p.Smax = a.Smax; p.D = a.D; p.G = a.H / a.Hkv;
    p.nchunks = decode_num_chunks(a.Smax);
    p.chunk = GTB_DECODE_CHUNK;
    p.scale_log2 = a.scale * 1.4426950408889634f;
    // rows per 16 bytes: 16 / gcd(row_bytes, 16) (row_bytes = 34 * D/32 is even)
    const int64_t row_bytes = a.D / QK * QBYTES;
    const int64_t low_bit = row_bytes & (-row_bytes);
    p.rows_align = (int)(16 / (low_bit < 16 ? low_bit : 16));
    p.bulk = ((uintptr_t)a.k % 16 == 0) && ((uintptr_t)a.v % 16 == 0) && (a.Smax % p.rows_align == 0);
    p.status = a.status;
    p.nhg = 1;
    if (scratch == nullptr) {
        set_error("decode_q8_0: scratch buffer missing");
        return -1;
    }
    p.part = (float*)((char*)scratch + decode_work_bytes(a.B, a.Hkv, a.Smax));
    const bool mma = decode_mma_supported(a);
    if (mma || decode_sm100_supported(a)) {
        const int rc = mma ? launch_decode_mma(a, (int*)scratch, p.part, p.nchunks, st)
                           : launch_decode_sm100(a, (int*)scratch, p.part, p.nchunks, st);
        if (rc != 0) return -1;
        if (p.nchunks > 1 && launch_decode_combine(p, st) != 0) return -1;
        return 0;
    }
    switch (a.D) {
        case 64: return run_decode<64>(p, st);
        case 128: return run_decode<128>(p, st);
        case 256: return run_decode<256>(p, st);
        default:
            set_errorf("decode_q8_0: head size %lld not supported (64, 128 or 256)", (long long)a.D);
            return -1;
    }
}

}  // namespace gtb
