// Q8_0-cache decode step on the sm_100a tensor cores: one persistent CTA per SM.
//
// The step is the one of gt_flash_decode_q8_0 (an f16 query row per head against the first
// seq_lens[b] rows of GGUF Q8_0 K/V caches, softmax scale applied to q.k, GQA head h -> kv head
// h / (H/Hkv)); the reference computes the same thing by dequantising the caches (gt_quantize /
// gt_tensor_to_dtype, csrc/gt_core.cpp:792-840) and calling gt_flash_attention
// (csrc/gt_ops_nn.cpp:2423-2525).
//
// Work item = (sequence b, kv head hk, chunk of GTB_DECODE_CHUNK cached rows). A one-block plan kernel
// writes the prefix of the per-sequence item counts and zeroes a counter; the producer warp of each
// CTA claims items from that counter and streams them as tiles of 128 cached rows:
//
//   warp 4       producer: claims items, copies the raw Q8_0 rows of K and V (136 B per row at D=128)
//                into a ring of shared-memory stages with cp.async.bulk
//   warps 6-9    K dequantiser, one cached row per thread: the 128 int8 quants -> f16 integers
//                (exact) in a 128-byte-swizzled K-major tile, the 4 block scales kept aside; the q
//                rows of a new item copied into the B operand of S
//   warps 10-13  V dequantiser: the same for V, plus the largest |scale| of the tile
//   warp 5       MMA issuer (one thread): for each Q8_0 block b, S_b = Kx[:, 32b:32b+32] q[:, 32b:32b+32]^T
//                (M = 128 rows, N = query heads padded to 16), and O~ = Vx^T P~ (M = 128 head dims,
//                N = 4 blocks x heads, A read MN-major straight from the row-major V tile)
//   warps 0-3    softmax (thread = cached row): s_h = scale * sum_b dK_b S_b[h], online softmax over
//                the tile, P~[t, (b, h)] = p_h(t) * dV_b(t) * 2^k as f16; then, one tile behind,
//                (thread = head dim d) O_h[d] = O_h[d] * alpha + O~[d, (block(d), h)] * 2^-k
//
// The quants are exact integers in f16, so K's products with the f16 query are exact and each
// (row, block) scale is applied once to an f32 block sum. In PV the scale varies along both the
// reduction (rows) and the output (head dims); it is folded into P~ per block, so O~ has one column
// group per block, of which head dim d keeps its own block's. The per-tile power of two 2^k puts the
// largest |dV| of the tile at 2^14, away from f16 subnormals for small-scale caches (p <= 1).
//
// Phase rule: a parity wait cannot tell phase n from phase n+2, so no barrier may complete twice
// while one of its waiters is still behind. The K tile of i+1 depends only on the softmax of tile
// i-1, so the K-ready barrier is double-buffered by tile parity; the V tile is double-buffered
// (V(i) waits for PV(i-2)), and so are its barriers; every other barrier's next phase needs its
// waiters to have passed (PV needs the softmax, S needs the K tile, ...).
//
// Every mbarrier wait is bounded (about a second); on timeout the kernel records a status code,
// stops, drains its own copies and MMAs with bounded waits, frees TMEM and returns.

#include <cstdio>
#include <cstdlib>

#include "gtb_common.cuh"
#include "q8_0_internal.h"
#include "sm100_ptx.cuh"

namespace gtb {
namespace {

using namespace sm100;

constexpr int TILE = 128;          // cached rows per tile
constexpr int HD = 128;            // head size of this kernel
constexpr int NBLK = HD / 32;      // Q8_0 blocks per row
constexpr int ROWB = NBLK * 34;    // bytes per cached row
constexpr int RAWB = TILE * ROWB;  // raw bytes of a K (or V) tile
constexpr int SLAB = TILE * 128;   // one 64-column slab of a dequantised tile
constexpr int DEQB = 2 * SLAB;     // a dequantised 128 x 128 f16 tile
constexpr int NTHREADS = 448;
constexpr int SMEM_LIMIT = 232448;  // dynamic shared memory per CTA on sm_100
constexpr uint32_t TMEM_COLS = 256;

enum : int { F_FIRST = 1, F_LAST = 2, F_END = 4 };

struct TileMeta {
    int b, hk, chunk, nrows, flags, seq, pad0, pad1;
};

template <int G>
struct DC {
    static constexpr int NS = 16;                           // S columns per block (heads padded)
    static constexpr int NP = ((NBLK * G + 15) / 16) * 16;  // O~ columns
    static constexpr int QSLAB = NS * 128;
    static constexpr int QBUF = 2 * QSLAB;
    static constexpr int PSLAB = NP * 128;
    static constexpr int PBUF = 2 * PSLAB;
    static constexpr int OFF_K = 0;
    static constexpr int OFF_V = DEQB;           // [2] by tile parity
    static constexpr int OFF_Q = 3 * DEQB;       // [2] by item parity
    static constexpr int OFF_P = OFF_Q + 2 * QBUF;  // [2] by tile parity
    static constexpr int OFF_RAW = OFF_P + 2 * PBUF;
    // tail: scales, reductions, metadata, barriers
    static constexpr int T_DK = 0;                    // uint2 [2][TILE]
    static constexpr int T_DV = T_DK + 2 * TILE * 8;  // uint2 [2][TILE]
    static constexpr int T_DVW = T_DV + 2 * TILE * 8; // float [2][4]
    static constexpr int T_RED = T_DVW + 32;          // float [2][4][G]
    static constexpr int T_REDL = T_RED + 2 * 4 * G * 4;  // float [2][4][G]
    static constexpr int T_META = ((T_REDL + 2 * 4 * G * 4) + 31) / 32 * 32;  // TileMeta [2]
    static constexpr int T_SMETA = T_META + 2 * 32;                        // TileMeta [R]
    static constexpr int TAIL_FIXED = T_SMETA + 4 * 32 + 8 * (2 * 4 + 20) + 16;
    static constexpr int TAIL = (TAIL_FIXED + 127) / 128 * 128;
    static constexpr int R0 = (SMEM_LIMIT - 1024 - OFF_RAW - TAIL) / (2 * RAWB);
    static constexpr int R = R0 > 4 ? 4 : R0;  // raw stages
    static_assert(R >= 2, "decode_sm100: not enough shared memory for two stages");
    static constexpr int OFF_TAIL = OFF_RAW + R * 2 * RAWB;
    static constexpr int T_BAR = T_SMETA + R * 32;
    static constexpr int NBAR = 2 * R + 20;
    static constexpr int T_SLOT = T_BAR + NBAR * 8;
    static constexpr int SMEM = OFF_TAIL + TAIL + 1024;
    static_assert(T_SLOT + 8 <= TAIL, "decode_sm100 tail layout");
    static_assert(SMEM <= SMEM_LIMIT, "decode_sm100 shared memory");
    // TMEM columns: S[2] (NBLK * NS each), then O~[2] (NP each)
    static constexpr uint32_t S_COLS = NBLK * NS;
    static_assert(2 * S_COLS + 2 * NP <= (int)TMEM_COLS, "decode_sm100 TMEM columns");
};

struct DecSmParams {
    const __half* q;
    const uint8_t* k;
    const uint8_t* v;
    const int32_t* lens;
    __half* out;
    float* part;  // [B][Hkv][nchunks][G][HD + 2] when nchunks > 1
    int* work;    // [0] item counter, [1 .. B+1] prefix of items per sequence
    int64_t B, H, Hkv, Smax;
    int nchunks, chunk;
    float scale_log2;
    int* status;
};

// the same bounded wait taken by a whole warp: every lane gets the same answer
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* status, int code) {
    const bool ok = mbar_wait(bar, parity, status, code);
    return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, off));
    return x;
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
    return x;
}

__device__ __forceinline__ float half_lo(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu))); }
__device__ __forceinline__ float half_hi(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }

// One cached row (4 Q8_0 blocks: fp16 scale + 32 int8) -> its 128 quants as f16 integers at row t
// of a 128-byte-swizzled tile (two 64-column slabs), and the 4 scales (f16 bits, block b in half b).
// int8 -> f16 without the conversion unit: flip the sign bit (u = x + 128), put u in the low mantissa
// byte of 1024.0 (0x6400 | u = 1024 + u) and subtract 1152. Exact for every int8.
__device__ __forceinline__ uint2 dequant_row(const unsigned char* row, unsigned char* deq, int t) {
    uint32_t w[34];
    const uint2* src = (const uint2*)row;  // rows are 8-byte aligned (136 = 17 * 8)
#pragma unroll
    for (int i = 0; i < 17; ++i) {
        const uint2 x = src[i];
        w[2 * i] = x.x;
        w[2 * i + 1] = x.y;
    }
    // block b starts at byte 34b: scales at bytes 0, 34, 68, 102
    const uint2 scales = make_uint2((w[0] & 0xFFFFu) | (w[8] & 0xFFFF0000u), (w[17] & 0xFFFFu) | (w[25] & 0xFFFF0000u));
    const uint32_t base = smem_u32(deq) + (uint32_t)t * 128u;
#pragma unroll
    for (int b = 0; b < NBLK; ++b) {
        uint32_t qw[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int byte = 34 * b + 2 + 4 * i;  // first quant byte of word i of block b
            const int wi = byte >> 2;
            qw[i] = (byte & 3) == 0 ? w[wi] : __funnelshift_r(w[wi], w[wi + 1], 16);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            uint32_t h[4];
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const uint32_t u = qw[2 * c + k] ^ 0x80808080u;
                const uint32_t lo = __byte_perm(u, 0x64u, 0x4140u);
                const uint32_t hi = __byte_perm(u, 0x64u, 0x4342u);
                asm("sub.f16x2 %0, %1, %2;" : "=r"(h[2 * k]) : "r"(lo), "r"(0x64806480u));
                asm("sub.f16x2 %0, %1, %2;" : "=r"(h[2 * k + 1]) : "r"(hi), "r"(0x64806480u));
            }
            const int chunk = 4 * b + c;  // 16-byte chunk of the row, 0..15
            const uint32_t addr = base + (uint32_t)((chunk >> 3) * SLAB) + (uint32_t)(((chunk & 7) ^ (t & 7)) << 4);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(h[0]), "r"(h[1]), "r"(h[2]),
                         "r"(h[3])
                         : "memory");
        }
    }
    return scales;
}

// Block-wide exclusive scan of one int64 per thread (blockDim.x a multiple of 32, at most 1024);
// returns the exclusive prefix, *total gets the sum.
__device__ __forceinline__ long long block_scan_excl(long long v, long long* wsum, long long* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    long long x = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const long long y = __shfl_up_sync(0xffffffffu, x, off);
        if (lane >= off) x += y;
    }
    if (lane == 31) wsum[warp] = x;
    __syncthreads();
    if (warp == 0) {
        long long s = lane < nw ? wsum[lane] : 0;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const long long y = __shfl_up_sync(0xffffffffu, s, off);
            if (lane >= off) s += y;
        }
        wsum[lane] = s;
    }
    __syncthreads();
    *total = wsum[nw - 1];
    return x - v + (warp > 0 ? wsum[warp - 1] : 0);
}

// One block plans the items of a decode call. work[0] = 0 (the claim counter); work[1 + b] = items of
// sequences < b and work[1 + B] = all items (the tcgen05 kernel maps an item index to its sequence
// with these); work[B + 2 + b] = full-chunk items of sequences < b. The item list at work + list_off
// holds (b, hk << 16 | c): first every full chunk (sequence-major), then the last, partial chunk of
// every sequence, by decreasing size (16 size classes), so that the persistent kernels end on small
// items and their groups run out of work at nearly the same time. Each warp writes the list entries
// of one sequence at a time.
__global__ void decode_plan_kernel(const int32_t* lens, int64_t B, int64_t Smax, int64_t Hkv, int chunk, int* work,
                                   int64_t list_off) {
    constexpr int NCLS = 17;  // size classes of a partial chunk: ceil(16 * rows / chunk), 0 .. 16
    __shared__ long long wsum[32];
    __shared__ int hist[NCLS], cursor[NCLS];
    const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5;
    if (tid < NCLS) hist[tid] = 0;
    __syncthreads();
    const int64_t per = (B + nt - 1) / nt;
    const int64_t b0 = (int64_t)tid * per, b1 = min(B, b0 + per);
    auto seq_len = [&](int64_t b) -> int64_t {
        const int64_t len = lens[b];
        return len < 0 ? 0 : (len > Smax ? Smax : len);
    };
    // per sequence: nch = max(1, ceil(len / chunk)) chunks, of which `full` hold chunk rows
    long long la = 0, lf = 0;
    for (int64_t b = b0; b < b1; ++b) {
        const int64_t len = seq_len(b);
        const int64_t nch = len == 0 ? 1 : (len + chunk - 1) / chunk;
        const int64_t full = len / chunk;
        la += Hkv * nch;
        lf += Hkv * full;
        if (nch > full) atomicAdd(&hist[(int)((16 * (len - full * chunk) + chunk - 1) / chunk)], (int)Hkv);
    }
    long long tot_all, tot_full;
    const long long pa = block_scan_excl((la << 32) | lf, wsum, &tot_all);  // both halves stay below 2^31
    tot_full = tot_all & 0xffffffffll;
    tot_all >>= 32;
    long long ra = pa >> 32, rf = pa & 0xffffffffll;
    for (int64_t b = b0; b < b1; ++b) {
        const int64_t len = seq_len(b);
        work[1 + b] = (int)ra;
        work[B + 2 + b] = (int)rf;
        ra += Hkv * (len == 0 ? 1 : (len + chunk - 1) / chunk);
        rf += Hkv * (len / chunk);
    }
    if (tid == 0) {
        work[0] = 0;
        work[1 + B] = (int)tot_all;
        work[2 * B + 2] = (int)tot_full;
        int start = (int)tot_full;  // partial chunks after the full ones, largest class first
        for (int k = NCLS - 1; k >= 0; --k) {
            cursor[k] = start;
            start += hist[k];
        }
    }
    __syncthreads();  // the prefixes (global, written by this block) and the cursors are visible
    int2* list = (int2*)(work + list_off);
    for (int64_t b = warp; b < B; b += nt >> 5) {
        const int64_t len = seq_len(b);
        const int full = (int)(len / chunk);
        const int nfull = full * (int)Hkv;
        const int base = work[B + 2 + b];
        for (int j = lane; j < nfull; j += 32) list[base + j] = make_int2((int)b, ((j / full) << 16) | (j % full));
        const int64_t nch = len == 0 ? 1 : (len + chunk - 1) / chunk;
        if (nch > full) {
            int pos = 0;
            if (lane == 0) pos = atomicAdd(&cursor[(int)((16 * (len - (int64_t)full * chunk) + chunk - 1) / chunk)], (int)Hkv);
            pos = __shfl_sync(0xffffffffu, pos, 0);
            for (int hk = lane; hk < Hkv; hk += 32) list[pos + hk] = make_int2((int)b, (hk << 16) | full);
        }
    }
}

template <int G>
__global__ void __launch_bounds__(NTHREADS, 1) decode_sm100_kernel(const DecSmParams p) {
    using C = DC<G>;
    constexpr int R = C::R;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    unsigned char* kdeq = smem + C::OFF_K;
    unsigned char* vdeq = smem + C::OFF_V;
    unsigned char* qbuf = smem + C::OFF_Q;
    unsigned char* pbuf = smem + C::OFF_P;
    unsigned char* raw = smem + C::OFF_RAW;
    unsigned char* tail = smem + C::OFF_TAIL;
    uint2* dks = (uint2*)(tail + C::T_DK);
    uint2* dvs = (uint2*)(tail + C::T_DV);
    float* dvw = (float*)(tail + C::T_DVW);
    float* red = (float*)(tail + C::T_RED);
    float* redl = (float*)(tail + C::T_REDL);
    TileMeta* meta = (TileMeta*)(tail + C::T_META);
    TileMeta* smeta = (TileMeta*)(tail + C::T_SMETA);
    uint64_t* bars = (uint64_t*)(tail + C::T_BAR);
    uint64_t* full = bars;              // [R] raw stage loaded (producer + tx bytes)
    uint64_t* empty = full + R;         // [R] raw stage consumed (256 dequantiser threads)
    uint64_t* k_full = empty + R;       // [2] by tile parity: K tile dequantised (128)
    uint64_t* k_empty = k_full + 2;     // S MMAs done with the K tile (commit)
    uint64_t* v_full = k_empty + 1;     // [2] by tile parity: V tile dequantised (128)
    uint64_t* v_empty = v_full + 2;     // [2] PV MMAs done with the V tile (commit)
    uint64_t* s_full = v_empty + 2;     // [2] S computed (commit)
    uint64_t* p_full = s_full + 2;      // [2] P~ written, S read (128)
    uint64_t* o_full = p_full + 2;      // [2] O~ computed (commit)
    uint64_t* o_empty = o_full + 2;     // [2] O~ read (128)
    uint64_t* red_bar = o_empty + 2;    // [2] per-warp tile maxima written (4)
    uint64_t* redl_bar = red_bar + 2;   // [2] per-warp row sums of a finished item written (4)
    uint64_t* drain = redl_bar + 2;     // error path
    uint32_t* tmem_slot = (uint32_t*)(tail + C::T_SLOT);
    int* abort_flag = (int*)(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < R; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 256); }
        mbar_init(&k_full[0], 128); mbar_init(&k_full[1], 128); mbar_init(k_empty, 1);
        for (int j = 0; j < 2; ++j) { mbar_init(&v_full[j], 128); mbar_init(&v_empty[j], 1); }
        for (int j = 0; j < 2; ++j) {
            mbar_init(&s_full[j], 1); mbar_init(&p_full[j], 128);
            mbar_init(&o_full[j], 1); mbar_init(&o_empty[j], 128);
            mbar_init(&red_bar[j], 4); mbar_init(&redl_bar[j], 4);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    // q buffers: the rows past the group's heads stay zero
    for (int i = threadIdx.x; i < 2 * C::QBUF / 16; i += NTHREADS) ((uint4*)qbuf)[i] = make_uint4(0, 0, 0, 0);
    fence_proxy_async_smem();
    if (warp == 5) tmem_alloc(tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const int* prefix = p.work + 1;
            const int total = prefix[p.B];
            int n = 0, seq = 0;
            bool ok = true;
            while (ok) {
                const int item = atomicAdd(p.work, 1);
                if (item >= total) break;
                int lo = 0, hi = (int)p.B - 1;  // last sequence whose first item is <= item
                while (lo < hi) {
                    const int mid = (lo + hi + 1) >> 1;
                    if (prefix[mid] <= item) lo = mid; else hi = mid - 1;
                }
                const int b = lo;
                const int nch = (prefix[b + 1] - prefix[b]) / (int)p.Hkv;
                const int rem = item - prefix[b];
                const int hk = rem / nch, chunk = rem % nch;
                int64_t len = p.lens[b];
                len = len < 0 ? 0 : (len > p.Smax ? p.Smax : len);
                const int64_t c0 = (int64_t)chunk * p.chunk;
                const int64_t c1 = min(len, c0 + p.chunk);
                const int nt = c1 > c0 ? (int)((c1 - c0 + TILE - 1) / TILE) : 1;
                const uint8_t* kb = p.k + ((int64_t)b * p.Hkv + hk) * p.Smax * ROWB;
                const uint8_t* vb = p.v + ((int64_t)b * p.Hkv + hk) * p.Smax * ROWB;
                for (int t = 0; t < nt; ++t) {
                    const int s = n % R;
                    if (n >= R) ok = mbar_wait(&empty[s], ((n / R) - 1) & 1, p.status, 41);
                    if (!ok || *(volatile int*)abort_flag) { ok = false; break; }
                    const int64_t r0 = c0 + (int64_t)t * TILE;
                    const int nrows = (int)max((int64_t)0, min((int64_t)TILE, c1 - r0));
                    TileMeta& m = smeta[s];
                    m.b = b; m.hk = hk; m.chunk = chunk; m.nrows = nrows; m.seq = seq;
                    m.flags = (t == 0 ? F_FIRST : 0) | (t == nt - 1 ? F_LAST : 0);
                    // whole row pairs: 2 * 136 bytes is a multiple of 16, and Smax is even on this path
                    const uint32_t bytes = (uint32_t)(((nrows + 1) & ~1) * ROWB);
                    unsigned char* kd = raw + s * 2 * RAWB;
                    unsigned char* vd = kd + RAWB;
                    const uint8_t* ks = kb + r0 * ROWB;
                    const uint8_t* vs = vb + r0 * ROWB;
                    if (bytes == 0 || (((uintptr_t)ks | (uintptr_t)vs | (uintptr_t)smem_u32(kd) | (uintptr_t)smem_u32(vd) |
                                        bytes) & 15) != 0) {
                        if (bytes != 0 && p.status) atomicExch(p.status, 2);  // never issue a misaligned copy
                        mbar_arrive(&full[s]);
                    } else {
                        mbar_expect_tx(&full[s], 2 * bytes);
                        bulk_load(kd, ks, bytes, &full[s]);
                        bulk_load(vd, vs, bytes, &full[s]);
                    }
                    ++n;
                }
                ++seq;
            }
            if (ok && !*(volatile int*)abort_flag) {
                const int s = n % R;
                if (n >= R) ok = mbar_wait(&empty[s], ((n / R) - 1) & 1, p.status, 43);
                if (ok) {
                    smeta[s].flags = F_END;
                    mbar_arrive(&full[s]);
                    ++n;
                }
            }
            if (!ok) *(volatile int*)abort_flag = 1;
            if (*(volatile int*)abort_flag) {
                for (int j = max(0, n - R); j < n; ++j) mbar_wait(&full[j % R], (j / R) & 1, nullptr, 0);
            }
        }
    } else if (warp == 5) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t IDESC_S = idesc_f16(128, C::NS, false, false);
            constexpr uint32_t IDESC_PV = idesc_f16_amn(128, C::NP, false, false);
            const uint32_t ka = smem_u32(kdeq), va = smem_u32(vdeq), qa = smem_u32(qbuf), pa = smem_u32(pbuf);
            auto issue_s = [&](int i) {
                const int par = i & 1;
                const uint32_t qb = qa + (uint32_t)((meta[par].seq & 1) * C::QBUF);
#pragma unroll
                for (int b = 0; b < NBLK; ++b) {
#pragma unroll
                    for (int kk = 0; kk < 2; ++kk) {
                        const int ks = 2 * b + kk;  // 16-column step along the head dim
                        const uint64_t ad = desc_sw128(ka + (ks >> 2) * SLAB + (ks & 3) * 32, 16, 1024);
                        const uint64_t bd = desc_sw128(qb + (ks >> 2) * C::QSLAB + (ks & 3) * 32, 16, 1024);
                        mma_ss(tmem + par * C::S_COLS + b * C::NS, ad, bd, IDESC_S, (uint32_t)kk);
                    }
                }
                mma_commit(&s_full[par]);
                mma_commit(k_empty);
            };
            auto issue_pv = [&](int i) {
                const int par = i & 1;
                const uint32_t pb = pa + (uint32_t)(par * C::PBUF);
                const uint32_t vb = va + (uint32_t)(par * DEQB);
#pragma unroll
                for (int kk = 0; kk < TILE / 16; ++kk) {
                    const uint64_t ad = desc_sw128(vb + kk * 2048, SLAB, 1024);  // MN-major: rows of the tile along K
                    const uint64_t bd = desc_sw128(pb + (kk >> 2) * C::PSLAB + (kk & 3) * 32, 16, 1024);
                    mma_ss(tmem + 2 * C::S_COLS + par * C::NP, ad, bd, IDESC_PV, kk > 0 ? 1u : 0u);
                }
                mma_commit(&o_full[par]);
                mma_commit(&v_empty[par]);
            };
            // Issue S(ns) as soon as its K tile is ready and PV(np) as soon as its P~ and V tile are,
            // in order within each kind. S(ns) reuses the S columns of tile ns-2, free once PV(ns-2)
            // was issued (which waited for the softmax of ns-2). No progress for ~2^31 cycles -> error.
            bool ok = true;
            int ns = 0, np = 0, end_tile = 0x7fffffff;
            long long t_last = clock64();
            while (np < end_tile) {
                bool progressed = false;
                if (ns < end_tile && ns <= np + 1 && mbar_test(&k_full[ns & 1], (ns >> 1) & 1)) {
                    if (meta[ns & 1].flags & F_END) {
                        end_tile = ns;
                    } else {
                        tc_fence_after();
                        issue_s(ns);
                        ++ns;
                    }
                    progressed = true;
                }
                if (np < ns && mbar_test(&p_full[np & 1], (np >> 1) & 1) && mbar_test(&v_full[np & 1], (np >> 1) & 1) &&
                    (np < 2 || mbar_test(&o_empty[np & 1], ((np - 2) >> 1) & 1))) {
                    tc_fence_after();
                    issue_pv(np);
                    ++np;
                    progressed = true;
                }
                if (progressed) {
                    t_last = clock64();
                } else if (clock64() - t_last > (1ll << 31)) {
                    if (p.status) atomicCAS(p.status, 0, 61);
                    ok = false;
                    break;
                }
                if (*(volatile int*)abort_flag) break;
            }
            if (!ok) *(volatile int*)abort_flag = 1;
            if (*(volatile int*)abort_flag) {
                mma_commit(drain);  // wait (bounded) for every MMA issued before TMEM is freed
                mbar_wait(drain, 0, nullptr, 0);
            }
        }
    } else if (warp >= 6) {
        // ------------------------------------------------------------ dequantisers
        const bool is_k = warp < 10;
        const int r = (warp - (is_k ? 6 : 10)) * 32 + lane;  // cached row of the tile
        unsigned char* deq = is_k ? kdeq : vdeq;
        bool ok = true;
        for (int i = 0;; ++i) {
            const int s = i % R;
            ok = warp_wait(&full[s], (i / R) & 1, p.status, is_k ? 71 : 81);
            if (!ok || *(volatile int*)abort_flag) break;
            const TileMeta m = smeta[s];
            const int par = i & 1;
            if (is_k) {
                if (i >= 1) ok = warp_wait(k_empty, (i - 1) & 1, p.status, 72);
                if (ok && i >= 2) ok = warp_wait(&p_full[par], ((i - 2) >> 1) & 1, p.status, 73);
                if (!ok) break;
                if (m.flags & F_END) {
                    if (r == 0) meta[par] = m;
                    mbar_arrive(&k_full[par]);
                    break;
                }
                if (m.flags & F_FIRST) {
                    // q rows of the item's heads -> rows 0..G-1 of the S operand (K-major, 128-byte swizzle)
                    unsigned char* qd = qbuf + (m.seq & 1) * C::QBUF;
                    for (int c = r; c < G * 16; c += 128) {
                        const int g = c >> 4, cc = c & 15;
                        const uint4 x = *(const uint4*)(p.q + ((int64_t)m.b * p.H + (int64_t)m.hk * G + g) * HD + cc * 8);
                        *(uint4*)(qd + (cc >> 3) * C::QSLAB + g * 128 + (((cc & 7) ^ (g & 7)) << 4)) = x;
                    }
                }
                dks[par * TILE + r] = dequant_row(raw + s * 2 * RAWB + r * ROWB, deq, r);
                if (r == 0) meta[par] = m;
                fence_proxy_async_smem();
                mbar_arrive(&k_full[par]);
                mbar_arrive(&empty[s]);
            } else {
                if (m.flags & F_END) break;
                if (i >= 2) ok = warp_wait(&v_empty[par], ((i - 2) >> 1) & 1, p.status, 82);
                if (!ok) break;
                const uint2 sc = dequant_row(raw + s * 2 * RAWB + RAWB + r * ROWB, deq + par * DEQB, r);
                dvs[par * TILE + r] = sc;
                float mx = 0.0f;
                if (r < m.nrows)
                    mx = fmaxf(fmaxf(fabsf(half_lo(sc.x)), fabsf(half_hi(sc.x))), fmaxf(fabsf(half_lo(sc.y)), fabsf(half_hi(sc.y))));
                mx = warp_max(mx);
                if (lane == 0) dvw[par * 4 + warp - 10] = mx;
                __syncwarp();
                fence_proxy_async_smem();
                mbar_arrive(&v_full[par]);
                mbar_arrive(&empty[s]);
            }
        }
        if (!ok) *(volatile int*)abort_flag = 1;
    } else if (warp < 4) {
        // ------------------------------------------------------------ softmax and accumulation
        const int u = warp * 32 + lane;  // cached row (softmax) / head dim (accumulation)
        const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
        float m_run[G], l_run[G], m_fin[G], l_fin[G], o[G], a_prev[G], alpha[G];
#pragma unroll
        for (int h = 0; h < G; ++h) {
            m_run[h] = -INFINITY; l_run[h] = 0.0f; m_fin[h] = -INFINITY; l_fin[h] = 0.0f;
            o[h] = 0.0f; a_prev[h] = 0.0f; alpha[h] = 0.0f;
        }
        float invf_prev = 1.0f, invf = 1.0f;
        bool have_prev = false, prev_last = false, ok = true;
        int fb = 0, fhk = 0, fch = 0, nfin = 0;
        for (int i = 0;; ++i) {
            const int par = i & 1;
            ok = warp_wait(&k_full[par], (i >> 1) & 1, p.status, 51);
            if (!ok || *(volatile int*)abort_flag) break;
            const TileMeta m = meta[par];
            const bool end = (m.flags & F_END) != 0;
            if (!end) {
                if (m.flags & F_FIRST) {
#pragma unroll
                    for (int h = 0; h < G; ++h) { m_run[h] = -INFINITY; l_run[h] = 0.0f; }
                }
                ok = warp_wait(&s_full[par], (i >> 1) & 1, p.status, 52);
                if (!ok) break;
                tc_fence_after();
                float sb[NBLK][G];
#pragma unroll
                for (int b = 0; b < NBLK; ++b)
                    tmem_ldx<G>(tmem + lane_base + par * C::S_COLS + b * C::NS, (uint32_t*)sb[b]);
                tmem_ld_wait();
                const uint2 dk2 = dks[par * TILE + u];
                const float dk[4] = {half_lo(dk2.x), half_hi(dk2.x), half_lo(dk2.y), half_hi(dk2.y)};
                const bool valid = u < m.nrows;
                float sc[G];
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    float a = dk[0] * sb[0][h];
#pragma unroll
                    for (int b = 1; b < NBLK; ++b) a = fmaf(dk[b], sb[b][h], a);
                    sc[h] = valid ? a * p.scale_log2 : -INFINITY;
                }
                // tile maxima of the 4 warps, exchanged through shared memory (double-buffered by tile parity)
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    const float mx = warp_max(sc[h]);
                    if (lane == 0) red[(par * 4 + warp) * G + h] = mx;
                }
                if (lane == 0) mbar_arrive(&red_bar[par]);
                ok = warp_wait(&red_bar[par], (i >> 1) & 1, p.status, 55);
                if (!ok) break;
                float pr[G];
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    const float mt = fmaxf(fmaxf(red[(par * 4 + 0) * G + h], red[(par * 4 + 1) * G + h]),
                                           fmaxf(red[(par * 4 + 2) * G + h], red[(par * 4 + 3) * G + h]));
                    const float m_new = fmaxf(m_run[h], mt);
                    const float neg = m_new == -INFINITY ? 0.0f : -m_new;
                    alpha[h] = ex2(m_run[h] + neg);  // 0 while nothing has been accumulated
                    pr[h] = ex2(sc[h] + neg);        // 0 for masked rows
                    l_run[h] = fmaf(l_run[h], alpha[h], pr[h]);
                    m_run[h] = m_new;
                }
                ok = warp_wait(&v_full[par], (i >> 1) & 1, p.status, 53);
                if (!ok) break;
                const float* dw = dvw + par * 4;
                const float dvmax = fmaxf(fmaxf(dw[0], dw[1]), fmaxf(dw[2], dw[3]));
                float f = 1.0f;
                invf = 1.0f;
                if (dvmax > 0.0f) {  // dvmax * f in [2^14, 2^15)
                    const int e = (int)((__float_as_uint(dvmax) >> 23) & 0xFF) - 127;
                    f = __uint_as_float((uint32_t)(127 + 14 - e) << 23);
                    invf = __uint_as_float((uint32_t)(127 - 14 + e) << 23);
                }
                const uint2 dv2 = dvs[par * TILE + u];
                const float dv[4] = {half_lo(dv2.x) * f, half_hi(dv2.x) * f, half_lo(dv2.y) * f, half_hi(dv2.y) * f};
                unsigned char* pb = pbuf + par * C::PBUF + (u >> 6) * C::PSLAB + (u & 7) * 2;
                const int chunk16 = (u & 63) >> 3;
#pragma unroll
                for (int b = 0; b < NBLK; ++b) {
#pragma unroll
                    for (int h = 0; h < G; ++h) {
                        const int n = b * G + h;
                        const float val = valid ? pr[h] * dv[b] : 0.0f;
                        *(__half*)(pb + n * 128 + ((chunk16 ^ (n & 7)) << 4)) = __float2half_rn(val);
                    }
                }
                fence_proxy_async_smem();
                tc_fence_before();
                mbar_arrive(&p_full[par]);
            }
            if (have_prev) {
                // accumulate tile i-1: O~ column (block of this head dim, h)
                const int pp = (i - 1) & 1;
                ok = warp_wait(&o_full[pp], ((i - 1) >> 1) & 1, p.status, 54);
                if (!ok) break;
                tc_fence_after();
                float tv[G];
                tmem_ldx<G>(tmem + lane_base + 2 * C::S_COLS + pp * C::NP + warp * G, (uint32_t*)tv);
                tmem_ld_wait();
                tc_fence_before();
                mbar_arrive(&o_empty[pp]);
#pragma unroll
                for (int h = 0; h < G; ++h) o[h] = fmaf(o[h], a_prev[h], tv[h] * invf_prev);
                if (prev_last) {
                    // item done: reduce the row sums, write the (normalised or partial) result
                    float lsum[G];
                    const int fp = nfin & 1;
                    float* rl = redl + fp * 4 * G;
#pragma unroll
                    for (int h = 0; h < G; ++h) {
                        const float x = warp_sum(l_fin[h]);
                        if (lane == 0) rl[warp * G + h] = x;
                    }
                    if (lane == 0) mbar_arrive(&redl_bar[fp]);
                    ok = warp_wait(&redl_bar[fp], (nfin >> 1) & 1, p.status, 56);
                    if (!ok) break;
                    ++nfin;
#pragma unroll
                    for (int h = 0; h < G; ++h)
                        lsum[h] = (rl[0 * G + h] + rl[1 * G + h]) + (rl[2 * G + h] + rl[3 * G + h]);
#pragma unroll
                    for (int h = 0; h < G; ++h) {
                        const int64_t head = (int64_t)fhk * G + h;
                        if (p.nchunks == 1) {
                            const float r = lsum[h] > 0.0f ? o[h] / lsum[h] : 0.0f;
                            p.out[((int64_t)fb * p.H + head) * HD + u] = __float2half_rn(r);
                        } else {
                            float* pp2 = p.part + ((((int64_t)fb * p.Hkv + fhk) * p.nchunks + fch) * G + h) * (HD + 2);
                            pp2[u] = o[h];
                            if (u == 0) { pp2[HD] = m_fin[h]; pp2[HD + 1] = lsum[h]; }
                        }
                        o[h] = 0.0f;
                    }
                }
            }
            if (end) break;
            have_prev = true;
            prev_last = (m.flags & F_LAST) != 0;
            invf_prev = invf;
#pragma unroll
            for (int h = 0; h < G; ++h) a_prev[h] = alpha[h];
            if (prev_last) {
#pragma unroll
                for (int h = 0; h < G; ++h) { m_fin[h] = m_run[h]; l_fin[h] = l_run[h]; }
                fb = m.b; fhk = m.hk; fch = m.chunk;
            }
        }
        if (!ok) *(volatile int*)abort_flag = 1;
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

int num_sms(int dev) {
    static int cache[64] = {0};
    if (dev < 0 || dev >= 64) return 148;
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

template <int G>
int run_decode_sm100(const DecodeArgs& a, int* work, float* part, int64_t nchunks, cudaStream_t st) {
    using C = DC<G>;
    if (cuda_failed(cudaFuncSetAttribute(decode_sm100_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM),
                    "cudaFuncSetAttribute(decode_sm100)"))
        return -1;
    if (launch_decode_plan(a, work, st) != 0) return -1;
    DecSmParams p;
    p.q = (const __half*)a.q;
    p.k = (const uint8_t*)a.k;
    p.v = (const uint8_t*)a.v;
    p.lens = a.lens;
    p.out = (__half*)a.out;
    p.part = part;
    p.work = work;
    p.B = a.B; p.H = a.H; p.Hkv = a.Hkv; p.Smax = a.Smax;
    p.nchunks = (int)nchunks;
    p.chunk = GTB_DECODE_CHUNK;
    p.scale_log2 = a.scale * 1.4426950408889634f;
    p.status = a.status;
    int dev = 0;
    cudaGetDevice(&dev);
    const int64_t max_items = a.B * a.Hkv * nchunks;
    const int grid = (int)min((int64_t)num_sms(dev), max_items);
    decode_sm100_kernel<G><<<grid, NTHREADS, C::SMEM, st>>>(p);
    return cuda_failed(cudaGetLastError(), "decode_sm100 launch") ? -1 : 0;
}

}  // namespace

int launch_decode_plan(const DecodeArgs& a, int* work, cudaStream_t st) {
    decode_plan_kernel<<<1, 1024, 0, st>>>(a.lens, a.B, a.Smax, a.Hkv, GTB_DECODE_CHUNK, work, decode_list_offset(a.B));
    return cuda_failed(cudaGetLastError(), "decode plan launch") ? -1 : 0;
}

bool decode_sm100_supported(const DecodeArgs& a) {
    static const int force_simt = [] {
        const char* e = getenv("GTB_DECODE_SIMT");
        return e ? atoi(e) : 0;
    }();
    const int64_t G = a.Hkv > 0 ? a.H / a.Hkv : 0;
    return !force_simt && a.D == HD && a.q_dtype == F16 && (G == 1 || G == 2 || G == 4 || G == 8) &&
           a.Smax > 0 && a.Smax % 2 == 0 && ((uintptr_t)a.q % 16 == 0) && ((uintptr_t)a.k % 16 == 0) &&
           ((uintptr_t)a.v % 16 == 0) && a.B * a.Hkv * decode_num_chunks(a.Smax) < (int64_t)INT32_MAX && a.B < INT32_MAX &&
           a.Hkv < 32768 && decode_num_chunks(a.Smax) < 65536;
}

int launch_decode_sm100(const DecodeArgs& a, int* work, float* part, int64_t nchunks, cudaStream_t st) {
    switch (a.H / a.Hkv) {
        case 1: return run_decode_sm100<1>(a, work, part, nchunks, st);
        case 2: return run_decode_sm100<2>(a, work, part, nchunks, st);
        case 4: return run_decode_sm100<4>(a, work, part, nchunks, st);
        case 8: return run_decode_sm100<8>(a, work, part, nchunks, st);
        default: set_error("decode_sm100: unsupported group size"); return -1;
    }
}

}  // namespace gtb
