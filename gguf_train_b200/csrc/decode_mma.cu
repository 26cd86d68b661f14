// Q8_0-cache decode step, memory-bound design: warp-level tensor-core MMAs on registers.
//
// The step is the one of gt_flash_decode_q8_0 (an f16 query row per head against the first
// seq_lens[b] rows of GGUF Q8_0 K/V caches, softmax scale applied to q.k, GQA head h -> kv head
// h / (H/Hkv)); the reference computes the same thing by dequantising the caches (gt_quantize /
// gt_tensor_to_dtype, csrc/gt_core.cpp:792-840) and calling gt_flash_attention
// (csrc/gt_ops_nn.cpp:2423-2525).
//
// Why this shape: per cached row the work is tiny (G = H/Hkv query heads, 2 x 4 x G x D FLOP), so the
// kernel must stream the cache at HBM speed with as few instructions per byte as possible. A
// tcgen05.mma of M = 128 occupies the tensor core for ~100 cycles whatever N is, and decode's shapes
// (N = heads) would pad it 8x; the warp-level m16n8k16 MMA pads 2x at most. Its rows are the
// (Q8_0 block b, head h) pairs, r = b * G + h (16 rows for G = 4):
//
//   S'[r, t]  = sum over d in block b of q_h[d] * Kx[t, d]   (A = block-diagonal q, B = int8 quants as f16)
//   s_h(t)    = scale * sum_b dK(t, b) * S'[b*G + h, t]       (the Q8_0 scale of each (row, block), in f32)
//   P~[r, t]  = p_h(t) * dV(t, b) * f                         (f = 2^k per warp keeps P~ in the f16 range)
//   O[r, d]  += P~[r, t] * Vx[t, d]                           (head dim d keeps row b(d)*G + h)
//
// The quants are exact integers in f16 (int8 -> f16 by a byte permute into 1024.0 + u; for K the
// bias 1152 is left in and removed after the MMA), so the products with the f16 query are exact;
// accumulation is f32.
//
// PV runs transposed, O^T[d, r] = Vx^T[d, t] P~^T[t, r], so that P~ (in the accumulator layout of
// S') is directly the B operand and each 16 head dims need one MMA with the 8 operand rows of their
// own Q8_0 block.
//
// Work: items (sequence b, kv head hk, chunk of GTB_DECODE_CHUNK rows) from the compacted list of the
// plan kernel (decode_sm100.cu), claimed through an atomic counter. The 8 consumer warps form two
// groups of 4 with their own items, their own 2-stage ring and their own producer warp, so that the
// groups' phases interleave; a producer streams 128-row tiles of raw K/V rows (and the item's q rows)
// into its ring with cp.async.bulk (issuing a tile's copies takes the issuing thread ~1000 cycles, so
// one producer per ring keeps a ring from waiting behind the other's issue). Warp wi of a group owns rows [32 wi, 32 wi + 32) of its tiles, as two
// 16-row slices: K fragments come straight from the raw rows (two int8 -> f16x2 per load), V rows are
// dequantised into a private f16 slice and read back transposed with ldmatrix. No barrier spans warps
// inside an item; at its end the group's 4 partial (max, sum, out) are merged through shared memory.
//
// Every mbarrier wait is bounded (about a second); on timeout the kernel records a status code and
// stops, draining its own copies with bounded waits before it returns.

#include <cstdio>
#include <cstdlib>

#include "gtb_common.cuh"
#include "q8_0_internal.h"
#include "sm100_ptx.cuh"

namespace gtb {
namespace {

using namespace sm100;

#ifndef GTB_DECODE_GROUPS
#define GTB_DECODE_GROUPS 3
#endif
#ifndef GTB_DECODE_SLICES
#define GTB_DECODE_SLICES 1
#endif
constexpr int HD = 128;             // head size
constexpr int NBLK = HD / 32;       // Q8_0 blocks per row
constexpr int ROWB = NBLK * 34;     // bytes per cached row
constexpr int NGRP = GTB_DECODE_GROUPS;  // consumer groups, each with its own items and stage ring
constexpr int GW = 4;               // warps per group
constexpr int SPW = GTB_DECODE_SLICES;   // 16-row slices per warp and tile
constexpr int TILE = GW * 16 * SPW; // cached rows per tile: warp wi owns rows [16 SPW wi, 16 SPW (wi + 1))
constexpr int RAWB = TILE * ROWB;   // raw bytes of a K (or V) tile
constexpr int NCW = NGRP * GW;
constexpr int RS = 3;               // stages per group ring
constexpr int NTHREADS = (NCW + NGRP) * 32;  // + one producer warp per group
static_assert(GTB_DECODE_CHUNK % TILE == 0, "tiles must divide a chunk");
constexpr int SMEM_LIMIT = 232448;

enum : int { F_FIRST = 1, F_LAST = 2, F_END = 4 };

// In-kernel plan (batches of at most FOLD_MAX_B sequences): every CTA derives the item order of the
// plan kernel (decode_sm100.cu) from the lengths in shared memory, so the step needs no plan launch,
// only a zeroed claim counter. Tables: full chunks [B], size class [B], full-item prefix [B + 1],
// partial-chunk sequences in list order [B], class starts [17], then full items and all items.
constexpr int FOLD_MAX_B = 256;
constexpr int PLAN_INTS = 4 * FOLD_MAX_B + 1 + 17 + 2;

struct TileMeta {
    int b, hk, chunk, nrows, flags, seq, pad0, pad1;
};

template <int G>
struct MC {
    static constexpr int QB = G * HD * 2;                        // q rows of the item's heads
    static constexpr int STAGE = 2 * RAWB + ((QB + 127) / 128) * 128;
    static constexpr int VST = 16 * 256;                         // per warp: one 16-row slice of V as f16
    // at the end of an item a warp's VST holds its partial: out [h][d] f32, then m [h], l [h]
    static_assert(G * HD * 4 + 2 * G * 4 <= VST, "decode_mma: partial does not fit the V slice buffer");
    static constexpr int OFF_RAW = 0;                            // [NGRP][RS] stages
    static constexpr int OFF_VST = OFF_RAW + NGRP * RS * STAGE;
    static constexpr int OFF_META = OFF_VST + NCW * VST;         // TileMeta [NGRP][RS]
    static constexpr int OFF_BAR = OFF_META + NGRP * RS * 32;
    static constexpr int NBAR = 2 * NGRP * RS + 2 * NGRP;        // full, empty [NGRP][RS]; mrg_full, mrg_done [NGRP]
    static constexpr int OFF_PLAN = OFF_BAR + NBAR * 8 + 16;     // item tables of the in-kernel plan
    static constexpr int SMEM = OFF_PLAN + PLAN_INTS * 4 + 128;
    static_assert(SMEM <= SMEM_LIMIT, "decode_mma shared memory");
};

struct DecMmaParams {
    const __half* q;
    const uint8_t* k;
    const uint8_t* v;
    const int32_t* lens;
    __half* out;
    float* part;  // [B][Hkv][nchunks][G][HD + 2] when nchunks > 1
    int* work;    // [0] item counter, [1 .. B+1] prefix of items per sequence (plan kernel)
    int fold;     // 1: no plan kernel ran; the item order is derived in the kernel (B <= FOLD_MAX_B)
    const int2* items;  // item list (b, hk << 16 | chunk), written by the plan kernel
    int64_t B, H, Hkv, Smax;
    int nchunks, chunk;
    float scale_log2;
    int* status;
};

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* status, int code) {
    const bool ok = mbar_wait(bar, parity, status, code);
    return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ float half_lo(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu))); }
__device__ __forceinline__ float half_hi(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }

__device__ __forceinline__ uint32_t pack_f16(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// D = A (16x16, row) * B (16x8, col) + D, f16 inputs, f32 accumulation
__device__ __forceinline__ void mma16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t lds_u16(const unsigned char* p) {
    uint32_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)));
    return v;
}

// two int8 (low 16 bits of x) -> f16x2 of the biased integers 1152 + x: flip the sign bits
// (u = x + 128) and place u in the low byte of 1024.0 (0x6400 | u = 1024 + u). Exact for every int8;
// the bias is removed after the MMA (1152 * the sum of the other operand over the reduction).
__device__ __forceinline__ uint32_t i8x2_to_f16x2_biased(uint32_t x) {
    return __byte_perm(x ^ 0x8080u, 0x64u, 0x4140u);
}

// Half of a cached row (Q8_0 blocks 2*hb and 2*hb+1: 68 bytes starting at row + 68*hb) -> 64 f16
// biased integers 1152 + x (exact; the bias is removed once per item, see vbias) at row r of a 16-row tile of 256-byte rows whose 16-byte chunks are XOR-swizzled by
// (r >> 1) & 7 (ldmatrix reads the even and the odd rows as separate 8-row matrices); returns the
// two scales.
__device__ __forceinline__ float2 dequant_half_row(const unsigned char* row, int hb, uint32_t out_row, int r) {
    uint32_t w[17];
    const uint32_t* src = (const uint32_t*)(row + 68 * hb);  // 4-byte aligned (136 and 68 are multiples of 4)
#pragma unroll
    for (int i = 0; i < 17; ++i) w[i] = src[i];
    const float2 sc = make_float2(half_lo(w[0]), half_hi(w[8]));  // scales at local bytes 0 and 34
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        uint32_t qw[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int byte = 34 * j + 2 + 4 * i;
            const int wi = byte >> 2;
            qw[i] = (byte & 3) == 0 ? w[wi] : __funnelshift_r(w[wi], w[wi + 1], 16);
        }
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
            uint32_t h[4];
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const uint32_t u = qw[2 * cc + k] ^ 0x80808080u;  // x + 128 in each byte
                h[2 * k] = __byte_perm(u, 0x64u, 0x4140u);          // 1024 + (x + 128) as f16
                h[2 * k + 1] = __byte_perm(u, 0x64u, 0x4342u);
            }
            const int chunk = 4 * (2 * hb + j) + cc;
            const uint32_t addr = out_row + (uint32_t)((chunk ^ ((r >> 1) & 7)) << 4);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(h[0]), "r"(h[1]), "r"(h[2]),
                         "r"(h[3])
                         : "memory");
        }
    }
    return sc;
}

template <int G>
__global__ void __launch_bounds__(NTHREADS, 1) decode_mma_kernel(const DecMmaParams p) {
    using C = MC<G>;
    constexpr int NR = NBLK * G;  // valid (block, head) rows, <= 16
    static_assert(NR <= 16 && 8 % G == 0, "decode_mma: G in {1, 2, 4}");
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 127) & ~(uintptr_t)127);
    TileMeta* smeta = (TileMeta*)(smem + C::OFF_META);            // [NGRP][RS]
    uint64_t* bars = (uint64_t*)(smem + C::OFF_BAR);
    uint64_t* full = bars;                                         // [NGRP][RS] stage loaded
    uint64_t* empty = full + NGRP * RS;                            // [NGRP][RS] stage released (GW warps)
    uint64_t* mrg_full = empty + NGRP * RS;                        // [NGRP] partials written (GW warps)
    uint64_t* mrg_done = mrg_full + NGRP;                          // [NGRP] merge done reading (GW warps)
    int* abort_flag = (int*)(bars + C::NBAR);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < NGRP * RS; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], GW); }
        for (int i = 0; i < NGRP; ++i) { mbar_init(&mrg_full[i], GW); mbar_init(&mrg_done[i], GW); }
        *abort_flag = 0;
        fence_mbar_init();
    }
    // in-kernel plan: the same order as the plan kernel's list (full chunks sequence-major, then
    // each sequence's partial last chunk by decreasing size class, sequences in order within a class)
    int* s_full = (int*)(smem + C::OFF_PLAN);  // full chunks of sequence b
    int* s_cls = s_full + FOLD_MAX_B;          // size class of its partial chunk, -1: none
    int* s_fpre = s_cls + FOLD_MAX_B;          // full items of sequences < b
    int* s_tail = s_fpre + FOLD_MAX_B + 1;     // sequences with a partial chunk, in list order
    int* s_cs = s_tail + FOLD_MAX_B;           // [17] class starts, [17] full items, [18] all items
    if (p.fold) {
        const int B = (int)p.B, ch = p.chunk, hkv = (int)p.Hkv;
        for (int b = threadIdx.x; b < B; b += NTHREADS) {
            int64_t len = p.lens[b];
            len = len < 0 ? 0 : (len > p.Smax ? p.Smax : len);
            const int fc = (int)(len / ch);
            const int nch = len == 0 ? 1 : (int)((len + ch - 1) / ch);
            s_full[b] = fc;
            s_cls[b] = nch > fc ? (int)((16 * (len - (int64_t)fc * ch) + ch - 1) / ch) : -1;
        }
        __syncthreads();
        if (warp == 0) {
            const int per = (B + 31) / 32, b0 = min(B, lane * per), b1 = min(B, b0 + per);
            int loc = 0;
            for (int b = b0; b < b1; ++b) loc += s_full[b];
            int x = loc;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, x, off);
                if (lane >= off) x += y;
            }
            int run = x - loc;
            for (int b = b0; b < b1; ++b) {
                s_fpre[b] = run * hkv;
                run += s_full[b];
            }
            const int fitems = __shfl_sync(0xffffffffu, x, 31) * hkv;
            int cnt = 0;
            if (lane < 17)
                for (int b = 0; b < B; ++b) cnt += (s_cls[b] == lane);
            int suf = cnt;  // sequences in classes >= lane (larger classes come first)
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int y = __shfl_down_sync(0xffffffffu, suf, off);
                if (lane + off < 17) suf += y;
            }
            if (lane < 17) s_cs[lane] = suf - cnt;  // first list slot (in sequences) of class lane
            const int ntail = __shfl_sync(0xffffffffu, suf, 0);
            if (lane == 0) {
                s_fpre[B] = fitems;
                s_cs[17] = fitems;
                s_cs[18] = fitems + ntail * hkv;
            }
        }
        __syncthreads();
        for (int b = threadIdx.x; b < B; b += NTHREADS) {
            const int k = s_cls[b];
            if (k >= 0) {
                int r = 0;
                for (int b2 = 0; b2 < b; ++b2) r += (s_cls[b2] == k);
                s_tail[s_cs[k] + r] = b;
            }
        }
    }
    __syncthreads();

    if (warp >= NCW) {
        // ------------------------------------------------------------ producer of group warp - NCW
        if (lane == 0) {
            const int gp = warp - NCW;
            const int total = p.fold ? s_cs[18] : p.work[1 + p.B];
            // item n -> (b, hk << 16 | chunk): from the plan kernel's list, or from the tables
            auto item = [&](int n) -> int2 {
                if (!p.fold) return p.items[n];
                const int hkv = (int)p.Hkv;
                if (n < s_cs[17]) {  // full chunk: the sequence with s_fpre[b] <= n < s_fpre[b + 1]
                    int lo = 0, hi = (int)p.B;
                    while (hi - lo > 1) {
                        const int mid = (lo + hi) >> 1;
                        if (s_fpre[mid] <= n) lo = mid; else hi = mid;
                    }
                    const int w = n - s_fpre[lo], fc = s_full[lo];
                    return make_int2(lo, ((w / fc) << 16) | (w % fc));
                }
                const int t = n - s_cs[17], b = s_tail[t / hkv];
                return make_int2(b, ((t % hkv) << 16) | s_full[b]);
            };
            // claims run two deep: the counter for item k+2 and the list entry of item k+1 are fetched
            // while item k's tiles are issued, so neither latency stalls the ring
            int n1 = atomicAdd(p.work, 1);
            int n2 = atomicAdd(p.work, 1);
            int2 d1 = n1 < total ? item(n1) : make_int2(0, 0);
            int n = 0, seq = 0;
            bool ok = true;
            while (ok && n1 < total) {  // claims only grow: once n1 is past the end, so is n2
                const int b = d1.x, hk = d1.y >> 16, chunk = d1.y & 0xFFFF;
                n1 = n2;
                d1 = n1 < total ? item(n1) : make_int2(0, 0);
                n2 = atomicAdd(p.work, 1);
                int64_t len = p.lens[b];
                len = len < 0 ? 0 : (len > p.Smax ? p.Smax : len);
                const int64_t c0 = (int64_t)chunk * p.chunk;
                const int64_t c1 = min(len, c0 + p.chunk);
                const int nt = c1 > c0 ? (int)((c1 - c0 + TILE - 1) / TILE) : 1;
                const int64_t slab = ((int64_t)b * p.Hkv + hk) * p.Smax;
                const __half* qs = p.q + ((int64_t)b * p.H + (int64_t)hk * G) * HD;
                for (int t = 0; t < nt; ++t) {
                    const int s = n % RS;
                    if (n >= RS) ok = mbar_wait(&empty[gp * RS + s], ((n / RS) - 1) & 1, p.status, 41);
                    if (!ok || *(volatile int*)abort_flag) { ok = false; break; }
                    const int64_t r0 = c0 + (int64_t)t * TILE;
                    const int nrows = (int)max((int64_t)0, min((int64_t)TILE, c1 - r0));
                    TileMeta& m = smeta[gp * RS + s];
                    m.b = b; m.hk = hk; m.chunk = chunk; m.nrows = nrows; m.seq = seq;
                    m.flags = (t == 0 ? F_FIRST : 0) | (t == nt - 1 ? F_LAST : 0);
                    // whole row pairs: 2 * 136 bytes is a multiple of 16, and Smax is even on this path
                    const uint32_t bytes = (uint32_t)(((nrows + 1) & ~1) * ROWB);
                    const uint32_t qbytes = t == 0 ? (uint32_t)C::QB : 0u;
                    unsigned char* kd = smem + C::OFF_RAW + (gp * RS + s) * C::STAGE;
                    unsigned char* vd = kd + RAWB;
                    unsigned char* qd = kd + 2 * RAWB;
                    const uint8_t* ks = p.k + (slab + r0) * ROWB;
                    const uint8_t* vs = p.v + (slab + r0) * ROWB;
                    uint64_t* fb = &full[gp * RS + s];
                    const bool aligned = ((((uintptr_t)ks | (uintptr_t)vs | (uintptr_t)qs | (uintptr_t)smem_u32(kd) |
                                            (uintptr_t)smem_u32(vd) | (uintptr_t)smem_u32(qd) | bytes) & 15) == 0);
                    if (!aligned && p.status) atomicCAS(p.status, 0, 2);  // never issue a misaligned copy
                    const uint32_t tx = aligned ? 2 * bytes + qbytes : 0u;
                    if (tx == 0) {
                        mbar_arrive(fb);
                    } else {
                        mbar_expect_tx(fb, tx);
                        if (bytes) {
                            bulk_load(kd, ks, bytes, fb);
                            bulk_load(vd, vs, bytes, fb);
                        }
                        if (qbytes) bulk_load(qd, qs, qbytes, fb);
                    }
                    ++n;
                }
                ++seq;
            }
            if (ok && !*(volatile int*)abort_flag) {
                const int s = n % RS;
                if (n >= RS) ok = mbar_wait(&empty[gp * RS + s], ((n / RS) - 1) & 1, p.status, 43);
                if (ok) {
                    smeta[gp * RS + s].flags = F_END;
                    mbar_arrive(&full[gp * RS + s]);
                    ++n;
                }
            }
            if (!ok) *(volatile int*)abort_flag = 1;
            if (*(volatile int*)abort_flag) {
                for (int j = max(0, n - RS); j < n; ++j) mbar_wait(&full[gp * RS + j % RS], (j / RS) & 1, nullptr, 0);
            }
        }
        return;
    }

    // ---------------------------------------------------------------- consumer warp
    const int gp = warp / GW, wi = warp % GW;
    const int g = lane >> 2, c = lane & 3;  // MMA fragment coordinates
    // rows g and g + 8 of the 16-row (block, head) operand
    const bool v0 = g < NR, v1 = g + 8 < NR;
    const int b0 = g / G, b1 = (g + 8) / G;
    const int hh = g % G;  // head of both rows
    const uint32_t vst = smem_u32(smem + C::OFF_VST + warp * C::VST);

    // q of the item for the block-diagonal A operand of S: row g is non-zero only in the two 16-column
    // steps of block b0 (qg), row g + 8 only in those of block b1 (qg8); [step parity][cols 2c / 2c+8]
    uint32_t qg[2][2] = {{0u, 0u}, {0u, 0u}}, qg8[2][2] = {{0u, 0u}, {0u, 0u}};
    // O^T[d, r] for head dims d = 16 mt + g (+8) and operand rows r = 8 * ntile(mt) + 2c (+1)
    float ot[8][4];
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) ot[mt][0] = ot[mt][1] = ot[mt][2] = ot[mt][3] = 0.0f;
    // vbias: the V operand holds 1152 + x, so O^T carries 1152 * sum_t P~[r, t] in every row of column
    // r; that sum comes from one more MMA per column tile with an all-ones A operand (rescaled with
    // O), and is subtracted at the end of the item. Same layout as ot: [column tile][c0..c3].
    constexpr int NTL = ((3 * G) >> 3) + 1;  // column tiles of operand rows in use
    float ps[NTL][4];
#pragma unroll
    for (int nt = 0; nt < NTL; ++nt) ps[nt][0] = ps[nt][1] = ps[nt][2] = ps[nt][3] = 0.0f;
    float m_run = -INFINITY, l_run = 0.0f;
    float f = 0.0f;  // power of two for P~; 0 = not chosen yet in this item
    float qbias0 = 0.0f, qbias1 = 0.0f;  // -1152 * sum of q over the block of row g / row g + 8
    int nitem = 0;
    bool ok = true;

    for (int i = 0;; ++i) {
        const int s = i % RS;
        ok = warp_wait(&full[gp * RS + s], (i / RS) & 1, p.status, 51);
        if (!ok || *(volatile int*)abort_flag) break;
        const TileMeta m = smeta[gp * RS + s];
        if (m.flags & F_END) break;
        const unsigned char* st = smem + C::OFF_RAW + (gp * RS + s) * C::STAGE;

        if (m.flags & F_FIRST) {
            const uint32_t* q0 = (const uint32_t*)((const __half*)(st + 2 * RAWB) + hh * HD);
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int d0 = 16 * (2 * (v0 ? b0 : 0) + e) + 2 * c;
                const int d1 = 16 * (2 * (v1 ? b1 : 0) + e) + 2 * c;
                qg[e][0] = v0 ? q0[d0 >> 1] : 0u;
                qg[e][1] = v0 ? q0[(d0 + 8) >> 1] : 0u;
                qg8[e][0] = v1 ? q0[d1 >> 1] : 0u;
                qg8[e][1] = v1 ? q0[(d1 + 8) >> 1] : 0u;
            }
            // sum of each operand row over its block: the K operand carries +1152 per element
            float qs0 = 0.0f, qs1 = 0.0f;
#pragma unroll
            for (int e = 0; e < 2; ++e) {
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    qs0 += half_lo(qg[e][j]) + half_hi(qg[e][j]);
                    qs1 += half_lo(qg8[e][j]) + half_hi(qg8[e][j]);
                }
            }
            qs0 += __shfl_xor_sync(0xffffffffu, qs0, 1);
            qs0 += __shfl_xor_sync(0xffffffffu, qs0, 2);
            qs1 += __shfl_xor_sync(0xffffffffu, qs1, 1);
            qs1 += __shfl_xor_sync(0xffffffffu, qs1, 2);
            qbias0 = -1152.0f * qs0;
            qbias1 = -1152.0f * qs1;
            m_run = -INFINITY;
            l_run = 0.0f;
            f = 0.0f;
        }

#pragma unroll 1
        for (int sl = 0; sl < SPW; ++sl) {
            const int rb = 16 * (SPW * wi + sl);  // first tile row of this 16-row slice
            // V rows of the slice -> f16 (two lanes per row), and the largest |dV| of the valid rows
            float dvm = 0.0f;
            {
                // a quarter-warp stores 8 different swizzle phases: lanes 0-7 even rows, 8-15 odd rows
                const int r = 2 * (lane & 7) + ((lane >> 3) & 1), hb = lane >> 4;
                const float2 sv = dequant_half_row(st + RAWB + (rb + r) * ROWB, hb, vst + r * 256, r);
                if (rb + r < m.nrows) dvm = fmaxf(fabsf(sv.x), fabsf(sv.y));
            }
            // S'[(block, head), t] for the slice's 16 rows, straight from the raw K rows
            float sacc[2][2][4];  // [column tile][accumulation chain]
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int ch = 0; ch < 2; ++ch) sacc[nt][ch][0] = sacc[nt][ch][1] = sacc[nt][ch][2] = sacc[nt][ch][3] = 0.0f;
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                const bool r0 = v0 && b0 == (ks >> 1), r1 = v1 && b1 == (ks >> 1);
                const uint32_t qa[4] = {r0 ? qg[ks & 1][0] : 0u, r1 ? qg8[ks & 1][0] : 0u, r0 ? qg[ks & 1][1] : 0u,
                                        r1 ? qg8[ks & 1][1] : 0u};
                const int off = 34 * (ks >> 1) + 2 + 16 * (ks & 1) + 2 * c;  // byte of quant (16ks + 2c) in a row
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) {
                    // column tile nt holds the slice's rows 2n + nt (row order inside an MMA is free; rows
                    // 2 apart start 4 banks apart, so the 8 rows' 2-byte reads never share a bank)
                    const unsigned char* kr = st + (rb + 2 * g + nt) * ROWB + off;
                    mma16816(sacc[nt][ks & 1], qa, i8x2_to_f16x2_biased(lds_u16(kr)), i8x2_to_f16x2_biased(lds_u16(kr + 8)));
                }
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) dvm = fmaxf(dvm, __shfl_xor_sync(0xffffffffu, dvm, off));
            // scores of this thread's head hh; value k = 2 nt + e is column 2c + e of tile nt: slice row
            // t = 2 (2c + e) + nt = 4c + 2e + nt
            float sc4[4], dv0[4], dv1[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int t = 4 * c + 2 * (k & 1) + (k >> 1);
                const unsigned char* kr = st + (rb + t) * ROWB;
                const unsigned char* vr = kr + RAWB;
                const float s0 = sacc[k >> 1][0][k & 1] + sacc[k >> 1][1][k & 1] + qbias0;
                const float s1 = sacc[k >> 1][0][2 + (k & 1)] + sacc[k >> 1][1][2 + (k & 1)] + qbias1;
                float x = 0.0f;
                dv0[k] = dv1[k] = 0.0f;
                if (v0) {
                    x = half_lo(lds_u16(kr + 34 * b0)) * s0;
                    dv0[k] = half_lo(lds_u16(vr + 34 * b0));
                }
                if (v1) {
                    x = fmaf(half_lo(lds_u16(kr + 34 * b1)), s1, x);
                    dv1[k] = half_lo(lds_u16(vr + 34 * b1));
                }
                sc4[k] = x;
            }
            // sum over the lanes holding the other blocks of the same head
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                if constexpr (G == 4) {
                    sc4[k] += __shfl_xor_sync(0xffffffffu, sc4[k], 16);
                } else if constexpr (G == 2) {
                    sc4[k] += __shfl_xor_sync(0xffffffffu, sc4[k], 8);
                    sc4[k] += __shfl_xor_sync(0xffffffffu, sc4[k], 16);
                } else {
                    sc4[k] += __shfl_xor_sync(0xffffffffu, sc4[k], 4);
                    sc4[k] += __shfl_xor_sync(0xffffffffu, sc4[k], 8);
                }
            }
            float mx = -INFINITY;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int t = 4 * c + 2 * (k & 1) + (k >> 1);
                sc4[k] = (v0 && rb + t < m.nrows) ? sc4[k] * p.scale_log2 : -INFINITY;
                mx = fmaxf(mx, sc4[k]);
            }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            // lazy rescale: only when the running maximum grows by more than 2^8; p <= 2^8 otherwise
            float alpha = 1.0f;
            if (mx > m_run + 8.0f) {
                alpha = m_run == -INFINITY ? 0.0f : ex2(m_run - mx);
                l_run *= alpha;
                m_run = mx;
            }
            // f: dvm * f in [2^6, 2^7), so that P~ = p * dV * f < 2^15 with p <= 2^8; shrink when needed
            float fr = 1.0f;
            if (dvm > 0.0f) {
                const int e = (int)((__float_as_uint(dvm) >> 23) & 0xFF) - 127;
                const float f_want = __uint_as_float((uint32_t)(127 + 6 - e) << 23);
                if (f == 0.0f) {
                    f = f_want;
                } else if (f_want < f) {
                    fr = f_want / f;  // exact: both powers of two
                    f = f_want;
                }
            }
            if (__any_sync(0xffffffffu, alpha != 1.0f || fr != 1.0f)) {
                // O^T registers hold operand rows 2c + e of their column tile: head (2c + e) % G
                const float a0 = __shfl_sync(0xffffffffu, alpha, 4 * ((2 * c) % G)) * fr;
                const float a1 = __shfl_sync(0xffffffffu, alpha, 4 * ((2 * c + 1) % G)) * fr;
#pragma unroll
                for (int mt = 0; mt < 8; ++mt) {
                    ot[mt][0] *= a0; ot[mt][1] *= a1; ot[mt][2] *= a0; ot[mt][3] *= a1;
                }
#pragma unroll
                for (int nt = 0; nt < NTL; ++nt) {
                    ps[nt][0] *= a0; ps[nt][1] *= a1; ps[nt][2] *= a0; ps[nt][3] *= a1;
                }
            }
            const float neg = m_run == -INFINITY ? 0.0f : -m_run;
            float pr[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                pr[k] = ex2(sc4[k] + neg);
                l_run += pr[k];
            }
            // P~ rows g, g+8 as B fragments of PV. PV's reduction index k maps to slice row
            // 2 (k mod 8) + k / 8: k = 2c, 2c+1 are rows 4c, 4c+2 (tile 0), k = 2c+8, 2c+9 rows 4c+1, 4c+3
            uint32_t pa[4];
            {
                const float fv = f == 0.0f ? 1.0f : f;
                float w0[4], w1[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    // rows past the end of the sequence hold stale bytes: select, never multiply by 0
                    const bool tv = rb + 4 * c + 2 * (k & 1) + (k >> 1) < m.nrows;
                    w0[k] = (v0 && tv) ? pr[k] * dv0[k] * fv : 0.0f;
                    w1[k] = (v1 && tv) ? pr[k] * dv1[k] * fv : 0.0f;
                }
                pa[0] = pack_f16(w0[0], w0[1]);
                pa[1] = pack_f16(w1[0], w1[1]);
                pa[2] = pack_f16(w0[2], w0[3]);
                pa[3] = pack_f16(w1[2], w1[3]);
            }
            __syncwarp();  // the slice's f16 V rows are written
            // O^T[d, r] += Vx^T[d, t] P~^T[t, r]: one MMA per 16 head dims, with the column tile of
            // the operand rows of the dims' Q8_0 block
            {
                // matrices: k 0-7 / 8-15 (slice rows 2i / 2i+1) x head dims 16mt.. / 16mt+8..
                const int lr = 2 * (lane & 7) + (lane >> 4);  // V row (slice row) this lane addresses
                const int lc = (lane >> 3) & 1;
#pragma unroll
                for (int mt = 0; mt < 8; ++mt) {
                    uint32_t a[4];
                    ldsm_x4_t(vst + lr * 256 + (((2 * mt + lc) ^ ((lr >> 1) & 7)) << 4), a[0], a[1], a[2], a[3]);
                    const int ntile = ((mt >> 1) * G) >> 3;
                    mma16816(ot[mt], a, ntile ? pa[1] : pa[0], ntile ? pa[3] : pa[2]);
                }
                const uint32_t ones[4] = {0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u};  // f16 1.0
#pragma unroll
                for (int nt = 0; nt < NTL; ++nt) mma16816(ps[nt], ones, pa[nt], pa[2 + nt]);
            }
            __syncwarp();  // done with the slice's f16 V rows
        }
        if (lane == 0) mbar_arrive(&empty[gp * RS + s]);  // the stage is free for the producer

        if (m.flags & F_LAST) {
            // ---------------------------------------------------- merge the group's 4 partials of the item
            // Each warp's partial goes to its own V slice buffer (free after its PV); two group barriers
            // per item: partials written, and every warp done reading before any buffer is reused.
            float* mo = (float*)(smem + C::OFF_VST + warp * C::VST);  // [h][d]
            float* mm = mo + G * HD;                                  // [h]
            float* ml = mm + G;                                       // [h]
            float lsum = l_run;
            lsum += __shfl_xor_sync(0xffffffffu, lsum, 1);
            lsum += __shfl_xor_sync(0xffffffffu, lsum, 2);
            const float invf = f == 0.0f ? 1.0f : 1.0f / f;
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
                const int blk = mt >> 1;
                const int R0 = 8 * (((mt >> 1) * G) >> 3);
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int r = R0 + 2 * c + e;
                    if (r < NR && r / G == blk) {
                        const int h = r % G;
                        const float bias = 1152.0f * ps[R0 >> 3][e];
                        mo[h * HD + 16 * mt + g] = (ot[mt][e] - bias) * invf;
                        mo[h * HD + 16 * mt + g + 8] = (ot[mt][2 + e] - bias) * invf;
                    }
                }
            }
            if (v0 && b0 == 0 && c == 0) {  // one lane per head
                mm[hh] = m_run;
                ml[hh] = lsum;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&mrg_full[gp]);
            ok = warp_wait(&mrg_full[gp], nitem & 1, p.status, 53);
            if (!ok) break;
            const float* gbase = (const float*)(smem + C::OFF_VST + gp * GW * C::VST);
            constexpr int WSTRIDE = C::VST / 4;  // floats between the group's warps' buffers
            for (int pr2 = wi * 32 + lane; pr2 < G * HD; pr2 += GW * 32) {
                const int h = pr2 / HD, d = pr2 % HD;
                float M = -INFINITY;
#pragma unroll
                for (int w = 0; w < GW; ++w) M = fmaxf(M, gbase[w * WSTRIDE + G * HD + h]);
                float L = 0.0f, O = 0.0f;
#pragma unroll
                for (int w = 0; w < GW; ++w) {
                    const float mw = gbase[w * WSTRIDE + G * HD + h];
                    const float a = mw == -INFINITY ? 0.0f : ex2(mw - M);
                    L = fmaf(gbase[w * WSTRIDE + G * HD + G + h], a, L);
                    O = fmaf(gbase[w * WSTRIDE + h * HD + d], a, O);
                }
                const int64_t head = (int64_t)m.hk * G + h;
                if (p.nchunks == 1) {
                    p.out[((int64_t)m.b * p.H + head) * HD + d] = __float2half_rn(L > 0.0f ? O / L : 0.0f);
                } else {
                    float* pp = p.part + ((((int64_t)m.b * p.Hkv + m.hk) * p.nchunks + m.chunk) * G + h) * (HD + 2);
                    pp[d] = O;
                    if (d == 0) { pp[HD] = M; pp[HD + 1] = L; }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&mrg_done[gp]);
            ok = warp_wait(&mrg_done[gp], nitem & 1, p.status, 52);
            if (!ok) break;
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) ot[mt][0] = ot[mt][1] = ot[mt][2] = ot[mt][3] = 0.0f;
#pragma unroll
            for (int nt = 0; nt < NTL; ++nt) ps[nt][0] = ps[nt][1] = ps[nt][2] = ps[nt][3] = 0.0f;
            ++nitem;
        }
    }
    if (!ok) *(volatile int*)abort_flag = 1;
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
int run_decode_mma(const DecodeArgs& a, int* work, float* part, int64_t nchunks, cudaStream_t st) {
    using C = MC<G>;
    if (cuda_failed(cudaFuncSetAttribute(decode_mma_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM),
                    "cudaFuncSetAttribute(decode_mma)"))
        return -1;
    // small batches plan inside the kernel: only the claim counter needs zeroing
    const bool fold = a.B <= FOLD_MAX_B;
    if (fold) {
        if (cuda_failed(cudaMemsetAsync(work, 0, sizeof(int), st), "decode_mma counter reset")) return -1;
    } else if (launch_decode_plan(a, work, st) != 0) {
        return -1;
    }
    DecMmaParams p;
    p.fold = fold ? 1 : 0;
    p.q = (const __half*)a.q;
    p.k = (const uint8_t*)a.k;
    p.v = (const uint8_t*)a.v;
    p.lens = a.lens;
    p.out = (__half*)a.out;
    p.part = part;
    p.work = work;
    p.items = (const int2*)(work + decode_list_offset(a.B));
    p.B = a.B; p.H = a.H; p.Hkv = a.Hkv; p.Smax = a.Smax;
    p.nchunks = (int)nchunks;
    p.chunk = GTB_DECODE_CHUNK;
    p.scale_log2 = a.scale * 1.4426950408889634f;
    p.status = a.status;
    int dev = 0;
    cudaGetDevice(&dev);
    const int64_t max_items = a.B * a.Hkv * nchunks;
    const int grid = (int)min((int64_t)num_sms(dev), max_items);
    decode_mma_kernel<G><<<grid, NTHREADS, C::SMEM, st>>>(p);
    return cuda_failed(cudaGetLastError(), "decode_mma launch") ? -1 : 0;
}

}  // namespace

bool decode_mma_supported(const DecodeArgs& a) {
    static const int force_off = [] {
        const char* e = getenv("GTB_DECODE_MMA");
        return e ? (atoi(e) == 0) : 0;
    }();
    const int64_t G = a.Hkv > 0 ? a.H / a.Hkv : 0;
    return !force_off && a.D == HD && a.q_dtype == F16 && (G == 1 || G == 2 || G == 4) && a.Smax > 0 &&
           a.Smax % 2 == 0 && ((uintptr_t)a.q % 16 == 0) && ((uintptr_t)a.k % 16 == 0) && ((uintptr_t)a.v % 16 == 0) &&
           a.B * a.Hkv * decode_num_chunks(a.Smax) < (int64_t)INT32_MAX && a.B < INT32_MAX && a.Hkv < 32768 &&
           decode_num_chunks(a.Smax) < 65536;
}

int launch_decode_mma(const DecodeArgs& a, int* work, float* part, int64_t nchunks, cudaStream_t st) {
    switch (a.H / a.Hkv) {
        case 1: return run_decode_mma<1>(a, work, part, nchunks, st);
        case 2: return run_decode_mma<2>(a, work, part, nchunks, st);
        case 4: return run_decode_mma<4>(a, work, part, nchunks, st);
        default: set_error("decode_mma: unsupported group size"); return -1;
    }
}

}  // namespace gtb
