// Flash-style attention forward for sm_100a: tcgen05 tensor cores, TMEM accumulators, TMA tiles.
//
// One CTA computes two 128-row query tiles (rows 256c .. 256c+255) of one (batch, query head) that
// share every K/V tile it loads. Twelve warps, specialised:
//   warp 0       TMA producer: both Q tiles once, then K and V tiles of 128 keys into a ring of
//                shared-memory stages (128-byte swizzled, the layout the tcgen05 descriptors read);
//   warp 1       TMEM owner (512 columns) and MMA issuer (one thread), ping-ponging the two tiles:
//                  S_t = Q_t K_j^T        (M=128, N=128, K=D; both operands K-major in shared memory)
//                  O_t += P_t V_j         (M=128, N=D, K=128; P_t from TMEM, V read MN-major)
//                in the order  PV_0(j), S_0(j+1), PV_1(j), S_1(j+1), ...  so that while one softmax
//                warpgroup works on its S the tensor core runs the other tile's MMAs;
//   warps 2-3    idle;
//   warps 4-7    softmax + epilogue of tile 0, warps 8-11 of tile 1: one query row per thread (TMEM
//                lane = row). A whole 128-key block of S is read from TMEM into registers at once (the
//                softmax warpgroups run with 200 registers a thread, taken from warpgroup 0 with
//                setmaxnreg); online softmax in the log2 domain with lazy rescaling (the exponent
//                offset is raised only when the block's maximum exceeds it by more than 2^8, and O and
//                the running sum are rescaled then); P (bf16/f16) of each 32-key chunk is written over
//                the first 16 of the chunk's S columns, where the PV MMA reads it as its A operand.
// TMEM columns: S_0 [0,128), S_1 [128,256), O_0 [256,256+D), O_1 [384,384+D).
//
// Semantics are those of gt_flash_attention (reference csrc/gt_ops_nn.cpp:2423-2525): causal is
// top-left aligned (key s masked for query l when s > l), GQA maps query head h to kv head
// h / (H/Hkv), rows are normalised by the sum of exp over allowed keys. Accumulation is f32.
//
// tcgen05 MMAs issued by one thread complete in issue order, and tcgen05.commit arrives once all
// earlier MMAs of the thread are done. Two consequences the schedule relies on: S_t(j+1) may reuse
// the TMEM columns PV_t(j) reads P_t(j) from, and when S_t(j+1) is reported complete, PV_t(j) is
// complete too, so the softmax may rescale O_t without waiting on anything else.
//
// Every wait on an mbarrier is bounded (about a second); on timeout the kernel records a status
// code, skips its remaining work, drains its own in-flight copies and MMAs with bounded waits,
// frees TMEM and returns.

#include <cmath>
#include <cstdio>
#include <mutex>

#include <cudaTypedefs.h>

#include "dropout.cuh"
#include "gtb_common.cuh"
#include "mask_tiles.cuh"
#include "sdpa_args.h"
#include "sm100_ptx.cuh"

namespace gtb {
namespace {

using namespace sm100;

constexpr int BM = 128;          // rows per query tile
constexpr int BN = 128;          // keys per K/V tile
constexpr int NTHREADS = 384;
constexpr int REG_LO = 104;      // registers per thread of warpgroup 0 (TMA, MMA) after the split
constexpr int REG_HI = 200;      // ... of the softmax warpgroups
constexpr uint32_t TMEM_COLS = 512;

template <int D>
struct Cfg {
    static constexpr int ATOMS = D / 64;                  // 128-byte swizzle atoms along D
    static constexpr int TILE = BM * D * 2;               // bytes of a 128-row Q, K or V tile
    static constexpr int ATOM_BYTES = BM * 128;           // 16 KB: one 64-column slab of a tile
    static constexpr int KS = 2;                          // K stages
    static constexpr int VS = 2;                          // V stages
    static constexpr int OFF_Q = 0;                       // Q_0, Q_1
    static constexpr int OFF_K = 2 * TILE;
    static constexpr int OFF_V = OFF_K + KS * TILE;
    static constexpr int OFF_BAR = OFF_V + VS * TILE;
    static constexpr int NBAR = 1 + 2 * KS + 2 * VS + 2 + 2 + 2 + 1 + 1 + 2 + 4 + 1;
    static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;  // + TMEM slot and flag, + alignment slack
};

__device__ __forceinline__ uint32_t s_col(int t) { return (uint32_t)t * 128u; }
__device__ __forceinline__ uint32_t o_col(int t) { return 256u + (uint32_t)t * 128u; }

// 2^x on the FMA/ALU pipes, to take part of the softmax's exponentials off the MUFU unit, for a
// packed pair of floats. Range reduction x = n + f with n = round(x) (adding 1.5 * 2^23 rounds to an
// integer held in the low mantissa bits) and f in [-1/2, 1/2]; 2^f from a cubic fitted for this
// kernel (minimax in relative error on [-1/2, 1/2], max error 7.5e-5, far below the 2^-9 of the
// bf16 P it feeds); 2^n is added to the exponent field. x is clamped below at -126 so the exponent
// cannot wrap. The reduction and the cubic run as two-lane f32 operations.
__device__ __forceinline__ uint64_t exp2_poly2(uint64_t x2) {
    constexpr float C0 = 0.9999280571937561f, C1 = 0.6932609677314758f;
    constexpr float C2 = 0.2426111400127411f, C3 = 0.0551716573536396f;
    constexpr float SHIFT = 12582912.0f;  // 1.5 * 2^23
    float x0, x1;
    f2_unpack(x2, x0, x1);
    x2 = f2_pack(fmaxf(x0, -126.0f), fmaxf(x1, -126.0f));
    const uint64_t t2 = f2_add(x2, f2_pack(SHIFT, SHIFT));
    const uint64_t f2 = f2_add(x2, f2_add(t2, f2_pack(-SHIFT, -SHIFT)) ^ 0x8000000080000000ull);  // x - (t - SHIFT)
    uint64_t q2 = f2_fma(f2_pack(C3, C3), f2, f2_pack(C2, C2));
    q2 = f2_fma(q2, f2, f2_pack(C1, C1));
    q2 = f2_fma(q2, f2, f2_pack(C0, C0));
    float q0, q1, t0, t1;
    f2_unpack(q2, q0, q1);
    f2_unpack(t2, t0, t1);
    // n = bits(t) - bits(1.5 * 2^23); n << 23 == bits(t) << 23 (mod 2^32): the low 9 bits of the shift's bits are 0
    return f2_pack(__uint_as_float(__float_as_uint(q0) + (__float_as_uint(t0) << 23)),
                   __uint_as_float(__float_as_uint(q1) + (__float_as_uint(t1) << 23)));
}

// two floats -> one 32-bit word of two 16-bit values (lo in the low half), round to nearest even
template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    uint32_t r;
    if constexpr (BF16) asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    else asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// RoPE of one Q tile in shared memory, in place, by the 64 threads of warps 2-3 (rt = 0..63): the
// tile is ATOMS 128-byte-swizzled slabs of 64 columns (16-byte chunk c of row r at r * 128 +
// 16 (c ^ (r & 7))); row r is query row0 + r, rotated with row (row0 + r) of the (cos, sin) table,
// x0' = x0 c - x1 s, x1' = x0 s + x1 c in f32 with round-to-nearest products, rounded back to the
// 16-bit type, as the rope kernels compute it (so the rotated tile equals rope(q) in HBM bit for bit).
// Rows past L (zero-filled by the TMA) and dimensions past n_dims are left as they are.
template <bool BF16>
__device__ __forceinline__ float h16_lo(uint32_t w) {
    if constexpr (BF16) return __uint_as_float(w << 16);
    else return __half2float(__ushort_as_half((unsigned short)(w & 0xffffu)));
}
template <bool BF16>
__device__ __forceinline__ float h16_hi(uint32_t w) {
    if constexpr (BF16) return __uint_as_float(w & 0xffff0000u);
    else return __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}
__device__ __forceinline__ void rope_rot(float x0, float x1, float c, float sn, float& a, float& b) {
    a = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
    b = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
}
__device__ __forceinline__ unsigned char* swz_chunk(unsigned char* tile, int r, int g) {
    return tile + (g >> 3) * (BM * 128) + r * 128 + (((g & 7) ^ (r & 7)) << 4);
}
template <bool BF16>
__device__ void rope_q_tile(unsigned char* tile, int row0, int64_t L, const float* __restrict__ tab, int pairs,
                            int mode, int rt) {
    constexpr int NB = 2;  // chunks in flight a thread: their table loads issued before any is used
    if (mode != 2) {
        const int cpr = pairs / 4;  // rotated 16-byte chunks per row (4 pairs each)
        for (int u0 = rt; u0 < BM * cpr; u0 += 64 * NB) {
            uint4 w[NB];
            float4 t0[NB], t1[NB];
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                const int u = u0 + 64 * b, r = u / cpr, g = u - r * cpr;
                if (u < BM * cpr && row0 + r < L) {
                    const float4* tr = (const float4*)(tab + 2 * ((int64_t)(row0 + r) * pairs + 4 * g));
                    t0[b] = __ldg(tr);      // (c, s) of pairs 4g, 4g+1
                    t1[b] = __ldg(tr + 1);  // ... 4g+2, 4g+3
                    w[b] = *(const uint4*)swz_chunk(tile, r, g);
                }
            }
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                const int u = u0 + 64 * b, r = u / cpr, g = u - r * cpr;
                if (!(u < BM * cpr && row0 + r < L)) continue;
                float a, c;
                rope_rot(h16_lo<BF16>(w[b].x), h16_hi<BF16>(w[b].x), t0[b].x, t0[b].y, a, c); w[b].x = pack2<BF16>(a, c);
                rope_rot(h16_lo<BF16>(w[b].y), h16_hi<BF16>(w[b].y), t0[b].z, t0[b].w, a, c); w[b].y = pack2<BF16>(a, c);
                rope_rot(h16_lo<BF16>(w[b].z), h16_hi<BF16>(w[b].z), t1[b].x, t1[b].y, a, c); w[b].z = pack2<BF16>(a, c);
                rope_rot(h16_lo<BF16>(w[b].w), h16_hi<BF16>(w[b].w), t1[b].z, t1[b].w, a, c); w[b].w = pack2<BF16>(a, c);
                *(uint4*)swz_chunk(tile, r, g) = w[b];
            }
        }
    } else {
        const int cph = pairs / 8;  // chunks of the first half of a row; chunk g pairs with chunk g + cph
        constexpr int NBX = NB / 2;
        for (int u0 = rt; u0 < BM * cph; u0 += 64 * NBX) {
            uint4 w0[NBX], w1[NBX];
            float4 t[NBX][4];
#pragma unroll
            for (int b = 0; b < NBX; ++b) {
                const int u = u0 + 64 * b, r = u / cph, g = u - r * cph;
                if (u < BM * cph && row0 + r < L) {
                    const float4* tr = (const float4*)(tab + 2 * ((int64_t)(row0 + r) * pairs + 8 * g));
#pragma unroll
                    for (int k = 0; k < 4; ++k) t[b][k] = __ldg(tr + k);  // (c, s) of pairs 8g .. 8g+7
                    w0[b] = *(const uint4*)swz_chunk(tile, r, g);
                    w1[b] = *(const uint4*)swz_chunk(tile, r, g + cph);
                }
            }
#pragma unroll
            for (int b = 0; b < NBX; ++b) {
                const int u = u0 + 64 * b, r = u / cph, g = u - r * cph;
                if (!(u < BM * cph && row0 + r < L)) continue;
                uint32_t* x0 = (uint32_t*)&w0[b];
                uint32_t* x1 = (uint32_t*)&w1[b];
#pragma unroll
                for (int k = 0; k < 4; ++k) {  // word k holds pairs 8g+2k (low halves) and 8g+2k+1 (high)
                    float a0, b0, a1, b1;
                    rope_rot(h16_lo<BF16>(x0[k]), h16_lo<BF16>(x1[k]), t[b][k].x, t[b][k].y, a0, b0);
                    rope_rot(h16_hi<BF16>(x0[k]), h16_hi<BF16>(x1[k]), t[b][k].z, t[b][k].w, a1, b1);
                    x0[k] = pack2<BF16>(a0, a1);
                    x1[k] = pack2<BF16>(b0, b1);
                }
                *(uint4*)swz_chunk(tile, r, g) = w0[b];
                *(uint4*)swz_chunk(tile, r, g + cph) = w1[b];
            }
        }
    }
}

// max of three (one instruction on sm_100)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// the same bounded wait taken by a whole warp: every lane gets the same answer
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* status, int code) {
    const bool ok = mbar_wait(bar, parity, status, code);
    return __all_sync(0xffffffffu, ok);
}

struct Params {
    int64_t H, Hkv, L, S;
    int group;
    int n_pairs;  // work items along the query dimension (two 128-row tiles each)
    int n_items;  // n_pairs * H * B: item i = (batch, kv head, pair heaviest first, query head)
    int64_t B;
    int* claim;   // zeroed item counter: CTAs claim items in order (persistent launch)
    float scale_log2;
    int causal;
    void* o;
    int64_t os0, os1, os2;  // output strides of b, h, l (elements); d stride is 1
    float* lse;
    int* status;
    MaskView mk;  // attention mask (MASK instances only)
    uint32_t drop_thr;   // dropout (DROP instances only): keep threshold, seed, 1 / (1 - p)
    uint64_t drop_seed;
    float inv_keep;
    const float* rope_tab;  // ROPE instances: (cos, sin) of query row l, pair i at rope_tab[2 (l n_pairs + i)]
    int rope_pairs;         // n_dims / 2
    int rope_mode;          // 0: pairs (2i, 2i+1); 2: NeoX, pairs (i, i + n_dims / 2)
};

// keys a row of tile t may see: [0, n_kv*BN) minus causal / ragged masking
__device__ __forceinline__ int tile_blocks(int row0, const Params& p, int n_kv) {
    if (row0 >= p.L) return 0;
    if (!p.causal) return n_kv;
    const int last = (int)min((int64_t)row0 + BM - 1, p.L - 1);
    return min(n_kv, last / BN + 1);
}

// Scores of one 32-column chunk, masked: column s (absolute key index kv0 + i) is excluded when
// s >= S or, for causal attention, s > row.
__device__ __forceinline__ void mask_chunk(float* x, int kv0, int lim) {
#pragma unroll
    for (int i = 0; i < 32; ++i)
        if (kv0 + i > lim) x[i] = -INFINITY;
}

template <int D, bool BF16, int EMU, bool PERSIST, bool MASK, bool DROP, bool ROPE>
__global__ void __launch_bounds__(NTHREADS, 1)
fwd_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                 const __grid_constant__ CUtensorMap tmV, const Params p) {
    using C = Cfg<D>;
    using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = (uint64_t*)(smem + C::OFF_BAR);
    uint64_t* q_full = bars;
    uint64_t* k_full = bars + 1;
    uint64_t* k_empty = k_full + C::KS;
    uint64_t* v_full = k_empty + C::KS;
    uint64_t* v_empty = v_full + C::VS;
    uint64_t* s_full = v_empty + C::VS;      // [2] per tile: S_t(j) computed
    uint64_t* p_full = s_full + 2;           // [2] per tile: P_t(j) written (128 arrivals)
    uint64_t* o_final = p_full + 2;          // [2] per tile: every MMA of the tile done
    uint64_t* drain = o_final + 2;           // error path only
    uint64_t* q_empty = drain + 1;           // every S MMA of an item done: its Q buffers are free
    uint64_t* o_empty = q_empty + 1;         // [2] per tile: the epilogue has read O_t (128 arrivals)
    uint64_t* item_full = o_empty + 2;       // [2] ring of claimed items: index written
    uint64_t* item_empty = item_full + 2;    // [2] ... read by the MMA warp and the 8 softmax warps (+ 2 RoPE warps)
    uint64_t* q_rot = item_empty + 2;        // ROPE: the item's Q tiles rotated in place (64 arrivals)
    uint32_t* tmem_slot = (uint32_t*)(bars + C::NBAR);
    int* abort_flag = (int*)(tmem_slot + 1);
    int* item_slot = abort_flag + 1;         // [2] claimed item index, -1: no more items

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_kv = (int)((p.S + BN - 1) / BN);
    // Work item = (pair of 128-row query tiles, head, batch). Persistent launch (short sequences):
    // one CTA per SM claims items from a counter, pairs heaviest first and (batch, head) fastest, so
    // that the CTAs take the longest work first; the TMA warp claims and passes each item on through
    // a two-slot ring in shared memory, and the K/V ring, the barrier phases and TMEM carry over from
    // item to item (the next item's K/V loads start as soon as ring slots free up, its Q load as soon
    // as the previous item's S MMAs are done), which hides each item's start-up. One CTA per item
    // (long sequences): blockIdx order, (batch, head) major and pairs heaviest first, so that the
    // CTAs running together stream the same head's K/V and share it through L2; measured faster
    // when a sequence's K/V is far larger than L2.
    struct Item {
        int h, b, hk, row0[2], nblk[2], n;
    };
    auto item_of = [&](int i) {
        Item it;
        int pr, bh;
        if constexpr (PERSIST) {  // pairs heaviest first, (batch, head) fastest
            const int hb = (int)(p.H * p.B);
            pr = i / hb;
            bh = i - pr * hb;
        } else {             // (batch, head) major, pairs heaviest first
            bh = i / p.n_pairs;
            pr = i - bh * p.n_pairs;
        }
        const int pair = p.causal ? (p.n_pairs - 1 - pr) : pr;
        it.b = (int)(bh / p.H);
        it.h = (int)(bh % p.H);
        it.hk = it.h / p.group;
        it.row0[0] = pair * 2 * BM;
        it.row0[1] = pair * 2 * BM + BM;
        it.nblk[0] = tile_blocks(it.row0[0], p, n_kv);  // >= 1: row0[0] < L for every pair
        it.nblk[1] = tile_blocks(it.row0[1], p, n_kv);
        it.n = max(it.nblk[0], it.nblk[1]);
        return it;
    };

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < C::KS; ++i) { mbar_init(&k_full[i], 1); mbar_init(&k_empty[i], 1); }
        for (int i = 0; i < C::VS; ++i) { mbar_init(&v_full[i], 1); mbar_init(&v_empty[i], 1); }
        for (int t = 0; t < 2; ++t) {
            mbar_init(&s_full[t], 1); mbar_init(&p_full[t], 128); mbar_init(&o_final[t], 1); mbar_init(&o_empty[t], 128);
        }
        mbar_init(q_empty, 1);
        for (int i = 0; i < 2; ++i) { mbar_init(&item_full[i], 1); mbar_init(&item_empty[i], ROPE ? 11 : 9); }
        mbar_init(q_rot, 64);
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // Registers: warpgroup 0 (TMA, MMA, two idle warps) hands registers to the two softmax warpgroups,
    // which hold a whole 128-key block of scores. Every thread executes its warpgroup's setmaxnreg at
    // the top of its role's branch below, converged (the instruction is .sync.aligned and
    // warpgroup-wide; the compiler allocates the code a setmaxnreg dominates within its count):
    // 128 x REG_LO + 256 x REG_HI stays within the 384 x 168 registers the block is launched with.
    static_assert(128 * REG_LO + 256 * REG_HI <= NTHREADS * 168, "register split above the launch's registers");

    if (warp < 4) {
        setmaxnreg_dec<REG_LO>();
        if (warp == 0) {
            // ------------------------------------------------------------ TMA producer
            if (lane == 0) {
                prefetch_tmap(&tmQ);
                prefetch_tmap(&tmK);
                prefetch_tmap(&tmV);
                int J = 0, nitem = 0;  // K/V blocks and items started so far
                int nk = 0, nv = 0, nql = 0;  // K, V and Q loads issued
                bool ok = true;
                // claims run one item ahead (the atomic's latency is hidden); one item per CTA otherwise
                int next = PERSIST ? atomicAdd(p.claim, 1) : (int)blockIdx.x;
                for (;; ++nitem) {
                    const int i = next;
                    if constexpr (PERSIST) {
                        const int slot = nitem & 1;
                        if (nitem >= 2) ok = mbar_wait(&item_empty[slot], ((nitem >> 1) - 1) & 1, p.status, 14);
                        if (!ok || *(volatile int*)abort_flag) { ok = false; break; }
                        item_slot[slot] = i < p.n_items ? i : -1;
                        mbar_arrive(&item_full[slot]);
                    }
                    if (i >= p.n_items) break;
                    next = PERSIST ? atomicAdd(p.claim, 1) : p.n_items;
                    const Item it = item_of(i);
                    const int nq = it.nblk[1] > 0 ? 2 : 1;
                    auto load_q = [&]() {
                        mbar_expect_tx(q_full, nq * C::TILE);
                        for (int t = 0; t < nq; ++t)
                            for (int a = 0; a < C::ATOMS; ++a)
                                tma_load_4d(smem + C::OFF_Q + t * C::TILE + a * C::ATOM_BYTES, &tmQ, a * 64, it.row0[t], it.h,
                                            it.b, q_full);
                        ++nql;
                    };
                    if (nitem == 0) load_q();  // the CTA's first item: nothing to wait for, Q first
                    for (int j = 0; j < it.n && ok; ++j, ++J) {
                        const int ks = J % C::KS;
                        if (J >= C::KS) ok = mbar_wait(&k_empty[ks], ((J / C::KS) - 1) & 1, p.status, 11);
                        if (!ok || *(volatile int*)abort_flag) { ok = false; break; }
                        mbar_expect_tx(&k_full[ks], C::TILE);
                        for (int a = 0; a < C::ATOMS; ++a)
                            tma_load_4d(smem + C::OFF_K + ks * C::TILE + a * C::ATOM_BYTES, &tmK, a * 64, j * BN, it.hk, it.b,
                                        &k_full[ks]);
                        ++nk;
                        const int vs = J % C::VS;
                        if (J >= C::VS) ok = mbar_wait(&v_empty[vs], ((J / C::VS) - 1) & 1, p.status, 12);
                        if (!ok || *(volatile int*)abort_flag) { ok = false; break; }
                        mbar_expect_tx(&v_full[vs], C::TILE);
                        for (int a = 0; a < C::ATOMS; ++a)
                            tma_load_4d(smem + C::OFF_V + vs * C::TILE + a * C::ATOM_BYTES, &tmV, a * 64, j * BN, it.hk, it.b,
                                        &v_full[vs]);
                        ++nv;
                        if (j == 0 && nitem > 0) {
                            // Q of a later item, once the previous item's S MMAs have read theirs (after this
                            // item's first K/V block, whose slots may free up earlier)
                            ok = mbar_wait(q_empty, (nitem - 1) & 1, p.status, 13);
                            if (!ok || *(volatile int*)abort_flag) { ok = false; break; }
                            load_q();
                        }
                    }
                }
                if (!ok) *(volatile int*)abort_flag = 1;
                if (*(volatile int*)abort_flag) {
                    // drain our own copies before the CTA exits (bounded): the last Q and the last K/V blocks
                    if (nql > 0) mbar_wait(q_full, (nql - 1) & 1, nullptr, 0);
                    for (int jj = max(0, nk - C::KS); jj < nk; ++jj) mbar_wait(&k_full[jj % C::KS], (jj / C::KS) & 1, nullptr, 0);
                    for (int jj = max(0, nv - C::VS); jj < nv; ++jj) mbar_wait(&v_full[jj % C::VS], (jj / C::VS) & 1, nullptr, 0);
                }
            }
        } else if (warp == 1) {
            // ------------------------------------------------------------ MMA issuer
            if (lane == 0) {
                constexpr uint32_t IDESC_S = idesc_f16(BM, BN, BF16, false);
                constexpr uint32_t IDESC_PV = idesc_f16(BM, D, BF16, true);
                // operand descriptors of every buffer, built once: per MMA only a constant is added to the
                // start address
                static_assert(C::KS == 2 && C::VS == 2, "descriptor selection below assumes two K and two V stages");
                const uint64_t qd0 = desc_sw128(smem_u32(smem + C::OFF_Q), 16, 1024);
                const uint64_t qd1 = desc_sw128(smem_u32(smem + C::OFF_Q + C::TILE), 16, 1024);
                const uint64_t kd0 = desc_sw128(smem_u32(smem + C::OFF_K), 16, 1024);
                const uint64_t kd1 = desc_sw128(smem_u32(smem + C::OFF_K + C::TILE), 16, 1024);
                const uint64_t vd0 = desc_sw128(smem_u32(smem + C::OFF_V), C::ATOM_BYTES, 1024);
                const uint64_t vd1 = desc_sw128(smem_u32(smem + C::OFF_V + C::TILE), C::ATOM_BYTES, 1024);
                // J: K/V block of the ring (over all items); u[t]: blocks of tile t so far (s_full / p_full
                // phases); nf[t]: items with a tile t so far (o_final / o_empty phases)
                int J = 0, u[2] = {0, 0}, nf[2] = {0, 0}, nitem = 0;
                auto issue_s = [&](int t, int jg) -> bool {  // S_t of ring block jg
                    const int ks = jg % C::KS;
                    if (!mbar_wait(&k_full[ks], (jg / C::KS) & 1, p.status, 22)) return false;
                    tc_fence_after();
                    const uint64_t qb = t ? qd1 : qd0, kb = ks ? kd1 : kd0;
                    const uint32_t dst = tmem + s_col(t);
    #pragma unroll
                    for (int kk = 0; kk < D / 16; ++kk) {
                        const uint32_t off = (uint32_t)((kk / 4) * C::ATOM_BYTES + (kk % 4) * 32);
                        mma_ss(dst, desc_advance(qb, off), desc_advance(kb, off), IDESC_S, kk > 0 ? 1u : 0u);
                    }
                    mma_commit(&s_full[t]);
                    return true;
                };
                auto issue_pv = [&](int t, int jg, int ut, bool first) -> bool {  // PV_t of ring block jg
                    if (!mbar_wait(&p_full[t], ut & 1, p.status, 23)) return false;
                    const int vs = jg % C::VS;
                    if (!mbar_wait(&v_full[vs], (jg / C::VS) & 1, p.status, 24)) return false;
                    tc_fence_after();
                    const uint64_t vb = vs ? vd1 : vd0;
                    const uint32_t dst = tmem + o_col(t), pa = tmem + s_col(t);
    #pragma unroll
                    for (int kk = 0; kk < BN / 16; ++kk) {
                        // A = P_t(j): 16-bit values packed two per TMEM column; keys 32c..32c+31 sit in
                        // columns 32c..32c+15, 8 columns per K step
                        mma_ts(dst, pa + 32 * (kk >> 1) + 8 * (kk & 1), desc_advance(vb, kk * 2048), IDESC_PV,
                               (!first || kk > 0) ? 1u : 0u);
                    }
                    return true;
                };
                bool ok = true;
                for (;; ++nitem) {
                    int i;
                    if constexpr (PERSIST) {
                        const int slot = nitem & 1;
                        ok = mbar_wait(&item_full[slot], (nitem >> 1) & 1, p.status, 27);
                        if (!ok) break;
                        i = item_slot[slot];
                        mbar_arrive(&item_empty[slot]);
                    } else {
                        i = nitem == 0 ? (int)blockIdx.x : -1;
                    }
                    if (i < 0) break;
                    const Item it = item_of(i);
                    ok = mbar_wait(q_full, nitem & 1, p.status, 21);
                    if (ROPE && ok) ok = mbar_wait(q_rot, nitem & 1, p.status, 28);  // and rotated by warps 2-3
                    for (int t = 0; t < 2 && ok; ++t)
                        if (it.nblk[t] > 0) ok = issue_s(t, J);
                    if (!ok) break;
                    mma_commit(&k_empty[J % C::KS]);
                    if (it.n == 1) mma_commit(q_empty);  // every S of the item issued
                    for (int j = 0; j < it.n && ok; ++j) {
                        for (int t = 0; t < 2 && ok; ++t) {
                            if (j >= it.nblk[t]) continue;
                            // the first PV of an item overwrites O_t: the previous item's epilogue must have read it
                            if (j == 0 && nf[t] > 0) ok = mbar_wait(&o_empty[t], (nf[t] - 1) & 1, p.status, 26);
                            if (ok) ok = issue_pv(t, J + j, u[t] + j, j == 0);
                            if (ok && j + 1 < it.nblk[t]) ok = issue_s(t, J + j + 1);
                            if (ok && j + 1 == it.nblk[t]) mma_commit(&o_final[t]);
                        }
                        if (!ok || *(volatile int*)abort_flag) { ok = false; break; }
                        mma_commit(&v_empty[(J + j) % C::VS]);
                        if (j + 1 < it.n) mma_commit(&k_empty[(J + j + 1) % C::KS]);
                        if (j + 2 == it.n) mma_commit(q_empty);  // the item's last S MMAs were issued at this j
                    }
                    J += it.n;
                    for (int t = 0; t < 2; ++t) {
                        u[t] += it.nblk[t];
                        nf[t] += it.nblk[t] > 0 ? 1 : 0;
                    }
                }
                if (!ok) *(volatile int*)abort_flag = 1;
                if (*(volatile int*)abort_flag) {
                    mma_commit(drain);  // wait (bounded) for every MMA we issued before TMEM is freed
                    mbar_wait(drain, 0, nullptr, 0);
                }
            }
        } else if constexpr (ROPE) {
            // ------------------------------------------------------------ RoPE of each item's Q tiles
            // (warps 2-3): once both Q tiles have landed, rotate them in place, make the generic-proxy
            // writes visible to the tensor core (async proxy), then release them to the MMA warp. The
            // next item's Q lands while this item's last blocks are computed, so the rotation overlaps.
            const int rt = (int)threadIdx.x - 64;
            bool ok = true;
            for (int nitem = 0;; ++nitem) {
                int i;
                if constexpr (PERSIST) {
                    const int slot = nitem & 1;
                    ok = warp_wait(&item_full[slot], (nitem >> 1) & 1, p.status, 17);
                    if (!ok) break;
                    i = item_slot[slot];
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&item_empty[slot]);
                } else {
                    i = nitem == 0 ? (int)blockIdx.x : -1;
                }
                if (i < 0) break;
                const Item it = item_of(i);
                ok = warp_wait(q_full, nitem & 1, p.status, 18);
                if (!ok || __any_sync(0xffffffffu, *(volatile int*)abort_flag)) { ok = false; break; }
                for (int t = 0; t < 2; ++t)
                    if (it.nblk[t] > 0)
                        rope_q_tile<BF16>(smem + C::OFF_Q + t * C::TILE, it.row0[t], p.L, p.rope_tab, p.rope_pairs,
                                          p.rope_mode, rt);
                fence_proxy_async_smem();
                mbar_arrive(q_rot);
            }
            if (!ok) *(volatile int*)abort_flag = 1;
        }
    } else {
        setmaxnreg_inc<REG_HI>();
        // ------------------------------------------------------------ softmax + epilogue of tile t
        const int t = (warp - 4) >> 2;
        const int quad = warp & 3;                    // TMEM lanes this warp may access
        const int r = quad * 32 + lane;               // row of the tile
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        const uint32_t s_tmem = tmem + lane_addr + s_col(t);
        const uint32_t o_tmem = tmem + lane_addr + o_col(t);
        const int lim_s = (int)min(p.S, (int64_t)INT32_MAX) - 1;
        int u = 0, nf = 0;  // blocks and items of tile t so far (barrier phases)
        bool ok = true;
        for (int nitem = 0; ok; ++nitem) {
            int i;
            if constexpr (PERSIST) {
                const int slot = nitem & 1;
                ok = warp_wait(&item_full[slot], (nitem >> 1) & 1, p.status, 34);
                if (!ok) break;
                i = item_slot[slot];
                __syncwarp();
                if (lane == 0) mbar_arrive(&item_empty[slot]);
            } else {
                i = nitem == 0 ? (int)blockIdx.x : -1;
            }
            if (i < 0) break;
            const Item it = item_of(i);
            const int nb = it.nblk[t];
            if (nb == 0) continue;
            const int h = it.h, b = it.b;
            const int row0t = it.row0[t];
            const int grow = row0t + r;                   // query index
            const int lim = p.causal ? min(lim_s, grow) : lim_s;  // last key this row may see
            // mask entries of this row (padding rows past L read row L-1; their results are dropped)
            const unsigned char* mrow = nullptr;
            if constexpr (MASK) mrow = p.mk.row(b, h, min((int64_t)grow, p.L - 1));
            // dropout: this row's key of the counter-based keep decisions (dropout.cuh)
            const uint32_t rkey = DROP ? drop_row_key(drop_head_key(p.drop_seed, (uint32_t)(b * p.H + h)), (uint32_t)grow) : 0u;
            float m_used = -INFINITY, lsum = 0.0f;
            for (int j = 0; j < nb; ++j) {
                // the attention mask's class for this tile and key block (the same for every row), read
                // before the wait for the block's scores so that the load completes during the wait
                const uint8_t mcls = MASK ? p.mk.tile_class(b, h, row0t / BM, j) : (uint8_t)MASK_NONE;
                ok = warp_wait(&s_full[t], (u + j) & 1, p.status, 31);
                if (!ok || __any_sync(0xffffffffu, *(volatile int*)abort_flag)) break;
                tc_fence_after();
                const int kv0 = j * BN;
                const bool need_mask = (kv0 + BN > p.S) || (p.causal && kv0 + BN - 1 > row0t);
                auto attn_mask = [&](float* x, int s0) {
                    if constexpr (MASK) {
                        if (mcls == MASK_MIXED) {
                            mask_apply32(x, p.mk, mrow, s0, p.S);
                        } else if (mcls == MASK_ALL) {
#pragma unroll
                            for (int i = 0; i < 32; ++i) x[i] = -INFINITY;
                        }
                    }
                };
                // The block's scores in registers, the running maximum m_used as the exponent's offset
                // (raised when the block's maximum exceeds it by more than 2^8; O and the running sum
                // are rescaled at the end of the block when it moved). P of chunk c (keys 32c..32c+31)
                // is written over S's columns 32c..32c+15, already read, as packed 16-bit pairs (the
                // PV MMA's A operand). The scale-and-subtract and the sums run as packed two-lane f32.
                const float m_start = m_used;
                const uint64_t sc2 = f2_pack(p.scale_log2, p.scale_log2);
                uint64_t ps2[2] = {0ull, 0ull};
                auto emit = [&](const float* x, int c) {
                    const float neg_m = (m_used == -INFINITY) ? 0.0f : -m_used;
                    const uint64_t nm2 = f2_pack(neg_m, neg_m);
                    uint32_t pk[16];
                    uint32_t kbits = 0;  // dropout: keep decisions of keys kv0 + 32c .. kv0 + 32c + 31
                    if constexpr (DROP) {
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            kbits |= (drop_keep(rkey, (uint32_t)(kv0 + 32 * c + i), p.drop_thr) ? 1u : 0u) << i;
                    }
#pragma unroll
                    for (int i = 0; i < 32; i += 2) {
                        const uint64_t a2 = f2_fma(f2_pack(x[i], x[i + 1]), sc2, nm2);
                        uint64_t p2;
                        if ((i & 7) < EMU) {  // this pair on the FMA pipe
                            p2 = exp2_poly2(a2);
                        } else {
                            float a0, a1;
                            f2_unpack(a2, a0, a1);
                            p2 = f2_pack(ex2(a0), ex2(a1));
                        }
                        ps2[(i >> 1) & 1] = f2_add(ps2[(i >> 1) & 1], p2);  // the normaliser: undropped
                        float p0, p1;
                        f2_unpack(p2, p0, p1);
                        if constexpr (DROP) {  // the PV product takes only the kept probabilities
                            if (!((kbits >> i) & 1u)) p0 = 0.0f;
                            if (!((kbits >> (i + 1)) & 1u)) p1 = 0.0f;
                        }
                        pk[i / 2] = pack2<BF16>(p0, p1);
                    }
                    tmem_st16(s_tmem + 32 * c, pk);
                };
                {
                    // the block's 128 scores in registers: one maximum, one decision per row (nothing of
                    // this block is written before it), then the four chunks' probabilities
                    uint32_t ra[32], rb[32], rc[32], rd[32];
                    tmem_ld32(s_tmem + 0, ra);
                    tmem_ld32(s_tmem + 32, rb);
                    tmem_ld32(s_tmem + 64, rc);
                    tmem_ld32(s_tmem + 96, rd);
                    tmem_ld_wait();
                    float* xa = (float*)ra;
                    float* xb = (float*)rb;
                    float* xc = (float*)rc;
                    float* xd = (float*)rd;
                    attn_mask(xa, kv0);
                    attn_mask(xb, kv0 + 32);
                    attn_mask(xc, kv0 + 64);
                    attn_mask(xd, kv0 + 96);
                    if (need_mask) {
                        mask_chunk(xa, kv0, lim);
                        mask_chunk(xb, kv0 + 32, lim);
                        mask_chunk(xc, kv0 + 64, lim);
                        mask_chunk(xd, kv0 + 96, lim);
                    }
                    float pm[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) pm[u] = fmax3(xa[u], xb[u], xc[u]);
#pragma unroll
                    for (int u = 0; u < 8; ++u) pm[u] = fmax3(pm[u], xd[u], xa[u + 8]);
#pragma unroll
                    for (int i = 8; i < 32; ++i) pm[i & 7] = fmax3(pm[i & 7], xb[i], xc[i]);
#pragma unroll
                    for (int i = 8; i < 32; ++i) pm[i & 7] = fmaxf(pm[i & 7], xd[i]);
#pragma unroll
                    for (int i = 16; i < 32; i += 2) pm[i & 7] = fmax3(pm[i & 7], xa[i], xa[i + 1]);
                    const float cm =
                        fmax3(fmax3(pm[0], pm[1], pm[2]), fmax3(pm[3], pm[4], pm[5]), fmaxf(pm[6], pm[7])) * p.scale_log2;
                    const float m_new = fmaxf(m_used, cm);
                    if (m_new > m_used + 8.0f) m_used = m_new;  // false while the row has no finite score
                    emit(xa, 0);
                    emit(xb, 1);
                    emit(xc, 2);
                    emit(xd, 3);
                }
                const bool grew = m_used != m_start;
                if (__any_sync(0xffffffffu, grew && j > 0)) {
                    // PV_t(j-1) is complete: it was issued before S_t(j), whose completion we have seen
                    const float alpha = grew ? ex2(m_start - m_used) : 1.0f;
#pragma unroll
                    for (int c = 0; c < D / 32; ++c) {
                        uint32_t ov[32];
                        tmem_ld32(o_tmem + c * 32, ov);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
                        tmem_st32(o_tmem + c * 32, ov);
                    }
                }
                {
                    float s0, s1, s2, s3;
                    f2_unpack(ps2[0], s0, s1);
                    f2_unpack(ps2[1], s2, s3);
                    lsum = (grew ? lsum * ex2(m_start - m_used) : lsum) + ((s0 + s1) + (s2 + s3));
                }
                tmem_st_wait();
                tc_fence_before();
                mbar_arrive(&p_full[t]);
            }
            u += nb;
            if (!ok) break;
            if (!*(volatile int*)abort_flag) {
                ok = warp_wait(&o_final[t], nf & 1, p.status, 33);
                if (ok) {
                    tc_fence_after();
                    const float inv = lsum > 0.0f ? (DROP ? p.inv_keep : 1.0f) / lsum : 0.0f;
                    T* orow = (T*)p.o + (int64_t)b * p.os0 + (int64_t)h * p.os1 + (int64_t)grow * p.os2;
#pragma unroll
                    for (int c = 0; c < D / 32; ++c) {
                        uint32_t ov[32];
                        tmem_ld32(o_tmem + c * 32, ov);
                        tmem_ld_wait();
                        if (grow < p.L) {
                            uint32_t w[16];
#pragma unroll
                            for (int i = 0; i < 32; i += 2)
                                w[i / 2] = pack2<BF16>(__uint_as_float(ov[i]) * inv, __uint_as_float(ov[i + 1]) * inv);
                            uint4* dst = (uint4*)(orow + c * 32);
#pragma unroll
                            for (int q4 = 0; q4 < 4; ++q4)
                                dst[q4] = make_uint4(w[4 * q4], w[4 * q4 + 1], w[4 * q4 + 2], w[4 * q4 + 3]);
                        }
                    }
                    if (p.lse && grow < p.L)
                        p.lse[((int64_t)b * p.H + h) * p.L + grow] =
                            lsum > 0.0f ? (m_used + log2f(lsum)) * 0.69314718055994531f : -INFINITY;
                    tc_fence_before();
                    mbar_arrive(&o_empty[t]);  // O_t has been read: the next item's PV may overwrite it
                    ++nf;
                }
            } else {
                ok = false;
            }
        }
        if (!ok) *(volatile int*)abort_flag = 1;
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

}  // namespace

// ------------------------------------------------------------------ host side

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)ptr;
    });
    return fn;
}

// 4-D map over (d, row, head, batch) with a 64 x box_rows box and 128-byte swizzle
bool make_tma_map_4d(CUtensorMap* tm, const gtb_tensor4& t, int64_t d_extent, bool bf16, int box_rows) {
    auto enc = encode_fn();
    if (!enc) {
        set_error("flash_attention: cuTensorMapEncodeTiled is unavailable");
        return false;
    }
    cuuint64_t dims[4] = {(cuuint64_t)d_extent, (cuuint64_t)t.shape[2], (cuuint64_t)t.shape[1], (cuuint64_t)t.shape[0]};
    int64_t st[3] = {t.stride[2], t.stride[1], t.stride[0]};
    // a size-1 dimension is never stepped: give it a legal stride
    int64_t run = d_extent;
    for (int i = 0; i < 3; ++i) {
        if (dims[i + 1] == 1) st[i] = run;
        run = st[i] * (int64_t)dims[i + 1];
    }
    cuuint64_t strides[3];
    for (int i = 0; i < 3; ++i) {
        const int64_t bytes = st[i] * 2;
        if (bytes <= 0 || bytes % 16 != 0 || bytes >= (1ll << 40)) {
            set_error("flash_attention: a stride is not a positive multiple of 16 bytes");
            return false;
        }
        strides[i] = (cuuint64_t)bytes;
    }
    cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(tm, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, t.data, dims,
                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_errorf("flash_attention: cuTensorMapEncodeTiled failed (%d)", (int)r);
        return false;
    }
    return true;
}

namespace {

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

template <int D, bool BF16, int EMU, bool MASK, bool DROP, bool ROPE = false>
int run(const FwdArgs& a, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const MaskView& mview,
        cudaStream_t st) {
    using C = Cfg<D>;
    auto kern_p = fwd_sm100_kernel<D, BF16, EMU, true, MASK, DROP, ROPE>;
    auto kern_1 = fwd_sm100_kernel<D, BF16, EMU, false, MASK, DROP, ROPE>;
    static bool attr_set = false;  // benign race: setting the same attribute twice is harmless
    if (!attr_set) {
        if (cuda_failed(cudaFuncSetAttribute(kern_p, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM),
                        "cudaFuncSetAttribute(fwd_sm100)") ||
            cuda_failed(cudaFuncSetAttribute(kern_1, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM),
                        "cudaFuncSetAttribute(fwd_sm100)"))
            return -1;
        // setmaxnreg.inc waits until the block's registers cover the split: refuse to launch a build
        // whose kernels were compiled with fewer registers a thread than the split assumes
        for (auto kern : {kern_p, kern_1}) {
            cudaFuncAttributes fa;
            if (cuda_failed(cudaFuncGetAttributes(&fa, kern), "cudaFuncGetAttributes(fwd_sm100)")) return -1;
            if ((int64_t)fa.numRegs * NTHREADS < 128 * REG_LO + 256 * REG_HI) {
                set_errorf("flash_attention (sm100): kernel built with %d registers a thread, below the %d the "
                           "register split needs", fa.numRegs, (128 * REG_LO + 256 * REG_HI + NTHREADS - 1) / NTHREADS);
                return -1;
            }
        }
        attr_set = true;
    }
    Params p;
    p.H = a.sh.H; p.Hkv = a.sh.Hkv; p.L = a.sh.L; p.S = a.sh.S;
    p.group = (int)(a.sh.H / a.sh.Hkv);
    p.n_pairs = (int)((a.sh.L + 2 * BM - 1) / (2 * BM));
    p.scale_log2 = a.scale * 1.4426950408889634f;
    p.causal = a.causal;
    p.o = a.o.data;
    p.os0 = a.o.stride[0]; p.os1 = a.o.stride[1]; p.os2 = a.o.stride[2];
    p.lse = (float*)a.lse;
    p.mk = mview;
    p.drop_thr = a.drop_thr;
    p.drop_seed = a.drop_seed;
    p.inv_keep = 1.0f / (1.0f - a.drop_p);
    p.rope_tab = a.rope_q_tab;
    p.rope_pairs = a.rope_n_dims / 2;
    p.rope_mode = a.rope_mode;
    int dev = 0;
    cudaGetDevice(&dev);
    p.status = device_status_word(dev);
    p.B = a.sh.B;
    const int64_t items = (int64_t)p.n_pairs * a.sh.H * a.sh.B;
    if (items >= INT32_MAX) {
        set_error("flash_attention (sm100): too many work items");
        return -1;
    }
    p.n_items = (int)items;
    static int n_sm = 0;
    if (n_sm == 0 && (cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n_sm <= 0))
        n_sm = 148;
    // persistent for sequences of up to 32 tile pairs (8192 rows): there the start-up of each short
    // item is worth hiding; longer ones keep the blockIdx order (see the kernel's comment)
    p.claim = nullptr;
    if (p.n_pairs > 32) {
        kern_1<<<(unsigned)items, NTHREADS, C::SMEM, st>>>(mq, mk, mv, p);
        return cuda_failed(cudaGetLastError(), "flash_attention (sm100) launch") ? -1 : 0;
    }
    const int grid = (int)min((int64_t)n_sm, items);  // one CTA per SM
    // the item counter: 4 bytes of the stream-ordered pool, zeroed on the stream
    retain_pool_memory(dev);
    int* claim = nullptr;
    if (cuda_failed(cudaMallocAsync((void**)&claim, sizeof(int), st), "flash_attention (sm100): item counter") ||
        cuda_failed(cudaMemsetAsync(claim, 0, sizeof(int), st), "flash_attention (sm100): item counter reset"))
        return -1;
    p.claim = claim;
    kern_p<<<grid, NTHREADS, C::SMEM, st>>>(mq, mk, mv, p);
    const bool bad = cuda_failed(cudaGetLastError(), "flash_attention (sm100) launch");
    cudaFreeAsync(claim, st);
    return bad ? -1 : 0;
}

// Exponentials computed by exp2_poly2 per 8 (GTB_FWD_EMU=0|2|4, default 0).
int emu_setting() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("GTB_FWD_EMU");
        v = e ? atoi(e) : 0;
        if (v != 0 && v != 2 && v != 4) v = 0;
    }
    return v;
}

template <int D, bool BF16>
int run_emu(const FwdArgs& a, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const MaskView& mview,
            cudaStream_t st) {
    // RoPE of q inside the kernel: no mask, no dropout (the caller checks), MUFU exponentials
    if (a.rope_q_tab) return run<D, BF16, 0, false, false, true>(a, mq, mk, mv, mview, st);
    // masked or dropout: MUFU exponentials only
    if (a.drop_p > 0.0f)
        return mview.data ? run<D, BF16, 0, true, true>(a, mq, mk, mv, mview, st)
                          : run<D, BF16, 0, false, true>(a, mq, mk, mv, mview, st);
    if (mview.data) return run<D, BF16, 0, true, false>(a, mq, mk, mv, mview, st);
    switch (emu_setting()) {
        case 4: return run<D, BF16, 4, false, false>(a, mq, mk, mv, mview, st);
        case 2: return run<D, BF16, 2, false, false>(a, mq, mk, mv, mview, st);
        default: return run<D, BF16, 0, false, false>(a, mq, mk, mv, mview, st);
    }
}

}  // namespace

bool fwd_sm100_supported(const FwdArgs& a) {
    if (a.has_mask && !mask_supported(a.mask)) return false;
    if (a.q.dtype != BF16 && a.q.dtype != F16) return false;
    if (a.k.dtype != a.q.dtype || a.v.dtype != a.q.dtype || a.o.dtype != a.q.dtype) return false;
    if (a.sh.D != a.sh.Dv || (a.sh.D != 64 && a.sh.D != 128)) return false;
    if (a.q.stride[3] != 1 || a.k.stride[3] != 1 || a.v.stride[3] != 1 || a.o.stride[3] != 1) return false;
    if (!aligned16(a.q.data) || !aligned16(a.k.data) || !aligned16(a.v.data) || !aligned16(a.o.data)) return false;
    for (int i = 0; i < 3; ++i) {
        if (a.o.stride[i] % 8 != 0) return false;  // 16-byte vector stores of output rows
        if ((a.q.shape[i] > 1 && a.q.stride[i] % 8 != 0) || (a.k.shape[i] > 1 && a.k.stride[i] % 8 != 0) ||
            (a.v.shape[i] > 1 && a.v.stride[i] % 8 != 0))
            return false;
    }
    if (a.sh.L >= (1ll << 30) || a.sh.S >= (1ll << 30) || a.sh.H > 65535 || a.sh.B > 65535) return false;
    if (a.sh.L < 1 || a.sh.S < 1) return false;
    return encode_fn() != nullptr;
}

int launch_fwd_sm100(const FwdArgs& a, cudaStream_t st) {
    const bool bf16 = a.q.dtype == BF16;
    CUtensorMap mq, mk, mv;
    if (!make_tma_map_4d(&mq, a.q, a.sh.D, bf16, BM) || !make_tma_map_4d(&mk, a.k, a.sh.D, bf16, BN) ||
        !make_tma_map_4d(&mv, a.v, a.sh.Dv, bf16, BN))
        return -1;
    MaskView mview;
    void* table = nullptr;
    if (a.has_mask && build_mask_view(a.mask, a.sh.B, a.sh.H, a.sh.L, a.sh.S, a.scale, mview, &table, st) != 0) return -1;
    int rc;
    if (a.sh.D == 128)
        rc = bf16 ? run_emu<128, true>(a, mq, mk, mv, mview, st) : run_emu<128, false>(a, mq, mk, mv, mview, st);
    else
        rc = bf16 ? run_emu<64, true>(a, mq, mk, mv, mview, st) : run_emu<64, false>(a, mq, mk, mv, mview, st);
    if (table) cudaFreeAsync(table, st);  // after the kernel on the same stream
    return rc;
}

}  // namespace gtb
