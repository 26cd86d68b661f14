// Attention backward for sm_100a: tcgen05 tensor cores, TMEM accumulators, TMA tiles.
//
// The reference's backward (FlashAttentionFn.backward, gguf_train/_functions.py:1934-1965) recomputes
// the probabilities with separate matmul / softmax / elementwise ops and materialises several
// (B, H, L, S) tensors. Here it is a few kernels that never hold more than 128x128 tiles:
//
//   preprocess  per query row: -delta = -sum(dO * O), -lse2 = -lse * log2(e) (-inf for rows that are
//               padding or had no allowed key, so their probabilities come out 0); both stored negated
//               (the main kernels add them) in (B, H, Lpad) buffers, Lpad = L rounded up to 128, so
//               tiles load with bulk copies.
//   dK/dV       one CTA per 128-key block of one (batch, kv head); it loops over the 128-row query
//               tiles of every query head of the kv head's group, so dK and dV are complete when the
//               CTA ends (no cross-CTA reduction). Each query tile is two sub-items of 64 queries;
//               per sub-item h, in TMEM (lane = key):
//                 S^T = K Q_h^T, dP^T = V dO_h^T                  (M=128 keys, N=64 queries, K=D)
//                 P^T = exp2(S^T * scale*log2e - lse2), dS^T = P^T * (dP^T - delta)
//                 dV += P^T dO_h, dK += dS^T Q_h                   (M=128, N=D, K=64; P^T from TMEM)
//               With D = 128 the same CTA also forms the sub-item's share of dQ (fused dQ):
//                 dQ_h^T = K^T dS^T                                (M=128 head dims, N=64, K=128 keys)
//               with dS^T written to shared memory (the B operand here and the A operand of dK) and
//               dQ_h^T accumulated into the dP^T columns it no longer needs; the compute warps add it
//               to f32 sums (B, H, Lpad, D) in global memory with reductions performed at L2, and a
//               conversion kernel writes dq = scale * sums. Five GEMM-shaped products per tile
//               instead of seven; the bits of dq may vary in the last place from run to run.
//   dQ          (D = 64, or GTB_BWD_SPLIT_DQ=1) one CTA per 128-row query tile; it loops over the
//               128-key blocks the tile attends, each two sub-items of 64 keys:
//                 S = Q K_h^T, dP = dO V_h^T, dS = P * (dP - delta), dQ += dS K_h  (A from TMEM)
// TMEM columns: dK/dV kernel: dV [0,D), dK [128,128+D), S^T of sub-item h [256+64h, 320+64h),
//               dP^T (then dQ_h^T) of sub-item h [384+64h, 448+64h); dQ kernel: S_h [64h, 64h+64),
//               dP_h [128+64h, 192+64h), dQ [256,256+D), and the tile's Q [384, 384+D/2) and
//               dO [448, 448+D/2) (16-bit pairs), the A operands of S and dP (TS-form MMAs: Q and
//               dO are the same for every key block, so they are read from TMEM, not shared memory).
// P^T / dS^T / dS (bf16 or f16, packed two per column) are written back over the first 32 of the
// S / dP columns of their sub-item: chunk c (32 columns) lands in columns 16c..16c+15, read before
// (dS^T goes to shared memory instead when dQ is fused).
//
// Warps (both main kernels): 0 = TMA producer, 1 = TMEM owner and MMA issuer (one thread), 2-9 =
// two compute warpgroups, one key (dK/dV) or query (dQ) row per thread: warpgroup h computes
// sub-item h of every tile (ping-pong). While one warpgroup exponentiates, the tensor core runs the
// other sub-item's MMAs; the MMA thread issues sub-item h of the next tile right after the
// gradient MMAs of sub-item h of this one (tcgen05 MMAs of one thread run in issue order, which
// is what lets them reuse the columns those MMAs read). Causal masking is top-left (key s masked for
// query l when s > l), as in gt_flash_attention (csrc/gt_ops_nn.cpp:2476). Every wait is bounded as in
// the forward kernel: a timeout records a status code, drains, frees TMEM and returns.

#include <cmath>
#include <mutex>
#include <type_traits>

#include "dropout.cuh"
#include "gtb_common.cuh"
#include "mask_tiles.cuh"
#include "sdpa_args.h"
#include "sm100_ptx.cuh"

namespace gtb {
namespace {

using namespace sm100;

constexpr int BT = 128;        // rows of a query tile and of a key block
constexpr int NTHREADS = 320;  // 10 warps: TMA, MMA, two compute warpgroups
constexpr int HB = BT / 2;     // rows of a sub-item
constexpr int NCOMP = 256;     // compute threads (two warpgroups)
constexpr int SB_UNITS = 4;    // (batch, head) units per superblock of the block order
constexpr uint32_t TMEM_COLS = 512;
constexpr float LOG2E = 1.4426950408889634f;

template <int D>
struct BCfg {
    static constexpr int ATOMS = D / 64;      // 64-column (128-byte) slabs along D
    static constexpr int TILE = BT * D * 2;   // one 128-row tile of Q, K, V or dO
    static constexpr int SLAB = BT * 128;     // one slab of a tile
};

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    uint32_t r;
    if constexpr (BF16) asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    else asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* status, int code) {
    const bool ok = mbar_wait(bar, parity, status, code);
    return __all_sync(0xffffffffu, ok);
}

// K-major operand descriptor: k-step kk (16 elements) of a 128-row tile made of 64-column slabs
__device__ __forceinline__ uint64_t kmajor(uint32_t base, int kk, int slab_bytes) {
    return desc_sw128(base + (uint32_t)((kk / 4) * slab_bytes + (kk % 4) * 32), 16, 1024);
}
// MN-major operand descriptor: k-step kk = rows 16kk..16kk+15 of a tile (rows are the K dimension)
__device__ __forceinline__ uint64_t mnmajor(uint32_t base, int kk, int slab_bytes) {
    return desc_sw128(base + (uint32_t)(kk * 2048), (uint32_t)slab_bytes, 1024);
}

// store 32 accumulator columns (f32 in registers) of one row as 16-bit values, times `mul`
template <bool BF16>
__device__ __forceinline__ void store_row32(void* dst, const uint32_t* v, float mul) {
    uint32_t w[16];
#pragma unroll
    for (int i = 0; i < 32; i += 2) w[i / 2] = pack2<BF16>(__uint_as_float(v[i]) * mul, __uint_as_float(v[i + 1]) * mul);
    uint4* d = (uint4*)dst;
#pragma unroll
    for (int q = 0; q < 4; ++q) d[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
}

// ------------------------------------------------------------------ preprocess

struct PreP {
    const void* o;
    const void* g;            // dO
    int64_t os0, os1, os2;    // strides of O (b, h, l); d stride 1
    int64_t gs0, gs1, gs2;    // strides of dO
    const float* lse;         // (B, H, L)
    float* lse2;              // (B, H, Lpad): -lse * log2(e)
    float* delta;             // (B, H, Lpad): -sum(dO * O)
    int64_t B, H, L, Lpad, D;
};

template <typename T>
__global__ void __launch_bounds__(128) bwd_pre_kernel(PreP p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * 4 + warp;  // over B*H*Lpad
    if (row >= p.B * p.H * p.Lpad) return;
    const int64_t l = row % p.Lpad, bh = row / p.Lpad, h = bh % p.H, b = bh / p.H;
    float acc = 0.0f;
    if (l < p.L) {
        const T* o = (const T*)p.o + b * p.os0 + h * p.os1 + l * p.os2;
        const T* g = (const T*)p.g + b * p.gs0 + h * p.gs1 + l * p.gs2;
        for (int64_t d = lane; d < p.D; d += 32) acc += (float)Elem<T>::load(o + d) * (float)Elem<T>::load(g + d);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) {
        float nl2 = -INFINITY;  // padding rows and rows without an allowed key: probabilities 0
        if (l < p.L) {
            const float lse = p.lse[bh * p.L + l];
            if (lse != -INFINITY) nl2 = -lse * LOG2E;
        }
        p.lse2[row] = nl2;
        p.delta[row] = -acc;
    }
}

// The same for 16-bit rows of D = 128 whose starts are 8-byte aligned: a warp takes 4 consecutive
// rows (l .. l+3 of one (b, h)) and issues all 8 of a lane's 8-byte loads before reducing, so that
// enough bytes are in flight to stream O and dO at HBM speed.
template <typename T>
__global__ void __launch_bounds__(128) bwd_pre128_kernel(PreP p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r0 = ((int64_t)blockIdx.x * 4 + warp) * 4;  // over B*H*Lpad; Lpad % 4 == 0
    if (r0 >= p.B * p.H * p.Lpad) return;
    const int64_t l0 = r0 % p.Lpad, bh = r0 / p.Lpad, h = bh % p.H, b = bh / p.H;
    uint2 ov[4], gv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        ov[u] = make_uint2(0u, 0u);
        gv[u] = make_uint2(0u, 0u);
        if (l0 + u < p.L) {
            ov[u] = *(const uint2*)((const T*)p.o + b * p.os0 + h * p.os1 + (l0 + u) * p.os2 + 4 * lane);
            gv[u] = *(const uint2*)((const T*)p.g + b * p.gs0 + h * p.gs1 + (l0 + u) * p.gs2 + 4 * lane);
        }
    }
    float acc[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const T* oe = (const T*)&ov[u];
        const T* ge = (const T*)&gv[u];
        acc[u] = 0.0f;
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[u] = fmaf((float)Elem<T>::load(oe + e), (float)Elem<T>::load(ge + e), acc[u]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc[u] += __shfl_xor_sync(0xffffffffu, acc[u], off);
    }
    if (lane < 4) {
        const int64_t l = l0 + lane;
        const float a = lane == 0 ? acc[0] : lane == 1 ? acc[1] : lane == 2 ? acc[2] : acc[3];
        float nl2 = -INFINITY;  // padding rows and rows without an allowed key: probabilities 0
        if (l < p.L) {
            const float lse = p.lse[bh * p.L + l];
            if (lse != -INFINITY) nl2 = -lse * LOG2E;
        }
        p.lse2[r0 + lane] = nl2;
        p.delta[r0 + lane] = l < p.L ? -a : 0.0f;
    }
}

// ------------------------------------------------------------------ dK / dV

struct KvP {
    int64_t H, Hkv, L, S, Lpad;
    int group, n_qt, n_kvt;
    float scale_log2, scale;
    int causal;
    void* dk;
    int64_t ks0, ks1, ks2;
    void* dv;
    int64_t vs0, vs1, vs2;
    const float* lse2;
    const float* delta;
    float* dqacc;  // (B, H, Lpad, D) f32, zeroed: unscaled dQ sums (fused dQ only)
    int* status;
    MaskView mk;   // attention mask (AMASK instances only)
    uint32_t drop_thr;  // dropout of the forward (DROP instances only): keep threshold, seed, 1 / (1 - p)
    uint64_t drop_seed;
    float inv_keep;
};

// Shared memory of the dK/dV kernel: K, V, two stages of (Q, dO, lse2, delta), with the fused dQ
// two 16 KB dS^T tiles, then the barrier block. The fused layout uses all 227 KB a block may have,
// so its base may sit at most SMEM_SLACK bytes past the start of dynamic shared memory.
template <int D, bool FUSE>
struct KvSmem {
    static constexpr int ST_BYTES = 2 * BCfg<D>::TILE + 1024;  // Q, dO, lse2[128], delta[128]
    static constexpr int OFF_ST = 2 * BCfg<D>::TILE;
    static constexpr int OFF_DS = OFF_ST + 2 * ST_BYTES;       // dS^T of sub-item h: 128 keys x 64 queries
    static constexpr int DS_BYTES = BT * HB * 2;
    static constexpr int OFF_BAR = OFF_DS + (FUSE ? 2 * DS_BYTES : 0);
    static constexpr int USED = OFF_BAR + 32 * 8;              // + barriers, TMEM slot, flag
    static constexpr int ALLOC = FUSE ? 232448 : USED + 1024;  // 232448 = 227 KB, the per-block maximum
    static constexpr int SLACK = ALLOC - USED;
};

template <int D, bool BF16, bool FUSE, bool AMASK, bool DROP>
__global__ void __launch_bounds__(NTHREADS, 1)
bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmG, const KvP p) {
    static_assert(!FUSE || D == 128, "the fused dQ needs M = D = 128");
    using C = BCfg<D>;
    using M = KvSmem<D, FUSE>;
    using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    constexpr int OFF_K = 0, OFF_V = C::TILE, OFF_ST = M::OFF_ST;
    constexpr int ST_BYTES = M::ST_BYTES;
    constexpr int OFF_BAR = M::OFF_BAR;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    if constexpr (M::SLACK < 1023) {
        // the tiles need 1024-byte alignment and the fused layout leaves less slack than that
        if ((uintptr_t)(smem - smem_raw) > (uintptr_t)M::SLACK) {
            if (threadIdx.x == 0) atomicCAS(p.status, 0, 40);
            return;
        }
    }
    uint64_t* bars = (uint64_t*)(smem + OFF_BAR);
    uint64_t* kv_full = bars;
    uint64_t* st_full = bars + 1;     // [2]
    uint64_t* st_empty = bars + 3;    // [2]
    uint64_t* s_full = bars + 5;      // [2] S^T, dP^T of sub-item h computed
    uint64_t* p_full = bars + 7;      // [2] P^T, dS^T of sub-item h written (128 arrivals)
    uint64_t* acc_final = bars + 9;   // every MMA done
    uint64_t* drain = bars + 10;
    uint64_t* dq_full = bars + 11;    // [2] dQ^T of sub-item h computed (fused dQ)
    uint64_t* dq_empty = bars + 13;   // [2] dQ^T of sub-item h read out of TMEM (128 arrivals)
    uint32_t* tmem_slot = (uint32_t*)(bars + 15);
    int* abort_flag = (int*)(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Block order: superblocks of SB_UNITS (batch, kv head) units, key blocks outer (block 0, the
    // heaviest under a causal mask, first) and the units inner. Every heavy CTA starts early, so no
    // long CTA is still running after the rest of the grid is done, and a superblock's Q/dO streams
    // (about 16 MB per unit at L = 8192) stay in L2 for all of its CTAs.
    int jt, hk, b;
    {
        const int nunits = (int)(gridDim.y * gridDim.z);
        const int lin = (int)(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z));
        const int per_sb = SB_UNITS * (int)gridDim.x;
        const int sb = lin / per_sb, r = lin - sb * per_sb;
        const int sbsize = min(SB_UNITS, nunits - sb * SB_UNITS);
        jt = r / sbsize;
        const int unit = sb * SB_UNITS + r % sbsize;
        hk = unit % (int)gridDim.y;
        b = unit / (int)gridDim.y;
    }
    const int key0 = jt * BT;
    // query tiles that see this key block: rows l >= key0 when causal (top-left)
    const int i_start = p.causal ? min(p.n_qt, key0 / BT) : 0;
    const int nq = p.n_qt - i_start;
    const int nit = p.group * nq;

    if (threadIdx.x == 0) {
        mbar_init(kv_full, 1);
        for (int i = 0; i < 2; ++i) { mbar_init(&st_full[i], 1); mbar_init(&st_empty[i], 1); }
        for (int h = 0; h < 2; ++h) {
            mbar_init(&s_full[h], 1); mbar_init(&p_full[h], 128);
            mbar_init(&dq_full[h], 1); mbar_init(&dq_empty[h], 128);
        }
        mbar_init(acc_final, 1);
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0 && nit > 0) {
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmG);
            mbar_expect_tx(kv_full, 2 * C::TILE);
            for (int a = 0; a < C::ATOMS; ++a) {
                tma_load_4d(smem + OFF_K + a * C::SLAB, &tmK, a * 64, key0, hk, b, kv_full);
                tma_load_4d(smem + OFF_V + a * C::SLAB, &tmV, a * 64, key0, hk, b, kv_full);
            }
            int last = -1;
            bool ok = true;
            for (int it = 0; it < nit && ok; ++it) {
                const int st = it & 1;
                if (it >= 2) ok = mbar_wait(&st_empty[st], ((it >> 1) - 1) & 1, p.status, 41);
                if (!ok || *(volatile int*)abort_flag) break;
                const int g = it / nq, i = i_start + it % nq;
                const int h = hk * p.group + g;
                unsigned char* sb = smem + OFF_ST + st * ST_BYTES;
                mbar_expect_tx(&st_full[st], ST_BYTES);
                for (int a = 0; a < C::ATOMS; ++a) {
                    tma_load_4d(sb + a * C::SLAB, &tmQ, a * 64, i * BT, h, b, &st_full[st]);
                    tma_load_4d(sb + C::TILE + a * C::SLAB, &tmG, a * 64, i * BT, h, b, &st_full[st]);
                }
                const int64_t r0 = ((int64_t)b * p.H + h) * p.Lpad + (int64_t)i * BT;
                bulk_load(sb + 2 * C::TILE, p.lse2 + r0, 512, &st_full[st]);
                bulk_load(sb + 2 * C::TILE + 512, p.delta + r0, 512, &st_full[st]);
                last = it;
            }
            if (!ok) *(volatile int*)abort_flag = 1;
            if (*(volatile int*)abort_flag) {
                mbar_wait(kv_full, 0, nullptr, 0);
                for (int it = max(0, last - 1); it <= last; ++it) mbar_wait(&st_full[it & 1], (it >> 1) & 1, nullptr, 0);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && nit > 0) {
            constexpr uint32_t IDESC_S = idesc_f16(BT, HB, BF16, false);
            constexpr uint32_t IDESC_ACC = idesc_f16(BT, D, BF16, true);
            // operand descriptors built once; per MMA only a constant is added to the start address
            const uint64_t kdk = kmajor(smem_u32(smem + OFF_K), 0, C::SLAB), vdk = kmajor(smem_u32(smem + OFF_V), 0, C::SLAB);
            const uint64_t qk0 = kmajor(smem_u32(smem + OFF_ST), 0, C::SLAB);
            const uint64_t qk1 = kmajor(smem_u32(smem + OFF_ST + ST_BYTES), 0, C::SLAB);
            const uint64_t qm0 = mnmajor(smem_u32(smem + OFF_ST), 0, C::SLAB);
            const uint64_t qm1 = mnmajor(smem_u32(smem + OFF_ST + ST_BYTES), 0, C::SLAB);
            // S^T of sub-item h (queries 64h.. of the stage's tile: 64 rows = 8 KB into each slab)
            auto issue_s = [&](int st, int h) {
                const uint64_t qk = st ? qk1 : qk0;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t off = (uint32_t)((kk / 4) * C::SLAB + (kk % 4) * 32);
                    mma_ss(tmem + 256 + HB * h, desc_advance(kdk, off), desc_advance(qk, off + h * HB * 128), IDESC_S, kk > 0);
                }
            };
            // dP^T of sub-item h; the commit covers S^T as well
            auto issue_dp = [&](int st, int h) {
                const uint64_t qk = st ? qk1 : qk0;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t off = (uint32_t)((kk / 4) * C::SLAB + (kk % 4) * 32);
                    mma_ss(tmem + 384 + HB * h, desc_advance(vdk, off), desc_advance(qk, off + h * HB * 128 + C::TILE),
                           IDESC_S, kk > 0);
                }
                mma_commit(&s_full[h]);
            };
            auto issue_sdp = [&](int st, int h) {
                issue_s(st, h);
                issue_dp(st, h);
            };
            // dS^T of sub-item h in shared memory (fused dQ): rows = keys, 64 queries per 128-byte row
            const uint32_t ds0 = smem_u32(smem + M::OFF_DS), ds1 = ds0 + M::DS_BYTES;
            // dV += P^T dO_h, dK += dS^T Q_h (k-steps over the sub-item's 64 queries)
            auto issue_grad = [&](int st, int h, bool first) {
                const uint64_t qm = st ? qm1 : qm0;
#pragma unroll
                for (int kk = 0; kk < HB / 16; ++kk) {
                    const uint32_t acc = (!first || kk > 0) ? 1u : 0u;
                    const uint32_t rows = (uint32_t)((h * (HB / 16) + kk) * 2048);
                    mma_ts(tmem + 0, tmem + 256 + HB * h + kk * 8, desc_advance(qm, rows + C::TILE), IDESC_ACC, acc);  // dV
                    if constexpr (FUSE)  // A = dS^T from shared memory (K-major)
                        mma_ss(tmem + 128, kmajor(h ? ds1 : ds0, kk, 0), desc_advance(qm, rows), IDESC_ACC, acc);  // dK
                    else
                        mma_ts(tmem + 128, tmem + 384 + HB * h + kk * 8, desc_advance(qm, rows), IDESC_ACC, acc);  // dK
                }
            };
            // dQ^T_h = K^T dS^T_h (M = 128 head dims, N = 64 queries, K = 128 keys; both operands
            // MN-major) into the columns of dP^T_h, which the compute warps have read by now
            auto issue_dq = [&](int h) {
                constexpr uint32_t IDESC_DQ = idesc_f16_amn(BT, HB, BF16, true);
                const uint64_t km = mnmajor(smem_u32(smem + OFF_K), 0, C::SLAB);
                const uint64_t dm = desc_sw128(h ? ds1 : ds0, 8192, 1024);  // one 64-query atom: LBO unused
#pragma unroll
                for (int kk = 0; kk < BT / 16; ++kk)
                    mma_ss(tmem + 384 + HB * h, desc_advance(km, (uint32_t)(kk * 2048)), desc_advance(dm, (uint32_t)(kk * 2048)),
                           IDESC_DQ, kk > 0);
                mma_commit(&dq_full[h]);
            };
            bool ok = mbar_wait(kv_full, 0, p.status, 42);
            if (ok) ok = mbar_wait(&st_full[0], 0, p.status, 43);
            if (ok && !*(volatile int*)abort_flag) {
                tc_fence_after();
                issue_sdp(0, 0);
                issue_sdp(0, 1);
            } else {
                ok = false;
            }
            for (int it = 0; it < nit && ok; ++it) {
                const int st = it & 1;
                const bool more = it + 1 < nit;
                ok = mbar_wait(&p_full[0], it & 1, p.status, 44);
                if (!ok) break;
                tc_fence_after();
                // dQ^T first: the compute warps read it out while the gradient MMAs run, so the next
                // tile's dP^T rarely waits for its columns
                if constexpr (FUSE) issue_dq(0);
                issue_grad(st, 0, it == 0);
                if (more) {  // sub-item 0 of the next tile, into the columns just read
                    ok = mbar_wait(&st_full[st ^ 1], ((it + 1) >> 1) & 1, p.status, 43);
                    if (!ok || *(volatile int*)abort_flag) { ok = false; break; }
                    tc_fence_after();
                    if constexpr (FUSE) {
                        // dP^T waits for dQ^T_0 to leave its columns; S^T keeps the tensor core busy meanwhile
                        issue_s(st ^ 1, 0);
                        ok = mbar_wait(&dq_empty[0], it & 1, p.status, 49);
                        if (!ok) break;
                        tc_fence_after();
                        issue_dp(st ^ 1, 0);
                    } else {
                        issue_sdp(st ^ 1, 0);
                    }
                }
                ok = mbar_wait(&p_full[1], it & 1, p.status, 44);
                if (!ok) break;
                tc_fence_after();
                if constexpr (FUSE) issue_dq(1);
                issue_grad(st, 1, false);
                mma_commit(&st_empty[st]);  // this tile's Q / dO are read by every MMA issued so far
                if (more) {
                    if constexpr (FUSE) {
                        issue_s(st ^ 1, 1);
                        ok = mbar_wait(&dq_empty[1], it & 1, p.status, 49);
                        if (!ok) break;
                        tc_fence_after();
                        issue_dp(st ^ 1, 1);
                    } else {
                        issue_sdp(st ^ 1, 1);
                    }
                }
            }
            if (!ok) *(volatile int*)abort_flag = 1;
            if (ok && !*(volatile int*)abort_flag) {
                mma_commit(acc_final);
            } else {
                mma_commit(drain);
                mbar_wait(drain, 0, nullptr, 0);
            }
        }
    } else {
        const int wg = (warp - 2) >> 2;  // compute warpgroup = sub-item: queries [64 wg, 64 wg + 64) of a tile
        const int quad = warp & 3;
        const int r = quad * 32 + lane;
        const int key = key0 + r;
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        unsigned char* const ds_row = smem + M::OFF_DS + wg * M::DS_BYTES + r * 128;
        bool ok = true;
        for (int it = 0; it < nit; ++it) {
            const int st = it & 1;
            const int q0 = (i_start + it % nq) * BT + wg * HB;  // first query of the sub-item
            // the attention mask's class for this query tile and key block, and the query head (the
            // class byte is read before the waits so that the load completes during them)
            const int hq_it = hk * p.group + it / nq;
            const uint8_t mcls = AMASK ? p.mk.tile_class(b, hq_it, i_start + it % nq, jt) : (uint8_t)MASK_NONE;
            const uint32_t hkey = DROP ? drop_head_key(p.drop_seed, (uint32_t)(b * p.H + hq_it)) : 0u;
            ok = warp_wait(&st_full[st], (it >> 1) & 1, p.status, 45);  // lse2 / delta of this tile
            if (ok) ok = warp_wait(&s_full[wg], it & 1, p.status, 46);
            if (!ok || __any_sync(0xffffffffu, *(volatile int*)abort_flag)) break;
            tc_fence_after();
            const float* lse_s = (const float*)(smem + OFF_ST + st * ST_BYTES + 2 * C::TILE) + wg * HB;  // -lse2
            const float* dl_s = lse_s + 128;                                                                 // -delta
            const uint64_t sc2 = f2_pack(p.scale_log2, p.scale_log2);
            // masking only where the causal diagonal crosses the sub-item: one branch per sub-item
            auto chunks = [&](auto masked) {
                constexpr bool MASK = decltype(masked)::value;
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    uint32_t ra[32], rb[32], pk[16], dk[16];
                    tmem_ld32(tmem + lane_addr + 256 + HB * wg + c * 32, ra);
                    tmem_ld32(tmem + lane_addr + 384 + HB * wg + c * 32, rb);
                    tmem_ld_wait();
                    if constexpr (AMASK) {  // scores of queries q0 + 32c .. for this thread's key
                        if (mcls == MASK_MIXED) {
                            mask_apply_col32((float*)ra, p.mk, b, hq_it, q0 + c * 32, p.L, min((int64_t)key, p.S - 1));
                        } else if (mcls == MASK_ALL) {
#pragma unroll
                            for (int i = 0; i < 32; ++i) ra[i] = __float_as_uint(-INFINITY);
                        }
                    }
                    uint32_t kbits = 0xffffffffu;  // dropout: which of the 32 queries keep this key
                    if constexpr (DROP) {
                        // lane i holds the row key of query q0 + 32c + i; every thread tests its own key
                        const uint32_t rk_lane = drop_row_key(hkey, (uint32_t)(q0 + c * 32 + lane));
                        kbits = 0;
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            kbits |= (drop_keep(__shfl_sync(0xffffffffu, rk_lane, i), (uint32_t)key, p.drop_thr) ? 1u : 0u) << i;
#pragma unroll
                        for (int i = 0; i < 32; ++i)  // dP of a dropped element contributes nothing; kept ones / (1 - p)
                            rb[i] = ((kbits >> i) & 1u) ? __float_as_uint(__uint_as_float(rb[i]) * p.inv_keep) : 0u;
                    }
#pragma unroll
                    for (int i = 0; i < 32; i += 2) {
                        // packed two-lane f32: a = S * scale - lse2, ds = p * (dP - delta)
                        const int qc = c * 32 + i;
                        float a0, a1;
                        f2_unpack(f2_fma(f2_pack(__uint_as_float(ra[i]), __uint_as_float(ra[i + 1])), sc2,
                                         *(const uint64_t*)(lse_s + qc)), a0, a1);
                        float p0 = ex2(a0), p1 = ex2(a1);
                        if constexpr (MASK) {
                            if (key > q0 + qc) p0 = 0.0f;
                            if (key > q0 + qc + 1) p1 = 0.0f;
                        }
                        float d0, d1;
                        f2_unpack(f2_mul(f2_pack(p0, p1), f2_add(f2_pack(__uint_as_float(rb[i]), __uint_as_float(rb[i + 1])),
                                                                 *(const uint64_t*)(dl_s + qc))), d0, d1);
                        if constexpr (DROP) {  // dV takes the kept probabilities (scaled at the store)
                            if (!((kbits >> i) & 1u)) p0 = 0.0f;
                            if (!((kbits >> (i + 1)) & 1u)) p1 = 0.0f;
                        }
                        pk[i / 2] = pack2<BF16>(p0, p1);
                        dk[i / 2] = pack2<BF16>(d0, d1);
                    }
                    tmem_st16(tmem + lane_addr + 256 + HB * wg + c * 16, pk);
                    if constexpr (FUSE) {
                        // row r of the 128-byte-swizzled dS^T tile: 16-byte chunk j sits at j ^ (r & 7)
                        unsigned char* row = ds_row;
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            *(uint4*)(row + (((4 * c + j) ^ (r & 7)) << 4)) =
                                make_uint4(dk[4 * j], dk[4 * j + 1], dk[4 * j + 2], dk[4 * j + 3]);
                    } else {
                        tmem_st16(tmem + lane_addr + 384 + HB * wg + c * 16, dk);
                    }
                }
            };
            if (p.causal && (q0 < key0 + BT - 1)) chunks(std::true_type{});
            else chunks(std::false_type{});
            tmem_st_wait();
            if constexpr (FUSE) fence_proxy_async_smem();  // dS^T is read by the tensor core
            tc_fence_before();
            mbar_arrive(&p_full[wg]);
            if constexpr (FUSE) {
                // dQ^T of the sub-item (lane = head dim r, column = query): read it out of TMEM, free the
                // columns for the next dP^T, and add it to the f32 sums in global memory (each warp's
                // reduction covers 32 consecutive head dims of one query row: 128 contiguous bytes)
                ok = warp_wait(&dq_full[wg], it & 1, p.status, 48);
                if (!ok) break;
                tc_fence_after();
                uint32_t v[64];
                tmem_ld32(tmem + lane_addr + 384 + HB * wg, v);
                tmem_ld32(tmem + lane_addr + 384 + HB * wg + 32, v + 32);
                tmem_ld_wait();
                tc_fence_before();
                mbar_arrive(&dq_empty[wg]);
                const int hq = hk * p.group + it / nq;
                float* dst = p.dqacc + (((int64_t)b * p.H + hq) * p.Lpad + q0) * D + r;
#pragma unroll
                for (int q = 0; q < HB; ++q) red_add_f32(dst + (int64_t)q * D, __uint_as_float(v[q]));
            }
        }
        if (!ok) *(volatile int*)abort_flag = 1;
        if (nit > 0 && ok && !*(volatile int*)abort_flag) {
            ok = warp_wait(acc_final, 0, p.status, 47);
            if (ok) {
                tc_fence_after();
                T* dvrow = (T*)p.dv + (int64_t)b * p.vs0 + (int64_t)hk * p.vs1 + (int64_t)key * p.vs2;
                T* dkrow = (T*)p.dk + (int64_t)b * p.ks0 + (int64_t)hk * p.ks1 + (int64_t)key * p.ks2;
#pragma unroll
                for (int c2 = 0; c2 < D / 64; ++c2) {
                    const int c = wg * (D / 64) + c2;  // this warpgroup's half of the D columns
                    uint32_t v[32];
                    tmem_ld32(tmem + lane_addr + c * 32, v);
                    tmem_ld_wait();
                    if (key < p.S) store_row32<BF16>(dvrow + c * 32, v, DROP ? p.inv_keep : 1.0f);
                    tmem_ld32(tmem + lane_addr + 128 + c * 32, v);
                    tmem_ld_wait();
                    if (key < p.S) store_row32<BF16>(dkrow + c * 32, v, p.scale);
                }
            } else {
                *(volatile int*)abort_flag = 1;
            }
        } else if (nit == 0 && key < p.S) {
            // no query sees this key block: its gradients are zero
            T* dvrow = (T*)p.dv + (int64_t)b * p.vs0 + (int64_t)hk * p.vs1 + (int64_t)key * p.vs2;
            T* dkrow = (T*)p.dk + (int64_t)b * p.ks0 + (int64_t)hk * p.ks1 + (int64_t)key * p.ks2;
            for (int d = wg * (D / 2); d < (wg + 1) * (D / 2); d += 8) {
                *(uint4*)(dvrow + d) = make_uint4(0, 0, 0, 0);
                *(uint4*)(dkrow + d) = make_uint4(0, 0, 0, 0);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

// ------------------------------------------------------------------ dQ

struct DqP {
    int64_t H, Hkv, L, S, Lpad;
    int group, n_qt, n_kvt;
    float scale_log2, scale;
    int causal;
    void* dq;
    int64_t s0, s1, s2;
    const float* lse2;
    const float* delta;
    int* status;
    MaskView mk;  // attention mask (AMASK instances only)
    uint32_t drop_thr;
    uint64_t drop_seed;
    float inv_keep;
};

template <int D, bool BF16, bool AMASK, bool DROP>
__global__ void __launch_bounds__(NTHREADS, 1)
bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
              const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmG, const DqP p) {
    using C = BCfg<D>;
    using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    constexpr int OFF_Q = 0, OFF_G = C::TILE, OFF_K = 2 * C::TILE, OFF_V = 4 * C::TILE, OFF_BAR = 6 * C::TILE;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = (uint64_t*)(smem + OFF_BAR);
    uint64_t* qg_full = bars;
    uint64_t* k_full = bars + 1;    // [2]
    uint64_t* k_empty = bars + 3;   // [2]
    uint64_t* v_full = bars + 5;    // [2]
    uint64_t* v_empty = bars + 7;   // [2]
    uint64_t* s_full = bars + 9;    // [2] S, dP of sub-item h computed
    uint64_t* ds_full = bars + 11;  // [2] dS of sub-item h written (128 arrivals)
    uint64_t* dq_final = bars + 13;
    uint64_t* drain = bars + 14;
    uint64_t* qt_full = bars + 15;  // Q and dO copied into TMEM (NCOMP arrivals)
    uint32_t* tmem_slot = (uint32_t*)(bars + 16);
    int* abort_flag = (int*)(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Block order: superblocks of SB_UNITS (batch, head) units (the query heads of one kv head when
    // H / Hkv = SB_UNITS), query tiles outer (the heaviest, last tile first under a causal mask) and
    // the units inner, for the same reason as in the dK/dV kernel.
    int tile, h, b;
    {
        const int nunits = (int)(gridDim.y * gridDim.z);
        const int lin = (int)(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z));
        const int per_sb = SB_UNITS * (int)gridDim.x;
        const int sb = lin / per_sb, r = lin - sb * per_sb;
        const int sbsize = min(SB_UNITS, nunits - sb * SB_UNITS);
        const int ti = r / sbsize;
        const int unit = sb * SB_UNITS + r % sbsize;
        tile = p.causal ? (p.n_qt - 1 - ti) : ti;
        h = unit % (int)gridDim.y;
        b = unit / (int)gridDim.y;
    }
    const int hk = h / p.group;
    const int row0 = tile * BT;
    const int last_row = (int)min((int64_t)row0 + BT - 1, p.L - 1);
    const int nblk = p.causal ? min(p.n_kvt, last_row / BT + 1) : p.n_kvt;

    if (threadIdx.x == 0) {
        mbar_init(qg_full, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&k_full[i], 1); mbar_init(&k_empty[i], 1);
            mbar_init(&v_full[i], 1); mbar_init(&v_empty[i], 1);
        }
        for (int h = 0; h < 2; ++h) { mbar_init(&s_full[h], 1); mbar_init(&ds_full[h], 128); }
        mbar_init(dq_final, 1);
        mbar_init(drain, 1);
        mbar_init(qt_full, NCOMP);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    constexpr uint32_t QCOL = 384, GCOL = 448;  // Q, dO in TMEM (16-bit pairs)

    if (warp == 0) {
        if (lane == 0) {
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmV);
            int last_k = -1, last_v = -1;
            bool ok = true;
            mbar_expect_tx(qg_full, 2 * C::TILE);
            for (int a = 0; a < C::ATOMS; ++a) {
                tma_load_4d(smem + OFF_Q + a * C::SLAB, &tmQ, a * 64, row0, h, b, qg_full);
                tma_load_4d(smem + OFF_G + a * C::SLAB, &tmG, a * 64, row0, h, b, qg_full);
            }
            for (int j = 0; j < nblk && ok; ++j) {
                const int s = j & 1;
                if (j >= 2) ok = mbar_wait(&k_empty[s], ((j >> 1) - 1) & 1, p.status, 51);
                if (!ok || *(volatile int*)abort_flag) break;
                mbar_expect_tx(&k_full[s], C::TILE);
                for (int a = 0; a < C::ATOMS; ++a)
                    tma_load_4d(smem + OFF_K + s * C::TILE + a * C::SLAB, &tmK, a * 64, j * BT, hk, b, &k_full[s]);
                last_k = j;
                if (j >= 2) ok = mbar_wait(&v_empty[s], ((j >> 1) - 1) & 1, p.status, 52);
                if (!ok || *(volatile int*)abort_flag) break;
                mbar_expect_tx(&v_full[s], C::TILE);
                for (int a = 0; a < C::ATOMS; ++a)
                    tma_load_4d(smem + OFF_V + s * C::TILE + a * C::SLAB, &tmV, a * 64, j * BT, hk, b, &v_full[s]);
                last_v = j;
            }
            if (!ok) *(volatile int*)abort_flag = 1;
            if (*(volatile int*)abort_flag) {
                mbar_wait(qg_full, 0, nullptr, 0);
                for (int j = max(0, last_k - 1); j <= last_k; ++j) mbar_wait(&k_full[j & 1], (j >> 1) & 1, nullptr, 0);
                for (int j = max(0, last_v - 1); j <= last_v; ++j) mbar_wait(&v_full[j & 1], (j >> 1) & 1, nullptr, 0);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t IDESC_S = idesc_f16(BT, HB, BF16, false);
            constexpr uint32_t IDESC_DQ = idesc_f16(BT, D, BF16, true);
            const uint64_t kb0 = kmajor(smem_u32(smem + OFF_K), 0, C::SLAB), kb1 = kmajor(smem_u32(smem + OFF_K + C::TILE), 0, C::SLAB);
            const uint64_t vb0 = kmajor(smem_u32(smem + OFF_V), 0, C::SLAB), vb1 = kmajor(smem_u32(smem + OFF_V + C::TILE), 0, C::SLAB);
            const uint64_t km0 = mnmajor(smem_u32(smem + OFF_K), 0, C::SLAB), km1 = mnmajor(smem_u32(smem + OFF_K + C::TILE), 0, C::SLAB);
            // S_h = Q K_h^T (keys 64h.. of the block: 64 rows = 8 KB into each slab)
            auto issue_s = [&](int s, int h) {
                const uint64_t kb = s ? kb1 : kb0;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t off = (uint32_t)((kk / 4) * C::SLAB + (kk % 4) * 32);
                    mma_ts(tmem + HB * h, tmem + QCOL + kk * 8, desc_advance(kb, off + h * HB * 128), IDESC_S, kk > 0);
                }
            };
            // dP_h = dO V_h^T
            auto issue_dp = [&](int s, int h) {
                const uint64_t vb = s ? vb1 : vb0;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t off = (uint32_t)((kk / 4) * C::SLAB + (kk % 4) * 32);
                    mma_ts(tmem + 128 + HB * h, tmem + GCOL + kk * 8, desc_advance(vb, off + h * HB * 128), IDESC_S, kk > 0);
                }
                mma_commit(&s_full[h]);
            };
            // dQ += dS_h K_h (k-steps over the sub-item's 64 keys)
            auto issue_dq = [&](int s, int h, bool first) {
                const uint64_t km = s ? km1 : km0;
#pragma unroll
                for (int kk = 0; kk < HB / 16; ++kk)
                    mma_ts(tmem + 256, tmem + HB * h + kk * 8, desc_advance(km, (uint32_t)((h * (HB / 16) + kk) * 2048)), IDESC_DQ,
                           (!first || kk > 0) ? 1u : 0u);
            };
            // both sub-items of block j: S needs K, dP needs V
            auto issue_block_sdp = [&](int j, int h) -> bool {
                const int s = j & 1;
                if (h == 0) {
                    if (!mbar_wait(&k_full[s], (j >> 1) & 1, p.status, 54) || *(volatile int*)abort_flag) return false;
                    if (!mbar_wait(&v_full[s], (j >> 1) & 1, p.status, 55)) return false;
                    tc_fence_after();
                }
                issue_s(s, h);
                issue_dp(s, h);
                if (h == 1) mma_commit(&v_empty[s]);  // V of block j is read by both dP MMAs
                return true;
            };
            bool ok = mbar_wait(qt_full, 0, p.status, 53);  // Q and dO in TMEM
            if (ok) tc_fence_after();
            if (ok && nblk > 0) ok = issue_block_sdp(0, 0) && issue_block_sdp(0, 1);
            for (int j = 0; j < nblk && ok; ++j) {
                const int s = j & 1;
                const bool more = j + 1 < nblk;
                ok = mbar_wait(&ds_full[0], j & 1, p.status, 56);
                if (!ok) break;
                tc_fence_after();
                issue_dq(s, 0, j == 0);
                if (more && !(ok = issue_block_sdp(j + 1, 0))) break;  // into the columns just read
                ok = mbar_wait(&ds_full[1], j & 1, p.status, 56);
                if (!ok) break;
                tc_fence_after();
                issue_dq(s, 1, false);
                mma_commit(&k_empty[s]);  // K of block j is read by every MMA issued so far
                if (more) issue_block_sdp(j + 1, 1);
            }
            if (!ok) *(volatile int*)abort_flag = 1;
            if (ok && !*(volatile int*)abort_flag) {
                mma_commit(dq_final);
            } else {
                mma_commit(drain);
                mbar_wait(drain, 0, nullptr, 0);
            }
        }
    } else {
        const int wg = (warp - 2) >> 2;  // compute warpgroup = sub-item: keys [64 wg, 64 wg + 64) of a block
        const int quad = warp & 3;
        const int r = quad * 32 + lane;
        const int row = row0 + r;
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        const int64_t prow = ((int64_t)b * p.H + h) * p.Lpad + row;  // row < Lpad
        const float nlse2 = p.lse2[prow];  // stored negated
        const float ndl = p.delta[prow];
        const uint64_t sc2 = f2_pack(p.scale_log2, p.scale_log2), nl2 = f2_pack(nlse2, nlse2), nd2 = f2_pack(ndl, ndl);
        const int lim_s = (int)min(p.S, (int64_t)INT32_MAX) - 1;
        const int lim = p.causal ? min(lim_s, row) : lim_s;  // last key this row may see
        const unsigned char* mrow = nullptr;  // mask entries of this row (padding rows read row L-1)
        if constexpr (AMASK) mrow = p.mk.row(b, h, min((int64_t)row, p.L - 1));
        const uint32_t rkey = DROP ? drop_row_key(drop_head_key(p.drop_seed, (uint32_t)(b * p.H + h)), (uint32_t)row) : 0u;
        // warpgroup 0 copies its row of Q, warpgroup 1 its row of dO, from the 128-byte-swizzled tile
        // into TMEM (16-byte chunk c of row r of a 64-column slab sits at chunk c ^ (r & 7))
        bool ok = warp_wait(qg_full, 0, p.status, 59);
        if (ok) {
            const unsigned char* src = smem + (wg ? OFF_G : OFF_Q) + r * 128;
#pragma unroll
            for (int a = 0; a < C::ATOMS; ++a) {
                uint32_t w[32];
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const uint4 v = *(const uint4*)(src + a * C::SLAB + ((c ^ (r & 7)) << 4));
                    w[4 * c] = v.x; w[4 * c + 1] = v.y; w[4 * c + 2] = v.z; w[4 * c + 3] = v.w;
                }
                tmem_st32(tmem + lane_addr + (wg ? GCOL : QCOL) + a * 32, w);
            }
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(qt_full);
        }
        for (int j = 0; j < nblk && ok; ++j) {
            // the attention mask's class of this key block, read before the wait
            const uint8_t mcls = AMASK ? p.mk.tile_class(b, h, tile, j) : (uint8_t)MASK_NONE;
            ok = warp_wait(&s_full[wg], j & 1, p.status, 57);
            if (!ok || __any_sync(0xffffffffu, *(volatile int*)abort_flag)) break;
            tc_fence_after();
            const int kv0 = j * BT + wg * HB;  // first key of the sub-item
            // masking only on ragged or diagonal blocks: one branch per sub-item
            auto chunks = [&](auto masked) {
                constexpr bool MASK = decltype(masked)::value;
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    uint32_t ra[32], rb[32], pk[16];
                    tmem_ld32(tmem + lane_addr + HB * wg + c * 32, ra);
                    tmem_ld32(tmem + lane_addr + 128 + HB * wg + c * 32, rb);
                    tmem_ld_wait();
                    if constexpr (AMASK) {  // keys kv0 + 32c .. of this thread's query row
                        if (mcls == MASK_MIXED) {
                            mask_apply32((float*)ra, p.mk, mrow, kv0 + c * 32, p.S);
                        } else if (mcls == MASK_ALL) {
#pragma unroll
                            for (int i = 0; i < 32; ++i) ra[i] = __float_as_uint(-INFINITY);
                        }
                    }
                    if constexpr (DROP) {  // dP of a dropped element contributes nothing; kept ones / (1 - p)
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            rb[i] = drop_keep(rkey, (uint32_t)(kv0 + c * 32 + i), p.drop_thr)
                                        ? __float_as_uint(__uint_as_float(rb[i]) * p.inv_keep) : 0u;
                    }
#pragma unroll
                    for (int i = 0; i < 32; i += 2) {
                        // packed two-lane f32: a = S * scale - lse2, ds = p * (dP - delta)
                        float a0, a1;
                        f2_unpack(f2_fma(f2_pack(__uint_as_float(ra[i]), __uint_as_float(ra[i + 1])), sc2, nl2), a0, a1);
                        float p0 = ex2(a0), p1 = ex2(a1);
                        if constexpr (MASK) {
                            if (kv0 + c * 32 + i > lim) p0 = 0.0f;
                            if (kv0 + c * 32 + i + 1 > lim) p1 = 0.0f;
                        }
                        float d0, d1;
                        f2_unpack(f2_mul(f2_pack(p0, p1), f2_add(f2_pack(__uint_as_float(rb[i]), __uint_as_float(rb[i + 1])), nd2)),
                                  d0, d1);
                        pk[i / 2] = pack2<BF16>(d0, d1);
                    }
                    tmem_st16(tmem + lane_addr + HB * wg + c * 16, pk);
                }
            };
            if ((kv0 + HB > p.S) || (p.causal && kv0 + HB - 1 > row0)) chunks(std::true_type{});
            else chunks(std::false_type{});
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(&ds_full[wg]);
        }
        if (!ok) *(volatile int*)abort_flag = 1;
        if (ok && !*(volatile int*)abort_flag) {
            ok = warp_wait(dq_final, 0, p.status, 58);
            if (ok) {
                tc_fence_after();
                T* qrow = (T*)p.dq + (int64_t)b * p.s0 + (int64_t)h * p.s1 + (int64_t)row * p.s2;
#pragma unroll
                for (int c2 = 0; c2 < D / 64; ++c2) {
                    const int c = wg * (D / 64) + c2;  // this warpgroup's half of the D columns
                    uint32_t v[32];
                    tmem_ld32(tmem + lane_addr + 256 + c * 32, v);
                    tmem_ld_wait();
                    if (row < p.L) store_row32<BF16>(qrow + c * 32, v, p.scale);
                }
            } else {
                *(volatile int*)abort_flag = 1;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

// ------------------------------------------------------------------ dQ from the fused sums

// dq[b, h, l, :] = scale * dqacc[b, h, l, :] in the 16-bit type; 16 threads per row of D = 128,
// each converting 8 values (two 16-byte loads, one 16-byte store)
template <typename T>
__global__ void __launch_bounds__(256) bwd_dq_convert_kernel(const float* __restrict__ acc, T* __restrict__ dq, int64_t s0,
                                                             int64_t s1, int64_t s2, int64_t H, int64_t L, int64_t Lpad,
                                                             int64_t n, float scale) {
    const int64_t idx = (int64_t)blockIdx.x * 256 + threadIdx.x;  // over B*H*L*16
    if (idx >= n) return;
    const int seg = (int)(idx & 15);
    const int64_t row = idx >> 4, l = row % L, bh = row / L, h = bh % H, b = bh / H;
    const float4* src = (const float4*)(acc + ((bh * Lpad + l) * 128 + seg * 8));
    const float4 x = src[0], y = src[1];
    uint32_t w[4];
    w[0] = pack2<std::is_same<T, __nv_bfloat16>::value>(x.x * scale, x.y * scale);
    w[1] = pack2<std::is_same<T, __nv_bfloat16>::value>(x.z * scale, x.w * scale);
    w[2] = pack2<std::is_same<T, __nv_bfloat16>::value>(y.x * scale, y.y * scale);
    w[3] = pack2<std::is_same<T, __nv_bfloat16>::value>(y.z * scale, y.w * scale);
    *(uint4*)(dq + b * s0 + h * s1 + l * s2 + seg * 8) = make_uint4(w[0], w[1], w[2], w[3]);
}

// ------------------------------------------------------------------ host side

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

bool fast_view(const gtb_tensor4& t, int dtype) {
    if (t.dtype != dtype || t.stride[3] != 1 || !aligned16(t.data)) return false;
    for (int i = 0; i < 3; ++i)
        if (t.shape[i] > 1 && t.stride[i] % 8 != 0) return false;
    return true;
}

int64_t lpad_of(int64_t L) { return (L + BT - 1) / BT * BT; }

// dQ summed inside the dK/dV kernel (D = 128): f32 reductions in global memory, so the bits of dQ
// may differ from run to run in the last place. A deterministic call (gtb_sdpa_bwd_ex with
// GTB_BWD_DETERMINISTIC) or GTB_BWD_SPLIT_DQ=1 in the environment selects the separate dQ kernel
// instead (recomputes S and dP per query tile; the same bits on every run).
bool fused_dq(const BwdArgs& a) {
    static const bool split = [] {
        const char* e = getenv("GTB_BWD_SPLIT_DQ");
        return e && e[0] == '1';
    }();
    return a.sh.D == 128 && !split && !a.deterministic;
}

// A non-blocking stream per device for the dQ kernel (created once, kept for the process).
cudaStream_t side_stream(int dev) {
    static cudaStream_t streams[64] = {};
    static std::once_flag once[64];
    if (dev < 0 || dev >= 64) return nullptr;
    std::call_once(once[dev], [dev] {
        if (cudaStreamCreateWithFlags(&streams[dev], cudaStreamNonBlocking) != cudaSuccess) streams[dev] = nullptr;
        cudaGetLastError();
    });
    return streams[dev];
}

template <int D, bool BF16, bool FUSE, bool AMASK, bool DROP>
int run_bwd(const BwdArgs& a, const MaskView& mview, cudaStream_t st) {
    using C = BCfg<D>;
    const int64_t B = a.sh.B, H = a.sh.H, L = a.sh.L, S = a.sh.S, Lpad = lpad_of(L);
    float* lse2 = (float*)a.scratch;
    float* delta = lse2 + B * H * Lpad;
    int dev = 0;
    cudaGetDevice(&dev);
    int* status = device_status_word(dev);

    PreP pp{a.o.data, a.dout.data, a.o.stride[0], a.o.stride[1], a.o.stride[2], a.dout.stride[0], a.dout.stride[1],
            a.dout.stride[2], (const float*)a.lse, lse2, delta, B, H, L, Lpad, a.sh.Dv};
    const int64_t rows = B * H * Lpad;
    using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    // 8-byte vector loads need every row of O and dO to start on an 8-byte boundary
    const bool vec = a.sh.Dv == 128 && (uintptr_t)a.o.data % 8 == 0 && (uintptr_t)a.dout.data % 8 == 0 &&
                     a.o.stride[0] % 4 == 0 && a.o.stride[1] % 4 == 0 && a.o.stride[2] % 4 == 0 &&
                     a.dout.stride[0] % 4 == 0 && a.dout.stride[1] % 4 == 0 && a.dout.stride[2] % 4 == 0;
    if (vec) bwd_pre128_kernel<T><<<(unsigned)((rows / 4 + 3) / 4), 128, 0, st>>>(pp);
    else bwd_pre_kernel<T><<<(unsigned)((rows + 3) / 4), 128, 0, st>>>(pp);
    if (cuda_failed(cudaGetLastError(), "flash_attention_backward: preprocess launch")) return -1;

    CUtensorMap mq, mk, mv, mg;
    if (!make_tma_map_4d(&mq, a.q, D, BF16, BT) || !make_tma_map_4d(&mk, a.k, D, BF16, BT) ||
        !make_tma_map_4d(&mv, a.v, D, BF16, BT) || !make_tma_map_4d(&mg, a.dout, D, BF16, BT))
        return -1;
    const int n_qt = (int)((L + BT - 1) / BT), n_kvt = (int)((S + BT - 1) / BT);
    const int group = (int)(H / a.sh.Hkv);
    const float scale_log2 = a.scale * LOG2E;

    static bool attr_set = false;
    constexpr int SMEM_KV = KvSmem<D, FUSE>::ALLOC;
    constexpr int SMEM_DQ = 6 * C::TILE + 32 * 8 + 1024;  // + barriers, TMEM slot, flag
    if (!attr_set) {
        if (cuda_failed(cudaFuncSetAttribute(bwd_dkdv_kernel<D, BF16, FUSE, AMASK, DROP>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_KV),
                        "cudaFuncSetAttribute(bwd dkdv)") ||
            (!FUSE && cuda_failed(cudaFuncSetAttribute(bwd_dq_kernel<D, BF16, AMASK, DROP>,
                                                       cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_DQ),
                                  "cudaFuncSetAttribute(bwd dq)")))
            return -1;
        attr_set = true;
    }
    float* dqacc = FUSE ? delta + B * H * Lpad : nullptr;
    KvP kp{H, a.sh.Hkv, L, S, Lpad, group, n_qt, n_kvt, scale_log2, a.scale, a.causal,
           a.dk.data, a.dk.stride[0], a.dk.stride[1], a.dk.stride[2],
           a.dv.data, a.dv.stride[0], a.dv.stride[1], a.dv.stride[2], lse2, delta, dqacc, status, mview,
           a.drop_thr, a.drop_seed, 1.0f / (1.0f - a.drop_p)};
    if constexpr (FUSE) {
        if (cuda_failed(cudaMemsetAsync(dqacc, 0, sizeof(float) * (size_t)(B * H * Lpad * D), st),
                        "flash_attention_backward: dQ sums reset"))
            return -1;
        bwd_dkdv_kernel<D, BF16, true, AMASK, DROP><<<dim3((unsigned)n_kvt, (unsigned)a.sh.Hkv, (unsigned)B), NTHREADS, SMEM_KV, st>>>(
            mq, mk, mv, mg, kp);
        if (cuda_failed(cudaGetLastError(), "flash_attention_backward: dK/dV/dQ launch")) return -1;
        const int64_t n = B * H * L * 16;
        bwd_dq_convert_kernel<T><<<(unsigned)((n + 255) / 256), 256, 0, st>>>(dqacc, (T*)a.dq.data, a.dq.stride[0],
                                                                          a.dq.stride[1], a.dq.stride[2], H, L, Lpad, n, a.scale);
        return cuda_failed(cudaGetLastError(), "flash_attention_backward: dQ conversion launch") ? -1 : 0;
    }
    DqP dp{H, a.sh.Hkv, L, S, Lpad, group, n_qt, n_kvt, scale_log2, a.scale, a.causal,
           a.dq.data, a.dq.stride[0], a.dq.stride[1], a.dq.stride[2], lse2, delta, status, mview,
           a.drop_thr, a.drop_seed, 1.0f / (1.0f - a.drop_p)};
    // dK/dV and dQ only share the preprocess output: dQ runs on a side stream, forked after the
    // preprocess and joined before returning, so that each kernel's last partial wave of CTAs leaves
    // no SM idle while the other still has work
    cudaStream_t side = side_stream(dev);
    cudaEvent_t fork = nullptr, join = nullptr;
    const bool two = side && cudaEventCreateWithFlags(&fork, cudaEventDisableTiming) == cudaSuccess &&
                     cudaEventCreateWithFlags(&join, cudaEventDisableTiming) == cudaSuccess &&
                     cudaEventRecord(fork, st) == cudaSuccess && cudaStreamWaitEvent(side, fork, 0) == cudaSuccess;
    cudaGetLastError();  // a failed fork falls back to one stream
    cudaStream_t dq_st = two ? side : st;
    bwd_dkdv_kernel<D, BF16, false, AMASK, DROP><<<dim3((unsigned)n_kvt, (unsigned)a.sh.Hkv, (unsigned)B), NTHREADS, SMEM_KV, st>>>(
        mq, mk, mv, mg, kp);
    bool bad = cuda_failed(cudaGetLastError(), "flash_attention_backward: dK/dV launch");
    if (!bad) {
        bwd_dq_kernel<D, BF16, AMASK, DROP><<<dim3((unsigned)n_qt, (unsigned)H, (unsigned)B), NTHREADS, SMEM_DQ, dq_st>>>(mq, mk, mv, mg, dp);
        bad = cuda_failed(cudaGetLastError(), "flash_attention_backward: dQ launch");
    }
    if (two) {
        // join even after a failed launch: later work on st (the scratch's release) must follow dQ
        if (cuda_failed(cudaEventRecord(join, side), "flash_attention_backward: join record") ||
            cuda_failed(cudaStreamWaitEvent(st, join, 0), "flash_attention_backward: join wait"))
            bad = true;
    }
    if (fork) cudaEventDestroy(fork);
    if (join) cudaEventDestroy(join);
    return bad ? -1 : 0;
}

}  // namespace

bool bwd_sm100_supported(const BwdArgs& a) {
    if (a.has_mask && !mask_supported(a.mask)) return false;
    const int dt = a.q.dtype;
    if (dt != BF16 && dt != F16) return false;
    if (a.sh.D != a.sh.Dv || (a.sh.D != 64 && a.sh.D != 128)) return false;
    const gtb_tensor4* ts[] = {&a.q, &a.k, &a.v, &a.o, &a.dout, &a.dq, &a.dk, &a.dv};
    for (const gtb_tensor4* t : ts)
        if (!fast_view(*t, dt)) return false;
    if (a.sh.L < 1 || a.sh.S < 1 || a.sh.L >= (1ll << 30) || a.sh.S >= (1ll << 30)) return false;
    if (a.sh.H > 65535 || a.sh.B > 65535 || a.sh.Hkv > 65535) return false;
    return encode_fn() != nullptr;
}

size_t bwd_sm100_scratch_bytes(const BwdArgs& a) {
    const size_t rows = (size_t)(a.sh.B * a.sh.H * lpad_of(a.sh.L));
    return sizeof(float) * rows * (2 + (fused_dq(a) ? (size_t)a.sh.D : 0));  // lse2, delta (+ dQ sums)
}

template <bool AMASK, bool DROP>
int launch_bwd_variant(const BwdArgs& a, const MaskView& mview, cudaStream_t st) {
    const bool bf16 = a.q.dtype == BF16;
    if (a.sh.D == 128) {
        if (fused_dq(a))
            return bf16 ? run_bwd<128, true, true, AMASK, DROP>(a, mview, st) : run_bwd<128, false, true, AMASK, DROP>(a, mview, st);
        return bf16 ? run_bwd<128, true, false, AMASK, DROP>(a, mview, st) : run_bwd<128, false, false, AMASK, DROP>(a, mview, st);
    }
    return bf16 ? run_bwd<64, true, false, AMASK, DROP>(a, mview, st) : run_bwd<64, false, false, AMASK, DROP>(a, mview, st);
}

template <bool AMASK>
int launch_bwd_masked(const BwdArgs& a, const MaskView& mview, cudaStream_t st) {
    return a.drop_p > 0.0f ? launch_bwd_variant<AMASK, true>(a, mview, st) : launch_bwd_variant<AMASK, false>(a, mview, st);
}

int launch_bwd_sm100(const BwdArgs& a, cudaStream_t st) {
    if (!a.has_mask) return launch_bwd_masked<false>(a, MaskView{}, st);
    MaskView mview;
    void* table = nullptr;
    if (build_mask_view(a.mask, a.sh.B, a.sh.H, a.sh.L, a.sh.S, a.scale, mview, &table, st) != 0) return -1;
    const int rc = launch_bwd_masked<true>(a, mview, st);
    if (table) cudaFreeAsync(table, st);  // after the kernels: the dq kernel's side stream is joined into st
    return rc;
}

}  // namespace gtb
