// Attention weights on the tensor cores: MultiheadAttention's need_weights output for 16-bit q/k.
//
// The reference forms the weights explicitly (gguf_train/nn/modules/transformer.py:153-166): scores =
// q k^T * scale, the causal and attention masks, softmax over keys, dropout in training, the mean over
// heads (average_attn_weights) or every head. The forward kernel has already produced each row's
// log-sum-exp, so a weight is one exponential of a recomputed score:
//   P[b,h,l,s] = exp2(q.k * scale * log2(e) + mask - lse[b,h,l] * log2(e)),
// 0 where masked, times the forward's dropout decisions / (1 - p). No (B, H, L, S) score tensor exists.
//
// One CTA per (batch, 128 query rows, 128 keys), looping over the heads. Twelve warps:
//   warp 0       TMA: per head the Q tile (128 rows) and the K tile (128 keys of the head's kv head)
//                into a two-stage ring of 128-byte-swizzled shared-memory stages;
//   warp 1       TMEM owner (256 columns) and MMA issuer: S_h = Q_h K_h^T (M = N = 128, K = D) into one
//                of two 128-column buffers, so the next head's product runs while this one's scores
//                are exponentiated;
//   warps 2-3    idle;
//   warps 4-11   two warpgroups, one query row per thread (TMEM lane = row), warpgroup g taking keys
//                64g..64g+63: masks as the forward applies them (the per-tile class table of
//                mask_tiles.cuh), the exponential, dropout, and the head mean accumulated in registers
//                (or every head's weights stored), then the output rows; whole 64-key spans go
//                through a per-warp staging area in shared memory, so that each store instruction
//                writes 4 rows x 128 contiguous bytes.
// Every wait is bounded as in the attention kernels: a timeout records a status code, drains the
// CTA's own copies and MMAs, frees TMEM and returns.

#include <cmath>
#include <type_traits>

#include "dropout.cuh"
#include "gtb_common.cuh"
#include "mask_tiles.cuh"
#include "sdpa_args.h"
#include "sm100_ptx.cuh"

namespace gtb {
namespace {

using namespace sm100;

constexpr int WB = 128;            // rows and keys of a tile
constexpr int WTHREADS = 384;
constexpr uint32_t WTMEM = 256;    // two S buffers
constexpr int WREG_LO = 104;       // registers a thread of warpgroup 0 (TMA, MMA) after the split
constexpr int WREG_HI = 200;       // ... of the two compute warpgroups
constexpr float WLOG2E = 1.4426950408889634f;

template <int D>
struct WCfg {
    static constexpr int ATOMS = D / 64;
    static constexpr int TILE = WB * D * 2;          // a 128-row tile of Q or K
    static constexpr int ATOM_BYTES = WB * 128;
    static constexpr int ST_BYTES = 2 * TILE;        // Q and K of one head
    static constexpr int OFF_BAR = 2 * ST_BYTES;     // two stages
    static constexpr int NBAR = 2 + 2 + 2 + 2 + 1;   // st_full, st_empty, s_full, s_empty, drain
    static constexpr int STG_ROW = 144;              // a staged output row: 64 keys x 2 B + 16 B of padding
    static constexpr int OFF_STG = (OFF_BAR + NBAR * 8 + 16 + 127) / 128 * 128;  // [8 warps][32 rows]
    static constexpr int SMEM = OFF_STG + 8 * 32 * STG_ROW + 1024;
};

struct WParams {
    int64_t B, H, L, S;
    int group;
    float scale_log2;
    int causal, average;
    void* out;          // (B, L, S) or (B, H, L, S) contiguous, q's dtype
    const float* lse;   // (B, H, L)
    int* status;
    MaskView mk;
    uint32_t drop_thr;
    uint64_t drop_seed;
    float inv_keep;
};

template <bool BF16>
__device__ __forceinline__ uint32_t pack2w(float lo, float hi) {
    uint32_t r;
    if constexpr (BF16) asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    else asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// N consecutive values of one output row (keys s..s+N-1, s relative to the row start): 16-byte stores
// where the row is aligned for them and all N keys exist, else one value at a time up to S
template <int N, bool BF16, typename T>
__device__ __forceinline__ void store_row(T* row, int64_t s, int64_t S, const float* v, bool vec) {
    if (vec && s + N <= S) {
        uint4* dst = (uint4*)(row + s);
#pragma unroll
        for (int q = 0; q < N / 8; ++q)
            dst[q] = make_uint4(pack2w<BF16>(v[8 * q], v[8 * q + 1]), pack2w<BF16>(v[8 * q + 2], v[8 * q + 3]),
                                pack2w<BF16>(v[8 * q + 4], v[8 * q + 5]), pack2w<BF16>(v[8 * q + 6], v[8 * q + 7]));
    } else {
#pragma unroll
        for (int i = 0; i < N; ++i)  // unrolled with constant indices: v stays in registers
            if (s + i < S) Elem<T>::store(row + s + i, v[i]);
    }
}

// A warp's 32 rows of 64 weights (keys sk..sk+63, the thread's row = lane) written through the warp's
// staging rows in shared memory, so that each store instruction covers 4 rows x 128 contiguous bytes
// instead of 32 rows x 16 bytes. base: row 0 of the 32 at key sk (16-byte aligned), row_stride in
// elements; rows_valid (warp-uniform) of the 32 exist.
template <bool BF16, typename T>
__device__ __forceinline__ void store_rows_staged(unsigned char* stg, const float* xa, const float* xb, T* base,
                                                  int64_t row_stride, int rows_valid, int lane) {
    uint4* my = (uint4*)(stg + lane * WCfg<64>::STG_ROW);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        my[q] = make_uint4(pack2w<BF16>(xa[8 * q], xa[8 * q + 1]), pack2w<BF16>(xa[8 * q + 2], xa[8 * q + 3]),
                           pack2w<BF16>(xa[8 * q + 4], xa[8 * q + 5]), pack2w<BF16>(xa[8 * q + 6], xa[8 * q + 7]));
        my[4 + q] = make_uint4(pack2w<BF16>(xb[8 * q], xb[8 * q + 1]), pack2w<BF16>(xb[8 * q + 2], xb[8 * q + 3]),
                               pack2w<BF16>(xb[8 * q + 4], xb[8 * q + 5]), pack2w<BF16>(xb[8 * q + 6], xb[8 * q + 7]));
    }
    __syncwarp();
    const int c = lane & 7;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int r = (lane >> 3) + 4 * j;
        if (r < rows_valid)
            *(uint4*)(base + r * row_stride + 8 * c) = *(const uint4*)(stg + r * WCfg<64>::STG_ROW + 16 * c);
    }
    __syncwarp();  // the rows are read before the next call overwrites them
}

// one 32-key chunk of a row (keys sc..sc+31): scores in x -> weights, in place
template <bool MASK, bool DROP>
__device__ __forceinline__ void weights_chunk(float* x, uint8_t mcls, const MaskView& mk, const unsigned char* mrow,
                                              int sc, int64_t S, int lim, float scale_log2, float nl2,
                                              uint32_t rkey, uint32_t drop_thr, float inv_keep) {
    if constexpr (MASK) {
        if (mcls == MASK_MIXED) {
            mask_apply32(x, mk, mrow, sc, S);
        } else if (mcls == MASK_ALL) {
#pragma unroll
            for (int i = 0; i < 32; ++i) x[i] = -INFINITY;
        }
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const bool in = sc + i <= lim;
        float e = in ? ex2(fmaf(x[i], scale_log2, nl2)) : 0.0f;  // ex2(-inf) = 0
        if constexpr (DROP) e = drop_keep(rkey, (uint32_t)(sc + i), drop_thr) ? e * inv_keep : 0.0f;
        x[i] = e;
    }
}

template <int D, bool BF16, bool MASK, bool DROP, bool AVG>
__global__ void __launch_bounds__(WTHREADS, 1)
weights_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK, const WParams p) {
    using C = WCfg<D>;
    using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = (uint64_t*)(smem + C::OFF_BAR);
    uint64_t* st_full = bars;        // [2] Q and K of a head landed
    uint64_t* st_empty = bars + 2;   // [2] the head's MMAs have read them
    uint64_t* s_full = bars + 4;     // [2] S of a head computed
    uint64_t* s_empty = bars + 6;    // [2] S read by both compute warpgroups (256 arrivals)
    uint64_t* drain = bars + 8;
    uint32_t* tmem_slot = (uint32_t*)(bars + C::NBAR);
    int* abort_flag = (int*)(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t b = blockIdx.z;
    const int lt = (int)blockIdx.y, kt = (int)blockIdx.x;
    const int64_t l0 = (int64_t)lt * WB, s0 = (int64_t)kt * WB;
    // causal: every key of the tile after every row -> weights 0, nothing to compute
    const int64_t nh = (p.causal && s0 > l0 + WB - 1) ? 0 : p.H;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&st_full[i], 1); mbar_init(&st_empty[i], 1);
            mbar_init(&s_full[i], 1); mbar_init(&s_empty[i], 256);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, WTMEM);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // Registers: warpgroup 0 (TMA, MMA, two idle warps) hands registers to the compute warpgroups, which
    // hold 64 scores and 64 head-sum accumulators a thread. Every thread executes its warpgroup's
    // setmaxnreg at the top of its role's branch, converged (.sync.aligned, warpgroup-wide).
    static_assert(128 * WREG_LO + 256 * WREG_HI <= WTHREADS * 168, "register split above the launch's registers");
    if (warp < 4) {
    setmaxnreg_dec<WREG_LO>();
    if (warp == 0) {
        if (lane == 0 && nh > 0) {
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmK);
            int64_t h = 0;
            bool ok = true;
            for (; h < nh; ++h) {
                const int st = (int)(h & 1);
                if (h >= 2) ok = mbar_wait(&st_empty[st], (uint32_t)(((h >> 1) - 1) & 1), p.status, 81);
                if (!ok || *(volatile int*)abort_flag) { ok = false; break; }
                unsigned char* sb = smem + st * C::ST_BYTES;
                mbar_expect_tx(&st_full[st], C::ST_BYTES);
                for (int a = 0; a < C::ATOMS; ++a) {
                    tma_load_4d(sb + a * C::ATOM_BYTES, &tmQ, a * 64, (int)l0, (int)h, (int)b, &st_full[st]);
                    tma_load_4d(sb + C::TILE + a * C::ATOM_BYTES, &tmK, a * 64, (int)s0, (int)(h / p.group), (int)b,
                                &st_full[st]);
                }
            }
            if (!ok) *(volatile int*)abort_flag = 1;
            if (*(volatile int*)abort_flag)  // drain our own copies in flight (bounded)
                for (int64_t j = (h > 2 ? h - 2 : 0); j < h; ++j) mbar_wait(&st_full[j & 1], (uint32_t)((j >> 1) & 1), nullptr, 0);
        }
    } else if (warp == 1) {
        if (lane == 0 && nh > 0) {
            constexpr uint32_t IDESC = idesc_f16(WB, WB, BF16, false);
            const uint64_t qd0 = desc_sw128(smem_u32(smem), 16, 1024);
            const uint64_t kd0 = desc_sw128(smem_u32(smem + C::TILE), 16, 1024);
            const uint64_t qd1 = desc_sw128(smem_u32(smem + C::ST_BYTES), 16, 1024);
            const uint64_t kd1 = desc_sw128(smem_u32(smem + C::ST_BYTES + C::TILE), 16, 1024);
            bool ok = true;
            for (int64_t h = 0; h < nh; ++h) {
                const int st = (int)(h & 1);
                ok = mbar_wait(&st_full[st], (uint32_t)((h >> 1) & 1), p.status, 82);
                if (ok && h >= 2) ok = mbar_wait(&s_empty[st], (uint32_t)(((h >> 1) - 1) & 1), p.status, 83);
                if (!ok || *(volatile int*)abort_flag) { ok = false; break; }
                tc_fence_after();
                const uint64_t qd = st ? qd1 : qd0, kd = st ? kd1 : kd0;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t off = (uint32_t)((kk / 4) * C::ATOM_BYTES + (kk % 4) * 32);
                    mma_ss(tmem + (uint32_t)(st * WB), desc_advance(qd, off), desc_advance(kd, off), IDESC, kk > 0 ? 1u : 0u);
                }
                mma_commit(&s_full[st]);
                mma_commit(&st_empty[st]);
            }
            if (!ok) *(volatile int*)abort_flag = 1;
            if (*(volatile int*)abort_flag) {
                mma_commit(drain);  // every MMA issued is done before TMEM is freed (bounded)
                mbar_wait(drain, 0, nullptr, 0);
            }
        }
    }
    } else {
        setmaxnreg_inc<WREG_HI>();
        const int wg = (warp - 4) >> 2;           // keys 64 wg .. of the tile
        const int quad = warp & 3;
        const int64_t l = l0 + quad * 32 + lane;  // this thread's query row
        const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(wg * 64);
        const int sk = (int)s0 + wg * 64;         // first key of this thread's 64 (S < 2^30)
        const int lim = (int)(p.causal ? min(l, p.S - 1) : p.S - 1);  // last key the row may see
        T* const out = (T*)p.out;
        const bool vec = (p.S % 8) == 0;          // rows start 16-byte aligned
        // per-head weights: whole 64-key spans of 16-byte-aligned rows go through the warp's staging rows
        // AVG instances fix the head mean at compile time; the per-head instances test the flag at
        // run time (measured: per head 0.53 ms at B=2 on config 3's shape, 0.74 with the flag removed)
        const bool avg = AVG || p.average != 0;
        const bool staged = !avg && vec && (int64_t)sk + 64 <= p.S;
        const int64_t wrow0 = l0 + quad * 32;     // the warp's first row
        float acc[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) acc[i] = 0.0f;
        bool ok = true;
        const float* lse_row = p.lse + b * p.H * p.L + min(l, p.L - 1);  // head h at lse_row[h * L]
        float lse_next = nh > 0 ? lse_row[0] : 0.0f;                     // one head ahead of its use
        for (int64_t h = 0; h < nh && ok; ++h) {
            const int st = (int)(h & 1);
            const float lse = l < p.L ? lse_next : -INFINITY;
            if (h + 1 < nh) lse_next = lse_row[(h + 1) * p.L];
            const float nl2 = lse == -INFINITY ? -INFINITY : -lse * WLOG2E;
            const uint8_t mcls = MASK ? p.mk.tile_class(b, h, lt, kt) : (uint8_t)MASK_NONE;
            const unsigned char* mrow = nullptr;
            if constexpr (MASK) mrow = p.mk.row(b, h, min(l, p.L - 1));
            const uint32_t rkey = DROP ? drop_row_key(drop_head_key(p.drop_seed, (uint32_t)(b * p.H + h)), (uint32_t)l) : 0u;
            ok = mbar_wait(&s_full[st], (uint32_t)((h >> 1) & 1), p.status, 84);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok || __any_sync(0xffffffffu, *(volatile int*)abort_flag)) { ok = false; break; }
            tc_fence_after();
            uint32_t ra[32], rb[32];
            tmem_ld32(taddr + (uint32_t)(st * WB), ra);
            tmem_ld32(taddr + (uint32_t)(st * WB) + 32, rb);
            tmem_ld_wait();
            tc_fence_before();
            mbar_arrive(&s_empty[st]);  // the buffer is free for the head after next
            float* const xa = (float*)ra;  // scores, then (in place) the weights
            float* const xb = (float*)rb;
            weights_chunk<MASK, DROP>(xa, mcls, p.mk, mrow, sk, p.S, lim, p.scale_log2, nl2, rkey, p.drop_thr, p.inv_keep);
            weights_chunk<MASK, DROP>(xb, mcls, p.mk, mrow, sk + 32, p.S, lim, p.scale_log2, nl2, rkey, p.drop_thr,
                                      p.inv_keep);
            if (avg) {
#pragma unroll
                for (int i = 0; i < 32; ++i) { acc[i] += xa[i]; acc[32 + i] += xb[i]; }
            } else if (staged) {
                store_rows_staged<BF16>(smem + C::OFF_STG + (warp - 4) * 32 * C::STG_ROW, xa, xb,
                                        out + ((b * p.H + h) * p.L + wrow0) * p.S + sk, p.S,
                                        (int)min((int64_t)32, p.L - wrow0), lane);
            } else if (l < p.L) {
                T* row = out + ((b * p.H + h) * p.L + l) * p.S;
                store_row<32, BF16>(row, sk, p.S, xa, vec);
                store_row<32, BF16>(row, sk + 32, p.S, xb, vec);
            }
        }
        if (!ok) {
            *(volatile int*)abort_flag = 1;
        } else if (staged && nh == 0) {  // per head, a tile wholly above the causal diagonal: zeros (warp-uniform)
            for (int64_t h = 0; h < p.H; ++h)
                store_rows_staged<BF16>(smem + C::OFF_STG + (warp - 4) * 32 * C::STG_ROW, acc, acc + 32,
                                        out + ((b * p.H + h) * p.L + wrow0) * p.S + sk, p.S,
                                        (int)min((int64_t)32, p.L - wrow0), lane);
        } else if (l < p.L && sk < p.S) {
            if (avg) {
                const float inv_h = 1.0f / (float)p.H;
#pragma unroll
                for (int i = 0; i < 64; ++i) acc[i] *= inv_h;
                store_row<64, BF16>(out + (b * p.L + l) * p.S, sk, p.S, acc, vec);
            } else if (nh == 0) {  // a tile wholly above the causal diagonal: zeros for every head
                for (int64_t h = 0; h < p.H; ++h) store_row<64, BF16>(out + ((b * p.H + h) * p.L + l) * p.S, sk, p.S, acc, vec);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, WTMEM);
    }
}

template <int D, bool BF16, bool MASK, bool DROP, bool AVG>
int run_weights_sm100(const CUtensorMap& mq, const CUtensorMap& mk, const WParams& p, int64_t B, int64_t L, int64_t S,
                      cudaStream_t st) {
    using C = WCfg<D>;
    auto kern = weights_sm100_kernel<D, BF16, MASK, DROP, AVG>;
    static bool attr = false;  // benign race: setting the same attribute twice is harmless
    if (!attr) {
        if (cuda_failed(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM),
                        "attention weights (sm100): shared memory"))
            return -1;
        // setmaxnreg.inc waits until the block's registers cover the split: refuse a build whose kernel
        // was compiled with fewer registers a thread than the split assumes
        cudaFuncAttributes fa;
        if (cuda_failed(cudaFuncGetAttributes(&fa, kern), "cudaFuncGetAttributes(weights_sm100)")) return -1;
        if ((int64_t)fa.numRegs * WTHREADS < 128 * WREG_LO + 256 * WREG_HI) {
            set_errorf("attention weights (sm100): kernel built with %d registers a thread, below the %d the "
                       "register split needs", fa.numRegs, (128 * WREG_LO + 256 * WREG_HI + WTHREADS - 1) / WTHREADS);
            return -1;
        }
        attr = true;
    }
    dim3 grid((unsigned)((S + WB - 1) / WB), (unsigned)((L + WB - 1) / WB), (unsigned)B);
    // the head mean never touches the per-warp staging rows: launch it without them
    const int smem = AVG ? C::OFF_STG + 1024 : C::SMEM;
    kern<<<grid, WTHREADS, smem, st>>>(mq, mk, p);
    return cuda_failed(cudaGetLastError(), "attention weights (sm100) launch") ? -1 : 0;
}

template <int D, bool BF16>
int dispatch_weights_sm100(const CUtensorMap& mq, const CUtensorMap& mk, const WParams& p, bool mask, bool drop,
                           int64_t B, int64_t L, int64_t S, cudaStream_t st) {
    if (p.average) {
        if (mask) return drop ? run_weights_sm100<D, BF16, true, true, true>(mq, mk, p, B, L, S, st)
                              : run_weights_sm100<D, BF16, true, false, true>(mq, mk, p, B, L, S, st);
        return drop ? run_weights_sm100<D, BF16, false, true, true>(mq, mk, p, B, L, S, st)
                    : run_weights_sm100<D, BF16, false, false, true>(mq, mk, p, B, L, S, st);
    }
    if (mask) return drop ? run_weights_sm100<D, BF16, true, true, false>(mq, mk, p, B, L, S, st)
                          : run_weights_sm100<D, BF16, true, false, false>(mq, mk, p, B, L, S, st);
    return drop ? run_weights_sm100<D, BF16, false, true, false>(mq, mk, p, B, L, S, st)
                : run_weights_sm100<D, BF16, false, false, false>(mq, mk, p, B, L, S, st);
}

bool aligned16w(const void* p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace

bool weights_sm100_supported(const FwdArgs& a, const void* out) {
    if (a.q.dtype != BF16 && a.q.dtype != F16) return false;
    if (a.k.dtype != a.q.dtype || (a.sh.D != 64 && a.sh.D != 128)) return false;
    if (a.has_mask && !mask_supported(a.mask)) return false;
    if (a.q.stride[3] != 1 || a.k.stride[3] != 1 || !aligned16w(a.q.data) || !aligned16w(a.k.data) || !aligned16w(out))
        return false;
    for (int i = 0; i < 3; ++i)
        if ((a.q.shape[i] > 1 && a.q.stride[i] % 8 != 0) || (a.k.shape[i] > 1 && a.k.stride[i] % 8 != 0)) return false;
    if (a.sh.L < 1 || a.sh.S < 1 || a.sh.L >= (1ll << 30) || a.sh.S >= (1ll << 30) || a.sh.H > 65535 || a.sh.B > 65535)
        return false;
    return encode_fn() != nullptr;
}

int launch_weights_sm100(const FwdArgs& a, const void* lse, void* out, bool average, cudaStream_t st) {
    const bool bf16 = a.q.dtype == BF16;
    CUtensorMap mq, mk;
    if (!make_tma_map_4d(&mq, a.q, a.sh.D, bf16, WB) || !make_tma_map_4d(&mk, a.k, a.sh.D, bf16, WB)) return -1;
    MaskView mview;
    void* table = nullptr;
    if (a.has_mask && build_mask_view(a.mask, a.sh.B, a.sh.H, a.sh.L, a.sh.S, a.scale, mview, &table, st) != 0) return -1;
    int dev = 0;
    cudaGetDevice(&dev);
    WParams p;
    p.B = a.sh.B; p.H = a.sh.H; p.L = a.sh.L; p.S = a.sh.S;
    p.group = (int)(a.sh.H / a.sh.Hkv);
    p.scale_log2 = a.scale * WLOG2E;
    p.causal = a.causal;
    p.average = average ? 1 : 0;
    p.out = out;
    p.lse = (const float*)lse;
    p.status = device_status_word(dev);
    p.mk = mview;
    p.drop_thr = a.drop_thr;
    p.drop_seed = a.drop_seed;
    p.inv_keep = 1.0f / (1.0f - a.drop_p);
    const bool drop = a.drop_p > 0.0f;
    int rc;
    if (a.sh.D == 128)
        rc = bf16 ? dispatch_weights_sm100<128, true>(mq, mk, p, a.has_mask, drop, a.sh.B, a.sh.L, a.sh.S, st)
                  : dispatch_weights_sm100<128, false>(mq, mk, p, a.has_mask, drop, a.sh.B, a.sh.L, a.sh.S, st);
    else
        rc = bf16 ? dispatch_weights_sm100<64, true>(mq, mk, p, a.has_mask, drop, a.sh.B, a.sh.L, a.sh.S, st)
                  : dispatch_weights_sm100<64, false>(mq, mk, p, a.has_mask, drop, a.sh.B, a.sh.L, a.sh.S, st);
    if (table) cudaFreeAsync(table, st);  // after the kernel on the same stream
    return rc;
}

}  // namespace gtb
