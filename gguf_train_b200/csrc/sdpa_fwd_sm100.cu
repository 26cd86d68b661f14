// Flash-style attention forward for sm_100a: tcgen05 tensor cores, TMEM accumulators, TMA tiles.
//
// One CTA computes one 128-row query tile of one (batch, query head). Six warps, specialised:
//   warp 0      TMA producer: the Q tile once, then K and V tiles of 128 keys into a ring of
//               shared-memory stages (128-byte swizzled, the layout tcgen05 descriptors read);
//   warp 1      MMA issuer (one thread) and TMEM owner:
//                 S_j = Q K_j^T         (M=128, N=128, K=D; A, B from shared memory, K-major)
//                 O  += P_j V_j         (M=128, N=D,  K=128; A = P, B = V read MN-major)
//               S is double-buffered in TMEM so S_{j+2} is computed while the softmax works on S_j;
//   warps 2..5  softmax, one query row per thread (TMEM lane = row): read S_j from TMEM, mask,
//               online softmax in the log2 domain with lazy rescaling (O and the running sum are
//               rescaled only when the row maximum grows by more than 2^8), write P_j (bf16/f16)
//               back to TMEM or to shared memory, and at the end normalise O and store it.
// TMEM: S0 = columns [0,128), S1 = [128,256), O = [256, 256+D); 512 columns allocated.
//
// Semantics are those of gt_flash_attention (reference csrc/gt_ops_nn.cpp:2423-2525): causal is
// top-left aligned (key s masked for query l when s > l), GQA maps query head h to kv head
// h / (H/Hkv), rows are normalised by the sum of exp over allowed keys. Accumulation is f32.
//
// Every wait on an mbarrier is bounded (about a second); on timeout the kernel records a status
// code, skips its remaining work, drains its own in-flight copies and MMAs with bounded waits,
// frees TMEM and returns.

#include <cmath>
#include <cstdio>
#include <mutex>

#include <cudaTypedefs.h>

#include "gtb_common.cuh"
#include "sdpa_args.h"
#include "sm100_ptx.cuh"

namespace gtb {
namespace {

using namespace sm100;

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int NTHREADS = 192;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t S_COL0 = 0;
constexpr uint32_t O_COL = 256;

template <int D, bool P_TMEM>
struct Cfg {
    static constexpr int ATOMS = D / 64;                  // 128-byte swizzle atoms along D
    static constexpr int TILE = BM * D * 2;               // bytes of a 128-row Q, K or V tile
    static constexpr int ATOM_BYTES = BM * 128;           // 16 KB: one 64-column slab of a tile
    static constexpr int KS = 2;                          // K stages
    static constexpr int VS = 2;                          // V stages
    static constexpr int P_TILE = BM * BN * 2;            // P tile in shared memory (if used)
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_K = OFF_Q + TILE;
    static constexpr int OFF_V = OFF_K + KS * TILE;
    static constexpr int OFF_P = OFF_V + VS * TILE;
    static constexpr int OFF_BAR = OFF_P + (P_TMEM ? 0 : 2 * P_TILE);
    static constexpr int NBAR = 1 + 2 * KS + 2 * VS + 2 + 2 + 3;
    static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;  // + TMEM slot, + alignment slack
};

// two floats -> one 32-bit word of two 16-bit values (lo in the low half), round to nearest even
template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    uint32_t r;
    if constexpr (BF16) asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    else asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
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
    int n_qtiles;
    float scale_log2;
    int causal;
    void* o;
    int64_t os0, os1, os2;  // output strides of b, h, l (elements); d stride is 1
    float* lse;
    int* status;
};

template <int D, bool BF16, bool P_TMEM>
__global__ void __launch_bounds__(NTHREADS, 1)
fwd_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                 const __grid_constant__ CUtensorMap tmV, const Params p) {
    using C = Cfg<D, P_TMEM>;
    using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = (uint64_t*)(smem + C::OFF_BAR);
    uint64_t* q_full = bars;
    uint64_t* k_full = bars + 1;
    uint64_t* k_empty = k_full + C::KS;
    uint64_t* v_full = k_empty + C::KS;
    uint64_t* v_empty = v_full + C::VS;
    uint64_t* s_full = v_empty + C::VS;      // [2]
    uint64_t* p_full = s_full + 2;           // [2]
    uint64_t* o_full = p_full + 2;           // one phase per PV block
    uint64_t* o_final = o_full + 1;          // single phase: all MMAs done
    uint64_t* drain = o_final + 1;           // error path only
    uint32_t* tmem_slot = (uint32_t*)(bars + C::NBAR);
    int* abort_flag = (int*)(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = p.causal ? (p.n_qtiles - 1 - (int)blockIdx.x) : (int)blockIdx.x;  // heavy tiles first
    const int h = blockIdx.y, b = blockIdx.z;
    const int hk = h / p.group;
    const int row0 = tile * BM;
    const int n_kv = (int)((p.S + BN - 1) / BN);
    const int row_last = (int)min((int64_t)row0 + BM - 1, p.L - 1);
    const int nblk = p.causal ? min(n_kv, row_last / BN + 1) : n_kv;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < C::KS; ++i) { mbar_init(&k_full[i], 1); mbar_init(&k_empty[i], 1); }
        for (int i = 0; i < C::VS; ++i) { mbar_init(&v_full[i], 1); mbar_init(&v_empty[i], 1); }
        for (int i = 0; i < 2; ++i) { mbar_init(&s_full[i], 1); mbar_init(&p_full[i], 128); }
        mbar_init(o_full, 1);
        mbar_init(o_final, 1);
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
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmV);
            int last_k = -1, last_v = -1;
            bool ok = true;
            mbar_expect_tx(q_full, C::TILE);
            for (int a = 0; a < C::ATOMS; ++a)
                tma_load_4d(smem + C::OFF_Q + a * C::ATOM_BYTES, &tmQ, a * 64, row0, h, b, q_full);
            for (int j = 0; j < nblk && ok; ++j) {
                const int ks = j % C::KS;
                if (j >= C::KS) ok = mbar_wait(&k_empty[ks], ((j / C::KS) - 1) & 1, p.status, 11);
                if (!ok || *(volatile int*)abort_flag) break;
                mbar_expect_tx(&k_full[ks], C::TILE);
                for (int a = 0; a < C::ATOMS; ++a)
                    tma_load_4d(smem + C::OFF_K + ks * C::TILE + a * C::ATOM_BYTES, &tmK, a * 64, j * BN, hk, b, &k_full[ks]);
                last_k = j;
                const int vs = j % C::VS;
                if (j >= C::VS) ok = mbar_wait(&v_empty[vs], ((j / C::VS) - 1) & 1, p.status, 12);
                if (!ok || *(volatile int*)abort_flag) break;
                mbar_expect_tx(&v_full[vs], C::TILE);
                for (int a = 0; a < C::ATOMS; ++a)
                    tma_load_4d(smem + C::OFF_V + vs * C::TILE + a * C::ATOM_BYTES, &tmV, a * 64, j * BN, hk, b, &v_full[vs]);
                last_v = j;
            }
            if (!ok) *(volatile int*)abort_flag = 1;
            if (*(volatile int*)abort_flag) {
                // drain our own copies before the CTA exits (bounded)
                mbar_wait(q_full, 0, nullptr, 0);
                for (int j = max(0, last_k - C::KS + 1); j <= last_k; ++j)
                    mbar_wait(&k_full[j % C::KS], (j / C::KS) & 1, nullptr, 0);
                for (int j = max(0, last_v - C::VS + 1); j <= last_v; ++j)
                    mbar_wait(&v_full[j % C::VS], (j / C::VS) & 1, nullptr, 0);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t IDESC_S = idesc_f16(BM, BN, BF16, false);
            constexpr uint32_t IDESC_PV = idesc_f16(BM, D, BF16, true);
            const uint32_t q_addr = smem_u32(smem + C::OFF_Q);
            bool ok = mbar_wait(q_full, 0, p.status, 21);
            auto issue_s = [&](int j) -> bool {
                const int ks = j % C::KS;
                if (!mbar_wait(&k_full[ks], (j / C::KS) & 1, p.status, 22)) return false;
                tc_fence_after();
                const uint32_t k_addr = smem_u32(smem + C::OFF_K + ks * C::TILE);
                const uint32_t d_tmem = tmem + S_COL0 + (uint32_t)(j & 1) * BN;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t off = (uint32_t)((kk / 4) * C::ATOM_BYTES + (kk % 4) * 32);
                    mma_ss(d_tmem, desc_sw128(q_addr + off, 16, 1024), desc_sw128(k_addr + off, 16, 1024), IDESC_S,
                           kk > 0 ? 1u : 0u);
                }
                mma_commit(&s_full[j & 1]);
                mma_commit(&k_empty[ks]);
                return true;
            };
            if (ok) ok = issue_s(0);
            if (ok && nblk > 1) ok = issue_s(1);
            for (int j = 0; j < nblk && ok; ++j) {
                ok = mbar_wait(&p_full[j & 1], (j >> 1) & 1, p.status, 23);
                if (!ok || *(volatile int*)abort_flag) break;
                const int vs = j % C::VS;
                ok = mbar_wait(&v_full[vs], (j / C::VS) & 1, p.status, 24);
                if (!ok || *(volatile int*)abort_flag) break;
                tc_fence_after();
                const uint32_t v_addr = smem_u32(smem + C::OFF_V + vs * C::TILE);
#pragma unroll
                for (int kk = 0; kk < BN / 16; ++kk) {
                    const uint64_t bdesc = desc_sw128(v_addr + kk * 2048, C::ATOM_BYTES, 1024);
                    const uint32_t acc = (j > 0 || kk > 0) ? 1u : 0u;
                    if constexpr (P_TMEM) {
                        mma_ts(tmem + O_COL, tmem + S_COL0 + (uint32_t)(j & 1) * BN + kk * 8, bdesc, IDESC_PV, acc);
                    } else {
                        const uint32_t p_addr = smem_u32(smem + C::OFF_P + (j & 1) * C::P_TILE);
                        const uint32_t off = (uint32_t)((kk / 4) * C::ATOM_BYTES + (kk % 4) * 32);
                        mma_ss(tmem + O_COL, desc_sw128(p_addr + off, 16, 1024), bdesc, IDESC_PV, acc);
                    }
                }
                mma_commit(o_full);
                mma_commit(&v_empty[vs]);
                if (j + 2 < nblk) ok = issue_s(j + 2);
            }
            if (!ok) *(volatile int*)abort_flag = 1;
            if (ok && !*(volatile int*)abort_flag) {
                mma_commit(o_final);
            } else {
                mma_commit(drain);  // wait (bounded) for every MMA we issued before TMEM is freed
                mbar_wait(drain, 0, nullptr, 0);
            }
        }
    } else {
        // ------------------------------------------------------------ softmax + epilogue
        const int quad = warp & 3;                    // TMEM lanes this warp may access
        const int r = quad * 32 + lane;               // row of the tile
        const int grow = row0 + r;                    // query index
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        float m_used = -INFINITY, lsum = 0.0f;
        bool ok = true;
        for (int j = 0; j < nblk; ++j) {
            ok = warp_wait(&s_full[j & 1], (j >> 1) & 1, p.status, 31);
            if (!ok || __any_sync(0xffffffffu, *(volatile int*)abort_flag)) break;
            tc_fence_after();
            const uint32_t s_tmem = tmem + lane_addr + S_COL0 + (uint32_t)(j & 1) * BN;
            uint32_t xr[BN];
#pragma unroll
            for (int c = 0; c < BN / 32; ++c) tmem_ld32(s_tmem + c * 32, &xr[c * 32]);
            tmem_ld_wait();
            float x[BN];
#pragma unroll
            for (int i = 0; i < BN; ++i) x[i] = __uint_as_float(xr[i]);
            const int kv0 = j * BN;
            const bool need_mask = (kv0 + BN > p.S) || (p.causal && kv0 + BN - 1 > row0);
            if (need_mask) {
                const int lim = p.causal ? min((int)min(p.S, (int64_t)INT32_MAX) - 1, grow) : (int)p.S - 1;
#pragma unroll
                for (int i = 0; i < BN; ++i)
                    if (kv0 + i > lim) x[i] = -INFINITY;
            }
            float mx = x[0];
#pragma unroll
            for (int i = 1; i < BN; ++i) mx = fmaxf(mx, x[i]);
            const float m_new = fmaxf(m_used, mx * p.scale_log2);
            const bool rescale = m_new > m_used + 8.0f;  // false while the row has no finite score
            if (__any_sync(0xffffffffu, rescale && j > 0)) {
                // PV_{j-1} must be complete before O is read; PV_{j-2} is known complete here
                ok = warp_wait(o_full, (j - 1) & 1, p.status, 32);
                if (!ok) break;
                tc_fence_after();
                const float alpha = rescale ? ex2(m_used - m_new) : 1.0f;
                const uint32_t o_tmem = tmem + lane_addr + O_COL;
#pragma unroll
                for (int c = 0; c < D / 32; ++c) {
                    uint32_t ov[32];
                    tmem_ld32(o_tmem + c * 32, ov);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
                    tmem_st32(o_tmem + c * 32, ov);
                }
                tmem_st_wait();
            }
            if (rescale) {
                lsum *= ex2(m_used - m_new);
                m_used = m_new;
            }
            const float neg_m = (m_used == -INFINITY) ? 0.0f : -m_used;
            uint32_t pk[BN / 2];
            float rs = 0.0f;
#pragma unroll
            for (int i = 0; i < BN; i += 2) {
                const float p0 = ex2(fmaf(x[i], p.scale_log2, neg_m));
                const float p1 = ex2(fmaf(x[i + 1], p.scale_log2, neg_m));
                rs += p0 + p1;
                pk[i / 2] = pack2<BF16>(p0, p1);
            }
            lsum += rs;
            if constexpr (P_TMEM) {
                tmem_st32(s_tmem, pk);
                tmem_st32(s_tmem + 32, pk + 32);
                tmem_st_wait();
            } else {
                // row r of a K-major 128-byte-swizzled tile: 16-byte chunk c of a 128-byte row lands
                // at chunk c ^ (r % 8); 64 columns per 16 KB slab
                unsigned char* pbase = smem + C::OFF_P + (j & 1) * C::P_TILE;
#pragma unroll
                for (int c = 0; c < BN / 8; ++c) {
                    const int slab = c / 8, cc = c % 8;
                    uint4 v = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
                    *(uint4*)(pbase + slab * C::ATOM_BYTES + r * 128 + ((cc ^ (r & 7)) * 16)) = v;
                }
                fence_proxy_async_smem();
            }
            tc_fence_before();
            mbar_arrive(&p_full[j & 1]);
        }
        if (!ok) *(volatile int*)abort_flag = 1;
        if (ok && !*(volatile int*)abort_flag) {
            ok = warp_wait(o_final, 0, p.status, 33);
            if (ok) {
                tc_fence_after();
                const float inv = lsum > 0.0f ? 1.0f / lsum : 0.0f;
                const uint32_t o_tmem = tmem + lane_addr + O_COL;
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
                        for (int q4 = 0; q4 < 4; ++q4) dst[q4] = make_uint4(w[4 * q4], w[4 * q4 + 1], w[4 * q4 + 2], w[4 * q4 + 3]);
                    }
                }
                if (p.lse && grow < p.L)
                    p.lse[((int64_t)b * p.H + h) * p.L + grow] =
                        lsum > 0.0f ? (m_used + log2f(lsum)) * 0.69314718055994531f : -INFINITY;
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

// 4-D map over (d, row, head, batch) with a 64 x 128 box and 128-byte swizzle
bool make_map(CUtensorMap* tm, const gtb_tensor4& t, int64_t d_extent, bool bf16) {
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
    cuuint32_t box[4] = {64, (cuuint32_t)BM, 1, 1};
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

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

template <int D, bool BF16, bool P_TMEM>
int run(const FwdArgs& a, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, cudaStream_t st) {
    using C = Cfg<D, P_TMEM>;
    auto kern = fwd_sm100_kernel<D, BF16, P_TMEM>;
    static bool attr_set = false;  // benign race: setting the same attribute twice is harmless
    if (!attr_set) {
        if (cuda_failed(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM),
                        "cudaFuncSetAttribute(fwd_sm100)"))
            return -1;
        attr_set = true;
    }
    Params p;
    p.H = a.sh.H; p.Hkv = a.sh.Hkv; p.L = a.sh.L; p.S = a.sh.S;
    p.group = (int)(a.sh.H / a.sh.Hkv);
    p.n_qtiles = (int)((a.sh.L + BM - 1) / BM);
    p.scale_log2 = a.scale * 1.4426950408889634f;
    p.causal = a.causal;
    p.o = a.o.data;
    p.os0 = a.o.stride[0]; p.os1 = a.o.stride[1]; p.os2 = a.o.stride[2];
    p.lse = (float*)a.lse;
    int dev = 0;
    cudaGetDevice(&dev);
    p.status = device_status_word(dev);
    dim3 grid((unsigned)p.n_qtiles, (unsigned)a.sh.H, (unsigned)a.sh.B);
    kern<<<grid, NTHREADS, C::SMEM, st>>>(mq, mk, mv, p);
    return cuda_failed(cudaGetLastError(), "flash_attention (sm100) launch") ? -1 : 0;
}

// P staged in TMEM (aliasing S) by default; GTB_FWD_P_SMEM=1 stages it in shared memory instead.
bool p_in_tmem() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("GTB_FWD_P_SMEM");
        v = (e && atoi(e) == 1) ? 0 : 1;
    }
    return v == 1;
}

}  // namespace

bool fwd_sm100_supported(const FwdArgs& a) {
    if (a.has_mask) return false;
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
    if (a.sh.L >= (1ll << 31) || a.sh.S >= (1ll << 31) || a.sh.H > 65535 || a.sh.B > 65535) return false;
    if (a.sh.L < 1 || a.sh.S < 1) return false;
    return encode_fn() != nullptr;
}

int launch_fwd_sm100(const FwdArgs& a, cudaStream_t st) {
    const bool bf16 = a.q.dtype == BF16;
    CUtensorMap mq, mk, mv;
    if (!make_map(&mq, a.q, a.sh.D, bf16) || !make_map(&mk, a.k, a.sh.D, bf16) || !make_map(&mv, a.v, a.sh.Dv, bf16))
        return -1;
    const bool pt = p_in_tmem();
    if (a.sh.D == 128) {
        if (bf16) return pt ? run<128, true, true>(a, mq, mk, mv, st) : run<128, true, false>(a, mq, mk, mv, st);
        return pt ? run<128, false, true>(a, mq, mk, mv, st) : run<128, false, false>(a, mq, mk, mv, st);
    }
    if (bf16) return pt ? run<64, true, true>(a, mq, mk, mv, st) : run<64, true, false>(a, mq, mk, mv, st);
    return pt ? run<64, false, true>(a, mq, mk, mv, st) : run<64, false, false>(a, mq, mk, mv, st);
}

}  // namespace gtb
