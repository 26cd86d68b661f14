// Linear layer on the tensor cores: C (M, N) = A (M, K) B (N, K)^T (+ bias (N)), bf16 or f16 operands,
// f32 accumulation, C in the operands' dtype. This is F.linear(x, W, b) with x (M, K) and W (N, K)
// row-major: both operands are K-major, the layout tcgen05.mma reads from shared memory without a
// transpose. It replaces gt_linear (reference csrc/gt_ops_nn.cpp:256-335, a ggml_mul_mat graph) for
// MultiheadAttention's in/out projections in 16-bit; the backward products are the same kernel on
// transposed operands (gguf_train_b200.functional.linear).
//
// Persistent CTAs (one per SM) walk the 128 x BN output tiles in order tile = blockIdx.x + i * gridDim.x.
// Six warps:
//   warp 0     TMA producer: per tile, the K loop's A (128 x 64) and B (BN x 64) slabs into a 4-stage
//              ring of 128-byte-swizzled shared-memory stages;
//   warp 1     TMEM owner (2 x BN columns) and MMA issuer: per stage four tcgen05.mma (M=128, N=BN,
//              K=16) into the tile's accumulator buffer, alternating between the two buffers so the
//              epilogue of one tile overlaps the MMAs of the next;
//   warps 2-5  epilogue: one output row per thread (warp w reads TMEM lanes 32 * (w % 4) ..), 32
//              columns at a time: + bias, rounded to the 16-bit type, 16-byte stores.
// Rows past M, columns past N and the K tail come in as zeros from the tensor maps and are not stored.
// Every wait is bounded as in the attention kernels: a timeout records a status code, drains the
// CTA's own copies and MMAs, frees TMEM and returns.

#include <cmath>
#include <mutex>

#include <cudaTypedefs.h>

#include "gtb_common.cuh"
#include "sdpa_args.h"
#include "sm100_ptx.cuh"

namespace gtb {
namespace {

using namespace sm100;

constexpr int BM = 128, BK = 64, STAGES = 4, NTHREADS = 192;

template <int BN>
struct LCfg {
    static constexpr int A_BYTES = BM * BK * 2;   // 16 KB
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE = A_BYTES + B_BYTES;
    static constexpr int OFF_STG = STAGES * STAGE;  // per epilogue warp: 32 rows x 64 bytes (+16 padding)
    static constexpr int STG_ROW = 80;
    static constexpr int OFF_BAR = OFF_STG + 4 * 32 * STG_ROW;
    static constexpr int NBAR = 2 * STAGES + 4 + 1;
    static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;
    static constexpr uint32_t TMEM_COLS = 2 * BN;  // 256 or 512
};

struct LinP {
    int64_t M, N, K;
    int tiles_m, tiles_n, n_tiles;
    const void* bias;  // (N) in the operands' dtype, or null
    void* c;
    int64_t ldc;       // elements between rows of C
    int vec;           // 16-byte stores allowed (ldc % 8 == 0, aligned C)
    int bias_vec;      // 16-byte bias loads allowed (aligned bias)
    int* status;
};

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    uint32_t r;
    if constexpr (BF16) asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    else asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

template <int BN, bool BF16>
__global__ void __launch_bounds__(NTHREADS, 1)
linear_sm100_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const LinP p) {
    using C = LCfg<BN>;
    using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = (uint64_t*)(smem + C::OFF_BAR);
    uint64_t* full = bars;                  // [STAGES] a stage's A and B landed
    uint64_t* empty = bars + STAGES;        // [STAGES] the MMAs reading a stage are done
    uint64_t* acc_full = bars + 2 * STAGES; // [2] an accumulator buffer holds a finished tile
    uint64_t* acc_empty = acc_full + 2;     // [2] the epilogue has read a buffer (128 arrivals)
    uint64_t* drain = acc_empty + 2;
    uint32_t* tmem_slot = (uint32_t*)(bars + C::NBAR);
    int* abort_flag = (int*)(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kb_n = (int)((p.K + BK - 1) / BK);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(&acc_full[b], 1); mbar_init(&acc_empty[b], 128); }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            prefetch_tmap(&tmA);
            prefetch_tmap(&tmB);
            int it = 0;  // stage uses so far
            bool ok = true;
            for (int tile = blockIdx.x; tile < p.n_tiles && ok; tile += gridDim.x) {
                const int tm = tile / p.tiles_n, tn = tile % p.tiles_n;
                for (int kb = 0; kb < kb_n; ++kb, ++it) {
                    const int s = it % STAGES;
                    if (it >= STAGES) ok = mbar_wait(&empty[s], ((it / STAGES) - 1) & 1, p.status, 71);
                    if (!ok || *(volatile int*)abort_flag) { ok = false; break; }
                    unsigned char* st = smem + s * C::STAGE;
                    mbar_expect_tx(&full[s], C::STAGE);
                    asm volatile(
                        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                        ::"r"(smem_u32(st)), "l"((uint64_t)&tmA), "r"(kb * BK), "r"(tm * BM), "r"(smem_u32(&full[s])) : "memory");
                    asm volatile(
                        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                        ::"r"(smem_u32(st + C::A_BYTES)), "l"((uint64_t)&tmB), "r"(kb * BK), "r"(tn * BN), "r"(smem_u32(&full[s])) : "memory");
                }
            }
            if (!ok) *(volatile int*)abort_flag = 1;
            if (*(volatile int*)abort_flag)  // drain the copies in flight (bounded)
                for (int j = max(0, it - STAGES); j < it; ++j) mbar_wait(&full[j % STAGES], (j / STAGES) & 1, nullptr, 0);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t IDESC = idesc_f16(BM, BN, BF16, false);
            int it = 0, local = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < p.n_tiles && ok; tile += gridDim.x, ++local) {
                const int buf = local & 1;
                if (local >= 2) ok = mbar_wait(&acc_empty[buf], ((local >> 1) - 1) & 1, p.status, 72);
                if (!ok) break;
                tc_fence_after();
                const uint32_t acc = tmem + (uint32_t)(buf * BN);
                for (int kb = 0; kb < kb_n; ++kb, ++it) {
                    const int s = it % STAGES;
                    ok = mbar_wait(&full[s], (it / STAGES) & 1, p.status, 73);
                    if (!ok || *(volatile int*)abort_flag) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t ad = desc_sw128(smem_u32(smem + s * C::STAGE), 16, 1024);
                    const uint64_t bd = desc_sw128(smem_u32(smem + s * C::STAGE + C::A_BYTES), 16, 1024);
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)
                        mma_ss(acc, desc_advance(ad, k * 32), desc_advance(bd, k * 32), IDESC, (kb > 0 || k > 0) ? 1u : 0u);
                    mma_commit(&empty[s]);
                }
                if (ok) mma_commit(&acc_full[buf]);
            }
            if (!ok) *(volatile int*)abort_flag = 1;
            if (*(volatile int*)abort_flag) {
                mma_commit(drain);
                mbar_wait(drain, 0, nullptr, 0);
            }
        }
    } else {
        // epilogue: warp w reads TMEM lanes 32 * (w % 4) .. (rows of the tile)
        const int quad = warp & 3;
        const int r = quad * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        int local = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x, ++local) {
            const int buf = local & 1;
            ok = mbar_wait(&acc_full[buf], (local >> 1) & 1, p.status, 74);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok || __any_sync(0xffffffffu, *(volatile int*)abort_flag)) { ok = false; break; }
            tc_fence_after();
            const int tm = tile / p.tiles_n, tn = tile % p.tiles_n;
            const int64_t row = (int64_t)tm * BM + r;
            T* crow = (T*)p.c + row * p.ldc;
            unsigned char* stg = smem + C::OFF_STG + quad * 32 * C::STG_ROW;  // this warp's staging rows
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                const int64_t col0 = (int64_t)tn * BN + c * 32;
                // the chunk's 32 bias values in four 16-byte loads (the same address across the warp: one
                // transaction each), issued before the wait for the accumulator so the two overlap
                const bool bvec = p.bias && p.bias_vec && col0 + 32 <= p.N;
                uint4 bw[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) bw[q] = bvec ? ((const uint4*)((const T*)p.bias + col0))[q] : make_uint4(0, 0, 0, 0);
                uint32_t v[32];
                tmem_ld32(tmem + lane_addr + (uint32_t)(buf * BN + c * 32), v);
                tmem_ld_wait();
                if (col0 >= p.N) continue;  // the same for the whole warp
                float x[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) x[i] = __uint_as_float(v[i]);
                if (p.bias) {
                    const T* bb = (const T*)p.bias + col0;
                    if (bvec) {
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const uint4 w = bw[q];
                            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const T* pair = (const T*)&ww[e];
                                x[8 * q + 2 * e] += Elem<T>::load(pair);
                                x[8 * q + 2 * e + 1] += Elem<T>::load(pair + 1);
                            }
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (col0 + i < p.N) x[i] += Elem<T>::load(bb + i);
                    }
                }
                if (p.vec && col0 + 32 <= p.N) {
                    // through the warp's staging rows, so that each 16-byte store instruction writes 8 rows
                    // x 64 contiguous bytes instead of 32 rows x 16 bytes (rows of 80 bytes: the writes of
                    // a quarter warp hit eight different bank groups)
                    uint32_t w[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) w[i] = pack2<BF16>(x[2 * i], x[2 * i + 1]);
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        *(uint4*)(stg + lane * C::STG_ROW + 16 * q) = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
                    __syncwarp();
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const int rr = lane / 4 + 8 * k, seg = lane % 4;  // row of the warp's 32, 16-byte segment
                        const uint4 val = *(const uint4*)(stg + rr * C::STG_ROW + 16 * seg);
                        const int64_t grow = (int64_t)tm * BM + quad * 32 + rr;
                        if (grow < p.M) *(uint4*)((T*)p.c + grow * p.ldc + col0 + 8 * seg) = val;
                    }
                    __syncwarp();
                } else if (row < p.M) {
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (col0 + i < p.N) Elem<T>::store(crow + col0 + i, x[i]);
                }
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[buf]);
        }
        if (!ok) *(volatile int*)abort_flag = 1;
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// 2-D map over a row-major (rows, K) 16-bit matrix with a 64 x box_rows box and 128-byte swizzle
bool make_map_2d(CUtensorMap* tm, const void* p, int64_t rows, int64_t K, int64_t ld, bool bf16, int box_rows) {
    auto enc = encode_fn();
    if (!enc) {
        set_error("linear: cuTensorMapEncodeTiled is unavailable");
        return false;
    }
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
    cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(tm, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(p),
                     dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_errorf("linear: cuTensorMapEncodeTiled failed (%d)", (int)r);
        return false;
    }
    return true;
}

template <int BN, bool BF16>
int run_linear(const CUtensorMap& ma, const CUtensorMap& mb, LinP p, cudaStream_t st) {
    using C = LCfg<BN>;
    auto kern = linear_sm100_kernel<BN, BF16>;
    static bool attr = false;
    if (!attr) {
        if (cuda_failed(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM), "linear: smem"))
            return -1;
        attr = true;
    }
    int dev = 0;
    cudaGetDevice(&dev);
    static int n_sm = 0;
    if (n_sm == 0 && (cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n_sm <= 0))
        n_sm = 148;
    p.tiles_m = (int)((p.M + BM - 1) / BM);
    p.tiles_n = (int)((p.N + BN - 1) / BN);
    p.n_tiles = p.tiles_m * p.tiles_n;
    p.status = device_status_word(dev);
    const int grid = std::min(p.n_tiles, n_sm);
    kern<<<grid, NTHREADS, C::SMEM, st>>>(ma, mb, p);
    return cuda_failed(cudaGetLastError(), "linear launch") ? -1 : 0;
}

}  // namespace

int launch_linear_sm100(const void* a, const void* b, const void* bias, void* c, int64_t M, int64_t N, int64_t K,
                        int64_t lda, int64_t ldb, int64_t ldc, int dtype, cudaStream_t st) {
    const bool bf16 = dtype == BF16;
    // N of at most 128 takes 128-column tiles (less padding, more CTAs); otherwise 256
    const int bn = N <= 128 ? 128 : 256;
    CUtensorMap ma, mb;
    if (!make_map_2d(&ma, a, M, K, lda, bf16, BM) || !make_map_2d(&mb, b, N, K, ldb, bf16, bn)) return -1;
    LinP p{};
    p.M = M; p.N = N; p.K = K;
    p.bias = bias;
    p.c = c;
    p.ldc = ldc;
    p.vec = (ldc % 8 == 0) && (((uintptr_t)c & 15) == 0);
    p.bias_vec = bias && (((uintptr_t)bias & 15) == 0);
    if (bn == 128) return bf16 ? run_linear<128, true>(ma, mb, p, st) : run_linear<128, false>(ma, mb, p, st);
    return bf16 ? run_linear<256, true>(ma, mb, p, st) : run_linear<256, false>(ma, mb, p, st);
}

}  // namespace gtb
