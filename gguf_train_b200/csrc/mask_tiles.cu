// Class table of an attention mask for the tensor-core kernels (see mask_tiles.cuh).

#include <algorithm>

#include "mask_tiles.cuh"

namespace gtb {
namespace {

// One CTA per table entry (mask batch, mask head, row tile, key block): reads the entry's region
// (up to 128 x 128 mask entries, one row when the mask broadcasts over rows) and records whether
// every entry allows its key with nothing added (MASK_NONE), none allows it (MASK_ALL), or neither.
__global__ void __launch_bounds__(256) mask_class_kernel(MaskView m, int64_t rows, int64_t S, int64_t n_tiles,
                                                         int64_t n_blocks, int64_t Hm, uint8_t* out) {
    const int64_t e = blockIdx.x;
    const int64_t kb = e % n_blocks, lt = (e / n_blocks) % n_tiles, hm = (e / n_blocks / n_tiles) % Hm,
                  bm = e / n_blocks / n_tiles / Hm;
    const int64_t l0 = lt * MASK_TILE, s0 = kb * MASK_TILE;
    const int64_t nr = min((int64_t)MASK_TILE, rows - l0), ns = min((int64_t)MASK_TILE, S - s0);
    int allowed = 0, touched = 0;  // some entry lets its key through / some entry changes a score
    for (int64_t i = threadIdx.x; i < nr * ns; i += blockDim.x) {
        const int64_t l = l0 + i / ns, s = s0 + i % ns;
        const unsigned char* p = m.row(bm, hm, l) + s * m.s3 * m.esize;
        float v;
        switch (m.dtype) {
            case BOOL: v = *p ? 0.0f : -INFINITY; break;
            case F32: v = *(const float*)p; break;
            case F16: v = __half2float(*(const __half*)p); break;
            default: v = __bfloat162float(*(const __nv_bfloat16*)p); break;
        }
        allowed |= v != -INFINITY;
        touched |= v != 0.0f;
    }
    allowed = __syncthreads_or(allowed);
    touched = __syncthreads_or(touched);
    if (threadIdx.x == 0) out[e] = !touched ? MASK_NONE : (!allowed ? MASK_ALL : MASK_MIXED);
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace

bool mask_supported(const gtb_tensor4& mask) {
    if (mask.dtype != BOOL && mask.dtype != F32 && mask.dtype != F16 && mask.dtype != BF16) return false;
    for (int i = 0; i < 4; ++i)
        if (mask.stride[i] < 0 || (mask.shape[i] > 1 && mask.stride[i] >= (1ll << 40))) return false;
    return mask.data != nullptr;
}

int build_mask_view(const gtb_tensor4& mask, int64_t B, int64_t H, int64_t L, int64_t S, float scale, MaskView& mv,
                    void** table, cudaStream_t st) {
    (void)B;
    (void)H;
    mv = MaskView{};
    mv.data = (const unsigned char*)mask.data;
    mv.dtype = mask.dtype;
    mv.esize = (int)dtype_size(mask.dtype);
    // broadcast dimensions carry stride 0 (the C ABI layer has set them)
    mv.s0 = mask.shape[0] == 1 ? 0 : mask.stride[0];
    mv.s1 = mask.shape[1] == 1 ? 0 : mask.stride[1];
    mv.s2 = mask.shape[2] == 1 ? 0 : mask.stride[2];
    mv.s3 = mask.shape[3] == 1 ? 0 : mask.stride[3];
    mv.inv_scale = 1.0f / scale;
    bool vec = mv.s3 == 1 && aligned16(mask.data);
    const int64_t st3[3] = {mv.s0, mv.s1, mv.s2};
    for (int i = 0; i < 3; ++i) vec = vec && (st3[i] * mv.esize) % 16 == 0;
    mv.vec = vec ? 1 : 0;
    const int64_t Bm = mask.shape[0], Hm = mask.shape[1];
    const int64_t rows = mask.shape[2] == 1 ? 1 : L;
    const int64_t n_tiles = (rows + MASK_TILE - 1) / MASK_TILE;
    const int64_t n_blocks = (S + MASK_TILE - 1) / MASK_TILE;
    const int64_t entries = Bm * Hm * n_tiles * n_blocks;
    mv.c2 = mask.shape[2] == 1 ? 0 : n_blocks;
    mv.c1 = Hm == 1 ? 0 : n_tiles * n_blocks;
    mv.c0 = Bm == 1 ? 0 : Hm * n_tiles * n_blocks;
    *table = nullptr;
    if (entries <= 0) return 0;
    if (entries >= (1ll << 31)) {
        set_error("flash_attention: mask too large for the tile table");
        return -1;
    }
    if (cuda_failed(cudaMallocAsync(table, (size_t)entries, st), "flash_attention: mask tile table")) return -1;
    mv.cls = (const uint8_t*)*table;
    mask_class_kernel<<<(unsigned)entries, 256, 0, st>>>(mv, rows, S, n_tiles, n_blocks, Hm, (uint8_t*)*table);
    if (cuda_failed(cudaGetLastError(), "flash_attention: mask tile table launch")) {
        cudaFreeAsync(*table, st);
        *table = nullptr;
        return -1;
    }
    return 0;
}

}  // namespace gtb
