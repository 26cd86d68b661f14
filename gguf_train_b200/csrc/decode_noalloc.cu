// gtb_decode_q8_0_noalloc: the Q8_0 decode step with its scratch in a fixed device array.
//
// gtb_decode_q8_0 takes the split-KV partial results (one (max, sum, out) record per chunk of
// GTB_DECODE_CHUNK cached rows, per query head) and a small work area from the stream-ordered
// allocator. Some callers cannot let a library allocate device memory: a serving runtime that hands
// the whole GPU to its own allocator at start-up, or a latency-critical loop that must never reach
// cudaMalloc/cudaFree (they synchronise the device) or grow a memory pool mid-run. For them this
// entry point runs the same kernels with the work area and the partials in g_decode_scratch below,
// a file-scope array of GTB_DECODE_NOALLOC_SCRATCH_BYTES that every GPU which loads this library
// holds until the process exits.
//
// Set-up: the first call on each device (with that device current) looks up the device addresses
// of the array and of this entry point's status word with cudaGetSymbolAddress (a host-side use of
// their names would not be a device address) and registers the status word, so that
// gtb_device_status() reads and clears it with the library's own. That first call should come
// before any stream capture. Calls share the array: two calls whose kernels overlap on the GPU
// (other streams, other threads) race on it. Nothing in it has to start at zero: the work area
// (item counter and per-sequence item prefix) and every partial record the combine step reads are
// written earlier in the same call.

#include <cmath>
#include <mutex>

#include "gtb_common.cuh"
#include "q8_0_internal.h"

namespace gtb {
namespace {

static __device__ __align__(256) float g_decode_scratch[GTB_DECODE_NOALLOC_SCRATCH_BYTES / sizeof(float)];
// status word for the bounded waits of this entry point's kernels (zero at load; a timeout writes a code)
static __device__ int g_decode_noalloc_status;

struct DeviceSlot {
    std::once_flag once;
    float* scratch = nullptr;
    int* status = nullptr;
    cudaError_t err = cudaSuccess;
};

DeviceSlot g_slots[64];

// Device addresses of the fixed scratch and status word on the current device (set up once).
bool device_scratch(int dev, float** scratch, int** status) {
    if (dev < 0 || dev >= 64) {
        set_errorf("flash_decode_q8_0_noalloc: device %d out of range", dev);
        return false;
    }
    DeviceSlot& s = g_slots[dev];
    std::call_once(s.once, [&s, dev] {
        void* p = nullptr;
        s.err = cudaGetSymbolAddress(&p, g_decode_scratch);
        if (s.err == cudaSuccess) s.scratch = (float*)p;
        void* q = nullptr;
        if (s.err == cudaSuccess) s.err = cudaGetSymbolAddress(&q, g_decode_noalloc_status);
        if (s.err == cudaSuccess) s.status = (int*)q;
        if (s.err == cudaSuccess) register_status_word(dev, s.status);  // read by gtb_device_status()
    });
    if (s.err != cudaSuccess) {
        set_errorf("flash_decode_q8_0_noalloc: cudaGetSymbolAddress failed on cuda:%d: %s", dev,
                   cudaGetErrorString(s.err));
        return false;
    }
    *scratch = s.scratch;
    *status = s.status;
    return true;
}

bool on_device(const void* p, const char* name) {
    cudaPointerAttributes attr;
    if (!p || cudaPointerGetAttributes(&attr, p) != cudaSuccess ||
        (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged)) {
        cudaGetLastError();
        set_errorf("flash_decode_q8_0_noalloc: %s is not CUDA device memory", name);
        return false;
    }
    return true;
}

}  // namespace
}  // namespace gtb

using namespace gtb;

extern "C" GTB_API int gtb_decode_q8_0_noalloc(const void* q, int q_dtype, const void* k_q8, const void* v_q8,
                                               const int32_t* seq_lens, int64_t B, int64_t H, int64_t Hkv,
                                               int64_t Smax, int64_t D, float scale, void* out, void* stream) {
    const char* ctx = "flash_decode_q8_0_noalloc";
    if (B < 0 || H < 0 || Hkv <= 0 || Smax < 0 || D <= 0) {
        set_errorf("%s: bad sizes", ctx);
        return -1;
    }
    if (H % Hkv != 0) {
        set_errorf("%s: num_heads must be divisible by num_kv_heads", ctx);
        return -1;
    }
    if (D % 32 != 0) {
        set_errorf("%s: the head size must be a multiple of the Q8_0 block (32)", ctx);
        return -1;
    }
    if (q_dtype != F16 && q_dtype != BF16 && q_dtype != F32) {
        set_errorf("%s: q must be f16, bf16 or f32", ctx);
        return -1;
    }
    if (B == 0 || H == 0) return 0;
    // bounds first, so that the size below cannot wrap around and slip past the check
    if (B > INT32_MAX || Smax > INT32_MAX || H > 65535 || D > 256) {
        set_errorf("%s: sizes out of range (B and Smax at most 2^31 - 1, H at most 65535, D at most 256)", ctx);
        return -1;
    }
    // the scratch size of decode_scratch_bytes(), in 128-bit arithmetic: with the bounds above the
    // product stays below 2^31 * 2^16 * 2^20 * 2^16 * 2^9 * 4 < 2^128
    const unsigned __int128 nch = (unsigned __int128)decode_num_chunks(Smax);
    const unsigned __int128 items = (unsigned __int128)B * (unsigned __int128)Hkv * nch;
    const unsigned __int128 work = ((unsigned __int128)decode_list_offset(B) * 4 + items * 8 + 255) / 256 * 256;
    const unsigned __int128 part = nch <= 1 ? 0 : items * (unsigned __int128)(H / Hkv) * (unsigned __int128)(D + 2) * 4;
    const unsigned __int128 need128 = work + part;
    const size_t need = need128 > (unsigned __int128)SIZE_MAX ? SIZE_MAX : (size_t)need128;
    if (need128 > (unsigned __int128)GTB_DECODE_NOALLOC_SCRATCH_BYTES) {
        set_errorf("%s: this call needs %zu bytes of scratch, more than the fixed %zu bytes this entry point has "
                   "(a work area of 8 * (B + 2) + 8 * B * Hkv * ceil(Smax / %d) bytes rounded up to 256, plus "
                   "B * Hkv * ceil(Smax / %d) * (H / Hkv) * (D + 2) * 4 bytes of partials when Smax spans more than "
                   "one chunk); use gtb_decode_q8_0",
                   ctx, need, (size_t)GTB_DECODE_NOALLOC_SCRATCH_BYTES, GTB_DECODE_CHUNK, GTB_DECODE_CHUNK);
        return -1;
    }
    if (!on_device(q, "q") || !on_device(out, "out") || !on_device(seq_lens, "seq_lens")) return -1;
    if (Smax > 0 && (!on_device(k_q8, "k") || !on_device(v_q8, "v"))) return -1;
    int dev = 0;
    if (cuda_failed(cudaGetDevice(&dev), ctx)) return -1;
    float* scratch = nullptr;
    int* status = nullptr;
    if (!device_scratch(dev, &scratch, &status)) return -1;
    const float sc = scale <= 0.0f ? 1.0f / std::sqrt((float)D) : scale;
    DecodeArgs a{q, q_dtype, k_q8, v_q8, seq_lens, B, H, Hkv, Smax, D, sc, out, status};
    return launch_decode_q8_0(a, scratch, (cudaStream_t)stream);
}
