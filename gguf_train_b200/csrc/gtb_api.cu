// Raw-pointer C ABI of the attention engine (include/gtb_attn.h): argument checks, kernel choice,
// scratch from the stream-ordered allocator, error state.
//
// Error messages keep the wording of the reference's checks in gt_flash_attention
// (csrc/gt_ops_nn.cpp:2425-2454) where the same condition is tested, so callers that match on
// them (tests/test_pooling_and_attention.py:381,386 look for "cannot be broadcast") keep working.

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>
#include <vector>

#include "dropout.cuh"
#include "gtb_common.cuh"
#include "q8_0_internal.h"
#include "rope.cuh"
#include "sdpa_args.h"
#include "sm100_ptx.cuh"

namespace gtb {

constexpr long long WAIT_LIMIT_HOST = sm100::WAIT_LIMIT;

namespace {
thread_local std::string g_err;
thread_local const char* g_last_path = "";  // kernel family of the calling thread's last attention call
std::mutex g_status_mtx;
int* g_status[64] = {};
constexpr int MAX_EXTRA_WORDS = 4;
int* g_extra_status[64][MAX_EXTRA_WORDS] = {};
}  // namespace

void set_error(const std::string& msg) { g_err = msg; }

void set_errorf(const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
}

const char* last_error() { return g_err.c_str(); }
void clear_error() { g_err.clear(); }

bool cuda_failed(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return false;
    set_errorf("%s: CUDA error %d (%s)", what, (int)e, cudaGetErrorString(e));
    return true;
}

int* device_status_word(int device) {
    if (device < 0 || device >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(g_status_mtx);
    if (!g_status[device]) {
        int* p = nullptr;
        if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
        cudaMemset(p, 0, sizeof(int));
        g_status[device] = p;
    }
    return g_status[device];
}

void register_status_word(int device, int* word) {
    if (device < 0 || device >= 64 || !word) return;
    std::lock_guard<std::mutex> lk(g_status_mtx);
    for (int i = 0; i < MAX_EXTRA_WORDS; ++i) {
        if (g_extra_status[device][i] == word) return;
        if (!g_extra_status[device][i]) {
            g_extra_status[device][i] = word;
            return;
        }
    }
}

namespace {

// Every status word of a device that exists so far (none is allocated here).
int status_words(int device, int** out) {
    if (device < 0 || device >= 64) return 0;
    std::lock_guard<std::mutex> lk(g_status_mtx);
    int n = 0;
    if (g_status[device]) out[n++] = g_status[device];
    for (int i = 0; i < MAX_EXTRA_WORDS; ++i)
        if (g_extra_status[device][i]) out[n++] = g_extra_status[device][i];
    return n;
}

// A kernel whose mbarrier nothing ever arrives at: its bounded wait (the same mbar_wait every
// kernel uses) must give up after `limit` cycles, record code 90 in the status word and return.
__global__ void selftest_wait_kernel(int* status, long long limit) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        sm100::mbar_init(&bar, 1);
        sm100::fence_mbar_init();
    }
    __syncthreads();
    sm100::mbar_wait(&bar, 0, status, 90, limit);
    __syncthreads();  // no thread leaves while another still waits on the shared barrier
}

std::string shape_str(const int64_t* s, int n) {
    std::string r = "[";
    for (int i = 0; i < n; ++i) r += (i ? ", " : "") + std::to_string(s[i]);
    return r + "]";
}

// Every pointer handed to a kernel must be device (or managed) memory of the current device.
bool check_device_ptr(const void* p, const char* ctx, const char* name) {
    if (!p) {
        set_errorf("%s: %s is NULL", ctx, name);
        return false;
    }
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
        cudaGetLastError();
        set_errorf("%s: %s is not CUDA memory (this engine has no CPU path)", ctx, name);
        return false;
    }
    if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged) {
        set_errorf("%s: %s is not CUDA device memory (this engine has no CPU path)", ctx, name);
        return false;
    }
    int dev = 0;
    cudaGetDevice(&dev);
    if (attr.type == cudaMemoryTypeDevice && attr.device != dev) {
        set_errorf("%s: %s lives on cuda:%d but the current device is cuda:%d", ctx, name, attr.device, dev);
        return false;
    }
    return true;
}

int64_t numel4(const gtb_tensor4& t) { return t.shape[0] * t.shape[1] * t.shape[2] * t.shape[3]; }

// Shapes, dtypes and mask of an attention call (gt_ops_nn.cpp:2425-2454).
bool check_attn(const char* ctx, const gtb_tensor4* q, const gtb_tensor4* k, const gtb_tensor4* v,
                const gtb_tensor4* mask, AttnShape& sh) {
    if (!q || !k || !v) {
        set_errorf("%s expects 4D q, k, v tensors (B, H, L, D)", ctx);
        return false;
    }
    sh.B = q->shape[0]; sh.H = q->shape[1]; sh.L = q->shape[2]; sh.D = q->shape[3];
    sh.Hkv = k->shape[1]; sh.S = k->shape[2]; sh.Dv = v->shape[3];
    for (int i = 0; i < 4; ++i) {
        if (q->shape[i] < 0 || k->shape[i] < 0 || v->shape[i] < 0) {
            set_errorf("%s: negative size", ctx);
            return false;
        }
    }
    if (sh.Hkv <= 0 || sh.H % sh.Hkv != 0) {
        set_errorf("%s: num_heads must be divisible by num_kv_heads", ctx);
        return false;
    }
    if (k->shape[0] != sh.B || v->shape[0] != sh.B || v->shape[1] != sh.Hkv || v->shape[2] != sh.S ||
        k->shape[3] != sh.D) {
        set_errorf("%s: q (B, H, L, D), k (B, H_kv, S, D) and v (B, H_kv, S, Dv) do not fit together", ctx);
        return false;
    }
    if (!is_float_dtype(q->dtype) || k->dtype != q->dtype || v->dtype != q->dtype) {
        set_errorf("%s: q, k and v must share one floating dtype (f32, f16, bf16 or f64)", ctx);
        return false;
    }
    if (mask) {
        const int64_t want[4] = {sh.B, sh.H, sh.L, sh.S};
        bool fits = true;
        for (int i = 0; i < 4; ++i) fits = fits && (mask->shape[i] == 1 || mask->shape[i] == want[i]);
        if (!fits) {
            set_errorf("%s: attn_mask of shape %s cannot be broadcast to the attention weights %s", ctx,
                       shape_str(mask->shape, 4).c_str(), shape_str(want, 4).c_str());
            return false;
        }
        if (mask->dtype != BOOL && !is_float_dtype(mask->dtype)) {
            set_errorf("%s: attn_mask must be bool or floating point", ctx);
            return false;
        }
    }
    return true;
}

gtb_tensor4 broadcast_mask(const gtb_tensor4& m) {
    gtb_tensor4 r = m;
    for (int i = 0; i < 4; ++i)
        if (r.shape[i] == 1) r.stride[i] = 0;
    return r;
}

bool same_shape(const gtb_tensor4& a, const int64_t* s) {
    for (int i = 0; i < 4; ++i)
        if (a.shape[i] != s[i]) return false;
    return true;
}

float resolve_scale(float scale, int64_t D) { return scale <= 0.0f ? 1.0f / std::sqrt((float)D) : scale; }

// The scratch of the backward and of the split-KV decode comes from the device's stream-ordered
// pool. By default that pool hands unused memory back to the driver at every synchronisation, so a
// call after a synchronize would map its scratch afresh (milliseconds for tens of MB) while the GPU
// idles; keeping the memory in the pool makes repeated calls allocation-free after the first.
void keep_pool_memory(int dev) {
    static std::once_flag once[64];
    if (dev < 0 || dev >= 64) return;
    std::call_once(once[dev], [dev] {
        cudaMemPool_t pool;
        if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
            uint64_t keep = UINT64_MAX;
            cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
        }
        cudaGetLastError();
    });
}

int env_int(const char* name, int dflt) {
    const char* e = getenv(name);
    return e ? atoi(e) : dflt;
}

// RoPE arguments with the reference's checks and messages (gt_rope_check, csrc/gt_ops_nn.cpp:2316-2357)
bool rope_args(int64_t D, int n_dims, int mode, float freq_base, float freq_scale, bool backward, RopeArgs& r) {
    if (mode != 0 && mode != 2) {
        set_errorf("rope: mode must be 0 (normal) or 2 (NeoX), got %d; the multi-dimensional modes need per-section "
                   "position ids and are not supported", mode);
        return false;
    }
    if (n_dims < 2 || n_dims % 2 != 0 || n_dims > D) {
        set_errorf("rope: n_dims must be an even number between 2 and the head dimension %lld, got %d", (long long)D, n_dims);
        return false;
    }
    if (!(freq_base > 0.0f) || !std::isfinite(freq_base) || !std::isfinite(freq_scale)) {
        set_error("rope: freq_base must be positive and finite, and freq_scale finite");
        return false;
    }
    r.n_dims = n_dims;
    r.mode = mode;
    r.theta_scale = powf(freq_base, -2.0f / (float)n_dims);
    r.freq_scale = freq_scale;
    r.sin_sign = backward ? -1.0f : 1.0f;
    return true;
}

// Sizes and dtype of a Q8_0 cache append (both entry points)
bool append_args_ok(int x_dtype, int64_t B, int64_t Hkv, int64_t n_new, int64_t D, int64_t Smax) {
    if (B < 0 || Hkv < 0 || n_new < 0 || D < 0 || Smax < 0) {
        set_error("q8_0_append: negative size");
        return false;
    }
    if (D % 32 != 0) {
        set_error("Tensor size must be a multiple of ggml quantization block size");
        return false;
    }
    if (n_new > INT32_MAX) {
        set_error("q8_0_append: n_new must fit in int32");
        return false;
    }
    if (x_dtype != F32 && x_dtype != F16 && x_dtype != BF16) {
        set_error("q8_0_append: the new rows must be f32, f16 or bf16");
        return false;
    }
    return true;
}

// pointers checked, then the append kernel (and the length update) on `stream`
int append_run(const void* x, int x_dtype, int64_t B, int64_t Hkv, int64_t n_new, int64_t D, void* cache, int64_t Smax,
               int32_t* pos, int advance, const RopeArgs* rope, void* stream) {
    const char* ctx = "q8_0_append";
    if (B == 0 || n_new == 0) return 0;
    if (D > 0 && Hkv > 0) {
        if (!check_device_ptr(x, ctx, "x") || !check_device_ptr(cache, ctx, "cache")) return -1;
    }
    if (!check_device_ptr(pos, ctx, "pos")) return -1;
    return launch_q8_0_append(x, x_dtype, B, Hkv, n_new, D, cache, Smax, pos, advance != 0, rope, (cudaStream_t)stream);
}

// The two side streams of gtb_sdpa_fwd_host on a device (host -> device and device -> host copies),
// non-blocking, created once and kept for the process.
struct HostCopyStreams {
    cudaStream_t in = nullptr, out = nullptr;
};

HostCopyStreams host_copy_streams(int dev) {
    static HostCopyStreams hs[64];
    static std::once_flag once[64];
    if (dev < 0 || dev >= 64) return HostCopyStreams{};
    std::call_once(once[dev], [dev] {
        if (cudaStreamCreateWithFlags(&hs[dev].in, cudaStreamNonBlocking) != cudaSuccess ||
            cudaStreamCreateWithFlags(&hs[dev].out, cudaStreamNonBlocking) != cudaSuccess)
            hs[dev] = HostCopyStreams{};
        cudaGetLastError();
    });
    return hs[dev];
}

// host memory, pinned or not (not CUDA device or managed memory)
bool check_host_ptr(const void* p, const char* ctx, const char* name) {
    if (!p) {
        set_errorf("%s: %s is NULL", ctx, name);
        return false;
    }
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
        cudaGetLastError();
        return true;
    }
    if (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged) {
        set_errorf("%s: %s is CUDA memory; this call takes host memory (use gtb_sdpa_fwd for device tensors)", ctx, name);
        return false;
    }
    return true;
}

bool row_major(const gtb_tensor4& t) {
    int64_t s = 1;
    for (int i = 3; i >= 0; --i) {
        if (t.shape[i] > 1 && t.stride[i] != s) return false;
        s *= t.shape[i];
    }
    return true;
}

}  // namespace

void retain_pool_memory(int dev) { keep_pool_memory(dev); }

}  // namespace gtb

using namespace gtb;

extern "C" {

GTB_API const char* gtb_last_error(void) { return gtb::last_error(); }
GTB_API void gtb_clear_error(void) { gtb::clear_error(); }

GTB_API const char* gtb_last_path(void) { return g_last_path; }

GTB_API const char* gtb_version(void) { return "gguf_train_b200 attention engine 0.1 (sm_100a)"; }

GTB_API int gtb_device_status(void) {
    int dev = 0;
    if (cuda_failed(cudaGetDevice(&dev), "gtb_device_status")) return -1;
    if (cuda_failed(cudaDeviceSynchronize(), "gtb_device_status: synchronize")) return -1;
    int* words[1 + MAX_EXTRA_WORDS];
    const int n = status_words(dev, words);
    int first = 0;
    for (int i = 0; i < n; ++i) {
        int v = 0;
        if (cuda_failed(cudaMemcpy(&v, words[i], sizeof(int), cudaMemcpyDeviceToHost), "gtb_device_status: read"))
            return -1;
        if (v) {
            if (!first) first = v;
            if (cuda_failed(cudaMemset(words[i], 0, sizeof(int)), "gtb_device_status: clear")) return -1;
        }
    }
    return first;
}

GTB_API int gtb_selftest_wait_timeout(int64_t limit_cycles, void* stream) {
    if (limit_cycles < 1000 || limit_cycles > WAIT_LIMIT_HOST) {
        set_errorf("selftest_wait_timeout: limit_cycles must be in [1000, %lld]", (long long)WAIT_LIMIT_HOST);
        return -1;
    }
    int dev = 0;
    if (cuda_failed(cudaGetDevice(&dev), "selftest_wait_timeout")) return -1;
    int* w = device_status_word(dev);
    if (!w) {
        set_error("selftest_wait_timeout: no status word");
        return -1;
    }
    selftest_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(w, (long long)limit_cycles);
    return cuda_failed(cudaGetLastError(), "selftest_wait_timeout launch") ? -1 : 0;
}

GTB_API int gtb_sdpa_fwd(const gtb_tensor4* q, const gtb_tensor4* k, const gtb_tensor4* v, const gtb_tensor4* mask,
                         float scale, int is_causal, gtb_tensor4* out, void* lse, void* stream) {
    return gtb_sdpa_fwd_ex(q, k, v, mask, scale, is_causal, out, lse, nullptr, stream);
}

GTB_API int gtb_sdpa_fwd_ex(const gtb_tensor4* q, const gtb_tensor4* k, const gtb_tensor4* v, const gtb_tensor4* mask,
                            float scale, int is_causal, gtb_tensor4* out, void* lse, const gtb_sdpa_opts* opts,
                            void* stream) {
    const char* ctx = "flash_attention";
    FwdArgs a;
    if (opts && !(opts->dropout_p >= 0.0f && opts->dropout_p < 1.0f)) {
        set_errorf("%s: dropout probability has to be between 0 and 1, but got %g", ctx, (double)opts->dropout_p);
        return -1;
    }
    if (opts) {
        a.drop_p = opts->dropout_p;
        a.drop_thr = drop_threshold(opts->dropout_p);
        a.drop_seed = opts->dropout_seed;
    }
    if (!check_attn(ctx, q, k, v, mask, a.sh)) return -1;
    if (!out) {
        set_errorf("%s: out is NULL", ctx);
        return -1;
    }
    const int64_t osh[4] = {a.sh.B, a.sh.H, a.sh.L, a.sh.Dv};
    if (!same_shape(*out, osh) || out->dtype != q->dtype) {
        set_errorf("%s: out must be %s in q's dtype", ctx, shape_str(osh, 4).c_str());
        return -1;
    }
    if (numel4(*out) == 0) return 0;
    if (!check_device_ptr(q->data, ctx, "q") || !check_device_ptr(out->data, ctx, "out")) return -1;
    if (a.sh.S > 0 && (!check_device_ptr(k->data, ctx, "k") || !check_device_ptr(v->data, ctx, "v"))) return -1;
    if (mask && !check_device_ptr(mask->data, ctx, "attn_mask")) return -1;
    if (lse && !check_device_ptr(lse, ctx, "lse")) return -1;
    a.q = *q; a.k = *k; a.v = *v; a.o = *out;
    a.has_mask = mask != nullptr;
    if (mask) a.mask = broadcast_mask(*mask);
    a.scale = resolve_scale(scale, a.sh.D);
    a.causal = is_causal ? 1 : 0;
    a.lse = lse;
    cudaStream_t st = (cudaStream_t)stream;
    // GTB_FWD_SIMT=1 forces the SIMT kernel (used to cross-check the two kernels)
    static const int force_simt = env_int("GTB_FWD_SIMT", 0);
    if (!force_simt && fwd_sm100_supported(a)) {
        g_last_path = "tcgen05";
        return launch_fwd_sm100(a, st);
    }
    g_last_path = f32_tiled_supported(a.sh, a.q.dtype) ? "f32_tiled" : "simt";
    return launch_fwd_simt(a, st);
}

GTB_API int gtb_sdpa_fwd_rope(const gtb_tensor4* q, const gtb_tensor4* k, const gtb_tensor4* v, const gtb_tensor4* mask,
                              float scale, int is_causal, const int32_t* pos_q, int64_t n_pos_q, const int32_t* pos_k,
                              int64_t n_pos_k, int n_dims, int mode, float freq_base, float freq_scale,
                              int q_in_kernel, gtb_tensor4* k_rot, gtb_tensor4* out, void* lse, void* stream) {
    const char* ctx = "flash_attention (rope)";
    FwdArgs a;
    if (!check_attn(ctx, q, k, v, mask, a.sh)) return -1;
    if (q->dtype != F32 && q->dtype != F16 && q->dtype != BF16) {
        set_errorf("%s: q and k must be f32, f16 or bf16", ctx);
        return -1;
    }
    RopeArgs ra;
    if (!rope_args(a.sh.D, n_dims, mode, freq_base, freq_scale, false, ra)) return -1;
    if (!pos_q || !pos_k || n_pos_q < a.sh.L || n_pos_k < a.sh.S) {
        set_errorf("%s: pos_q needs a position for each of the %lld queries and pos_k one for each of the %lld keys", ctx,
                   (long long)a.sh.L, (long long)a.sh.S);
        return -1;
    }
    if (!out || !k_rot) {
        set_errorf("%s: out and k_rot are required", ctx);
        return -1;
    }
    const int64_t osh[4] = {a.sh.B, a.sh.H, a.sh.L, a.sh.Dv};
    if (!same_shape(*out, osh) || out->dtype != q->dtype) {
        set_errorf("%s: out must be %s in q's dtype", ctx, shape_str(osh, 4).c_str());
        return -1;
    }
    if (!same_shape(*k_rot, k->shape) || k_rot->dtype != k->dtype || !row_major(*k_rot) || !row_major(*k) ||
        !row_major(*q)) {
        set_errorf("%s: q, k and k_rot (k's shape and dtype) must be contiguous", ctx);
        return -1;
    }
    if (numel4(*out) == 0) return 0;
    if (!check_device_ptr(q->data, ctx, "q") || !check_device_ptr(out->data, ctx, "out") ||
        !check_device_ptr(pos_q, ctx, "pos_q") || !check_device_ptr(pos_k, ctx, "pos_k"))
        return -1;
    if (a.sh.S > 0 && (!check_device_ptr(k->data, ctx, "k") || !check_device_ptr(v->data, ctx, "v") ||
                       !check_device_ptr(k_rot->data, ctx, "k_rot")))
        return -1;
    if (mask && !check_device_ptr(mask->data, ctx, "attn_mask")) return -1;
    if (lse && !check_device_ptr(lse, ctx, "lse")) return -1;
    cudaStream_t st = (cudaStream_t)stream;
    // k: rotated once in HBM (every query tile reads each key tile), into the caller's k_rot
    if (a.sh.S > 0 && launch_rope(k->data, k->dtype, a.sh.B * a.sh.Hkv * a.sh.S, a.sh.S, a.sh.D, pos_k, ra, k_rot->data, st))
        return -1;
    a.q = *q; a.k = *k_rot; a.v = *v; a.o = *out;
    a.has_mask = mask != nullptr;
    if (mask) a.mask = broadcast_mask(*mask);
    a.scale = resolve_scale(scale, a.sh.D);
    a.causal = is_causal ? 1 : 0;
    a.lse = lse;
    int dev = 0;
    if (cuda_failed(cudaGetDevice(&dev), ctx)) return -1;
    retain_pool_memory(dev);
    const size_t q_bytes = (size_t)numel4(*q) * (q->dtype == F32 ? 4 : 2);
    if (q_in_kernel && !mask && n_dims % 16 == 0 && a.sh.L > 0 && fwd_sm100_supported(a)) {
        // q: rotated inside the tcgen05 forward, each Q tile in shared memory once it has landed, from a
        // (cos, sin) table of the L query positions
        float* tab = nullptr;
        const size_t tab_bytes = (size_t)a.sh.L * (size_t)(n_dims / 2) * 2 * sizeof(float);
        if (cuda_failed(cudaMallocAsync((void**)&tab, tab_bytes, st), "flash_attention (rope): angle table")) return -1;
        int rc = launch_rope_table(pos_q, a.sh.L, ra, tab, st);
        if (rc == 0) {
            a.rope_q_tab = tab;
            a.rope_n_dims = n_dims;
            a.rope_mode = mode;
            g_last_path = "tcgen05+rope";
            rc = launch_fwd_sm100(a, st);
        }
        cudaFreeAsync(tab, st);  // after the kernel on the same stream
        return rc;
    }
    // otherwise q is rotated into a scratch copy first and the forward runs as gtb_sdpa_fwd would
    void* qr = nullptr;
    if (cuda_failed(cudaMallocAsync(&qr, q_bytes, st), "flash_attention (rope): rotated q")) return -1;
    int rc = launch_rope(q->data, q->dtype, a.sh.B * a.sh.H * a.sh.L, a.sh.L, a.sh.D, pos_q, ra, qr, st);
    if (rc == 0) {
        a.q.data = qr;
        if (fwd_sm100_supported(a)) {
            g_last_path = "tcgen05";
            rc = launch_fwd_sm100(a, st);
        } else {
            g_last_path = f32_tiled_supported(a.sh, a.q.dtype) ? "f32_tiled" : "simt";
            rc = launch_fwd_simt(a, st);
        }
    }
    cudaFreeAsync(qr, st);
    return rc;
}

GTB_API int gtb_linear(const void* a, const void* b, const void* bias, void* c, int64_t M, int64_t N, int64_t K,
                       int64_t lda, int64_t ldb, int64_t ldc, int dtype, void* stream) {
    const char* ctx = "linear";
    if (M < 0 || N < 0 || K <= 0) {
        set_errorf("%s: sizes must be M, N >= 0 and K > 0 (got %lld, %lld, %lld)", ctx, (long long)M, (long long)N,
                   (long long)K);
        return -1;
    }
    if (dtype != BF16 && dtype != F16) {
        set_errorf("%s: the tensor-core linear takes bf16 or f16 operands", ctx);
        return -1;
    }
    if (lda < K || ldb < K || ldc < N || lda % 8 || ldb % 8 || ldc % 8) {
        set_errorf("%s: leading dimensions must cover the rows and be multiples of 8 elements", ctx);
        return -1;
    }
    if (M >= (1ll << 31) || N >= (1ll << 31) || K >= (1ll << 31)) {
        set_errorf("%s: sizes out of range", ctx);
        return -1;
    }
    if (M == 0 || N == 0) return 0;
    if (!check_device_ptr(a, ctx, "a") || !check_device_ptr(b, ctx, "b") || !check_device_ptr(c, ctx, "c")) return -1;
    if (bias && !check_device_ptr(bias, ctx, "bias")) return -1;
    if (((uintptr_t)a | (uintptr_t)b | (uintptr_t)c) & 15) {
        set_errorf("%s: a, b and c must be 16-byte aligned", ctx);
        return -1;
    }
    return launch_linear_sm100(a, b, bias, c, M, N, K, lda, ldb, ldc, dtype, (cudaStream_t)stream);
}

GTB_API int gtb_attn_weights(const gtb_tensor4* q, const gtb_tensor4* k, const gtb_tensor4* mask, const void* lse,
                             float scale, int is_causal, int average, const gtb_sdpa_opts* opts, gtb_tensor4* out,
                             void* stream) {
    const char* ctx = "attention_weights";
    FwdArgs a;
    if (!check_attn(ctx, q, k, k, mask, a.sh)) return -1;
    a.sh.Dv = a.sh.D;
    if (!out || !lse) {
        set_errorf("%s: out and lse are required", ctx);
        return -1;
    }
    const int64_t osh[4] = {a.sh.B, average ? 1 : a.sh.H, a.sh.L, a.sh.S};
    if (!same_shape(*out, osh) || out->dtype != q->dtype || !row_major(*out)) {
        set_errorf("%s: out must be a contiguous %s tensor in q's dtype", ctx, shape_str(osh, 4).c_str());
        return -1;
    }
    if (opts && !(opts->dropout_p >= 0.0f && opts->dropout_p < 1.0f)) {
        set_errorf("%s: dropout probability has to be between 0 and 1, but got %g", ctx, (double)opts->dropout_p);
        return -1;
    }
    if (numel4(*out) == 0) return 0;
    if (!check_device_ptr(q->data, ctx, "q") || !check_device_ptr(out->data, ctx, "out") ||
        !check_device_ptr(lse, ctx, "lse"))
        return -1;
    if (a.sh.S > 0 && !check_device_ptr(k->data, ctx, "k")) return -1;
    if (mask && !check_device_ptr(mask->data, ctx, "attn_mask")) return -1;
    a.q = *q; a.k = *k; a.v = *k;
    a.has_mask = mask != nullptr;
    if (mask) a.mask = broadcast_mask(*mask);
    a.scale = resolve_scale(scale, a.sh.D);
    a.causal = is_causal ? 1 : 0;
    if (opts) {
        a.drop_p = opts->dropout_p;
        a.drop_thr = drop_threshold(opts->dropout_p);
        a.drop_seed = opts->dropout_seed;
    }
    return launch_attn_weights(a, lse, out->data, average != 0, (cudaStream_t)stream);
}

GTB_API int gtb_sdpa_fwd_host(const gtb_tensor4* q, const gtb_tensor4* k, const gtb_tensor4* v, float scale, int is_causal,
                              gtb_tensor4* out, int pieces, void* stream) {
    const char* ctx = "flash_attention_host";
    AttnShape sh;
    if (!check_attn(ctx, q, k, v, nullptr, sh)) return -1;
    if (!out) {
        set_errorf("%s: out is NULL", ctx);
        return -1;
    }
    const int64_t osh[4] = {sh.B, sh.H, sh.L, sh.Dv};
    if (!same_shape(*out, osh) || out->dtype != q->dtype) {
        set_errorf("%s: out must be %s in q's dtype", ctx, shape_str(osh, 4).c_str());
        return -1;
    }
    if (!row_major(*q) || !row_major(*k) || !row_major(*v) || !row_major(*out)) {
        set_errorf("%s: q, k, v and out must be contiguous (row-major) host tensors", ctx);
        return -1;
    }
    if (numel4(*out) == 0) return 0;
    if (!check_host_ptr(q->data, ctx, "q") || !check_host_ptr(out->data, ctx, "out")) return -1;
    if (sh.S > 0 && (!check_host_ptr(k->data, ctx, "k") || !check_host_ptr(v->data, ctx, "v"))) return -1;
    int dev = 0;
    if (cuda_failed(cudaGetDevice(&dev), ctx)) return -1;
    const HostCopyStreams hs = host_copy_streams(dev);
    if (!hs.in || !hs.out) {
        set_errorf("%s: could not create the copy streams", ctx);
        return -1;
    }
    cudaStream_t st = (cudaStream_t)stream;
    const int64_t G = sh.H / sh.Hkv, P = pieces > 0 ? pieces : 8;
    // pieces of work: whole sequences, or one sequence's kv heads in groups (with their query heads);
    // either way each piece of q, k, v and out is one contiguous range of the host tensors
    struct Piece { int64_t b0, m, h0, mh; };
    std::vector<Piece> ps;
    if (sh.B >= P) {
        const int64_t n = sh.B / P;
        for (int64_t b0 = 0; b0 < sh.B; b0 += n) ps.push_back({b0, std::min(n, sh.B - b0), 0, sh.Hkv});
    } else {
        const int64_t parts = std::max<int64_t>(1, std::min<int64_t>(sh.Hkv, P / sh.B));
        const int64_t nh = (sh.Hkv + parts - 1) / parts;
        for (int64_t b = 0; b < sh.B; ++b)
            for (int64_t h0 = 0; h0 < sh.Hkv; h0 += nh) ps.push_back({b, 1, h0, std::min(nh, sh.Hkv - h0)});
    }
    int64_t nb = 0, nh = 0;
    for (const Piece& x : ps) { nb = std::max(nb, x.m); nh = std::max(nh, x.mh); }
    const size_t es = dtype_size(q->dtype);
    auto up = [](size_t b) { return (b + 255) / 256 * 256; };
    const size_t bq = up(es * nb * nh * G * sh.L * sh.D), bk = up(es * nb * nh * sh.S * sh.D),
                 bv = up(es * nb * nh * sh.S * sh.Dv), bo = up(es * nb * nh * G * sh.L * sh.Dv);
    const size_t slot = bq + bk + bv + bo;
    keep_pool_memory(dev);
    unsigned char* mem = nullptr;
    if (cuda_failed(cudaMallocAsync((void**)&mem, 2 * slot, st), "flash_attention_host: device slots")) return -1;
    const size_t ne = 3 * ps.size() + 3;
    std::vector<cudaEvent_t> ev(ne, nullptr);
    bool bad = false;
    for (size_t i = 0; i < ne && !bad; ++i) bad = cuda_failed(cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming), ctx);
    cudaEvent_t* ev_in = ev.data();
    cudaEvent_t* ev_comp = ev_in + ps.size();
    cudaEvent_t* ev_out = ev_comp + ps.size();
    cudaEvent_t ev_start = ev[ne - 3], ev_join_in = ev[ne - 2], ev_join_out = ev[ne - 1];
    // the slots were allocated on `st`: the copy streams start after that point
    if (!bad) bad = cuda_failed(cudaEventRecord(ev_start, st), ctx) || cuda_failed(cudaStreamWaitEvent(hs.in, ev_start, 0), ctx) ||
                    cuda_failed(cudaStreamWaitEvent(hs.out, ev_start, 0), ctx);
    const unsigned char* hq = (const unsigned char*)q->data;
    const unsigned char* hk = (const unsigned char*)k->data;
    const unsigned char* hv = (const unsigned char*)v->data;
    unsigned char* ho = (unsigned char*)out->data;
    for (size_t i = 0; i < ps.size() && !bad; ++i) {
        const Piece& x = ps[i];
        unsigned char* base = mem + (i & 1) * slot;
        const int64_t nq = x.m * x.mh * G;  // query heads of the piece (one range: m == 1 or mh == Hkv)
        const size_t oq = es * (x.b0 * sh.H + x.h0 * G) * sh.L * sh.D, nbq = es * nq * sh.L * sh.D;
        const size_t okv = (x.b0 * sh.Hkv + x.h0), nkv = x.m * x.mh;
        const size_t oo = es * (x.b0 * sh.H + x.h0 * G) * sh.L * sh.Dv, nbo = es * nq * sh.L * sh.Dv;
        if (i >= 2) bad = cuda_failed(cudaStreamWaitEvent(hs.in, ev_comp[i - 2], 0), ctx);  // slot read by piece i-2
        bad = bad || cuda_failed(cudaMemcpyAsync(base, hq + oq, nbq, cudaMemcpyHostToDevice, hs.in), ctx) ||
              cuda_failed(cudaMemcpyAsync(base + bq, hk + es * okv * sh.S * sh.D, es * nkv * sh.S * sh.D,
                                          cudaMemcpyHostToDevice, hs.in), ctx) ||
              cuda_failed(cudaMemcpyAsync(base + bq + bk, hv + es * okv * sh.S * sh.Dv, es * nkv * sh.S * sh.Dv,
                                          cudaMemcpyHostToDevice, hs.in), ctx) ||
              cuda_failed(cudaEventRecord(ev_in[i], hs.in), ctx) || cuda_failed(cudaStreamWaitEvent(st, ev_in[i], 0), ctx);
        if (!bad && i >= 2) bad = cuda_failed(cudaStreamWaitEvent(st, ev_out[i - 2], 0), ctx);  // slot's output copied out
        if (bad) break;
        gtb_tensor4 tq, tk, tv, to;
        const int64_t qs[4] = {x.m, x.mh * G, sh.L, sh.D}, ks[4] = {x.m, x.mh, sh.S, sh.D}, vs[4] = {x.m, x.mh, sh.S, sh.Dv},
                      os[4] = {x.m, x.mh * G, sh.L, sh.Dv};
        auto dense = [&](gtb_tensor4& t, void* p, const int64_t* s4) {
            t.data = p;
            t.dtype = q->dtype;
            int64_t str = 1;
            for (int d = 3; d >= 0; --d) {
                t.shape[d] = s4[d];
                t.stride[d] = str;
                str *= s4[d];
            }
        };
        dense(tq, base, qs);
        dense(tk, base + bq, ks);
        dense(tv, base + bq + bk, vs);
        dense(to, base + bq + bk + bv, os);
        if (gtb_sdpa_fwd(&tq, &tk, &tv, nullptr, scale, is_causal, &to, nullptr, st) != 0) {
            bad = true;
            break;
        }
        bad = cuda_failed(cudaEventRecord(ev_comp[i], st), ctx) || cuda_failed(cudaStreamWaitEvent(hs.out, ev_comp[i], 0), ctx) ||
              cuda_failed(cudaMemcpyAsync(ho + oo, base + bq + bk + bv, nbo, cudaMemcpyDeviceToHost, hs.out), ctx) ||
              cuda_failed(cudaEventRecord(ev_out[i], hs.out), ctx);
    }
    // join both copy streams into `st` (after an error too: the slots are released on `st`)
    const bool joined = ev_join_in && ev_join_out && cudaEventRecord(ev_join_in, hs.in) == cudaSuccess &&
                        cudaEventRecord(ev_join_out, hs.out) == cudaSuccess &&
                        cudaStreamWaitEvent(st, ev_join_in, 0) == cudaSuccess &&
                        cudaStreamWaitEvent(st, ev_join_out, 0) == cudaSuccess;
    if (!joined) {
        cudaGetLastError();
        cudaStreamSynchronize(hs.in);
        cudaStreamSynchronize(hs.out);
        bad = true;
    }
    cudaFreeAsync(mem, st);
    for (cudaEvent_t e : ev)
        if (e) cudaEventDestroy(e);
    return bad ? -1 : 0;
}

GTB_API int gtb_sdpa_bwd(const gtb_tensor4* dout, const gtb_tensor4* q, const gtb_tensor4* k, const gtb_tensor4* v,
                         const gtb_tensor4* mask, const gtb_tensor4* out, const void* lse, float scale, int is_causal,
                         gtb_tensor4* dq, gtb_tensor4* dk, gtb_tensor4* dv, void* stream) {
    return gtb_sdpa_bwd_ex(dout, q, k, v, mask, out, lse, scale, is_causal, dq, dk, dv, nullptr, stream);
}

GTB_API int gtb_sdpa_bwd_ex(const gtb_tensor4* dout, const gtb_tensor4* q, const gtb_tensor4* k, const gtb_tensor4* v,
                            const gtb_tensor4* mask, const gtb_tensor4* out, const void* lse, float scale, int is_causal,
                            gtb_tensor4* dq, gtb_tensor4* dk, gtb_tensor4* dv, const gtb_sdpa_opts* opts, void* stream) {
    const char* ctx = "flash_attention_backward";
    const int flags = opts ? opts->flags : 0;
    if (flags & ~GTB_BWD_DETERMINISTIC) {
        set_errorf("%s: unknown flags 0x%x", ctx, flags);
        return -1;
    }
    if (opts && !(opts->dropout_p >= 0.0f && opts->dropout_p < 1.0f)) {
        set_errorf("%s: dropout probability has to be between 0 and 1, but got %g", ctx, (double)opts->dropout_p);
        return -1;
    }
    BwdArgs a;
    if (!check_attn(ctx, q, k, v, mask, a.sh)) return -1;
    if (!dout || !out || !lse || !dq || !dk || !dv) {
        set_errorf("%s: dout, out, lse, dq, dk and dv are required", ctx);
        return -1;
    }
    const int64_t osh[4] = {a.sh.B, a.sh.H, a.sh.L, a.sh.Dv};
    if (!same_shape(*dout, osh) || !same_shape(*out, osh) || dout->dtype != q->dtype || out->dtype != q->dtype) {
        set_errorf("%s: dout and out must be %s in q's dtype", ctx, shape_str(osh, 4).c_str());
        return -1;
    }
    if (!same_shape(*dq, q->shape) || !same_shape(*dk, k->shape) || !same_shape(*dv, v->shape) ||
        dq->dtype != q->dtype || dk->dtype != q->dtype || dv->dtype != q->dtype) {
        set_errorf("%s: dq, dk, dv must match q, k, v in shape and dtype", ctx);
        return -1;
    }
    if (numel4(*q) == 0 && numel4(*k) == 0) return 0;
    const gtb_tensor4* all[] = {dout, q, k, v, out, dq, dk, dv};
    const char* names[] = {"dout", "q", "k", "v", "out", "dq", "dk", "dv"};
    for (int i = 0; i < 8; ++i)
        if (numel4(*all[i]) > 0 && !check_device_ptr(all[i]->data, ctx, names[i])) return -1;
    if (mask && !check_device_ptr(mask->data, ctx, "attn_mask")) return -1;
    if (a.sh.L > 0 && !check_device_ptr(lse, ctx, "lse")) return -1;
    a.q = *q; a.k = *k; a.v = *v; a.o = *out; a.dout = *dout; a.dq = *dq; a.dk = *dk; a.dv = *dv;
    a.has_mask = mask != nullptr;
    if (mask) a.mask = broadcast_mask(*mask);
    a.scale = resolve_scale(scale, a.sh.D);
    a.causal = is_causal ? 1 : 0;
    a.lse = lse;
    a.deterministic = (flags & GTB_BWD_DETERMINISTIC) != 0;
    if (opts) {
        a.drop_p = opts->dropout_p;
        a.drop_thr = drop_threshold(opts->dropout_p);
        a.drop_seed = opts->dropout_seed;
    }
    cudaStream_t st = (cudaStream_t)stream;
    // GTB_BWD_SIMT=1 forces the SIMT kernels (used to cross-check the two implementations)
    static const int force_simt = env_int("GTB_BWD_SIMT", 0);
    const bool fast = !force_simt && bwd_sm100_supported(a);
    g_last_path = fast ? "tcgen05" : f32_tiled_supported(a.sh, a.q.dtype) ? "f32_tiled" : "simt";
    const size_t bytes = fast ? bwd_sm100_scratch_bytes(a) : bwd_simt_scratch_bytes(a);
    int dev = 0;
    cudaGetDevice(&dev);
    keep_pool_memory(dev);
    void* scratch = nullptr;
    if (bytes && cuda_failed(cudaMallocAsync(&scratch, bytes, st), "flash_attention_backward: scratch allocation"))
        return -1;
    a.scratch = scratch;
    const int rc = fast ? launch_bwd_sm100(a, st) : launch_bwd_simt(a, st);
    if (scratch) cudaFreeAsync(scratch, st);
    return rc;
}

GTB_API int gtb_q8_0_quantize(const void* x, int x_dtype, int64_t n_rows, int64_t row_len, void* out, void* stream) {
    if (n_rows < 0 || row_len < 0) {
        set_error("quantize: negative size");
        return -1;
    }
    const int64_t n = n_rows * row_len;
    if (n % 32 != 0) {
        set_error("Tensor size must be a multiple of ggml quantization block size");
        return -1;
    }
    if (n == 0) return 0;
    if (!check_device_ptr(x, "quantize", "input") || !check_device_ptr(out, "quantize", "output")) return -1;
    return launch_q8_0_quantize(x, x_dtype, n / 32, out, (cudaStream_t)stream);
}

GTB_API int gtb_q8_0_append(const void* x, int x_dtype, int64_t B, int64_t Hkv, int64_t n_new, int64_t D, void* cache,
                            int64_t Smax, int32_t* pos, int advance, void* stream) {
    if (!append_args_ok(x_dtype, B, Hkv, n_new, D, Smax)) return -1;
    return append_run(x, x_dtype, B, Hkv, n_new, D, cache, Smax, pos, advance, nullptr, stream);
}

GTB_API int gtb_q8_0_append_rope(const void* x, int x_dtype, int64_t B, int64_t Hkv, int64_t n_new, int64_t D,
                                 void* cache, int64_t Smax, int32_t* pos, int advance, int n_dims, int mode,
                                 float freq_base, float freq_scale, void* stream) {
    if (!append_args_ok(x_dtype, B, Hkv, n_new, D, Smax)) return -1;
    RopeArgs ra;
    if (!rope_args(D, n_dims, mode, freq_base, freq_scale, false, ra)) return -1;
    return append_run(x, x_dtype, B, Hkv, n_new, D, cache, Smax, pos, advance, &ra, stream);
}

GTB_API int gtb_rope(const void* x, int dtype, int64_t B, int64_t H, int64_t S, int64_t D, const int32_t* pos,
                     int64_t n_pos, int n_dims, int mode, float freq_base, float freq_scale, int backward, void* out,
                     void* stream) {
    if (B < 0 || H < 0 || S < 0 || D < 0) {
        set_error("rope: negative size");
        return -1;
    }
    if (dtype != F32 && dtype != F16 && dtype != BF16) {
        set_error("rope: x must be f32, f16 or bf16");
        return -1;
    }
    RopeArgs ra;
    if (!rope_args(D, n_dims, mode, freq_base, freq_scale, backward != 0, ra)) return -1;
    if (n_pos < S) {
        set_errorf("rope: pos must be a 1-D tensor with a position for each of the %lld sequence elements, got %lld",
                   (long long)S, (long long)n_pos);
        return -1;
    }
    const int64_t rows = B * H * S;
    if (rows == 0 || D == 0) return 0;
    if (!check_device_ptr(x, "rope", "x") || !check_device_ptr(out, "rope", "out") || !check_device_ptr(pos, "rope", "pos"))
        return -1;
    return launch_rope(x, dtype, rows, S, D, pos, ra, out, (cudaStream_t)stream);
}

GTB_API int gtb_q8_0_dequantize(const void* blocks, int64_t n_rows, int64_t row_len, void* out, int out_dtype,
                                void* stream) {
    const int64_t n = n_rows * row_len;
    if (n_rows < 0 || row_len < 0 || n % 32 != 0) {
        set_error("dequantize: the value count must be a non-negative multiple of 32");
        return -1;
    }
    if (n == 0) return 0;
    if (!check_device_ptr(blocks, "dequantize", "input") || !check_device_ptr(out, "dequantize", "output")) return -1;
    return launch_q8_0_dequantize(blocks, n / 32, out, out_dtype, (cudaStream_t)stream);
}

GTB_API int gtb_decode_q8_0(const void* q, int q_dtype, const void* k_q8, const void* v_q8, const int32_t* seq_lens,
                            int64_t B, int64_t H, int64_t Hkv, int64_t Smax, int64_t D, float scale, void* out,
                            void* stream) {
    const char* ctx = "flash_decode_q8_0";
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
    if (!check_device_ptr(q, ctx, "q") || !check_device_ptr(out, ctx, "out") ||
        !check_device_ptr(seq_lens, ctx, "seq_lens"))
        return -1;
    if (Smax > 0 && (!check_device_ptr(k_q8, ctx, "k") || !check_device_ptr(v_q8, ctx, "v"))) return -1;
    int dev = 0;
    cudaGetDevice(&dev);
    DecodeArgs a{q, q_dtype, k_q8, v_q8, seq_lens, B, H, Hkv, Smax, D, resolve_scale(scale, D), out,
                 device_status_word(dev)};
    cudaStream_t st = (cudaStream_t)stream;
    const size_t bytes = decode_scratch_bytes(B, H, Hkv, Smax, D);
    keep_pool_memory(dev);
    void* scratch = nullptr;
    if (cuda_failed(cudaMallocAsync(&scratch, bytes, st), "flash_decode_q8_0: scratch allocation")) return -1;
    const int rc = launch_decode_q8_0(a, scratch, st);
    if (scratch) cudaFreeAsync(scratch, st);
    return rc;
}

}  // extern "C"
