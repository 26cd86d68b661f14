/* B200 (sm_100a) scaled-dot-product-attention engine: raw-pointer C ABI.
 *
 * Every entry point takes device pointers, sizes and element strides, and a CUDA stream
 * (cudaStream_t passed as void*; NULL = the legacy default stream). No entry point takes a
 * framework type. All return 0 on success and -1 on failure with a thread-local message in
 * gtb_last_error(), the convention of the reference's gt_last_error (csrc/gt_core.cpp:7-23).
 * Tensors must live on the current CUDA device. There is no CPU path: host pointers are an error.
 *
 * The reference-shaped handle ABI (gt_tensor *, gguf_train.h) is declared in gguf_train_attn.h and
 * is implemented on top of these functions.
 */
#ifndef GTB_ATTN_H
#define GTB_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GTB_API __attribute__((visibility("default")))

/* A strided 4-D view of device memory. data points at element [0,0,0,0]; strides count elements
 * (a stride of 0 broadcasts a size-1 dimension). dtype is a gt_dtype code (gguf_train.h:22-36):
 * 0 = f32, 1 = f16, 2 = bf16, 3 = f64, 9 = bool (masks only). */
typedef struct gtb_tensor4 {
    void *data;
    int64_t shape[4];
    int64_t stride[4];
    int32_t dtype;
} gtb_tensor4;

/* Attention forward.
 * Replaces the body of gt_flash_attention (reference csrc/gt_ops_nn.cpp:2423-2525, declared
 * csrc/gguf_train.h:311) for CUDA tensors.
 *   q (B,H,L,D), k (B,Hkv,S,D), v (B,Hkv,S,Dv); H % Hkv == 0 (query head h reads kv head
 *   h / (H/Hkv)); out (B,H,L,Dv) in q's dtype.
 *   mask: NULL or (B|1,H|1,L|1,S|1), bool (0 = may not attend) or float (added to the scores).
 *   scale <= 0 means 1/sqrt(D). is_causal masks s > l (top-left aligned).
 *   lse: NULL or a (B,H,L) contiguous buffer that receives the natural-log sum of exp(scores)
 *   per row (-inf for a row with no allowed key, whose output is 0): float64 for f64 inputs,
 *   float32 otherwise.
 * Kernel choice: bf16/f16 with D == Dv in {64,128}, unit inner stride, and no mask or a bool / f32 /
 * f16 / bf16 mask, runs the tcgen05/TMA kernel; everything else runs the SIMT kernel (f32/f64
 * accumulate as the input). With a mask, a pre-pass classifies each 128-row x 128-key block of it
 * (every key allowed with nothing added / none allowed / mixed) into a small table from the
 * stream-ordered allocator, and only mixed blocks read the mask entry by entry.
 * For L <= 8192 the tcgen05 kernel runs persistent CTAs that claim work from a 4-byte counter taken
 * from the stream-ordered allocator and zeroed on the stream. */
GTB_API int gtb_sdpa_fwd(const gtb_tensor4 *q, const gtb_tensor4 *k, const gtb_tensor4 *v,
                         const gtb_tensor4 *mask, float scale, int is_causal,
                         gtb_tensor4 *out, void *lse, void *stream);

/* Prefill attention with rotary position embedding fused in: out = attention(rope(q), rope(k), v) and
 * k_rot = rope(k), the rotation that of gtb_rope (backward = 0) with q's positions pos_q (>= L entries)
 * and k's positions pos_k (>= S entries). New export; replaces gt_rope on q and on k (reference
 * csrc/gt_ops_nn.cpp:2409-2421) followed by gt_flash_attention (csrc/gt_ops_nn.cpp:2423-2525).
 *   q (B,H,L,D), k (B,Hkv,S,D) contiguous f32/f16/bf16; v, mask, scale, is_causal, out and lse as in
 *   gtb_sdpa_fwd; k_rot: a contiguous buffer of k's shape and dtype that receives rope(k) (the rotated
 *   keys a caller keeps as its K cache).
 * k is rotated once in HBM (every query tile reads every key tile). q is rotated into a stream-ordered
 * scratch copy first, or, with q_in_kernel != 0 where the tcgen05 kernel runs with no mask and
 * n_dims % 16 == 0, inside the kernel: each Q tile in shared memory once it has landed, from a
 * (cos, sin) table of the L query positions (gtb_last_path "tcgen05+rope"; no q copy, but slower on
 * B200: the next item's Q lands only when the previous item's score products are issued, so the
 * rotation is not hidden). Either way the results equal gtb_rope on q and k followed by gtb_sdpa_fwd
 * bit for bit. */
GTB_API int gtb_sdpa_fwd_rope(const gtb_tensor4 *q, const gtb_tensor4 *k, const gtb_tensor4 *v,
                              const gtb_tensor4 *mask, float scale, int is_causal, const int32_t *pos_q,
                              int64_t n_pos_q, const int32_t *pos_k, int64_t n_pos_k, int n_dims, int mode,
                              float freq_base, float freq_scale, int q_in_kernel, gtb_tensor4 *k_rot,
                              gtb_tensor4 *out, void *lse, void *stream);

/* The forward for q, k, v and out in HOST memory (contiguous, row-major; pinned for the copies to
 * overlap, pageable works with serialised copies), no mask. New export for callers whose tensors live
 * on the host, as the reference's do (gt_flash_attention, csrc/gt_ops_nn.cpp:2423-2525, reads and
 * writes host tensors). The work is cut into `pieces` (<= 0: 8) pieces — whole sequences, or one
 * sequence's kv heads in groups when the batch is smaller than that — and on the calling thread's
 * device piece i's q, k, v are copied in on one internal stream while piece i-1 is attended on
 * `stream` and piece i-2's output is copied out on another; two device slots from the stream-ordered
 * allocator are reused in turn. Asynchronous like the other calls: `out` is complete once `stream`
 * has passed the call. Results are bit for bit those of gtb_sdpa_fwd on the same values. */
GTB_API int gtb_sdpa_fwd_host(const gtb_tensor4 *q, const gtb_tensor4 *k, const gtb_tensor4 *v, float scale,
                              int is_causal, gtb_tensor4 *out, int pieces, void *stream);

/* Attention backward: dq, dk, dv from dout, the forward inputs, the forward output and its lse.
 * Replaces FlashAttentionFn.backward (reference gguf_train/_functions.py:1934-1965), which
 * recomputes the probabilities with a chain of separate ops. dk/dv are summed over the query
 * heads of each kv head, as that function does (:1958-1962). Scratch (rowsum(dout*out) per row;
 * on the tcgen05 path with D = 128 also f32 dq sums, B*H*Lpad*128*4 bytes, Lpad = L rounded up to
 * 128) is taken from the stream-ordered allocator. With D = 128 dq is summed with f32 reductions
 * in global memory, so its bits may differ from run to run in the last place; the environment
 * variable GTB_BWD_SPLIT_DQ=1 (read once per process) selects a separate, deterministic dq kernel,
 * which then runs on an internal per-device stream forked from and joined back into `stream`
 * within the call, so the call's work stays ordered on `stream` (and under stream capture, in the
 * captured graph). */
GTB_API int gtb_sdpa_bwd(const gtb_tensor4 *dout, const gtb_tensor4 *q, const gtb_tensor4 *k,
                         const gtb_tensor4 *v, const gtb_tensor4 *mask, const gtb_tensor4 *out,
                         const void *lse, float scale, int is_causal,
                         gtb_tensor4 *dq, gtb_tensor4 *dk, gtb_tensor4 *dv, void *stream);

/* Options of gtb_sdpa_fwd_ex / gtb_sdpa_bwd_ex (NULL = all zero).
 *   flags: GTB_BWD_DETERMINISTIC (backward): dq from the separate dq kernel, the same bits on every
 *     run (what the environment variable GTB_BWD_SPLIT_DQ=1 selects for every call); needed where a
 *     recomputed backward must repeat exactly, as under activation checkpointing (reference
 *     gguf_train/utils/checkpoint.py:159-222) or torch.use_deterministic_algorithms.
 *   dropout_p in [0, 1): dropout on the attention probabilities, as the reference's
 *     F.scaled_dot_product_attention(dropout_p > 0) (gguf_train/nn/functional.py:750-767): each
 *     probability is dropped with probability dropout_p and the kept ones scaled by 1/(1 - dropout_p);
 *     the softmax normaliser and the lse are those of the undropped probabilities.
 *   dropout_seed: the keep / drop decision of element (b, h, l, s) is a pure function of the seed and
 *     the indices (a counter-based hash, no generator state), so the backward given the forward's
 *     seed reproduces the forward's mask exactly, on any kernel. */
typedef struct gtb_sdpa_opts {
    int32_t flags;
    float dropout_p;
    uint64_t dropout_seed;
} gtb_sdpa_opts;
#define GTB_BWD_DETERMINISTIC 1

/* gtb_sdpa_fwd with options (dropout). Replaces the same reference function as gtb_sdpa_fwd, and the
 * dropout branch of F.scaled_dot_product_attention (gguf_train/nn/functional.py:750-767). */
GTB_API int gtb_sdpa_fwd_ex(const gtb_tensor4 *q, const gtb_tensor4 *k, const gtb_tensor4 *v,
                            const gtb_tensor4 *mask, float scale, int is_causal,
                            gtb_tensor4 *out, void *lse, const gtb_sdpa_opts *opts, void *stream);

/* gtb_sdpa_bwd with options (determinism, dropout: pass the forward's dropout_p and seed).
 * Replaces the same reference function as gtb_sdpa_bwd. */
GTB_API int gtb_sdpa_bwd_ex(const gtb_tensor4 *dout, const gtb_tensor4 *q, const gtb_tensor4 *k,
                            const gtb_tensor4 *v, const gtb_tensor4 *mask, const gtb_tensor4 *out,
                            const void *lse, float scale, int is_causal,
                            gtb_tensor4 *dq, gtb_tensor4 *dk, gtb_tensor4 *dv, const gtb_sdpa_opts *opts,
                            void *stream);

/* Attention weights (probabilities) of a forward that has run, from its lse: the need_weights=True
 * output of MultiheadAttention (reference gguf_train/nn/modules/transformer.py:153-166, which forms
 * them with matmul + softmax). P[b,h,l,s] = exp(scale * q.k + mask - lse[b,h,l]), 0 where masked or
 * (causal) s > l; with opts->dropout_p > 0 and the forward's seed, times keep / (1 - p) with the
 * forward's decisions (the weights the output was formed with). q, k, mask, scale, is_causal as in
 * gtb_sdpa_fwd; lse as gtb_sdpa_fwd wrote it. out: contiguous in q's dtype, (B, 1, L, S) with
 * average != 0 (mean over the H heads) or (B, H, L, S). Any head size up to 256. */
GTB_API int gtb_attn_weights(const gtb_tensor4 *q, const gtb_tensor4 *k, const gtb_tensor4 *mask, const void *lse,
                             float scale, int is_causal, int average, const gtb_sdpa_opts *opts, gtb_tensor4 *out,
                             void *stream);

/* Linear layer on the tensor cores: c (M, N) = a (M, K) b (N, K)^T (+ bias (N)), i.e. F.linear(a, b, bias)
 * for row-major a and b. Replaces gt_linear (reference csrc/gt_ops_nn.cpp:256-335, a ggml_mul_mat graph)
 * for 16-bit operands: dtype bf16 or f16 for a, b, bias (nullable) and c; f32 accumulation.
 * lda, ldb, ldc: elements between consecutive rows, multiples of 8 (16-byte rows); pointers 16-byte
 * aligned; K > 0. MultiheadAttention's projections and their backward products use it. */
GTB_API int gtb_linear(const void *a, const void *b, const void *bias, void *c, int64_t M, int64_t N, int64_t K,
                       int64_t lda, int64_t ldb, int64_t ldc, int dtype, void *stream);

/* Q8_0 quantisation of n_rows rows of row_len values (row_len % 32 == 0) into GGUF Q8_0 blocks
 * (fp16 scale + 32 int8, 34 bytes per 32 values), bit-exact with ggml's reference quantiser.
 * Replaces gt_quantize(t, GT_Q_BASE + 8) (reference csrc/gt_ops_extra.cpp:2002, which goes
 * through a host float buffer in gt_tensor_to_dtype, csrc/gt_core.cpp:792-840).
 * x: contiguous f32/f16/bf16 (x_dtype); out: n_rows * row_len / 32 * 34 bytes. */
GTB_API int gtb_q8_0_quantize(const void *x, int x_dtype, int64_t n_rows, int64_t row_len,
                              void *out, void *stream);

/* KV-cache append on the device (new export; the reference appends by quantising on the host through
 * gt_tensor_to_dtype, csrc/gt_core.cpp:792-840, and concatenating). x: contiguous (B, Hkv, n_new, D)
 * f32/f16/bf16, D % 32 == 0; row t of (b, hk) is quantised exactly as gtb_q8_0_quantize does into
 * row pos[b] + t of cache (B, Hkv, Smax, D/32*34 bytes, the layout gtb_decode_q8_0 reads). pos:
 * device int32 (B), the sequences' current lengths (gtb_decode_q8_0's seq_lens); with advance != 0 a
 * second kernel then adds n_new to every pos[b]. A destination row outside [0, Smax) is skipped and
 * sets the device status word to 60 (read with gtb_device_status). */
GTB_API int gtb_q8_0_append(const void *x, int x_dtype, int64_t B, int64_t Hkv, int64_t n_new, int64_t D,
                            void *cache, int64_t Smax, int32_t *pos, int advance, void *stream);

/* The same with each new row first rotated (RoPE, as gtb_rope with backward = 0) for its cache
 * position pos[b] + t, in f32 before quantising: the rotated keys land in the cache without an
 * intermediate rounding. Replaces gt_rope (csrc/gt_ops_nn.cpp:2409) followed by the quantising append. */
GTB_API int gtb_q8_0_append_rope(const void *x, int x_dtype, int64_t B, int64_t Hkv, int64_t n_new, int64_t D,
                                 void *cache, int64_t Smax, int32_t *pos, int advance, int n_dims, int mode,
                                 float freq_base, float freq_scale, void *stream);

/* Rotary position embedding on the device. Replaces gt_rope / gt_rope_backward (reference
 * csrc/gt_ops_nn.cpp:2409-2421, ggml_rope_ext with ext_factor 0, attn_factor 1): x, out (B, H, S, D)
 * contiguous f32/f16/bf16 (computed in f32, stored in x's type), pos device int32 with n_pos >= S
 * entries (one per sequence element, shared by batch and heads), n_dims even in [2, D], mode 0
 * (pairs 2i, 2i+1) or 2 (NeoX: pairs i, i + n_dims/2), angle of pair i = freq_scale * p *
 * freq_base^(-2i/n_dims) accumulated as ggml's rope cache does; backward != 0 rotates by -angle.
 * Error texts are the reference's. */
GTB_API int gtb_rope(const void *x, int dtype, int64_t B, int64_t H, int64_t S, int64_t D, const int32_t *pos,
                     int64_t n_pos, int n_dims, int mode, float freq_base, float freq_scale, int backward, void *out,
                     void *stream);

/* Q8_0 -> f32/f16/bf16 (out_dtype), x = q * d. Replaces gt_dequantize (csrc/gt_ops_extra.cpp:2006). */
GTB_API int gtb_q8_0_dequantize(const void *blocks, int64_t n_rows, int64_t row_len,
                                void *out, int out_dtype, void *stream);

/* One decode step against a Q8_0 KV cache.
 * Replaces the reference's route for this step: k.dequantize(), v.dequantize(), then
 * F.scaled_dot_product_attention(q, k, v) with q (B,H,1,D) (gguf_train/_tensor.py:1188-1196,
 * csrc/gt_ops_nn.cpp:2423-2525), which has no fused path.
 *   q: (B,H,D) contiguous, q_dtype f16/bf16/f32; k_q8, v_q8: (B,Hkv,Smax,D) as rows of D/32
 *   Q8_0 blocks; seq_lens: int32 (B), sequence b attends its first seq_lens[b] rows (clamped to
 *   [0, Smax]); out: (B,H,D) in q_dtype. D % 32 == 0 and D <= 256.
 * Split-KV: each (b, kv head) is cut into chunks of up to GTB_DECODE_CHUNK rows that run in
 * parallel; a second kernel merges the partial results. The partials, and a small work area
 * (item counter, per-sequence item prefix and item list of the tensor-core kernels), live in scratch taken
 * from the stream-ordered allocator. With D = 128, an f16 q, H/Hkv in {1,2,4,8}, an even Smax
 * and 16-byte aligned q/k/v the step runs on the tensor cores; otherwise on CUDA cores. */
#define GTB_DECODE_CHUNK 2048
GTB_API int gtb_decode_q8_0(const void *q, int q_dtype, const void *k_q8, const void *v_q8,
                            const int32_t *seq_lens, int64_t B, int64_t H, int64_t Hkv, int64_t Smax,
                            int64_t D, float scale, void *out, void *stream);

/* The same decode step as gtb_decode_q8_0, for callers that cannot let the library allocate device
 * memory: a serving runtime whose own allocator owns the GPU, or a loop that must never reach
 * cudaMalloc/cudaFree (they synchronise the device) or grow a memory pool mid-run. It allocates
 * nothing: the split-KV partial results go to a fixed device array of
 * GTB_DECODE_NOALLOC_SCRATCH_BYTES that every GPU loading this library holds until the process
 * exits. A call needs a work area of 8*(B+2) + 8*B*Hkv*ceil(Smax/GTB_DECODE_CHUNK) bytes rounded up
 * to 256, plus B*Hkv*ceil(Smax/GTB_DECODE_CHUNK)*(H/Hkv)*(D+2)*4 bytes of partials when Smax spans
 * more than one chunk; calls needing more than the array holds, or with B, Smax above 2^31 - 1, H
 * above 65535 or D above 256, are rejected with an error before any kernel runs (config 5a, B=64
 * Hkv=8 H=32 D=128 Smax=32768, needs 17.1 MB).
 * The first call on a device sets up the array's device address (call it once before any stream
 * capture). Calls share the array: calls whose kernels overlap on the GPU race. Its kernels report
 * a bounded wait that ran out through gtb_device_status(), like every other kernel.
 * No counterpart in the reference: it is an addition of this engine. */
#define GTB_DECODE_NOALLOC_SCRATCH_BYTES (40u << 20)
GTB_API int gtb_decode_q8_0_noalloc(const void *q, int q_dtype, const void *k_q8, const void *v_q8,
                                    const int32_t *seq_lens, int64_t B, int64_t H, int64_t Hkv,
                                    int64_t Smax, int64_t D, float scale, void *out, void *stream);

/* Log-sum-exp merge of a partial attention result into an accumulator (the combine step of the
 * long-context K/V ring: a causal attention over a sequence sharded across GPUs):
 *   o_acc: groups x rows x D float32, lse_acc: groups x rows float32 (contiguous; start at 0 / -inf),
 *   o_part: element g*part_gstride + r*D + d of part_dtype (f32/f16/bf16), lse_part: g*lse_gstride + r
 *   (natural-log sums as gtb_sdpa_fwd writes them). Rows with lse -inf contribute nothing.
 * No counterpart in the reference, which has no multi-device path. */
GTB_API int gtb_attn_merge(float *o_acc, float *lse_acc, const void *o_part, const float *lse_part,
                           int part_dtype, int64_t groups, int64_t rows, int64_t D, int64_t part_gstride,
                           int64_t lse_gstride, void *stream);

/* Kernel family of the calling thread's last gtb_sdpa_fwd / gtb_sdpa_fwd_rope / gtb_sdpa_bwd call:
 * "tcgen05" (tensor cores, TMA), "tcgen05+rope" (the same with q rotated inside the kernel),
 * "f32_tiled" (fp32 with head size 64, register-blocked on the CUDA cores) or "simt" (one warp per
 * row; "" before the first). Lets a caller or a test see which path a call took. */
GTB_API const char *gtb_last_path(void);

/* Thread-local message of the last failure ("" if none). */
GTB_API const char *gtb_last_error(void);
GTB_API void gtb_clear_error(void);

/* Synchronises the current device and returns (then clears) its kernel status words: 0 = fine,
 * otherwise the code a kernel wrote when one of its bounded waits ran out or a check failed (the
 * first nonzero of the main word and of the fixed word of gtb_decode_q8_0_noalloc). Allocates
 * nothing. Replaces nothing in the reference, which runs no device kernels; its errors follow
 * gt_last_error (csrc/gt_core.cpp:7-23). */
GTB_API int gtb_device_status(void);

/* Failure-detection self-test: launches on `stream` a one-warp kernel that waits on an mbarrier
 * nothing ever arrives at, with the same bounded wait every kernel of this library uses but a limit
 * of `limit_cycles` SM cycles (1000 .. 2^31) instead of about a second. The wait gives up, the
 * kernel records status 90 and returns: gtb_device_status() then reports 90 once, and the device
 * stays usable. No counterpart in the reference, which has no device code. */
GTB_API int gtb_selftest_wait_timeout(int64_t limit_cycles, void *stream);

/* Build-time facts: number of sm_100a kernels compiled in, and a version string. */
GTB_API const char *gtb_version(void);

#ifdef __cplusplus
}
#endif

#endif /* GTB_ATTN_H */
