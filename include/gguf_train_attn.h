/* gguf_train-shaped handle ABI of the B200 attention engine.
 *
 * The same opaque-handle conventions as the reference's C ABI (csrc/gguf_train.h), reduced to what
 * the attention path needs: a gt_tensor * is an owned handle to a strided view of host or CUDA
 * storage; functions that produce a tensor return a new handle (NULL on failure), int functions
 * return 0 on success; failures leave a thread-local message in gt_last_error()
 * (csrc/gt_core.cpp:7-23). Dtype and device codes are the reference's (gguf_train.h:22-44).
 *
 * Attention entry points accept CUDA tensors only and run the sm_100a kernels declared in
 * gtb_attn.h; there is no CPU fallback. Reference lines each declaration stands in for are cited.
 */
#ifndef GGUF_TRAIN_ATTN_H
#define GGUF_TRAIN_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GT_API __attribute__((visibility("default")))
#define GT_MAX_DIMS 12

/* gguf_train.h:22-36 */
enum gt_dtype {
    GT_F32 = 0, GT_F16 = 1, GT_BF16 = 2, GT_F64 = 3, GT_I8 = 4, GT_U8 = 5, GT_I16 = 6, GT_I32 = 7,
    GT_I64 = 8, GT_BOOL = 9, GT_Q_BASE = 100
};
#define GT_Q8_0 (GT_Q_BASE + 8) /* GGUF Q8_0, gguf_train/_dtype.py:85 */

/* gguf_train.h:38-44 */
enum gt_device_type { GT_DEV_CPU = 0, GT_DEV_CUDA = 1 };

typedef struct gt_tensor gt_tensor;

/* ---- runtime (gguf_train.h:174-184) */
GT_API void gt_manual_seed(uint64_t seed);                               /* :174, gt_core.cpp:136 */
GT_API int gt_device_count(int device_type);                             /* :177 */
GT_API void gt_device_name(int device_type, int idx, char *buf, int buf_len);          /* :178 */
GT_API void gt_device_memory(int device_type, int idx, size_t *free_bytes, size_t *total_bytes); /* :179 */
GT_API void gt_synchronize(int device_type, int idx);                    /* :180 */
GT_API const char *gt_last_error(void);                                  /* :183 */
GT_API void gt_clear_error(void);                                        /* :184 */

/* ---- tensor lifecycle and metadata (gguf_train.h:189-227) */
GT_API gt_tensor *gt_tensor_empty(int ndim, const int64_t *shape, int dtype, int device_type, int device_index);
GT_API gt_tensor *gt_tensor_from_data(int ndim, const int64_t *shape, int dtype, int device_type, int device_index,
                                      const void *data, size_t nbytes);
/* Wraps memory the caller owns (host or CUDA device memory: the kind is detected), nothing copied.
 * Extends gguf_train.h:196, which wraps host memory only. `token` is informational. */
GT_API gt_tensor *gt_tensor_from_external(int ndim, const int64_t *shape, const int64_t *strides, int dtype,
                                          void *data, uint64_t token);
GT_API gt_tensor *gt_tensor_clone(const gt_tensor *t);
GT_API gt_tensor *gt_tensor_view(const gt_tensor *t, int ndim, const int64_t *shape, const int64_t *strides,
                                 int64_t offset);
GT_API gt_tensor *gt_tensor_contiguous(const gt_tensor *t);
GT_API gt_tensor *gt_tensor_to_dtype(const gt_tensor *t, int dtype);
GT_API gt_tensor *gt_tensor_to_device(const gt_tensor *t, int device_type, int device_index);
GT_API void gt_tensor_free(gt_tensor *t);
GT_API int gt_tensor_ndim(const gt_tensor *t);
GT_API void gt_tensor_shape(const gt_tensor *t, int64_t *out);
GT_API void gt_tensor_strides(const gt_tensor *t, int64_t *out);
GT_API int64_t gt_tensor_offset(const gt_tensor *t);
GT_API int64_t gt_tensor_numel(const gt_tensor *t);
GT_API int gt_tensor_dtype(const gt_tensor *t);
GT_API int gt_tensor_device_type(const gt_tensor *t);
GT_API int gt_tensor_device_index(const gt_tensor *t);
GT_API int gt_tensor_is_contiguous(const gt_tensor *t);
GT_API uint64_t gt_tensor_data_ptr(const gt_tensor *t);
GT_API size_t gt_tensor_nbytes(const gt_tensor *t);
GT_API size_t gt_tensor_elem_size(int dtype);
GT_API int gt_tensor_copy_to_host(const gt_tensor *t, void *dst, size_t dst_bytes);
GT_API int gt_tensor_copy_from_host(gt_tensor *t, const void *src, size_t src_bytes);

/* ---- seeded fills (gguf_train.h:235-240; gt_core.cpp:1182-1298): one global mt19937_64, a fresh
 * distribution per call, values drawn in row-major order on the host */
GT_API int gt_fill_uniform(gt_tensor *t, double low, double high);
GT_API int gt_fill_normal(gt_tensor *t, double mean, double std);
GT_API int gt_fill_bernoulli_prob(gt_tensor *t, double p);

/* ---- attention */
/* gguf_train.h:311 / gt_ops_nn.cpp:2423-2525, bound by gguf_train/_C.py:471-472 as
 * [c_void_p x4, c_float, c_int] -> c_void_p. mask: NULL, (L,S) or (B|1,H|1,L|1,S|1), bool
 * (true = may attend) or float (added). scale <= 0 -> 1/sqrt(D). */
GT_API gt_tensor *gt_flash_attention(const gt_tensor *q, const gt_tensor *k, const gt_tensor *v,
                                     const gt_tensor *mask, float scale, int is_causal);
/* The same forward, also returning the per-row log-sum-exp (B,H,L) the fused backward needs (f64 for
 * f64 inputs, else f32).
 * New export; replaces the saved-inputs-only FlashAttentionFn.forward (_functions.py:1924-1931). */
GT_API gt_tensor *gt_flash_attention_fwd_lse(const gt_tensor *q, const gt_tensor *k, const gt_tensor *v,
                                             const gt_tensor *mask, float scale, int is_causal, gt_tensor **lse_out);
/* New export; replaces the op-by-op FlashAttentionFn.backward (_functions.py:1934-1965). Writes three
 * new handles on success (the multi-output style of gt_layer_norm_backward, gt_ops_nn.cpp:720). */
GT_API int gt_flash_attention_backward(const gt_tensor *grad_out, const gt_tensor *q, const gt_tensor *k,
                                       const gt_tensor *v, const gt_tensor *mask, const gt_tensor *out,
                                       const gt_tensor *lse, float scale, int is_causal, gt_tensor **dq,
                                       gt_tensor **dk, gt_tensor **dv);
/* New export; replaces k.dequantize(), v.dequantize() then gt_flash_attention on q (B,H,1,D)
 * (_tensor.py:1188-1196). k_q8/v_q8: Q8_0 (B,Hkv,Smax,D); seq_lens: I32 (B). Returns (B,H,1,D). */
GT_API gt_tensor *gt_flash_decode_q8_0(const gt_tensor *q, const gt_tensor *k_q8, const gt_tensor *v_q8,
                                       const gt_tensor *seq_lens, float scale);

/* ---- RoPE (the reference's gt_rope / gt_rope_backward, bound at _C.py:467-470, csrc/gt_ops_nn.cpp:
 * 2409-2421): same signature and messages; CUDA tensors, x f32/f16/bf16 (B,H,S,D) or (H,S,D), pos 1-D
 * (converted to int32). Returns a new tensor of x's shape and dtype. */
GT_API gt_tensor *gt_rope(const gt_tensor *x, const gt_tensor *pos, int n_dims, int mode, int n_ctx_orig,
                          float freq_base, float freq_scale);
GT_API gt_tensor *gt_rope_backward(const gt_tensor *grad_out, const gt_tensor *pos, int n_dims, int mode,
                                   int n_ctx_orig, float freq_base, float freq_scale);

/* ---- Q8_0 (gguf_train.h:381-382, gt_ops_extra.cpp:2002-2008): CUDA tensors, rows along the last dim */
GT_API gt_tensor *gt_quantize(const gt_tensor *t, int quant_dtype);
GT_API gt_tensor *gt_dequantize(const gt_tensor *t, int target_dtype);

#ifdef __cplusplus
}
#endif

#endif /* GGUF_TRAIN_ATTN_H */
