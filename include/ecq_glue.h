/*
 * ecq_glue.h -- element-wise steps of a batch-1 transformer decode step that
 * sit between libecq's fused GEMVs (no counterpart in the reference, whose
 * model glue lives in the out-of-tree MLX fork; the model structure it
 * drives is experiments/real_model_test.py:18-113). fp16 in/out, fp32
 * arithmetic; every launch takes a cudaStream_t (as void*) and returns 0 or
 * a negative error.
 */
#ifndef ECQ_GLUE_H
#define ECQ_GLUE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* h_out = h + d (rounded to fp16; skipped when d is NULL) and
 * y = fp16(h_out * rsqrt(mean(h_out^2) + eps)) * w, for `rows` rows of n
 * (n <= 12256): one CTA per row, or for a single row of n >= 1024 one
 * thread-block cluster of 8 CTAs that add their partial sums of squares in
 * rank order through distributed shared memory. h_out may be h. */
int32_t ecq_add_rmsnorm_f16(const void *h, const void *d, const void *w, void *h_out, void *y, int32_t rows,
                            int32_t n, float eps, void *stream);

/* Rotary embedding of q (in place) and k for one position (angles cos_t /
 * sin_t, dim/2 each, pairs (2i, 2i+1)), storing the rotated k and v into the
 * KV cache slots k_cache / v_cache (head h at h * cache_head_stride
 * elements). q, k, v are [heads, dim]. */
int32_t ecq_rope_kv_f16(void *q, const void *k, const void *v, void *k_cache, void *v_cache, const void *cos_t,
                        const void *sin_t, int32_t heads, int32_t dim, int64_t cache_head_stride, void *stream);

/* m[r, c] = fp16(silu(gate[r, c])) * up[r, c] with gate_up = [rows, 2f]
 * (gate in the first f columns, up in the next f). */
int32_t ecq_silu_mul_f16(const void *gate_up, void *m, int32_t f, int32_t rows, void *stream);

/* Batch-1 decode attention: out[h] = softmax(q[h] . K[h]^T / sqrt(head_dim))
 * . V[h] for heads h < heads over keys t < keys, fp16 in/out, fp32 softmax
 * and accumulation (flash-decoding: the keys split over `splits` CTAs per
 * head, the last CTA of each head merging the partial results in split
 * order, so the result is deterministic). q and out are [heads, head_dim];
 * key t of head h is at k_cache + h * head_stride + t * head_dim (same for
 * v_cache). head_dim must be 128; pointers 8-byte aligned. The workspace
 * (ecq_decode_attention_workspace_bytes) must be zero-filled once; each call
 * leaves its counters zero again. ecq_decode_attention_splits gives a split
 * count that puts about two CTAs per SM, at least 32 keys per split and at
 * most 128 splits (the merge's limit; more returns ECQ_ERR_ARG). */
int64_t ecq_decode_attention_workspace_bytes(int32_t heads, int32_t splits);
int32_t ecq_decode_attention_splits(int32_t heads, int32_t keys);
int32_t ecq_decode_attention_f16(const void *q, const void *k_cache, const void *v_cache, void *out, int32_t heads,
                                 int32_t head_dim, int32_t keys, int64_t head_stride, int32_t splits, void *workspace,
                                 int64_t workspace_bytes, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* ECQ_GLUE_H */
