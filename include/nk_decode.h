/*
 * nk_decode.h — fused non-linear decode kernels of libnkgemm.so (sm_100a), the ops the
 * reference engine runs between its decode linears, with the same bf16 cast points.
 * Conventions as in nk_gemm.h: device pointers, a cudaStream_t, 0 or NK_ERR_* returned
 * before anything is launched, no allocation, no host synchronisation, capture-safe,
 * programmatic dependent launch. The position is a device int64 (as the reference's
 * `cache_position`, engine/engine.py:86), so a step needs no host value per token.
 */
#ifndef NK_DECODE_H
#define NK_DECODE_H

#include "nk_gemm.h"

#ifdef __cplusplus
extern "C" {
#endif

/* RMSNorm with optional residual: if branch != NULL, x <- bf16(x + branch) in place; then
 * out = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * weight), rows x width, contiguous rows,
 * width % 8 == 0 and <= 8192, 16-byte aligned. Replaces norm_out(x, weight, out, eps,
 * residual, summed) at engine/kernels/rmsnorm.py:28-41. */
NK_API int nk_rmsnorm_bf16(void* x, const void* branch, const void* weight, void* out,
                           int rows, int width, float eps, nk_stream_t stream);

/* Per-head RMSNorm of the query and key heads of the packed qkv row, RoPE with the bf16
 * cos/sin tables [capacity, head_dim] at *position (each product rounded, then the sum),
 * query heads to q_out [batch, q_heads * head_dim], key and value heads into the caches at
 * slot *position (strides in elements); cos_table and sin_table hold [capacity, 128]. head_dim
 * must be 128. A *position outside [0, capacity) writes nothing and sets the device error
 * word to NK_ERR_RANGE (nk_device_error). Replaces
 * qk_rope_cache_out(..., fused=True) at engine/kernels/elementwise.py:63-78. */
NK_API int nk_qk_norm_rope_cache_bf16(const void* qkv, int64_t ld_qkv, const void* q_norm,
                                      const void* k_norm, const void* cos_table,
                                      const void* sin_table, const int64_t* position,
                                      void* q_out, void* k_cache, void* v_cache, int batch,
                                      int q_heads, int kv_heads, int head_dim, int capacity,
                                      int64_t cache_batch_stride, int64_t cache_head_stride,
                                      int64_t cache_seq_stride, float eps, nk_stream_t stream);

/* The QKV linear and its consumer in one launch: qkv = x · Wqkvᵀ (nk_gemm_bf16's arithmetic,
 * W the packed [(q_heads + 2 kv_heads) * 128, K] weight) is never stored; each 128-row output
 * tile is one head, and the CTA that finishes a tile applies to it exactly what
 * nk_qk_norm_rope_cache_bf16 applies to the stored bf16 qkv row (same roundings, same sum
 * order, so the same bits): query and key heads RMSNorm + RoPE at *position into q_out and
 * the key cache, value heads into the value cache. Replaces torch.mm(norm, w.qkv, out=qkv)
 * followed by qk_rope_cache_out (engine/kernels/decode.py:54-55,
 * engine/kernels/elementwise.py:63-78); the reference's handoff names this "producer +
 * consumer" fusion as the next step (docs/NEXT_MODEL_HANDOFF.md:93-97).
 *   x: [M, K], row stride ldx; w, ldw, plan, ws, ws_bytes as nk_gemm_bf16, with a
 *   tensor-core plan of decode token tiles (M_max <= 16) in the balanced schedule (split_k 0;
 *   else NK_ERR_PLAN). Other arguments as nk_qk_norm_rope_cache_bf16 (head_dim 128; batch = M).
 *   A *position outside [0, capacity) writes nothing to q_out or the caches and sets the
 *   device error word to NK_ERR_RANGE. */
NK_API int nk_gemm_bf16_qkv_rope_cache(
    const void* x, int64_t ldx, const void* w, int64_t ldw, int M, int N, int K,
    const nk_plan* plan, void* ws, size_t ws_bytes, const void* q_norm, const void* k_norm,
    const void* cos_table, const void* sin_table, const int64_t* position, void* q_out,
    void* k_cache, void* v_cache, int q_heads, int kv_heads, int capacity,
    int64_t cache_batch_stride, int64_t cache_head_stride, int64_t cache_seq_stride, float eps,
    nk_stream_t stream);

/* Workspace bytes of nk_attention_decode_bf16 (fp32 split partials and their max/sum). */
NK_API size_t nk_attention_ws_bytes(int batch, int q_heads, int capacity);

/* Grouped split-KV decode attention over cache slots [0, *position]: out[b, h] =
 * softmax(q[b,h] . K[b, h/G]^T * scale) V[b, h/G] with fp32 scores, softmax and sums,
 * rounded once to bf16. q, out: [batch, q_heads, 128]; caches [batch, kv_heads, capacity,
 * 128] with the given strides (q and caches 8-byte aligned, strides multiples of 4); G =
 * q_heads / kv_heads in {1, 2, 4, 8}. A *position >= capacity attends over the whole cache and
 * a negative one writes nothing; both set the device error word to NK_ERR_RANGE. Replaces
 * attention_out(q, k, v, position, out, partial, lse) at engine/kernels/attention.py:53-62. */
NK_API int nk_attention_decode_bf16(const void* q, const void* k_cache, const void* v_cache,
                                    const int64_t* position, void* out, int batch, int q_heads,
                                    int kv_heads, int head_dim, int capacity,
                                    int64_t cache_batch_stride, int64_t cache_head_stride,
                                    int64_t cache_seq_stride, float scale, void* ws,
                                    size_t ws_bytes, nk_stream_t stream);

/* out[r, i] = bf16( bf16(g / (1 + exp(-g))) * u ) with [g | u] = gate_up[r, 0:2I].
 * Replaces silu_mul_out(packed, out, activation, fused=True) at
 * engine/kernels/elementwise.py:91-101. */
NK_API int nk_silu_mul_bf16(const void* gate_up, void* out, int rows, int intermediate,
                            nk_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* NK_DECODE_H */
