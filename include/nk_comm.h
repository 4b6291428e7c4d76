/* nk_comm.h — tensor-parallel all-reduce over NVLink peer memory (libnkgemm.so, sm_100a).
 *
 * In the tensor-parallel decode mode the linears split along K (o_proj at
 * engine/kernels/decode.py:58, down_proj at engine/kernels/decode.py:66) leave every rank with
 * an unrounded fp32 partial of the output; the sum over ranks, rounded once to bf16, is the
 * single-GPU result. nk_allreduce_bf16 does that exchange in one launch per rank: each CTA
 * writes its slice of the local partial into every rank's receive buffer over NVLink, raises
 * a flag there, waits (bounded) for every rank's flag in its own buffer and writes
 * bf16(x_0 + x_1 + ... + x_{world-1}) — ranks added in rank order, so every rank gets the same
 * bits. The reference engine is single-GPU (engine/engine.py:65) and has no collective; this
 * replaces the NCCL all-reduce of the library's own tensor-parallel mode for these sizes.
 *
 * Set-up, once per group: every rank allocates a receive buffer (nk_peer_alloc, zeroed),
 * exports it (nk_ipc_handle), exchanges the handles with the other ranks by any host channel,
 * opens theirs (nk_ipc_open) and fills an nk_peer_group. Every rank must then make the same
 * sequence of nk_allreduce_bf16 calls, each on one stream; calls are CUDA-graph capturable
 * (the kernel keeps its progress counter in the buffer). Plain peer loads and stores only.
 */
#ifndef NK_COMM_H
#define NK_COMM_H

#include <stddef.h>
#include <stdint.h>

#include "nk_gemm.h"

#ifdef __cplusplus
extern "C" {
#endif

#define NK_PEER_MAX_RANKS 8
#define NK_IPC_HANDLE_BYTES 64
#define NK_PEER_MAX_ELEMS (1 << 20) /* largest all-reduce, in fp32 elements */

typedef struct nk_peer_group {
    void* buf[NK_PEER_MAX_RANKS]; /* receive buffer of rank r as mapped in this process */
    int32_t rank;                 /* this process's rank in the group */
    int32_t world;                /* ranks in the group, 2..NK_PEER_MAX_RANKS */
    int32_t max_elems;            /* the size the buffers were made for (nk_peer_buffer_bytes) */
    int32_t reserved;
} nk_peer_group;

/* Bytes of one rank's receive buffer for all-reduces of up to max_elems fp32 elements among
 * world ranks; 0 for arguments out of range. */
NK_API size_t nk_peer_buffer_bytes(int max_elems, int world);

/* cudaMalloc + zero of a receive buffer on the current device, rounded up to whole 2 MiB so it
 * is a memory block of its own (CUDA IPC shares the underlying block, which for small
 * allocations may hold other allocations too); nk_peer_free releases it. */
NK_API int nk_peer_alloc(size_t bytes, void** ptr);
NK_API int nk_peer_free(void* ptr);

/* CUDA IPC handle (NK_IPC_HANDLE_BYTES bytes) of a buffer from nk_peer_alloc, and the mapping
 * of another process's buffer into this one (peer access enabled); nk_ipc_close unmaps it. */
NK_API int nk_ipc_handle(void* ptr, void* handle);
NK_API int nk_ipc_open(const void* handle, void** ptr);
NK_API int nk_ipc_close(void* ptr);

/* out[i] = bf16(x_0[i] + x_1[i] + ... ) over the group's ranks, x the caller's fp32 [n],
 * out bf16 [n] (both 16-byte aligned, n <= g->max_elems, n % 4 == 0). A rank that does not
 * arrive within ~2 s makes the others give up: NK_ERR_TIMEOUT in the device error word
 * (nk_device_error), out not written, and the group unusable until rebuilt. */
NK_API int nk_allreduce_bf16(const float* x, void* out, int n, const nk_peer_group* g,
                             nk_stream_t stream);

/*
 * The K-split linear of a tensor-parallel group fused with its all-reduce, in one launch per
 * rank: y = bf16( sum over ranks r, in rank order, of x_r · W_rᵀ ), where x_r · W_rᵀ is this
 * rank's fp32 partial (the nk_gemm_bf16_f32out product) and the group holds one rank per K
 * slice. As each output tile's fp32 values are final, the CTA that made them stores them into
 * every rank's receive buffer over NVLink (plain peer stores), publishes the tile's call number
 * to every rank, waits (bounded, about 2 s; NK_ERR_TIMEOUT through nk_device_error) for every
 * rank's, and stores the rank-order sum of the tile rounded once to bf16 — the bits
 * nk_gemm_bf16_f32out followed by nk_allreduce_bf16 give, without the second launch or a
 * separate pass over the partial. Replaces the pair mm_f32 + all-reduce of the library's
 * tensor-parallel o_proj / down (the split forms of engine/kernels/decode.py:58,66; the
 * reference itself is single-GPU, engine/engine.py:65).
 *   Arguments as nk_gemm_bf16 (y bf16 [M, N], row stride ldy; ws as nk_ws_bytes(plan)), plus
 *   the group, whose receive buffers must hold M * N elements (max_elems) and which serves no
 *   nk_allreduce_bf16 calls. Plans: the balanced tensor-core schedule (split_k 0, the AUTO
 *   choice for aligned shapes) with token tiles of up to 64 (M_max <= 64) and at most 1024
 *   output tiles; else NK_ERR_PLAN. Every rank makes the same sequence of calls, each on one
 *   stream, with the same plan; calls are CUDA-graph capturable.
 */
NK_API int nk_gemm_bf16_allreduce(const void* x, int64_t ldx, const void* w, int64_t ldw,
                                  void* y, int64_t ldy, int M, int N, int K,
                                  const nk_plan* plan, void* ws, size_t ws_bytes,
                                  const nk_peer_group* g, nk_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* NK_COMM_H */
