/*
 * nk_gemm.h — C ABI of the B200 (sm_100a) decode-GEMM library `libnkgemm.so`.
 *
 * The operation exported here is the bf16 decode linear (with its greedy-head form, which
 * also returns each row's argmax, and its fp32-output and workspace-free forms)
 *
 *     y[M, N] = bf16_rne( sum_k  f32(x[M, k]) * f32(W[N, k]) )      (fp32 accumulation)
 *
 * with W a row-major [N, K] weight whose rows are K-contiguous. This is exactly the call the
 * reference engine makes at every decode linear:
 *
 *     torch.mm(x, W.t(), out=y)
 *       engine/kernels/decode.py:54   (QKV:     norm     · Wqkvᵀ,    W = cat(q, k, v))
 *       engine/kernels/decode.py:58   (o_proj:  attn_flat · Woᵀ)
 *       engine/kernels/decode.py:64   (gate_up: norm     · [Wg; Wu]ᵀ)
 *       engine/kernels/decode.py:66   (down:    product  · Wdᵀ)
 *       engine/engine.py:114          (lm_head: norm     · Eᵀ)
 *
 * where `W.t()` is the transposed view built in engine/kernels/weights.py:12-13,24-25 and
 * engine/engine.py:70. The library reads that same storage: `w` below is the data pointer
 * of the row-major [N, K] weight (the storage behind the `.t()` view), `ldw` its row stride.
 *
 * Conventions
 *   - Every pointer is a CUDA device pointer except `plan` (host). No function allocates
 *     device memory, synchronizes the host, or touches any stream other than `stream`.
 *   - Functions return 0 (NK_OK) or a negative NK_ERR_* code and launch nothing on error.
 *   - `stream` is a cudaStream_t (0 = legacy default stream).
 *   - Launches are capture-safe: a sequence of nk_gemm_bf16 calls may be recorded into a
 *     CUDA graph and replayed, provided the workspace stays the one passed at capture.
 *   - Calls that share a workspace must be ordered (same stream, or joined by events): the
 *     split-K tickets and partials in the workspace belong to one call at a time.
 */
#ifndef NK_GEMM_H
#define NK_GEMM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define NK_API __attribute__((visibility("default")))
#else
#define NK_API
#endif

typedef struct CUstream_st* nk_stream_t; /* identical to cudaStream_t */

/* Status codes. */
#define NK_OK              0
#define NK_ERR_SHAPE      -1  /* M, N or K out of range, or M > plan->M_max            */
#define NK_ERR_ALIGN      -2  /* pointer or leading dimension violates the plan's layout  */
#define NK_ERR_WORKSPACE  -3  /* workspace missing or smaller than nk_ws_bytes(plan)     */
#define NK_ERR_SPLIT      -4  /* split_k outside [1, 16] or larger than K allows          */
#define NK_ERR_PLAN       -5  /* plan is NULL, corrupt, or made for another (N, K)        */
#define NK_ERR_CUDA       -6  /* a CUDA runtime call failed (launch, attribute, symbol)   */
#define NK_ERR_DEVICE     -7  /* current device is not sm_100 (B200 class)                */
#define NK_ERR_TIMEOUT    -8  /* a kernel's bounded wait expired (read by nk_device_error) */
#define NK_ERR_ARG        -9  /* any other invalid argument                               */
#define NK_ERR_RANGE      -10 /* a device-side decode position outside its cache (read by
                                  nk_device_error)                                       */

/* Kernel families a plan can select. */
#define NK_KIND_AUTO     0
#define NK_KIND_GEMV     1  /* CUDA-core weight-streaming GEMV, 128-bit loads, M <= 16        */
#define NK_KIND_TC       2  /* tcgen05/TMEM swap-AB tensor-core GEMM with a TMA smem ring     */
#define NK_KIND_GENERIC  3  /* unaligned / ragged fallback (still on the GPU), any layout    */

#define NK_MAX_SPLIT 16

/* A launch plan: chosen once per (M_max, N, K) at prepare time, never inside a graph. */
typedef struct nk_plan {
    int32_t magic;       /* NK_PLAN_MAGIC once made                                    */
    int32_t M_max;       /* largest M this plan accepts                                */
    int32_t N, K;
    int32_t kind;        /* NK_KIND_*                                                  */
    int32_t split_k;     /* K slices per tile (0 in the tensor-core family's balanced
                            schedule, where `segments` bounds the CTAs per tile)       */
    int32_t k_slice;     /* K elements per slice (multiple of the kernel's K step)     */
    int32_t tile_n;      /* weight rows per CTA                                        */
    int32_t tile_m;      /* token rows per CTA (padded M)                              */
    int32_t stages;      /* shared-memory pipeline depth (tensor-core kernel)          */
    int32_t n_tiles;     /* ceil(N / tile_n)                                           */
    int32_t m_tiles;     /* ceil(M_max / tile_m)                                       */
    int32_t grid;        /* CTAs launched (tensor-core family: persistent grid of the
                            balanced schedule)                                         */
    int32_t segments;    /* most CTAs sharing one output tile (1 = no partial sums)    */
    int32_t k_step;      /* K elements per pipeline step (tensor-core family's unit)   */
    int32_t slices;      /* tensor-core family, 16-token tile, split_k 0: K slices per
                            tile of the tile-aligned schedule (tiles x slices CTAs, two
                            per SM, one wave) that launches use when all of it is
                            resident; 0 = the balanced schedule only                   */
} nk_plan;

#define NK_PLAN_MAGIC 0x4E4B4731 /* "NKG1" */

/*
 * Choose kernel family, split-K factor and tiles for y[M<=M_max, N] = x · Wᵀ with W [N, K].
 *   split_k: 0 = choose automatically, else 1..16.   kind: NK_KIND_AUTO or a forced family.
 * Replaces the implicit per-call heuristic of torch.mm/cuBLAS at the call sites listed above.
 */
NK_API int nk_plan_make(nk_plan* plan, int M_max, int N, int K, int split_k, int kind);

/* Bytes of device workspace nk_gemm_bf16 needs for this plan: a fixed 288 KiB region (256
 * KiB of split-K tickets, then 32 KiB for nk_gemm_bf16_argmax's running maxima) followed by
 * the partial sums (8 bytes per partial value for the tensor-core family, 4 for the GEMV
 * family). 0 when the plan needs none (no tile is split). One workspace (zeroed once by
 * nk_ws_init) can serve any sequence of ordered calls whatever their plans, if it is as large
 * as the largest plan needs: every plan uses the same fixed regions and the kernels leave
 * them, and the partial slots they read, zeroed. Plans with split_k > 1 and more than 65536
 * output tiles are refused (NK_ERR_SPLIT). */
NK_API size_t nk_ws_bytes(const nk_plan* plan);

/* Zero a workspace once before its first use (the kernels keep it zeroed afterwards). After
 * nk_device_error has reported NK_ERR_TIMEOUT, zero it again: a launch that stopped on an
 * expired wait may have left split-K state behind.
 * Asynchronous on `stream`. */
NK_API int nk_ws_init(void* ws, size_t ws_bytes, nk_stream_t stream);

/*
 * y = x · Wᵀ  (bf16 in, fp32 accumulate, bf16 out, round-to-nearest-even).
 *   x: [M, K] with row stride ldx (elements)      — `a` of torch.mm(a, b, out=c)
 *   w: [N, K] with row stride ldw (elements)      — storage of `b` = W.t(), strides (1, ldw)
 *   y: [M, N] with row stride ldy (elements)      — `c`
 * Replaces torch.mm(x, W.t(), out=y) at engine/kernels/decode.py:54,58,64,66 and
 * engine/engine.py:114.
 */
NK_API int nk_gemm_bf16(const void* x, int64_t ldx,
                 const void* w, int64_t ldw,
                 void* y, int64_t ldy,
                 int M, int N, int K,
                 const nk_plan* plan, void* ws, size_t ws_bytes,
                 nk_stream_t stream);

/*
 * y = x · Wᵀ exactly as nk_gemm_bf16, for callers that cannot allocate device memory, so
 * cannot hand the library a workspace: an operator inside a host framework that owns every
 * device allocation and passes it only its inputs and outputs, a process whose device-memory
 * budget is fixed at start-up, or a latency-critical path that avoids cudaMalloc because a
 * device allocation serializes work in flight on other streams. No counterpart in the
 * reference: its torch.mm call sites let the library allocate as it pleases.
 *
 * The split-K scratch comes from an array of NK_STATIC_SCRATCH_BYTES (8 MiB) compiled into
 * the library, which every GPU that loads it holds until the process exits. Only plans of
 * the tensor-core family (NK_KIND_TC, what AUTO plans choose for aligned shapes) are taken
 * (else NK_ERR_PLAN); a plan whose nk_ws_bytes() exceeds the array is refused with
 * NK_ERR_WORKSPACE. Nothing is allocated. The first call on each device (with that device
 * current) looks up the array's device address, so make it before any stream capture on that
 * device; the address is kept for the life of the process (a cudaDeviceReset that unloads the
 * library is not supported here). `stream` must belong to the current device (else
 * NK_ERR_DEVICE). All calls on a device share the array and it keeps the last call's
 * contents: each call first clears the tickets and partial slots its plan uses, and calls that
 * overlap on the GPU race — order them (one stream, or streams joined by events). A call
 * refused for its arguments writes nothing.
 */
#define NK_STATIC_SCRATCH_BYTES (8u << 20)
NK_API int nk_gemm_bf16_static(const void* x, int64_t ldx,
                               const void* w, int64_t ldw,
                               void* y, int64_t ldy,
                               int M, int N, int K,
                               const nk_plan* plan, nk_stream_t stream);

/*
 * y32 = x · Wᵀ with fp32 accumulation and NO rounding: the fp32 partial of a linear split
 * along K across tensor-parallel ranks (o_proj, down), summed across ranks (all-reduce) and
 * rounded to bf16 once, so the sharded linear keeps the single-GPU rounding. Otherwise as
 * nk_gemm_bf16 (same plan, workspace and stream rules); y32 is [M, N] fp32, row stride ldy,
 * 4-byte aligned. No single call site in the reference: it is the split form of
 * torch.mm(x, W.t(), out=y) at engine/kernels/decode.py:58,66 for a K-split weight.
 */
NK_API int nk_gemm_bf16_f32out(const void* x, int64_t ldx,
                               const void* w, int64_t ldw,
                               float* y32, int64_t ldy,
                               int M, int N, int K,
                               const nk_plan* plan, void* ws, size_t ws_bytes,
                               nk_stream_t stream);

/*
 * Greedy head: y = x · Wᵀ as nk_gemm_bf16 and, per token m < M, idx[m] = the index n of the
 * largest bf16 y[m, n], the lowest such n on ties (a NaN counts as the largest, -0 equals +0)
 * — torch.argmax over the bf16 logits, fused into the linear's epilogue. Replaces
 * engine/engine.py:114-116 (lm_head linear, then argmax(dim=-1)); lm_head + lowest-index
 * argmax fusion is the reference's own next step for this path. y may be NULL: then no
 * logits are written (ldy is ignored). best, if not NULL, receives each token's largest
 * value (bf16, [M]). idx: int64 [M], 8-byte aligned.
 * Tensor-core plans of at most 255 tokens only (else NK_ERR_PLAN / NK_ERR_SHAPE; 0 from
 * nk_gemm_argmax_ws_bytes). The workspace is the one nk_gemm_bf16 uses, at least
 * nk_gemm_argmax_ws_bytes(plan) long — never 0, as the running maxima live in its fixed
 * region — zeroed once by nk_ws_init; the kernel leaves it zeroed, so ordered calls of both
 * entry points may share it.
 */
NK_API size_t nk_gemm_argmax_ws_bytes(const nk_plan* plan);
NK_API int nk_gemm_bf16_argmax(const void* x, int64_t ldx,
                               const void* w, int64_t ldw,
                               void* y, int64_t ldy,
                               int64_t* idx, void* best,
                               int M, int N, int K,
                               const nk_plan* plan, void* ws, size_t ws_bytes,
                               nk_stream_t stream);

/* Read and clear the device error word that bounded waits set on timeout (synchronizes
 * `stream`). Writes NK_OK or NK_ERR_TIMEOUT to *status. */
NK_API int nk_device_error(nk_stream_t stream, int* status);

/* Failure-detection tests only; no counterpart in the reference (its torch.mm has no
 * device-side wait). The next tensor-core launch (any entry point above) runs with the
 * rank-1 CTA of output tile `tile` keeping its fp32 partial to itself, so the CTA that
 * finishes that tile waits for it until its bounded wait expires (about 2 s): the tile's
 * outputs are not written, the launch returns, nk_device_error then reports NK_ERR_TIMEOUT,
 * and the workspace needs nk_ws_init before its next use. The request is consumed by that
 * one launch (a tile with a single CTA, a forced split_k grid larger than one resident wave,
 * or -1 withhold nothing). Nothing faults or hangs. */
NK_API int nk_test_withhold_partial(int tile);

/* Human-readable text for a status code (static storage). */
NK_API const char* nk_status_string(int status);

/* Library version, e.g. 0x000100 for 0.1.0. */
NK_API int nk_version(void);

#ifdef __cplusplus
}
#endif
#endif /* NK_GEMM_H */
