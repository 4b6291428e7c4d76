// C ABI of libnkgemm.so (declared in include/nk_gemm.h): plan selection, host-side
// validation and dispatch to the kernel families.
//
// The entry point nk_gemm_bf16 stands in for torch.mm(x, W.t(), out=y) at
// engine/kernels/decode.py:54,58,64,66 and engine/engine.py:114. Like the reference's Python
// wrappers (engine/kernels/decode.py:22,24; engine/kernels/rmsnorm.py:36), it rejects a bad
// configuration before launching anything; it never allocates and never synchronizes.
#include <string.h>

#include <atomic>

#include "nk_common.cuh"

namespace nk {

// Output tile whose rank-1 partial the next tensor-core launch withholds (-1 = none); set by
// nk_test_withhold_partial and consumed by that launch.
static std::atomic<int> g_withhold_tile{-1};

// Per-device "is this an sm_100 part" cache (checked once per device, then free).
static int g_device_ok[64];  // 0 = unknown, 1 = ok, -1 = not sm_100

static int check_device() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return NK_ERR_CUDA;
    if (dev < 0 || dev >= 64) return NK_ERR_DEVICE;
    if (g_device_ok[dev] == 0) {
        int major = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
            return NK_ERR_CUDA;
        g_device_ok[dev] = (major == 10) ? 1 : -1;
    }
    return g_device_ok[dev] == 1 ? NK_OK : NK_ERR_DEVICE;
}

static bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }
static bool aligned2(const void* p) { return ((uintptr_t)p & 1u) == 0; }

static int ceil_div(int a, int b) { return (a + b - 1) / b; }

// Split-K choice for the GEMV family: enough CTAs for about eight resident 256-thread CTAs
// on each of the 148 SMs, slices of at least two warp K-steps, at most NK_MAX_SPLIT slices.
static int gemv_auto_split(int tiles, int K) {
    const int target = kNumSMs * 8;
    int split = ceil_div(target, tiles);
    const int max_split = K / (2 * kGemvKStep);
    if (split > max_split) split = max_split;
    if (split > NK_MAX_SPLIT) split = NK_MAX_SPLIT;
    if (split < 1) split = 1;
    return split;
}

// Family choice for AUTO plans, from timings on B200 of whole decode steps (graph-replayed
// chains of the step's linears with weights far beyond L2). Past M = 1 the CUDA-core GEMV
// needs M FMAs per weight element and the tensor-core family wins every shape. At M = 1 the
// GEMV alone is a few percent faster on the widest weights, but in a chain of decode linears
// the persistent tensor-core kernel overlaps each launch with the previous one (programmatic
// dependent launch into a one-wave grid) and the all-tensor-core step is faster, so AUTO
// keeps the GEMV for explicit requests only.
static bool gemv_preferred(int M_max, int N, int K) {
    (void)M_max; (void)N; (void)K;
    return false;
}

// Round the slice to whole warp K-steps and drop slices that would be empty.
static void set_slices(nk_plan* p, int split, int step) {
    int ks = ceil_div(p->K, split);
    ks = ceil_div(ks, step) * step;
    p->k_slice = ks;
    p->split_k = ceil_div(p->K, ks);
}

}  // namespace nk

using namespace nk;

extern "C" int nk_plan_make(nk_plan* p, int M_max, int N, int K, int split_k, int kind) {
    if (!p) return NK_ERR_ARG;
    memset(p, 0, sizeof(*p));
    if (M_max < 1 || N < 1 || K < 1 || M_max > (1 << 20) || N > (1 << 28) || K > (1 << 28))
        return NK_ERR_SHAPE;
    if (split_k < 0 || split_k > NK_MAX_SPLIT) return NK_ERR_SPLIT;
    if (kind < NK_KIND_AUTO || kind > NK_KIND_GENERIC) return NK_ERR_ARG;

    if (kind == NK_KIND_AUTO) {
        if (K % 8 != 0) kind = NK_KIND_GENERIC;
        else kind = gemv_preferred(M_max, N, K) ? NK_KIND_GEMV : NK_KIND_TC;
    }
    if (kind != NK_KIND_GENERIC && K % 8 != 0) return NK_ERR_ALIGN;

    p->M_max = M_max;
    p->N = N;
    p->K = K;
    p->kind = kind;
    if (kind == NK_KIND_GENERIC) {
        if (split_k > 1) return NK_ERR_SPLIT;
        p->split_k = 1;
        p->k_slice = K;
        p->tile_n = kGenericRows;
        p->tile_m = kGenericTokens;
    } else if (kind == NK_KIND_TC) {
        // Persistent schedule (nk_tc.cu): one wave of CTAs, each streaming an equal run of
        // (tile, K block) units; a forced split_k instead gives each tile split_k CTAs.
        p->tile_m = tc_token_tile(M_max);
        p->tile_n = kTcRowsPerCta;
        p->stages = tc_stages(p->tile_m);
        p->k_step = tc_kstep(p->tile_m);
        const int KB = ceil_div(K, p->k_step);
        const int64_t T = (int64_t)ceil_div(N, p->tile_n) * ceil_div(M_max, p->tile_m);
        const int64_t U = T * KB;
        if (split_k > 0) {
            const int split = split_k < KB ? split_k : KB;
            if (T * split > (int64_t)1 << 30) return NK_ERR_SHAPE;
            p->split_k = split;
            p->grid = (int32_t)(T * split);
            p->segments = split;
            p->k_slice = ceil_div(KB, split) * p->k_step;
        } else {
            // A second CTA per SM pays only while each CTA keeps enough units: below that the
            // extra split tiles cost more finishing work, and a full SM leaves no room for
            // the next launch's prologue and first weight loads to overlap this one's tail.
            int per_sm = tc_ctas_per_sm(p->tile_m);
            if (per_sm > 1 && U < (int64_t)kNumSMs * per_sm * NK_TC_DUAL_MIN_UNITS) per_sm = 1;
            const int64_t slots = (int64_t)kNumSMs * per_sm;
            const int64_t G = U < slots ? U : slots;
            const int64_t q = U / G;  // units per CTA (the last ones may have one more)
            const int64_t seg = 1 + (KB - 1 + q - 1) / q;
            p->split_k = 0;
            p->grid = (int32_t)G;
            p->segments = (int32_t)(seg < G ? seg : G);
            p->k_slice = (int32_t)(q * p->k_step);
            // Tile-aligned schedule for decode launches with few output tiles: `slices` CTAs
            // per tile, one K slice each, two per SM, the whole grid resident. Every CTA then
            // holds one segment, and two CTAs per SM keep twice the loads in flight. Measured
            // on B200 (Qwen3-8B and Qwen3-0.6B decode linears, M = 1..16, 20 chained launches,
            // every forced split 3..12 against the balanced schedule): 5-20 % faster where it
            // gives at least four slices; more than 9 slices (7 above M = 8, whose partials
            // take the counted protocol) or fewer than two K steps per slice lose it again.
            // Only the 16-token tile (the one measured).
            const int full = tc_ctas_per_sm(p->tile_m);
            int64_t slices = (NK_TC_ALIGNED && p->tile_m == 16 && full > 1)
                                 ? ((int64_t)kNumSMs * full) / T : 0;
            const int64_t cap = M_max <= 8 ? 9 : 7;
            if (slices > cap) slices = cap;
            if (slices > KB / 2) slices = KB / 2;
            p->slices = slices >= NK_TC_MIN_SLICES ? (int32_t)slices : 0;
            if (p->slices > p->segments) p->segments = p->slices;
        }
    } else {  // NK_KIND_GEMV
        p->tile_m = gemv_token_tile(M_max);
        p->tile_n = gemv_rows_per_cta(p->tile_m);
        const int tiles = ceil_div(N, p->tile_n) * ceil_div(M_max, p->tile_m);
        const int split = split_k ? split_k : gemv_auto_split(tiles, K);
        set_slices(p, split, kGemvKStep);
    }
    p->n_tiles = ceil_div(N, p->tile_n);
    p->m_tiles = ceil_div(M_max, p->tile_m);
    if (p->kind == NK_KIND_GEMV || p->kind == NK_KIND_GENERIC) {
        p->grid = p->n_tiles * p->split_k * p->m_tiles;
        p->segments = p->split_k;
        p->k_step = p->kind == NK_KIND_GEMV ? kGemvKStep : 32;
    }
    if (p->segments > 1 && (size_t)p->n_tiles * (size_t)p->m_tiles > kTicketsMax) {
        memset(p, 0, sizeof(*p));
        return NK_ERR_SPLIT;  // more output tiles than the workspace's ticket region holds
    }
    p->magic = NK_PLAN_MAGIC;
    return NK_OK;
}

extern "C" size_t nk_ws_bytes(const nk_plan* p) {
    if (!p || p->magic != NK_PLAN_MAGIC) return 0;
    return ws_layout(*p).total;
}

extern "C" int nk_ws_init(void* ws, size_t ws_bytes, nk_stream_t stream) {
    if (ws_bytes == 0) return NK_OK;
    if (!ws) return NK_ERR_WORKSPACE;
    return cudaMemsetAsync(ws, 0, ws_bytes, (cudaStream_t)stream) == cudaSuccess ? NK_OK
                                                                                 : NK_ERR_CUDA;
}

namespace nk {

// Outputs of the greedy head (nk_gemm_bf16_argmax).
struct AmaxOut {
    int64_t* idx;
    void* best;
};

// The consumer of the fused QKV epilogue (nk_gemm_bf16_qkv_rope_cache), validated.
struct QkvIn {
    const void *q_norm, *k_norm, *cos_t, *sin_t;
    const int64_t* position;
    void *q_out, *k_cache, *v_cache;
    int hq, hkv, capacity;
    int64_t cb, ch, cs;
    float eps;
};

// The tensor-parallel group of the fused all-reduce (nk_gemm_bf16_allreduce), validated.
struct ArIn {
    void* buf[NK_PEER_MAX_RANKS_INTERNAL];
    int rank, world, max_elems;
};

// Every check of a linear's arguments that involves neither the workspace nor the device
// (plan, shape, pointers, alignment). Returns NK_OK or the NK_ERR_* the entry point reports.
static int gemm_validate(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* y,
                         int64_t ldy, bool y_f32, int M, int N, int K, const nk_plan* p,
                         const AmaxOut* amax, bool y_optional = false);

// Shared body of nk_gemm_bf16 (bf16 y), nk_gemm_bf16_f32out (fp32 y) and
// nk_gemm_bf16_argmax (bf16 y or none, plus the per-token argmax).
static int gemm_impl(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y,
                     int64_t ldy, bool y_f32, int M, int N, int K, const nk_plan* p, void* ws,
                     size_t ws_bytes, nk_stream_t stream, const AmaxOut* amax = nullptr,
                     const ArIn* ar = nullptr, const QkvIn* qk = nullptr);

}  // namespace nk

extern "C" int nk_gemm_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y,
                            int64_t ldy, int M, int N, int K, const nk_plan* p, void* ws,
                            size_t ws_bytes, nk_stream_t stream) {
    return gemm_impl(x, ldx, w, ldw, y, ldy, false, M, N, K, p, ws, ws_bytes, stream);
}

extern "C" int nk_gemm_bf16_f32out(const void* x, int64_t ldx, const void* w, int64_t ldw,
                                   float* y, int64_t ldy, int M, int N, int K, const nk_plan* p,
                                   void* ws, size_t ws_bytes, nk_stream_t stream) {
    return gemm_impl(x, ldx, w, ldw, y, ldy, true, M, N, K, p, ws, ws_bytes, stream);
}

static int nk::gemm_validate(const void* x, int64_t ldx, const void* w, int64_t ldw,
                             const void* y, int64_t ldy, bool y_f32, int M, int N, int K,
                             const nk_plan* p, const AmaxOut* amax, bool y_optional) {
    if (!p || p->magic != NK_PLAN_MAGIC) return NK_ERR_PLAN;
    if (p->N != N || p->K != K) return NK_ERR_PLAN;
    if (M < 1 || M > p->M_max) return NK_ERR_SHAPE;
    if (!x || !w || (!y && !amax && !y_optional)) return NK_ERR_ARG;
    if (ldx < K || ldw < K || (y && ldy < N)) return NK_ERR_SHAPE;
    if (amax) {
        if (p->kind != NK_KIND_TC) return NK_ERR_PLAN;  // the tensor-core family only
        if (!amax->idx) return NK_ERR_ARG;
        if (((uintptr_t)amax->idx & 7u) || ((uintptr_t)amax->best & 1u)) return NK_ERR_ALIGN;
        if (p->M_max > kAmaxMaxTokens) return NK_ERR_SHAPE;
    }
    if (!aligned2(x) || !aligned2(w) || !aligned2(y)) return NK_ERR_ALIGN;
    if (y_f32 && ((uintptr_t)y & 3u) != 0) return NK_ERR_ALIGN;
    if (p->kind == NK_KIND_GEMV || p->kind == NK_KIND_TC) {
        if (!aligned16(x) || !aligned16(w) || (ldx % 8) != 0 || (ldw % 8) != 0)
            return NK_ERR_ALIGN;
    }
    return NK_OK;
}

static int nk::gemm_impl(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y,
                         int64_t ldy, bool y_f32, int M, int N, int K, const nk_plan* p,
                         void* ws, size_t ws_bytes, nk_stream_t stream, const AmaxOut* amax,
                         const ArIn* ar, const QkvIn* qk) {
    const int valid = gemm_validate(x, ldx, w, ldw, y, ldy, y_f32, M, N, K, p, amax, qk != nullptr);
    if (valid != NK_OK) return valid;
    if (amax) {
        if (!ws || ws_bytes < amax_ws_bytes(*p)) return NK_ERR_WORKSPACE;
        if (((uintptr_t)ws & 255u) != 0) return NK_ERR_ALIGN;
    }
    const WsLayout L = ws_layout(*p);
    if (L.total > 0) {
        if (!ws || ws_bytes < L.total) return NK_ERR_WORKSPACE;
        if (((uintptr_t)ws & 255u) != 0) return NK_ERR_ALIGN;
    }
    const int dev_status = check_device();
    if (dev_status != NK_OK) return dev_status;

    GemmArgs a;
    a.x = static_cast<const __nv_bfloat16*>(x); a.ldx = ldx;
    a.w = static_cast<const __nv_bfloat16*>(w); a.ldw = ldw;
    a.y = y_f32 ? nullptr : static_cast<__nv_bfloat16*>(y);
    a.y32 = y_f32 ? static_cast<float*>(y) : nullptr;
    a.ldy = ldy;
    a.M = M; a.N = N; a.K = K;
    a.part = L.total ? reinterpret_cast<float*>(static_cast<char*>(ws) + L.part_offset) : nullptr;
    a.tickets = L.total ? static_cast<unsigned*>(ws) : nullptr;
    a.amax_keys = nullptr;
    a.amax_done = nullptr;
    a.amax_idx = nullptr;
    a.amax_best = nullptr;
    a.withhold_tile = p->kind == NK_KIND_TC ? g_withhold_tile.exchange(-1) : -1;
    for (int r = 0; r < NK_PEER_MAX_RANKS_INTERNAL; ++r)
        a.ar_buf[r] = ar && r < ar->world ? static_cast<uint8_t*>(ar->buf[r]) : nullptr;
    a.ar_rank = ar ? ar->rank : 0;
    a.ar_world = ar ? ar->world : 0;
    a.ar_max_elems = ar ? ar->max_elems : 0;
    a.qk_qnorm = qk ? static_cast<const __nv_bfloat16*>(qk->q_norm) : nullptr;
    a.qk_knorm = qk ? static_cast<const __nv_bfloat16*>(qk->k_norm) : nullptr;
    a.qk_cos = qk ? static_cast<const __nv_bfloat16*>(qk->cos_t) : nullptr;
    a.qk_sin = qk ? static_cast<const __nv_bfloat16*>(qk->sin_t) : nullptr;
    a.qk_pos = qk ? qk->position : nullptr;
    a.qk_q = qk ? static_cast<__nv_bfloat16*>(qk->q_out) : nullptr;
    a.qk_k = qk ? static_cast<__nv_bfloat16*>(qk->k_cache) : nullptr;
    a.qk_v = qk ? static_cast<__nv_bfloat16*>(qk->v_cache) : nullptr;
    a.qk_hq = qk ? qk->hq : 0;
    a.qk_hkv = qk ? qk->hkv : 0;
    a.qk_cap = qk ? qk->capacity : 0;
    a.qk_cb = qk ? qk->cb : 0;
    a.qk_ch = qk ? qk->ch : 0;
    a.qk_cs = qk ? qk->cs : 0;
    a.qk_eps = qk ? qk->eps : 0.f;
    if (amax) {
        a.amax_keys =  // keys kAmaxKeyStride bytes apart
            reinterpret_cast<unsigned long long*>(static_cast<char*>(ws) + kAmaxOffset);
        a.amax_done = reinterpret_cast<unsigned*>(static_cast<char*>(ws) + kAmaxCountOffset);
        a.amax_idx = amax->idx;
        a.amax_best = static_cast<__nv_bfloat16*>(amax->best);
    }

    cudaStream_t s = (cudaStream_t)stream;
    switch (p->kind) {
        case NK_KIND_GEMV: return launch_gemv(*p, a, s);
        case NK_KIND_GENERIC: return launch_generic(*p, a, s);
        case NK_KIND_TC: return launch_tc(*p, a, s);
        default: return NK_ERR_PLAN;
    }
}

extern "C" size_t nk_gemm_argmax_ws_bytes(const nk_plan* p) {
    if (!p || p->magic != NK_PLAN_MAGIC || p->kind != NK_KIND_TC) return 0;
    if (p->M_max > kAmaxMaxTokens) return 0;
    return amax_ws_bytes(*p);
}

extern "C" int nk_gemm_bf16_argmax(const void* x, int64_t ldx, const void* w, int64_t ldw,
                                   void* y, int64_t ldy, int64_t* idx, void* best, int M, int N,
                                   int K, const nk_plan* p, void* ws, size_t ws_bytes,
                                   nk_stream_t stream) {
    const AmaxOut out{idx, best};
    return gemm_impl(x, ldx, w, ldw, y, ldy, false, M, N, K, p, ws, ws_bytes, stream, &out);
}

extern "C" int nk_test_withhold_partial(int tile) {
    if (tile < -1) return NK_ERR_ARG;
    g_withhold_tile.store(tile);
    return NK_OK;
}

extern "C" int nk_device_error(nk_stream_t stream, int* status) {
    if (!status) return NK_ERR_ARG;
    int h = 0;
    cudaStream_t s = (cudaStream_t)stream;
    if (cudaMemcpyFromSymbolAsync(&h, g_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s) !=
        cudaSuccess)
        return NK_ERR_CUDA;
    if (cudaStreamSynchronize(s) != cudaSuccess) return NK_ERR_CUDA;
    if (h != 0) {
        const int zero = 0;
        if (cudaMemcpyToSymbolAsync(g_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s) !=
                cudaSuccess ||
            cudaStreamSynchronize(s) != cudaSuccess)
            return NK_ERR_CUDA;
    }
    *status = h;
    return NK_OK;
}

extern "C" const char* nk_status_string(int status) {
    switch (status) {
        case NK_OK: return "ok";
        case NK_ERR_SHAPE: return "shape out of range (M, N, K or leading dimension)";
        case NK_ERR_ALIGN: return "operand alignment or leading dimension not supported by plan";
        case NK_ERR_WORKSPACE: return "workspace missing or smaller than nk_ws_bytes(plan)";
        case NK_ERR_SPLIT: return "split_k out of range";
        case NK_ERR_PLAN: return "invalid plan or plan made for another shape";
        case NK_ERR_CUDA: return "CUDA runtime error";
        case NK_ERR_DEVICE: return "current device is not an sm_100 (B200-class) GPU";
        case NK_ERR_TIMEOUT: return "bounded device wait expired";
        case NK_ERR_ARG: return "invalid argument";
        case NK_ERR_RANGE: return "decode position outside the cache";
        default: return "unknown status";
    }
}

extern "C" int nk_version(void) { return 0x000100; }
