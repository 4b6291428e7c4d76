// C ABI of libnkgemm.so (declared in include/nk_gemm.h): plan selection, host-side
// validation and dispatch to the kernel families.
//
// The entry point nk_gemm_bf16 stands in for torch.mm(x, W.t(), out=y) at
// engine/kernels/decode.py:54,58,64,66 and engine/engine.py:114. Like the reference's Python
// wrappers (engine/kernels/decode.py:22,24; engine/kernels/rmsnorm.py:36), it rejects a bad
// configuration before launching anything; it never allocates and never synchronizes.
#include <string.h>

#include "nk_common.cuh"

namespace nk {

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

    if (kind == NK_KIND_AUTO) kind = (K % 8 != 0) ? NK_KIND_GENERIC : NK_KIND_GEMV;
    if (kind != NK_KIND_GENERIC && K % 8 != 0) return NK_ERR_ALIGN;
    if (kind == NK_KIND_TC) return NK_ERR_PLAN;  // tensor-core family not yet selectable

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
    } else {  // NK_KIND_GEMV
        p->tile_m = gemv_token_tile(M_max);
        p->tile_n = gemv_rows_per_cta(p->tile_m);
        const int tiles = ceil_div(N, p->tile_n) * ceil_div(M_max, p->tile_m);
        const int split = split_k ? split_k : gemv_auto_split(tiles, K);
        set_slices(p, split, kGemvKStep);
    }
    p->n_tiles = ceil_div(N, p->tile_n);
    p->m_tiles = ceil_div(M_max, p->tile_m);
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

extern "C" int nk_gemm_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y,
                            int64_t ldy, int M, int N, int K, const nk_plan* p, void* ws,
                            size_t ws_bytes, nk_stream_t stream) {
    if (!p || p->magic != NK_PLAN_MAGIC) return NK_ERR_PLAN;
    if (p->N != N || p->K != K) return NK_ERR_PLAN;
    if (M < 1 || M > p->M_max) return NK_ERR_SHAPE;
    if (!x || !w || !y) return NK_ERR_ARG;
    if (ldx < K || ldw < K || ldy < N) return NK_ERR_SHAPE;
    if (!aligned2(x) || !aligned2(w) || !aligned2(y)) return NK_ERR_ALIGN;
    if (p->kind == NK_KIND_GEMV || p->kind == NK_KIND_TC) {
        if (!aligned16(x) || !aligned16(w) || (ldx % 8) != 0 || (ldw % 8) != 0)
            return NK_ERR_ALIGN;
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
    a.y = static_cast<__nv_bfloat16*>(y);       a.ldy = ldy;
    a.M = M; a.N = N; a.K = K;
    a.part = L.total ? static_cast<float*>(ws) : nullptr;
    a.tickets = L.total ? reinterpret_cast<unsigned*>(static_cast<char*>(ws) + L.ticket_offset)
                        : nullptr;

    cudaStream_t s = (cudaStream_t)stream;
    switch (p->kind) {
        case NK_KIND_GEMV: return launch_gemv(*p, a, s);
        case NK_KIND_GENERIC: return launch_generic(*p, a, s);
        case NK_KIND_TC: return launch_tc(*p, a, s);
        default: return NK_ERR_PLAN;
    }
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
        default: return "unknown status";
    }
}

extern "C" int nk_version(void) { return 0x000100; }
