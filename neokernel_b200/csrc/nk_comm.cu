// One-shot all-reduce of fp32 partials over NVLink peer memory (include/nk_comm.h), launched
// with programmatic dependent launch so it starts while the GEMM that made the partial drains.
//
// The receive buffers and the call protocol (progress counters, two sets of flags and slots)
// are described with their layout in nk_common.cuh; here index i is CTA i, which moves
// elements [1024 i, 1024 i + 1024) of the partial.
#include <string.h>

#include "nk_common.cuh"
#include "../../include/nk_comm.h"

namespace nk {

constexpr int kArThreads = 256;
constexpr int kArElemsPerCta = kArThreads * 4;
constexpr int kArMaxCtas = NK_PEER_MAX_ELEMS / kArElemsPerCta;  // 1024
static_assert(kArMaxCtas == kArMaxIndex, "one flag per all-reduce CTA");
static_assert(NK_PEER_MAX_RANKS == NK_PEER_MAX_RANKS_INTERNAL, "group size");

struct PeerArgs {
    uint8_t* buf[NK_PEER_MAX_RANKS];
    int rank, world, max_elems;
};

__global__ void __launch_bounds__(kArThreads)
allreduce_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ out, int n,
                      PeerArgs g) {
    __shared__ unsigned s_e;
    __shared__ int s_ok;
    // Launched with programmatic dependent launch: the partial x comes from the previous
    // kernel (and this CTA's epoch counter from the previous call), so wait before any read.
    if (threadIdx.x == 0) griddep_launch_dependents();
    griddep_wait();
    const int c = blockIdx.x;
    uint8_t* own = g.buf[g.rank];
    unsigned* epo = reinterpret_cast<unsigned*>(own) + c;
    if (threadIdx.x == 0) {
        s_e = *epo + 1u;  // only CTA c of this rank ever touches this counter
        s_ok = 1;
    }
    __syncthreads();
    const unsigned e = s_e;
    const int set = (int)(e & 1u);
    const int i = c * kArElemsPerCta + threadIdx.x * 4;
    const bool live = i < n;  // n % 4 == 0, so [i, i + 4) is all in or all out
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (live) v = *reinterpret_cast<const float4*>(x + i);
    // this rank's slice into every rank's buffer (its own included)
    for (int r = 0; r < g.world; ++r)
        if (live)
            *reinterpret_cast<float4*>(ar_slot(g.buf[r], set, g.rank, g.world, g.max_elems) + i) = v;
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < g.world) st_release_sys(ar_flag(g.buf[threadIdx.x], set, g.rank, c), e);
    // every rank's slice of this call in the own buffer
    if (threadIdx.x < g.world) {
        const unsigned* f = ar_flag(own, set, threadIdx.x, c);
        const uint64_t t0 = global_ns();
        while (ld_acquire_sys(f) != e) {
            if (global_ns() - t0 > 2000000000ull) {
                atomicExch(&g_error, NK_ERR_TIMEOUT);
                s_ok = 0;
                break;
            }
            __nanosleep(64);
        }
    }
    __syncthreads();
    if (s_ok && live) {
        float4 a = __ldcg(reinterpret_cast<const float4*>(ar_slot(own, set, 0, g.world, g.max_elems) + i));
        for (int r = 1; r < g.world; ++r) {
            const float4 b =
                __ldcg(reinterpret_cast<const float4*>(ar_slot(own, set, r, g.world, g.max_elems) + i));
            a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
        }
        const uint32_t lo = (uint32_t)f32_to_bf16_bits(a.x) | ((uint32_t)f32_to_bf16_bits(a.y) << 16);
        const uint32_t hi = (uint32_t)f32_to_bf16_bits(a.z) | ((uint32_t)f32_to_bf16_bits(a.w) << 16);
        *reinterpret_cast<uint2*>(out + i) = make_uint2(lo, hi);
    }
    if (threadIdx.x == 0) *epo = e;
}

}  // namespace nk

using namespace nk;

extern "C" size_t nk_peer_buffer_bytes(int max_elems, int world) {
    if (max_elems < 1 || max_elems > NK_PEER_MAX_ELEMS || world < 2 || world > NK_PEER_MAX_RANKS)
        return 0;
    return kArHeader + 2ull * (size_t)world * (size_t)max_elems * sizeof(float);
}

// CUDA IPC shares the driver's underlying memory block, and small cudaMalloc allocations may
// be placed together in one block, so exporting one can expose its neighbours to the peer
// processes. Every peer buffer is rounded up to whole 2 MiB (the size CUDA's documentation
// recommends for shared allocations), so it is a block of its own and exposes nothing else.
constexpr size_t kIpcGranule = 2u << 20;

extern "C" int nk_peer_alloc(size_t bytes, void** ptr) {
    if (!ptr || bytes == 0) return NK_ERR_ARG;
    *ptr = nullptr;
    bytes = (bytes + kIpcGranule - 1) / kIpcGranule * kIpcGranule;
    if (cudaMalloc(ptr, bytes) != cudaSuccess) return NK_ERR_CUDA;
    if (cudaMemset(*ptr, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(*ptr);
        *ptr = nullptr;
        return NK_ERR_CUDA;
    }
    return NK_OK;
}

extern "C" int nk_peer_free(void* ptr) {
    if (!ptr) return NK_ERR_ARG;
    return cudaFree(ptr) == cudaSuccess ? NK_OK : NK_ERR_CUDA;
}

extern "C" int nk_ipc_handle(void* ptr, void* handle) {
    static_assert(sizeof(cudaIpcMemHandle_t) == NK_IPC_HANDLE_BYTES, "IPC handle size");
    if (!ptr || !handle) return NK_ERR_ARG;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) return NK_ERR_CUDA;
    memcpy(handle, &h, sizeof(h));
    return NK_OK;
}

extern "C" int nk_ipc_open(const void* handle, void** ptr) {
    if (!handle || !ptr) return NK_ERR_ARG;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    *ptr = nullptr;
    return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess
               ? NK_OK : NK_ERR_CUDA;
}

extern "C" int nk_ipc_close(void* ptr) {
    if (!ptr) return NK_ERR_ARG;
    return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? NK_OK : NK_ERR_CUDA;
}

extern "C" int nk_gemm_bf16_allreduce(const void* x, int64_t ldx, const void* w, int64_t ldw,
                                      void* y, int64_t ldy, int M, int N, int K,
                                      const nk_plan* p, void* ws, size_t ws_bytes,
                                      const nk_peer_group* g, nk_stream_t stream) {
    if (!g || !y) return NK_ERR_ARG;
    if (g->world < 2 || g->world > NK_PEER_MAX_RANKS || g->rank < 0 || g->rank >= g->world ||
        g->max_elems < 1 || g->max_elems > NK_PEER_MAX_ELEMS)
        return NK_ERR_ARG;
    if (!p || p->magic != NK_PLAN_MAGIC) return NK_ERR_PLAN;
    // the balanced tensor-core schedule (whole grid resident), token tiles of up to 64, one
    // flag index per output tile
    if (p->kind != NK_KIND_TC || p->split_k != 0 || p->tile_m > 64 ||
        (int64_t)p->n_tiles * p->m_tiles > kArMaxIndex)
        return NK_ERR_PLAN;
    if (M < 1 || N < 1 || (int64_t)M * N > g->max_elems) return NK_ERR_SHAPE;
    ArIn ar;
    for (int r = 0; r < NK_PEER_MAX_RANKS; ++r) {
        ar.buf[r] = r < g->world ? g->buf[r] : nullptr;
        if (r < g->world && (!ar.buf[r] || ((uintptr_t)ar.buf[r] & 255u))) return NK_ERR_ARG;
    }
    ar.rank = g->rank;
    ar.world = g->world;
    ar.max_elems = g->max_elems;
    return gemm_impl(x, ldx, w, ldw, y, ldy, false, M, N, K, p, ws, ws_bytes, stream, nullptr,
                     &ar);
}

extern "C" int nk_allreduce_bf16(const float* x, void* out, int n, const nk_peer_group* g,
                                 nk_stream_t stream) {
    if (!x || !out || !g) return NK_ERR_ARG;
    if (g->world < 2 || g->world > NK_PEER_MAX_RANKS || g->rank < 0 || g->rank >= g->world ||
        g->max_elems < 1 || g->max_elems > NK_PEER_MAX_ELEMS)
        return NK_ERR_ARG;
    if (n < 1 || n > g->max_elems || n % 4) return NK_ERR_SHAPE;
    if (((uintptr_t)x & 15u) || ((uintptr_t)out & 15u) || (g->max_elems % 4)) return NK_ERR_ALIGN;
    PeerArgs a;
    for (int r = 0; r < NK_PEER_MAX_RANKS; ++r) {
        a.buf[r] = static_cast<uint8_t*>(r < g->world ? g->buf[r] : nullptr);
        if (r < g->world && (!a.buf[r] || ((uintptr_t)a.buf[r] & 255u))) return NK_ERR_ARG;
    }
    a.rank = g->rank;
    a.world = g->world;
    a.max_elems = g->max_elems;
    const int grid = (n + kArElemsPerCta - 1) / kArElemsPerCta;
    return launch_pdl_smem(allreduce_bf16_kernel, dim3(grid), dim3(kArThreads), 0,
                           (cudaStream_t)stream, x, static_cast<__nv_bfloat16*>(out), n, a);
}
