// Workspace-free decode linear: nk_gemm_bf16_static (declared in include/nk_gemm.h).
//
// Who needs it. nk_gemm_bf16 takes its split-K scratch (tickets and fp32 partial sums) from
// the caller. Some callers have no way to provide one: an operator plugged into a host
// framework that owns every device allocation and hands the operator nothing but its input
// and output buffers; a process that fixes its device-memory budget at start-up and may not
// grow it afterwards; a latency-critical path that must not call cudaMalloc because a device
// allocation makes the CUDA runtime serialize work that is in flight on other streams. For
// them this entry point runs the tensor-core kernel family with its scratch in a fixed array
// compiled into this library instead.
//
// The array, g_static_scratch, is NK_STATIC_SCRATCH_BYTES (8 MiB) of device memory that every
// GPU which loads the library holds until the process exits. Plans whose scratch need
// (nk_ws_bytes) is larger are refused with NK_ERR_WORKSPACE before anything is launched.
// Nothing here allocates: no cudaMalloc, cudaFree or allocating library routine.
//
// Host code cannot use the array's name as a device address (on the host it names a host-side
// stand-in), so the first call on each device, with that device current, looks the address
// up with cudaGetSymbolAddress and keeps it for the life of the process (a cudaDeviceReset
// that unloads the library's module is not supported by this entry point); that first call
// on a device should therefore come before any stream capture on it. `stream` must belong to
// the current device, whose copy of the array is the one looked up (else NK_ERR_DEVICE).
// Every call on a device shares the one array, which keeps whatever the previous call left:
// each call first clears the parts of the array its plan uses (the plan's split-K tickets and
// its partial slots), and calls whose executions overlap on the GPU race on the array, so
// they must be ordered (one stream, or joined by events). A call refused for its arguments
// touches nothing.
#include <mutex>

#include "nk_common.cuh"

namespace nk {

static __device__ __align__(256) unsigned char g_static_scratch[NK_STATIC_SCRATCH_BYTES];

static std::mutex g_static_mutex;
static void* g_static_addr[64];  // device address of g_static_scratch, per device

// Device address of the static scratch on the current device (looked up once per device),
// provided `stream` runs on that device.
static int static_scratch_address(cudaStream_t stream, void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return NK_ERR_CUDA;
    if (dev < 0 || dev >= 64) return NK_ERR_DEVICE;
    if (stream != nullptr) {  // the legacy default stream is the current device's
        int sdev = -1;
        if (cudaStreamGetDevice(stream, &sdev) != cudaSuccess) return NK_ERR_CUDA;
        if (sdev != dev) return NK_ERR_DEVICE;
    }
    std::lock_guard<std::mutex> lock(g_static_mutex);
    if (!g_static_addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || p == nullptr)
            return NK_ERR_CUDA;
        g_static_addr[dev] = p;
    }
    *out = g_static_addr[dev];
    return NK_OK;
}

}  // namespace nk

extern "C" int nk_gemm_bf16_static(const void* x, int64_t ldx, const void* w, int64_t ldw,
                                   void* y, int64_t ldy, int M, int N, int K,
                                   const nk_plan* plan, nk_stream_t stream) {
    using namespace nk;
    if (!plan || plan->magic != NK_PLAN_MAGIC) return NK_ERR_PLAN;
    if (plan->kind != NK_KIND_TC) return NK_ERR_PLAN;  // the tensor-core family only
    const WsLayout L = ws_layout(*plan);
    if (L.total > (size_t)NK_STATIC_SCRATCH_BYTES) return NK_ERR_WORKSPACE;
    // Every argument check before the array is touched, so a refused call changes nothing.
    const int valid = gemm_validate(x, ldx, w, ldw, y, ldy, false, M, N, K, plan, nullptr);
    if (valid != NK_OK) return valid;
    const int dev_ok = check_device();
    if (dev_ok != NK_OK) return dev_ok;
    if (L.total == 0)  // no tile shared by two CTAs: no scratch at all
        return nk_gemm_bf16(x, ldx, w, ldw, y, ldy, M, N, K, plan, nullptr, 0, stream);
    void* scratch = nullptr;
    const int st = static_scratch_address((cudaStream_t)stream, &scratch);
    if (st != NK_OK) return st;
    // This plan's tickets and partial slots must start at zero. Every call leaves them so, but
    // one that stopped on an expired wait may not have, and all plans share the array.
    cudaStream_t s = (cudaStream_t)stream;
    if (cudaMemsetAsync(scratch, 0, L.ticket_count * sizeof(unsigned), s) != cudaSuccess ||
        cudaMemsetAsync(static_cast<char*>(scratch) + L.part_offset, 0, L.part_bytes, s) !=
            cudaSuccess)
        return NK_ERR_CUDA;
    return nk_gemm_bf16(x, ldx, w, ldw, y, ldy, M, N, K, plan, scratch,
                        (size_t)NK_STATIC_SCRATCH_BYTES, stream);
}
