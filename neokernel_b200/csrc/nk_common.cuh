// Shared device helpers and the internal launch interface of libnkgemm.so.
//
// Numerics follow the reference's decode linears (torch.mm on bf16 tensors, cuBLAS on the
// GPU, engine/kernels/decode.py:54-66): bf16 operands are widened exactly to fp32, products
// are accumulated in fp32, and the final sum is rounded once to bf16 (round-to-nearest-even).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/nk_gemm.h"

namespace nk {

// B200 (sm_100a): 148 SMs on two dies.
constexpr int kNumSMs = 148;

// Device-wide error word set by bounded waits that ran out (NK_ERR_TIMEOUT), read and
// cleared by nk_device_error(). The library is one translation unit (nk_lib.cu), so this
// definition exists once.
__device__ int g_error = 0;

// ---------------------------------------------------------------------------------------
// bf16 <-> fp32. Widening is exact by the format's definition (bf16 is the top half of an
// IEEE binary32); narrowing uses the CUDA intrinsic __float2bfloat16_rn.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ float bf16lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
    __nv_bfloat16 h = __float2bfloat16_rn(f);
    return *reinterpret_cast<uint16_t*>(&h);
}

// Streaming 128-bit load of weight data: read-only path, no L1 allocation (each weight byte
// is used by exactly one CTA once).
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(p));
    return r;
}

// Cached read-only 128-bit load (activations: tiny, reused by every CTA).
__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
    uint4 r;
    asm("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(p));
    return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

// ---------------------------------------------------------------------------------------
// Split-K epilogue shared by every kernel family.
//
// Each CTA of slice s stores its fp32 partial tile to part[s][m][n]. The CTA that takes the
// last ticket of its output tile sums the slices in the fixed order s = 0..S-1 (so the
// result does not depend on which CTA arrives last), rounds once to bf16, writes y and
// re-arms the ticket to zero so the workspace is ready for the next launch or graph replay.
// Returns true in the CTA that performed the reduction.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ bool splitk_last_cta(unsigned* ticket, int splits) {
    __shared__ unsigned s_last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned t = atomicAdd(ticket, 1u);
        s_last = (t == (unsigned)(splits - 1)) ? 1u : 0u;
    }
    __syncthreads();
    const bool last = s_last != 0u;
    if (last) __threadfence();
    return last;
}

// Workspace layout for a plan: [split][M_max][N] fp32 partials, then one ticket per
// (m_tile, n_tile), padded to 256 bytes.
struct WsLayout {
    size_t part_bytes;
    size_t ticket_offset;
    size_t ticket_count;
    size_t total;
};

inline WsLayout ws_layout(const nk_plan& p) {
    WsLayout L{};
    if (p.split_k <= 1) return L;
    L.part_bytes = (size_t)p.split_k * (size_t)p.M_max * (size_t)p.N * sizeof(float);
    L.ticket_offset = (L.part_bytes + 255) & ~(size_t)255;
    L.ticket_count = (size_t)p.n_tiles * (size_t)p.m_tiles;
    L.total = L.ticket_offset + ((L.ticket_count * sizeof(unsigned) + 255) & ~(size_t)255);
    return L;
}

// Launch arguments handed from the C ABI to a kernel family.
struct GemmArgs {
    const __nv_bfloat16* x; int64_t ldx;
    const __nv_bfloat16* w; int64_t ldw;
    __nv_bfloat16* y;       int64_t ldy;
    int M, N, K;
    float* part;            // split-K partials, or nullptr when split_k == 1
    unsigned* tickets;      // split-K tickets, or nullptr when split_k == 1
};

int launch_gemv(const nk_plan& p, const GemmArgs& a, cudaStream_t s);
int launch_generic(const nk_plan& p, const GemmArgs& a, cudaStream_t s);
int launch_tc(const nk_plan& p, const GemmArgs& a, cudaStream_t s);

// Tile geometry per family (host and device agree through these).
int gemv_token_tile(int M_max);          // MT: 1, 2, 4, 8 or 16
int gemv_rows_per_cta(int mt);           // weight rows per CTA for a given MT
constexpr int kGemvKStep = 256;          // K elements one warp covers per 128-bit load
constexpr int kGenericRows = 8;          // rows per CTA in the generic kernel
constexpr int kGenericTokens = 8;        // tokens per CTA in the generic kernel

}  // namespace nk
