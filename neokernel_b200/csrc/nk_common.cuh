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

// Largest tensor-parallel group (NK_PEER_MAX_RANKS in include/nk_comm.h).
#define NK_PEER_MAX_RANKS_INTERNAL 8

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
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(p));
    return r;
}

// Cached read-only 128-bit load (activations: tiny, reused by every CTA). Volatile, like the
// weight load, so neither moves across griddepcontrol.wait.
__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(p));
    return r;
}

// Programmatic dependent launch. A kernel launched with programmatic stream serialization
// may start while the previous kernel on the stream is still running; it must execute
// griddep_wait() before it reads anything that kernel writes (activations, workspace) and
// before it writes anything that kernel may still read. Weights are read-only, so their
// streaming may begin before the wait. Without the launch attribute both are no-ops.
#ifndef NK_PDL
#define NK_PDL 1  // launch with programmatic stream serialization
#endif
__device__ __forceinline__ void griddep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
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

// Store one output element: rounded once to bf16 into y, or unrounded into y32 (the fp32
// partial of a K-split tensor-parallel linear, summed across ranks before its one rounding).
template <typename GemmArgsT>
__device__ __forceinline__ void store_out(const GemmArgsT& a, int64_t idx, float v) {
    if (a.y32) a.y32[idx] = v;
    else a.y[idx] = __float2bfloat16_rn(v);
}

// The last CTA's share of the split-K reduction for one output tile of `rows` weight rows
// (from n_base) and `mcount` tokens (from m0). Thread i owns row i % rows and every
// (blockDim.x / rows)-th token from i / rows; for G of its tokens at a time it issues the
// loads of every slice before adding, so a batch costs about one L2 round trip instead of
// splits x G dependent ones. Slices are summed in ascending order, as in every other path.
template <int G, typename GemmArgsT>
__device__ __forceinline__ void splitk_reduce_tile(const GemmArgsT& a, int n_base, int rows,
                                                   int m0, int mcount, int splits) {
    const int lanes = blockDim.x / rows;
    const int r = threadIdx.x % rows;
    const int mfirst = threadIdx.x / rows;
    const int n = n_base + r;
    if (n >= a.N || mfirst >= lanes) return;
    const size_t slice = (size_t)a.M * a.N;
    for (int mb = mfirst; mb < mcount; mb += lanes * G) {
        float acc[G];
#pragma unroll
        for (int q = 0; q < G; ++q) acc[q] = 0.f;
        const float* p = a.part + (size_t)(m0 + mb) * a.N + n;
#pragma unroll 2
        for (int t = 0; t < splits; ++t) {
            float v[G];
#pragma unroll
            for (int q = 0; q < G; ++q)
                v[q] = (mb + q * lanes < mcount) ? __ldcg(p + (size_t)t * slice + (size_t)q * lanes * a.N)
                                                 : 0.f;
#pragma unroll
            for (int q = 0; q < G; ++q) acc[q] += v[q];
        }
#pragma unroll
        for (int q = 0; q < G; ++q)
            if (mb + q * lanes < mcount)
                store_out(a, (int64_t)(m0 + mb + q * lanes) * a.ldy + n, acc[q]);
    }
}

// Workspace layout: a fixed region of kTicketsMax split-K tickets at offset 0, then the
// greedy head's fixed region (the running (value, index) keys of up to kAmaxMaxTokens tokens
// and a count of finished CTAs), then the partials — [split][M_max][N] fp32 for the GEMV
// family, [tile][segment][token column][128 rows] 64-bit slots for the tensor-core family.
// Every plan puts its tickets and keys in the same fixed regions, the kernels leave tickets,
// keys and count at zero and clear every tagged slot they read, so any sequence of ordered
// calls may share one workspace whatever their plans (one plan's partials never overlay
// another's tickets or keys).
constexpr size_t kTicketsMax = 65536;
constexpr size_t kTicketBytes = kTicketsMax * sizeof(unsigned);
// One 128-byte line per token key: every warp of every tile updates each token's key, and
// atomics on keys sharing a line queue behind one another in its L2 slice (16 keys in one
// line cost lm_head at 16 tokens ~80 us).
constexpr size_t kAmaxOffset = kTicketBytes;
constexpr size_t kAmaxKeyStride = 128;
constexpr int kAmaxMaxTokens = 255;
constexpr size_t kAmaxBytes = (kAmaxMaxTokens + 1) * kAmaxKeyStride;  // 32 KiB: keys, count
constexpr size_t kAmaxCountOffset = kAmaxOffset + kAmaxMaxTokens * kAmaxKeyStride;
constexpr size_t kPartOffset = kAmaxOffset + kAmaxBytes;

struct WsLayout {
    size_t part_offset;
    size_t part_bytes;
    size_t ticket_count;
    size_t total;
};

inline WsLayout ws_layout(const nk_plan& p) {
    WsLayout L{};
    L.ticket_count = (size_t)p.n_tiles * (size_t)p.m_tiles;
    L.part_offset = kPartOffset;
    if (p.kind == NK_KIND_TC) {
        // [tile][segment][token column][128 rows] 64-bit {fp32 value, tag} slots, only when
        // some tile is shared
        if (p.segments <= 1) return WsLayout{};
        const size_t cols = (size_t)(p.M_max < p.tile_m ? p.M_max : p.tile_m);
        L.part_bytes = L.ticket_count * (size_t)p.segments * cols * 128 * sizeof(uint64_t);
    } else {
        // [slice][M][N] fp32
        if (p.split_k <= 1) return WsLayout{};
        L.part_bytes = (size_t)p.split_k * (size_t)p.M_max * (size_t)p.N * sizeof(float);
    }
    L.total = L.part_offset + ((L.part_bytes + 255) & ~(size_t)255);
    return L;
}

// Workspace bytes the greedy head (nk_gemm_bf16_argmax) needs: the plan's, and at least the
// fixed regions in front of the partials.
inline size_t amax_ws_bytes(const nk_plan& p) {
    const size_t t = ws_layout(p).total;
    return t > kPartOffset ? t : kPartOffset;
}

// ---------------------------------------------------------------------------------------
// Work partition of the tensor-core family. A "unit" is one 64-wide K block of one output
// tile (128 weight rows x NT tokens); tile t owns units [t*KB, (t+1)*KB). CTA c processes the
// contiguous units [begin(c), begin(c+1)):
//   balanced (split == 0): begin(c) = floor(U*c / G), so every CTA streams the same number
//                          of weight bytes (within one block) whatever the tile count;
//   split    (split  > 0): G = T*split and CTA c covers slice c % split of tile c / split.
// A tile whose units span several CTAs is summed from their fp32 partials in ascending
// rank (= ascending k) order by the CTA that finishes it last.
// ---------------------------------------------------------------------------------------
struct TcPartition {
    int64_t U;   // total units
    int KB;      // units (K blocks) per tile
    int G;       // CTAs
    int split;   // 0 = balanced
    int lead;    // split > 1: rank 0's slice is KB / split + lead units, the others share the
                 // rest evenly (0 = every slice KB / split)

    __host__ __device__ int lead_units() const {
        const int a = KB / split + lead;
        return a < KB - (split - 1) ? a : KB - (split - 1);
    }
    __host__ __device__ int64_t begin(int c) const {
        if (split == 0) return (U * (int64_t)c) / G;
        const int t = c / split, s = c % split;
        if (lead == 0 || split < 2 || s == 0) return (int64_t)t * KB + ((int64_t)s * KB) / split;
        const int A = lead_units();
        return (int64_t)t * KB + A + ((int64_t)(s - 1) * (KB - A)) / (split - 1);
    }
    // The CTA whose range contains unit u.
    __host__ __device__ int cta_of(int64_t u) const {
        if (split == 0) return (int)(((u + 1) * G + U - 1) / U - 1);
        const int64_t t = u / KB;
        const int64_t kb = u - t * KB;
        if (lead == 0 || split < 2) return (int)(t * split + ((kb + 1) * split + KB - 1) / KB - 1);
        const int A = lead_units();
        if (kb < A) return (int)(t * split);
        const int64_t v = kb - A, R = KB - A;
        return (int)(t * split + 1 + ((v + 1) * (split - 1) + R - 1) / R - 1);
    }
    __host__ __device__ int first_cta(int t) const { return cta_of((int64_t)t * KB); }
    __host__ __device__ int last_cta(int t) const { return cta_of((int64_t)(t + 1) * KB - 1); }
};

// ---------------------------------------------------------------------------------------
// Peer receive buffers of a tensor-parallel group (include/nk_comm.h). Buffer of one rank,
// zeroed once and mapped into every rank of the group:
//   [0, 4 KB)            progress counter per index (read and advanced by the one CTA that
//                        owns that index in a call)
//   [4 KB, 68 KB)        flags[2 sets][8 source ranks][1024 indices], u32
//   [68 KB, ...)         slots[2 sets][world source ranks][max_elems], fp32
// Call e (1, 2, ...) of index i uses set e & 1: its owner writes this rank's values into
// slots[set][rank] of every rank, fences at system scope, writes e into flags[set][rank][i] of
// every rank (release), waits for flags[set][r][i] == e for all r in its own buffer (acquire,
// bounded) and sums slots[set][0..world) in rank order. Two sets suffice: a rank can only
// start writing call e+2 into a peer once it has seen that peer's flag for call e+1, i.e. once
// the peer has finished call e on its stream. An index is a CTA of nk_allreduce_bf16 or an
// output tile of nk_gemm_bf16_allreduce; a group serves one of the two, as the elements an
// index covers differ between them.
// ---------------------------------------------------------------------------------------
constexpr int kArMaxIndex = 1024;
constexpr size_t kArEpochBytes = (size_t)kArMaxIndex * 4;
constexpr size_t kArFlagBytes = 2ull * NK_PEER_MAX_RANKS_INTERNAL * kArMaxIndex * 4;
constexpr size_t kArHeader = kArEpochBytes + kArFlagBytes;

__device__ __forceinline__ unsigned* ar_counter(uint8_t* base, int index) {
    return reinterpret_cast<unsigned*>(base) + index;
}

__device__ __forceinline__ unsigned* ar_flag(uint8_t* base, int set, int src, int index) {
    return reinterpret_cast<unsigned*>(base + kArEpochBytes) +
           ((size_t)(set * NK_PEER_MAX_RANKS_INTERNAL + src) * kArMaxIndex + index);
}

__device__ __forceinline__ float* ar_slot(uint8_t* base, int set, int src, int world,
                                          int max_elems) {
    return reinterpret_cast<float*>(base + kArHeader) + (size_t)(set * world + src) * max_elems;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Launch arguments handed from the C ABI to a kernel family.
struct GemmArgs {
    const __nv_bfloat16* x; int64_t ldx;
    const __nv_bfloat16* w; int64_t ldw;
    __nv_bfloat16* y;       int64_t ldy;
    int M, N, K;
    float* y32;             // when set: fp32 output [M, N] (row stride ldy) instead of y
    float* part;            // split-K partials, or nullptr when split_k == 1
    unsigned* tickets;      // split-K tickets, or nullptr when split_k == 1
    // tensor-core family only
    int n_tiles;            // ceil(N / 128)
    int segments;           // partial slots per tile
    int seg_max;            // most CTAs sharing one tile in this launch's partition (<= segments)
    int part_cols;          // token columns per partial slot (min(NT, M_max))
    int coresident;         // 1: every CTA of the grid is resident at once (see nk_tc.cu)
    int withhold_tile;      // failure-detection tests only (nk_test_withhold_partial): the
                            // rank-1 CTA of this output tile publishes no partial; -1 = none
    TcPartition part_map;
    // greedy head (nk_gemm_bf16_argmax) only; all nullptr otherwise
    unsigned long long* amax_keys;  // [M] (ordered value, inverted index) keys, zero between calls
    unsigned* amax_done;            // CTAs that have folded their rows in, zero between calls
    int64_t* amax_idx;              // [M] lowest index of each token's largest bf16 output
    __nv_bfloat16* amax_best;       // [M] that largest value, or nullptr
    // fused q/k-norm + RoPE + KV-cache epilogue (nk_gemm_bf16_qkv_rope_cache) only; qk_q is
    // nullptr otherwise
    const __nv_bfloat16* qk_qnorm;  // [128] query-head RMSNorm gain
    const __nv_bfloat16* qk_knorm;  // [128] key-head RMSNorm gain
    const __nv_bfloat16* qk_cos;    // [capacity, 128] rotary tables
    const __nv_bfloat16* qk_sin;
    const int64_t* qk_pos;          // device-side decode position
    __nv_bfloat16* qk_q;            // [M, Hq * 128] roped, normalised queries
    __nv_bfloat16* qk_k;            // key cache, element (b, h, p, d) at b*cb + h*ch + p*cs + d
    __nv_bfloat16* qk_v;            // value cache, same strides
    int qk_hq, qk_hkv, qk_cap;
    int64_t qk_cb, qk_ch, qk_cs;
    float qk_eps;
    // fused all-reduce (nk_gemm_bf16_allreduce) only; ar_world == 0 otherwise
    uint8_t* ar_buf[NK_PEER_MAX_RANKS_INTERNAL];  // every rank's receive buffer, as mapped here
    int ar_rank, ar_world, ar_max_elems;
};

int launch_gemv(const nk_plan& p, const GemmArgs& a, cudaStream_t s);
int launch_generic(const nk_plan& p, const GemmArgs& a, cudaStream_t s);
int launch_tc(const nk_plan& p, const GemmArgs& a, cudaStream_t s);

// Tile geometry per family (host and device agree through these).
int gemv_token_tile(int M_max);          // MT: 1, 2, 4, 8 or 16
int gemv_rows_per_cta(int mt);           // weight rows per CTA for a given MT
constexpr int kGemvKStep = 256;          // K elements one warp covers per 128-bit load
int tc_token_tile(int M_max);            // NT: 16, 32, 64, 128 or 256
int tc_stages(int nt);                   // shared-memory ring depth for a token tile
int tc_ctas_per_sm(int nt);              // resident CTAs per SM for a token tile
constexpr int kTcRowsPerCta = 128;       // weight rows per CTA (tcgen05 MMA M)
constexpr int kTcBox = 64;               // K elements per TMA box (one 128-byte swizzle row)
#ifndef NK_TC_UK
#define NK_TC_UK 2
#endif
// TMA boxes along K per pipeline stage (one "unit" of the schedule): the 256-token tile takes
// one, so that a stage (16 KB of weights, 32 KB of tokens) still leaves four stages in flight.
__host__ __device__ constexpr int tc_uk(int nt) { return nt >= 256 ? 1 : NK_TC_UK; }
__host__ __device__ constexpr int tc_kstep(int nt) { return kTcBox * tc_uk(nt); }  // K per unit
// fewest units per CTA for which the plan puts two CTAs on an SM (when both fit)
#ifndef NK_TC_DUAL_MIN_UNITS
#define NK_TC_DUAL_MIN_UNITS 16
#endif
// the tile-aligned schedule (nk_plan.slices): on, and the fewest slices per tile it takes
#ifndef NK_TC_ALIGNED
#define NK_TC_ALIGNED 1
#endif
#ifndef NK_TC_MIN_SLICES
#define NK_TC_MIN_SLICES 4
#endif
// Extra K blocks for the tile-aligned schedule's rank-0 slice (see tc_lead in nk_tc.cu): for
// tiles of at least 32 K blocks, by finishing protocol; the counted protocol's for 16..31.
#ifndef NK_TC_LEAD_TAGGED
#define NK_TC_LEAD_TAGGED 2
#endif
#ifndef NK_TC_LEAD_COUNTED
#define NK_TC_LEAD_COUNTED 4
#endif
#ifndef NK_TC_LEAD_COUNTED_WIDE  // counted, tiles of >= 32 K blocks split 7 or more ways
#define NK_TC_LEAD_COUNTED_WIDE 6
#endif
#ifndef NK_TC_LEAD_COUNTED_SHORT
#define NK_TC_LEAD_COUNTED_SHORT 3
#endif
constexpr int kGenericRows = 8;          // rows per CTA in the generic kernel
constexpr int kGenericTokens = 8;        // tokens per CTA in the generic kernel

}  // namespace nk
