// tcgen05/TMEM tensor-core family for the decode linears (sm_100a).
//
// Replaces the cuBLAS GEMM behind torch.mm(x, W.t(), out=y) at engine/kernels/decode.py:54,
// 58,64,66 and engine/engine.py:114 for decode batches where CUDA-core FMA throughput, not
// HBM, would bound the GEMV, and for the M = 64..256 tree-verify contraction.
//
// Swap-AB: the weight tile is the MMA's A operand (M_mma = 128 weight rows) and the decode
// tokens are its B operand (N_mma = NT = 16..256 tokens), so a decode batch of a few tokens
// still fills a legal MMA shape; the accumulator D[n, t] = sum_k W[n,k] x[t,k] lives in TMEM.
//
// Persistent schedule: the grid is one wave (148 SMs x resident CTAs) and CTA c streams the
// contiguous run of (tile, 64-wide K block) units given by TcPartition (nk_common.cuh), so
// every CTA moves the same number of weight bytes whatever the tile count. Six warps:
//   warp 0 lane 0 : TMA producer. For each unit it loads the W tile [128 x 64] and the x
//                   tile [NT x 64] (bf16, 128-byte rows, SWIZZLE_128B) into stage s of a
//                   STAGES-deep shared-memory ring, completing on full[s].
//   warp 1 lane 0 : MMA issuer. Per unit: four tcgen05.mma.kind::f16 (K = 16 each) into one
//                   of two TMEM accumulators, then tcgen05.commit -> empty[s]; at the end of
//                   each tile segment tcgen05.commit -> tfull[buf].
//   warps 2..5    : epilogue. Warp w reads TMEM lanes 32*(w%4).. (row n of the tile) with
//                   tcgen05.ld, frees the accumulator (tempty[buf]) and stores bf16 y when the
//                   segment covers the whole K range. A tile shared by several CTAs is
//                   finished by its rank-0 CTA (the one holding its first K blocks) from the
//                   other ranks' fp32 partials, added in rank order (protocols below).
// The two accumulators let the epilogue of one segment overlap the MMAs of the next.
//
// Programmatic dependent launch: weights do not depend on the previous kernel, so the
// producer fills the ring with weight tiles before griddepcontrol.wait, and every CTA lets
// the next launch begin once it is resident.
//
// Every mbarrier wait is bounded: on expiry the thread records NK_ERR_TIMEOUT in the device
// error word and the CTA stops storing, drains its outstanding copies and MMAs (bounded),
// frees its TMEM and exits. Every TMA load here fills only the issuing CTA's own shared memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "nk_common.cuh"

namespace nk {

constexpr int kTcRows = kTcRowsPerCta;
// Warps 0 and 1 load and issue; the epilogue has four warps (one per TMEM lane quarter) for
// the decode token tiles, eight for the 64-token tile and twelve for wider ones, whose CTA is
// alone on its SM: two or three warps then share each lane quarter and take 16-column chunks
// in turn. The epilogue's chunk loops run latency-bound on one warp per scheduler (~2.5 k
// cycles a chunk measured on B200), so every added warp shortens the tail in which one CTA
// stores, publishes or sums a wide tile. Measured (verify M = 64 / 128 / 256, µs, four ->
// eight -> twelve warps): o_proj 16.9 -> 14.0 -> 14.1, 25.4 -> 19.6 -> 18.3, 27.6 -> 21.8 ->
// 20.5; sixteen warps would leave 96 registers a thread and spill.
#ifndef NK_TC_EPI_WARPS_64
#define NK_TC_EPI_WARPS_64 8
#endif
#ifndef NK_TC_EPI_WARPS_128
#define NK_TC_EPI_WARPS_128 12
#endif
__host__ __device__ constexpr int tc_epi_warps(int nt) {
    return nt >= 128 ? NK_TC_EPI_WARPS_128 : (nt >= 64 ? NK_TC_EPI_WARPS_64 : 4);
}
__host__ __device__ constexpr int tc_threads(int nt) { return 64 + 32 * tc_epi_warps(nt); }
// Registers a thread may use. Every CTA of the grid must be resident at once (rank-0 CTAs of
// shared tiles wait for higher CTAs), and the launch caps the grid by the CTAs that fit per
// SM: two CTAs of six warps per SM need at most 128 registers a thread (each SM sub-partition
// holds up to four of the twelve warps), the cap for token tiles <= 64; a wide tile's CTA,
// alone on its SM, may use a sub-partition's 16K registers over the warps it places there
// (ceil(warps / 4)), at most 255.
__host__ __device__ constexpr int tc_reg_budget(int nt) {
    return (16384 / (((tc_threads(nt) / 32 + 3) / 4) * 32)) & ~7;
}
__host__ __device__ constexpr int tc_maxnreg(int nt) {
    return (nt <= 64 ? 128 : 255) < tc_reg_budget(nt) ? (nt <= 64 ? 128 : 255) : tc_reg_budget(nt);
}
constexpr int kTcEpiThreads = 128;         // the four-warp epilogue
constexpr uint32_t kWaitLimit = 1u << 26;  // polls before a wait gives up (seconds)

// ---------------------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity; false (error recorded) on expiry.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    for (uint32_t i = 0; i < kWaitLimit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    atomicExch(&g_error, NK_ERR_TIMEOUT);
    return false;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
        : "memory");
}

// Weight-tile load marked evict-first in L2: every weight byte is read once per decode step,
// so these lines should be the first to leave and not push out the activations, partials and
// KV rows that are read again.
__device__ __forceinline__ void tma_load_w(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                           int c0, int c1, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Untiled bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned) from global
// into this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
        : "memory");
}

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 32 lanes x 16 consecutive 32-bit TMEM columns -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32"
        " {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait until *count >= target (another CTA of this grid increments it after
// publishing). Gives up after ~2 s, recording NK_ERR_TIMEOUT; returns whether it was reached.
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Count one more published partial of a tile: a release, so every store the CTA made before
// the barrier that precedes this call (its partial) is visible to whoever acquires the count.
__device__ __forceinline__ void count_release(unsigned* count) {
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(count) : "memory");
}

__device__ __forceinline__ bool spin_until_count(const unsigned* count, unsigned target) {
    const uint64_t t0 = global_ns();
    while (ld_acquire_gpu(count) < target) {
        if (global_ns() - t0 > 2000000000ull) {
            atomicExch(&g_error, NK_ERR_TIMEOUT);
            return false;
        }
        __nanosleep(32);
    }
    return true;
}

template <int THREADS>
__device__ __forceinline__ void epi_bar_n() {  // named barrier over the epilogue warps
    asm volatile("bar.sync 1, %0;" ::"n"(THREADS) : "memory");
}
__device__ __forceinline__ void epi_bar() {  // the four-warp epilogue's
    epi_bar_n<kTcEpiThreads>();
}

// Shared-memory matrix descriptor for a K-major operand tile stored as 128-byte rows with
// the 128-byte swizzle (8-row x 128-byte swizzle atoms, atoms 1024 bytes apart):
//   bits  0-13 start address >> 4     bits 16-29 leading byte offset >> 4 (unused here: 1)
//   bits 32-45 stride byte offset >> 4 (1024 B between 8-row groups)
//   bits 46-47 descriptor version (1 on sm_100)   bits 61-63 layout (2 = SWIZZLE_128B)
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) |
           ((uint64_t)(1024u >> 4) << 32) | ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

// Instruction descriptor, kind::f16: fp32 accumulator (bits 4-5 = 1), A and B bf16 (bits
// 7-9 = 1, 10-12 = 1), both K-major (bits 15, 16 = 0), N >> 3 at bits 17-22, M >> 4 at 24-28.
__host__ __device__ constexpr uint32_t tc_idesc(int m, int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(m >> 4) << 24);
}

#ifndef NK_TC_SMEM_SMALL
#define NK_TC_SMEM_SMALL (110 * 1024)  // token tiles <= 64: two CTAs per SM
#endif
#ifndef NK_TC_SMALL_MAX_NT
// Widest token tile given the two-per-SM budget. Token tiles of 64 (the M = 33..64 verify
// batches) take the large ring: measured on B200, verify M = 64 QKV 20.6 -> 18.8 us, o_proj
// 18.1 -> 16.8, down 30.6 -> 27.2, gate_up 41.5 -> 42.0.
#define NK_TC_SMALL_MAX_NT 32
#endif
#ifndef NK_TC_SMEM_LARGE
#define NK_TC_SMEM_LARGE (200 * 1024)  // token tiles >= 128: one CTA per SM
#endif
#ifndef NK_TC_L2_PROMO
#define NK_TC_L2_PROMO CU_TENSOR_MAP_L2_PROMOTION_L2_256B
#endif

// Shared memory of the fused QKV epilogue (kModeQkv, below) for a head in the middle of a CTA's
// range, whose ring is still in use: one column at a time, (4 warp sums + 128 elements) for two
// columns in turn. It keeps the kernel within the footprint that lets two launches share an SM;
// a head finished last (the usual case: heads are split over several CTAs) uses the idle ring.
constexpr int kQkvSmemBytes = 2 * (4 + 128) * 4;

// EXTRA: bytes after the barriers and flags for a mode's own use (they do not change the
// number of stages the budget gives).
template <int NT, int EXTRA = 0>
struct TcSmem {
    static constexpr int kBoxA = kTcRows * kTcBox * 2;  // 16 KB: 128 weight rows x 128 B
    static constexpr int kBoxB = NT * kTcBox * 2;       // NT tokens x 128 B
    static constexpr int kUK = tc_uk(NT);  // boxes along K per stage
    static constexpr int kA = kUK * kBoxA;
    static constexpr int kB = kUK * kBoxB;
    static constexpr int kStage = kA + kB;
    static constexpr int kBudget = NT <= NK_TC_SMALL_MAX_NT ? NK_TC_SMEM_SMALL : NK_TC_SMEM_LARGE;
    static constexpr int kStagesFit = (kBudget - 2048) / kStage;
    static constexpr int kStages = kStagesFit > 8 ? 8 : (kStagesFit < 2 ? 2 : kStagesFit);
    static constexpr int kBarOff = kStages * kStage;
    static constexpr int kPartBars = 8;                  // partial chunks in flight (finisher)
    static constexpr int kNumBars = 2 * kStages + 4 + kPartBars;  // full, empty, tfull[2], tempty[2], part
    static constexpr int kMiscOff = kBarOff + kNumBars * 8;
    // tmem slot, abort, last, all-reduce call, ok; then the fused QKV epilogue's buffers
    static constexpr int kBytes = kMiscOff + 32 + EXTRA;
    static constexpr int kAlloc = kBytes + 1024;         // slack to align the base to 1 KB
    static constexpr int kTmemCols = 2 * NT < 32 ? 32 : 2 * NT;  // two accumulators
    // 228 KB of shared memory per SM, 1 KB of it reserved per resident CTA
    static constexpr int kPerSm = (233472 / (kAlloc + 1024)) > 2 ? 2 : (233472 / (kAlloc + 1024));
    static_assert(kAlloc <= 232448, "shared-memory footprint above the 227 KB per-CTA limit");
    static_assert(kBoxB % 1024 == 0, "activation boxes must keep 1 KB swizzle-atom alignment");
};

// Partials of shared tiles. For decode-sized launches (M <= NK_TC_TAG_MAX_M, with few enough
// slots to poll, see the epilogue) they live in 64-bit slots {fp32 value, tag}: a rank
// publishes a value and its tag in one store, so a reader that sees the tag has the value
// without a fence, a count or a second round trip, and the reader clears the slot after use.
// The tag is a signalling-NaN bit pattern, which no arithmetic produces, so no value left by
// another plan, launch or kernel family can pose as a published slot. Other launches, whose
// partials would need many slot rounds, publish plain fp32 and then the tile's count (one
// release per CTA).
#ifndef NK_TC_TAG_MAX_M
#define NK_TC_TAG_MAX_M 8
#endif
constexpr uint32_t kSlotTag = 0x7FBADC0Du;

__device__ __forceinline__ void st_slot(uint64_t* p, float v) {
    const uint64_t x = ((uint64_t)kSlotTag << 32) | (uint64_t)__float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(x) : "memory");
}

__device__ __forceinline__ uint64_t ld_slot(const uint64_t* p) {
    uint64_t x;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(x) : "l"(p) : "memory");
    return x;
}

__device__ __forceinline__ void clear_slot(uint64_t* p) {
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"((uint64_t)0) : "memory");
}

// ps[j] += the plain fp32 partials of ranks 1, 2, ..., nseg-1 (in that order) at token
// columns c0 + j < mcount of one tile row (part0: the row's rank-0, column-0 value); the caller
// has seen the tile's count complete. The loads of up to six ranks for eight columns are in
// flight together, so a tile shared by seven CTAs costs two L2 round trips, not six.
__device__ __forceinline__ void sum_partials16(const float* part0, int part_cols, int c0,
                                               int nseg, int mcount, float (&ps)[16]) {
    constexpr int RB = 6;
#pragma unroll
    for (int h = 0; h < 16; h += 8) {
        if (c0 + h >= mcount) break;
        for (int r0 = 1; r0 < nseg; r0 += RB) {
            float p[RB][8];
#pragma unroll
            for (int i = 0; i < RB; ++i) {
                const float* pr = part0 + ((size_t)(r0 + i) * part_cols + c0 + h) * kTcRows;
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    p[i][j] = (r0 + i < nseg && c0 + h + j < mcount) ? __ldcg(pr + (size_t)j * kTcRows)
                                                                     : 0.f;
            }
#pragma unroll
            for (int i = 0; i < RB; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) ps[h + j] += p[i][j];
        }
    }
}

// ps[j] += the partials of ranks 1, 2, ..., nseg-1 (in that order) at token columns
// c0 + j < mcount of one tile row (slot0: the row's rank-0, column-0 slot), clearing each
// slot it reads. Slots are read RB ranks x CB columns at a time; while some are not yet
// published, all of those are read again together (one L2 round trip per round), bounded by
// ~2 s (then NK_ERR_TIMEOUT is recorded and false returned).
template <int RB, int CB>
__device__ __forceinline__ bool collect_rounds(uint64_t* slot0, int part_cols, int c0, int nseg,
                                               int mcount, float (&ps)[16]) {
    for (int r0 = 1; r0 < nseg; r0 += RB) {
#pragma unroll
        for (int j0 = 0; j0 < 16; j0 += CB) {
            if (c0 + j0 >= mcount) break;
            uint64_t x[RB][CB];
#pragma unroll
            for (int i = 0; i < RB; ++i)
#pragma unroll
                for (int j = 0; j < CB; ++j)
                    x[i][j] = (r0 + i < nseg && c0 + j0 + j < mcount)
                                  ? ld_slot(slot0 + ((size_t)(r0 + i) * part_cols + c0 + j0 + j) * kTcRows)
                                  : ((uint64_t)kSlotTag << 32);
            uint64_t t0 = 0;
            for (;;) {
                bool all = true;
#pragma unroll
                for (int i = 0; i < RB; ++i)
#pragma unroll
                    for (int j = 0; j < CB; ++j) all &= (uint32_t)(x[i][j] >> 32) == kSlotTag;
                if (all) break;
                if (t0 == 0) t0 = global_ns();
                if (global_ns() - t0 > 2000000000ull) {
                    atomicExch(&g_error, NK_ERR_TIMEOUT);
                    return false;
                }
                __nanosleep(32);
#pragma unroll
                for (int i = 0; i < RB; ++i)
#pragma unroll
                    for (int j = 0; j < CB; ++j)
                        if ((uint32_t)(x[i][j] >> 32) != kSlotTag)
                            x[i][j] = ld_slot(slot0 + ((size_t)(r0 + i) * part_cols + c0 + j0 + j) * kTcRows);
            }
#pragma unroll
            for (int i = 0; i < RB; ++i)
#pragma unroll
                for (int j = 0; j < CB; ++j)
                    if (r0 + i < nseg && c0 + j0 + j < mcount) {
                        ps[j0 + j] += __uint_as_float((uint32_t)x[i][j]);
                        clear_slot(slot0 + ((size_t)(r0 + i) * part_cols + c0 + j0 + j) * kTcRows);
                    }
        }
    }
    return true;
}

// The round shape follows the chunk's width: one token column reads up to 16 ranks per round
// (a small tile is shared by 5-7 CTAs), wider chunks four ranks by four columns.
__device__ __forceinline__ bool collect_partials16(uint64_t* slot0, int part_cols, int c0,
                                                   int nseg, int mcount, float (&ps)[16]) {
    const int w = mcount - c0;
    if (w <= 1) return collect_rounds<16, 1>(slot0, part_cols, c0, nseg, mcount, ps);
    if (w <= 2) return collect_rounds<8, 2>(slot0, part_cols, c0, nseg, mcount, ps);
    return collect_rounds<4, 4>(slot0, part_cols, c0, nseg, mcount, ps);
}

// Greedy head: a token's best output is its largest bf16 value, the lowest vocabulary index
// on ties (torch.argmax over the bf16 logits; a NaN counts as the largest, -0 equals +0). The
// key packs an order-preserving 16-bit image of the bf16 value above the inverted index, so
// the largest key is that (value, index); a valid key is never zero.
__device__ __forceinline__ unsigned long long amax_key(float v, int n) {
    uint32_t h = __bfloat16_as_ushort(__float2bfloat16_rn(v));
    if (h == 0x8000u) h = 0u;
    uint32_t o;
    if ((h & 0x7FFFu) > 0x7F80u) o = 0xFFFFu;
    else o = (h & 0x8000u) ? (~h & 0xFFFFu) : (h | 0x8000u);
    return ((unsigned long long)o << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)n);
}

__device__ __forceinline__ __nv_bfloat16 amax_value(unsigned long long k) {
    const uint32_t o = (uint32_t)(k >> 32);
    const uint32_t h = o == 0xFFFFu ? 0x7FC0u : (o & 0x8000u) ? (o & 0x7FFFu) : (~o & 0xFFFFu);
    return __ushort_as_bfloat16((unsigned short)h);
}

// Folds one 16-column chunk of this thread's output row n (values v, tokens m..m+cols-1) into
// the tokens' keys: a warp-wide maximum per column, then one atomicMax per warp. Every lane of
// the warp calls it; `live` is false for a lane whose row is past N or whose values are not
// final. cols is warp-uniform.
__device__ __forceinline__ void amax_fold16(const GemmArgs& a, bool live, int n, int m, int cols,
                                            const float (&v)[16]) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        if (j >= cols) break;
        unsigned long long k = live ? amax_key(v[j], n) : 0ull;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const unsigned long long o = __shfl_xor_sync(0xffffffffu, k, off);
            k = o > k ? o : k;
        }
        if ((threadIdx.x & 31) == 0 && k != 0ull)
            atomicMax(a.amax_keys + (size_t)(m + j) * (kAmaxKeyStride / 8), k);
    }
}

// One tile segment of this CTA's unit range.
struct Segment {
    int t;         // tile index
    int kb0, kb1;  // K blocks [kb0, kb1) of the tile
};

__device__ __forceinline__ Segment segment_at(int64_t u, int64_t u_end, int KB) {
    Segment sg;
    sg.t = (int)(u / KB);
    sg.kb0 = (int)(u - (int64_t)sg.t * KB);
    const int64_t tile_end = (int64_t)(sg.t + 1) * KB;
    sg.kb1 = (int)((u_end < tile_end ? u_end : tile_end) - (int64_t)sg.t * KB);
    return sg;
}

// Kernel variants (template MODE), each compiled only with its own code:
//   kModePlain: y = x · Wᵀ (nk_gemm_bf16, nk_gemm_bf16_f32out, nk_gemm_bf16_static);
//   kModeAmax:  the greedy head (nk_gemm_bf16_argmax) — folds every final output into the
//               tokens' (value, index) keys and may skip storing y;
//   kModeAr:    the K-split linear of a tensor-parallel group fused with its all-reduce
//               (nk_gemm_bf16_allreduce) — each output tile's fp32 values go straight into
//               every rank's receive buffer, and the CTA that made them adds up all ranks'
//               values of the tile in rank order and stores y.
//   kModeQkv:   the QKV linear fused with its consumer (nk_gemm_bf16_qkv_rope_cache) — each
//               output tile is one 128-wide head; the CTA that finishes it applies the
//               per-head RMSNorm and RoPE of query and key heads and writes queries, keys
//               and values where the attention reads them (decode token tiles only).
constexpr int kModePlain = 0, kModeAmax = 1, kModeAr = 2, kModeQkv = 3;

// What the kModeQkv epilogue of one head needs besides the accumulator, loaded while the
// head's last MMAs still run: the decode position and, for a query or key head, this thread's
// gain and rotary cos/sin at that position.
struct QkvOperands {
    int64_t pos;
    bool pos_ok, is_q, is_v;
    float wgt, c, sn;
};

__device__ __forceinline__ QkvOperands qkv_operands(const GemmArgs& a, int head, int d) {
    QkvOperands o;
    o.pos = *a.qk_pos;
    o.pos_ok = o.pos >= 0 && o.pos < a.qk_cap;
    o.is_q = head < a.qk_hq;
    o.is_v = head >= a.qk_hq + a.qk_hkv;  // value heads follow the keys
    o.wgt = o.c = o.sn = 0.f;
    if (!o.is_v) {
        o.wgt = __bfloat162float(o.is_q ? a.qk_qnorm[d] : a.qk_knorm[d]);
        const int64_t p = o.pos_ok ? o.pos : 0;
        o.c = __bfloat162float(a.qk_cos[p * 128 + d]);
        o.sn = __bfloat162float(a.qk_sin[p * 128 + d]);
    }
    return o;
}

// The kModeQkv epilogue for the `cols` token columns of one head tile (values v, tokens
// b0 + j): exactly nk_qk_norm_rope_cache_bf16 (nk_decode.cu) applied to the bf16-rounded
// outputs, with the same sum-of-squares order, so the same bits. All columns at once: each
// warp reduces its 32 rows of every column, one barrier, every thread normalises its element
// of every column, one barrier, the RoPE partner comes from shared memory. `sm` holds
// 16 x (4 + 128) floats. Every epilogue thread calls it (it holds CTA-wide barriers); `live`
// only gates the stores.
__device__ __forceinline__ void qkv_rope_tile(const GemmArgs& a, const QkvOperands& o,
                                              float (&v)[16], int cols, int b0, int head, int d,
                                              int quarter, int lane, bool live, float* sm) {
    const int hq = a.qk_hq, hkv = a.qk_hkv;
    if (!o.pos_ok && head == 0 && d == 0 && b0 == 0) atomicExch(&g_error, NK_ERR_RANGE);
    live = live && o.pos_ok;
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __bfloat162float(__float2bfloat16_rn(v[j]));  // bf16 qkv
    if (o.is_v) {
        const int kh = head - hq - hkv;
        if (live)
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (j < cols)
                    a.qk_v[(int64_t)(b0 + j) * a.qk_cb + (int64_t)kh * a.qk_ch + o.pos * a.qk_cs + d] =
                        __float2bfloat16_rn(v[j]);
        return;
    }
    float* red = sm;            // [16 columns][4 quarters]
    float* xs = sm + 16 * 4;    // [16 columns][128]
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const float s = warp_sum(v[j] * v[j]);
        if (lane == 0 && j < cols) red[j * 4 + quarter] = s;
    }
    epi_bar();
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        if (j < cols) {
            const float* r = red + j * 4;
            const float ss = (r[0] + r[2]) + (r[1] + r[3]);  // the block_sum order
            const float inv = rsqrtf(ss / 128.f + a.qk_eps);
            v[j] = __bfloat162float(__float2bfloat16_rn(
                __bfloat162float(__float2bfloat16_rn(v[j] * inv)) * o.wgt));  // normalised
            xs[j * 128 + d] = v[j];
        }
    }
    epi_bar();
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        if (j < cols) {
            const float other = xs[j * 128 + ((d + 64) & 127)];
            const float rotated = d < 64 ? -other : other;
            const float y = __bfloat162float(__float2bfloat16_rn(v[j] * o.c)) +
                            __bfloat162float(__float2bfloat16_rn(rotated * o.sn));
            if (live) {
                const int b = b0 + j;
                if (o.is_q)
                    a.qk_q[((int64_t)b * hq + head) * 128 + d] = __float2bfloat16_rn(y);
                else
                    a.qk_k[(int64_t)b * a.qk_cb + (int64_t)(head - hq) * a.qk_ch + o.pos * a.qk_cs +
                           d] = __float2bfloat16_rn(y);
            }
        }
    }
    epi_bar();  // `sm` is free again for the next head
}

// qkv_rope_tile for a head whose CTA's ring is still in use: the same arithmetic, one column
// at a time through `sm` (2 x (4 + 128) floats, alternating between columns).
__device__ __forceinline__ void qkv_rope_columns(const GemmArgs& a, const QkvOperands& o,
                                                 float (&v)[16], int cols, int b0, int head,
                                                 int d, int quarter, int lane, bool live,
                                                 float* sm) {
    const int hq = a.qk_hq, hkv = a.qk_hkv;
    if (!o.pos_ok && head == 0 && d == 0 && b0 == 0) atomicExch(&g_error, NK_ERR_RANGE);
    live = live && o.pos_ok;
#pragma unroll 1
    for (int j = 0; j < cols; ++j) {
        float x = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i)
            if (i == j) x = v[i];
        x = __bfloat162float(__float2bfloat16_rn(x));  // bf16 qkv
        const int b = b0 + j;
        if (o.is_v) {
            if (live)
                a.qk_v[(int64_t)b * a.qk_cb + (int64_t)(head - hq - hkv) * a.qk_ch +
                       o.pos * a.qk_cs + d] = __float2bfloat16_rn(x);
            continue;
        }
        float* red = sm + (j & 1) * (4 + 128);
        float* xs = red + 4;
        const float s = warp_sum(x * x);
        if (lane == 0) red[quarter] = s;
        epi_bar();
        const float ss = (red[0] + red[2]) + (red[1] + red[3]);  // the block_sum order
        const float inv = rsqrtf(ss / 128.f + a.qk_eps);
        const float xn = __bfloat162float(__float2bfloat16_rn(
            __bfloat162float(__float2bfloat16_rn(x * inv)) * o.wgt));
        xs[d] = xn;
        epi_bar();
        const float other = xs[(d + 64) & 127];
        const float rotated = d < 64 ? -other : other;
        const float y = __bfloat162float(__float2bfloat16_rn(xn * o.c)) +
                        __bfloat162float(__float2bfloat16_rn(rotated * o.sn));
        if (live) {
            if (o.is_q)
                a.qk_q[((int64_t)b * hq + head) * 128 + d] = __float2bfloat16_rn(y);
            else
                a.qk_k[(int64_t)b * a.qk_cb + (int64_t)(head - hq) * a.qk_ch + o.pos * a.qk_cs + d] =
                    __float2bfloat16_rn(y);
        }
    }
    if (!o.is_v) epi_bar();  // `sm` is free again for the next head
}

// The fused all-reduce's final value of output (m, n): this rank's fp32 value into the tile's
// slot of every rank of the group (the sum follows once every rank has published the tile).
__device__ __forceinline__ void ar_publish(const GemmArgs& a, int set, int m, int n, float v) {
    const size_t off = (size_t)m * a.N + n;
    for (int r = 0; r < a.ar_world; ++r)
        ar_slot(a.ar_buf[r], set, a.ar_rank, a.ar_world, a.ar_max_elems)[off] = v;
}

template <int NT, int MODE>
__global__ void __launch_bounds__(tc_threads(NT)) __maxnreg__(tc_maxnreg(NT))
tc_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
          GemmArgs a) {
    constexpr bool AMAX = MODE == kModeAmax;
    constexpr bool AR = MODE == kModeAr;
    constexpr bool QKV = MODE == kModeQkv;
    static_assert(!QKV || NT == 16, "the fused QKV epilogue takes decode token tiles");
    static_assert(((tc_threads(NT) / 32 + 3) / 4) * 32 * tc_maxnreg(NT) <= 16384,
                  "one CTA's warps must fit a sub-partition's register file");
    constexpr int kTcUK = tc_uk(NT);       // boxes along K per stage
    constexpr int kTcKStep = tc_kstep(NT);  // K elements per unit
    using L = TcSmem<NT, QKV ? kQkvSmemBytes : 0>;
    constexpr int STAGES = L::kStages;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* gbase = smem_raw + (base - raw);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const TcPartition& P = a.part_map;
    const int c = blockIdx.x;
    const int64_t u_begin = P.begin(c);
    const int64_t u_end = P.begin(c + 1);
    const int n_units = (int)(u_end - u_begin);
    const int KB = P.KB;

    const uint32_t bar_full = base + L::kBarOff;
    const uint32_t bar_empty = bar_full + STAGES * 8;
    const uint32_t bar_tfull = bar_empty + STAGES * 8;
    const uint32_t bar_tempty = bar_tfull + 2 * 8;
    const uint32_t bar_part = bar_tempty + 2 * 8;
    volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(gbase + L::kMiscOff);
    volatile uint32_t* tmem_slot = misc;
    volatile uint32_t* abort_flag = misc + 1;
    volatile uint32_t* last_flag = misc + 2;
    volatile uint32_t* ar_call = misc + 3;  // fused all-reduce: this tile's call number
    volatile uint32_t* ar_ok = misc + 4;    // fused all-reduce: every rank's tile arrived
    float* qk_smem = reinterpret_cast<float*>(gbase + L::kMiscOff + 32);  // kModeQkv epilogue

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(bar_full + 8 * i, 1);
            mbar_init(bar_empty + 8 * i, 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(bar_tfull + 8 * i, 1);
            mbar_init(bar_tempty + 8 * i, tc_epi_warps(NT));
        }
        for (int i = 0; i < L::kPartBars; ++i) mbar_init(bar_part + 8 * i, 1);
        *abort_flag = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tma_prefetch_desc(&tmap_w);
        tma_prefetch_desc(&tmap_x);
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32((const void*)tmem_slot)),
                     "r"((uint32_t)L::kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (threadIdx.x == 0) griddep_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            const int n_pre = n_units < STAGES ? n_units : STAGES;
            const uint64_t wpol = l2_evict_first_policy();
            // The first stages' weight tiles need nothing from the previous kernel.
            for (int i = 0; i < n_pre; ++i) {
                const int64_t u = u_begin + i;
                const int t = (int)(u / KB);
                const int kb = (int)(u - (int64_t)t * KB);
                mbar_expect_tx(bar_full + 8 * i, (uint32_t)L::kStage);
#pragma unroll
                for (int ub = 0; ub < kTcUK; ++ub)
                    tma_load_w(base + i * L::kStage + ub * L::kBoxA, &tmap_w, bar_full + 8 * i,
                               kb * kTcKStep + ub * kTcBox, (t % a.n_tiles) * kTcRows, wpol);
            }
            griddep_wait();
            for (int i = 0; i < n_pre; ++i) {
                const int64_t u = u_begin + i;
                const int t = (int)(u / KB);
                const int kb = (int)(u - (int64_t)t * KB);
#pragma unroll
                for (int ub = 0; ub < kTcUK; ++ub)
                    tma_load_2d(base + i * L::kStage + L::kA + ub * L::kBoxB, &tmap_x,
                                bar_full + 8 * i, kb * kTcKStep + ub * kTcBox, (t / a.n_tiles) * NT);
            }
            int issued = n_pre;
            for (int i = n_pre; i < n_units; ++i) {
                const int st = i % STAGES;
                const uint32_t use = (uint32_t)(i / STAGES);
                if (!mbar_wait(bar_empty + 8 * st, (use & 1u) ^ 1u)) { *abort_flag = 1u; break; }
                if (*abort_flag) break;
                const int64_t u = u_begin + i;
                const int t = (int)(u / KB);
                const int kb = (int)(u - (int64_t)t * KB);
                const uint32_t sa = base + st * L::kStage;
                mbar_expect_tx(bar_full + 8 * st, (uint32_t)L::kStage);
#pragma unroll
                for (int ub = 0; ub < kTcUK; ++ub)
                    tma_load_w(sa + ub * L::kBoxA, &tmap_w, bar_full + 8 * st,
                               kb * kTcKStep + ub * kTcBox, (t % a.n_tiles) * kTcRows, wpol);
#pragma unroll
                for (int ub = 0; ub < kTcUK; ++ub)
                    tma_load_2d(sa + L::kA + ub * L::kBoxB, &tmap_x, bar_full + 8 * st,
                                kb * kTcKStep + ub * kTcBox, (t / a.n_tiles) * NT);
                ++issued;
            }
            // Drain: every stage's last load has landed and (unless the MMA issuer gave up)
            // every MMA that read it has completed before this CTA may exit.
            for (int i = (issued > STAGES ? issued - STAGES : 0); i < issued; ++i) {
                const int st = i % STAGES;
                const uint32_t use = (uint32_t)(i / STAGES);
                mbar_wait(bar_full + 8 * st, use & 1u);
                if (*abort_flag == 0u) mbar_wait(bar_empty + 8 * st, use & 1u);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t idesc = tc_idesc(kTcRows, NT);
            int i = 0, seg = 0;
            for (int64_t u = u_begin; u < u_end; ++seg) {
                const Segment sg = segment_at(u, u_end, KB);
                const int buf = seg & 1;
                const uint32_t use_b = (uint32_t)(seg >> 1);
                if (!mbar_wait(bar_tempty + 8 * buf, (use_b & 1u) ^ 1u)) { *abort_flag = 1u; break; }
                tc_fence_after();
                const uint32_t dacc = tmem + (uint32_t)(buf * NT);
                bool stop = false;
                for (int kb = sg.kb0; kb < sg.kb1; ++kb, ++i) {
                    const int st = i % STAGES;
                    const uint32_t use = (uint32_t)(i / STAGES);
                    if (!mbar_wait(bar_full + 8 * st, use & 1u)) { stop = true; break; }
                    tc_fence_after();
                    const uint32_t sa = base + st * L::kStage;
                    const uint32_t sb = sa + L::kA;
#pragma unroll
                    for (int ub = 0; ub < kTcUK; ++ub)
#pragma unroll
                        for (int j = 0; j < kTcBox / 16; ++j)  // 32 bytes of K per MMA
                            tc_mma(dacc, sw128_desc(sa + ub * L::kBoxA + 32 * j),
                                   sw128_desc(sb + ub * L::kBoxB + 32 * j), idesc,
                                   (kb > sg.kb0 || ub > 0 || j > 0) ? 1u : 0u);
                    tc_commit(bar_empty + 8 * st);
                }
                tc_commit(bar_tfull + 8 * buf);  // arrives when this segment's MMAs are done
                if (stop) { *abort_flag = 1u; break; }
                u += sg.kb1 - sg.kb0;
            }
        }
    } else {
        // ---------------- epilogue (warps 2 and up) ----------------
        griddep_wait();
        constexpr int kEpiW = tc_epi_warps(NT);
        constexpr int kEpiT = 32 * kEpiW;
        constexpr int kHalves = kEpiW / 4;        // warps sharing one TMEM lane quarter
        // which of them this warp is (a constant 0 with one warp per quarter, so that the
        // decode token tile's single-chunk loops fold as before)
        const int half = kHalves > 1 ? (warp - 2) >> 2 : 0;
        const int ep = threadIdx.x - 64;          // 0..kEpiT-1
        const int q = warp & 3;                   // TMEM lane quarter this warp may access
        const int row = 32 * q + lane;            // tile row owned by this thread
        const uint32_t tlane = (uint32_t)(32 * q) << 16;
        const bool wait_mode = a.coresident != 0;
        // Tagged slots cost rank 0 a poll of every partner's slot of every column; the count
        // protocol a fixed handful of round trips. Measured on B200 (Qwen3-8B, M = 8): tagged
        // wins QKV (11.8 vs 12.3 us) and gate_up (33.4 vs 33.7), loses o_proj (10.7 vs 9.7)
        // and down (20.8 vs 20.3), whose tiles are shared by 7 and 6 CTAs; M <= 4 always
        // tagged, M = 16 always counted. The same for every CTA of the launch.
        const bool tagged = wait_mode && a.M <= NK_TC_TAG_MAX_M &&
                            a.M * (a.seg_max - 1) <= 4 * NK_TC_TAG_MAX_M;
        const bool store_y = !AMAX || a.y != nullptr;            // the greedy head may skip y
        int seg = 0;
        for (int64_t u = u_begin; u < u_end; ++seg) {
            const Segment sg = segment_at(u, u_end, KB);
            u += sg.kb1 - sg.kb0;
            const int buf = seg & 1;
            const int n = (sg.t % a.n_tiles) * kTcRows + row;
            const int m0 = (sg.t / a.n_tiles) * NT;
            const int mcount = min(NT, a.M - m0);
            const bool whole = (sg.kb0 == 0 && sg.kb1 == KB);
            const int first = P.first_cta(sg.t);
            const int rank = c - first;
            const int nseg = whole ? 1 : P.last_cta(sg.t) - first + 1;
            // This row's partials of the tile, [rank][token column], 128 rows apart: 64-bit
            // tagged slots, or plain fp32 in the same region.
            const size_t row0 = ((size_t)sg.t * a.segments * a.part_cols) * kTcRows + row;
            uint64_t* const slot0 = reinterpret_cast<uint64_t*>(a.part) + row0;
            float* const part0 = a.part + row0;
            const bool finisher = !whole && rank == 0 && wait_mode;
            // Failure-detection tests only: this CTA keeps its partial to itself, so the tile's
            // finisher's bounded wait runs out (NK_ERR_TIMEOUT) instead of completing.
            const bool withhold = wait_mode && rank == 1 && sg.t == a.withhold_tile;
            // Fused QKV epilogue: the head's position, gain and rotary operands, loaded while the
            // head's last MMAs still run.
            QkvOperands qo{};
            if constexpr (QKV) {
                if (whole || finisher) qo = qkv_operands(a, sg.t, row);
            }
            // Fused all-reduce: the call number of this output tile (its progress counter in
            // this rank's receive buffer, plus one) picks the set of flags and slots.
            unsigned ar_e = 0;
            int ar_set = 0;
            if constexpr (AR) {
                if (whole || finisher) {
                    if (ep == 0) *ar_call = *ar_counter(a.ar_buf[a.ar_rank], sg.t) + 1u;
                    epi_bar_n<kEpiT>();
                    ar_e = *ar_call;
                    ar_set = (int)(ar_e & 1u);
                }
            }
            // Rank 0 of a shared tile holds the tile's first K blocks as its last segment; the
            // other ranks (higher CTAs) hold the rest. It waits for them while its own last
            // MMAs still run and, for the decode token tile, already adds up their partials
            // (rank 1 + rank 2 + ...), so that once its accumulator is ready only own + that
            // sum is left.
            float psum[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) psum[j] = 0.f;
            bool got = true;
            if (finisher && !tagged) {
                // one thread acquires the count; the barrier orders every thread's partial
                // loads (through L2) after that acquire
                if (ep == 0)
                    *last_flag = spin_until_count(a.tickets + sg.t, (unsigned)(nseg - 1)) ? 1u : 0u;
                epi_bar_n<kEpiT>();
                got = *last_flag != 0u;
            }
            if constexpr (NT == 16) {
                if (finisher) {
                    if (tagged) got = collect_partials16(slot0, a.part_cols, 0, nseg, mcount, psum);
                    else if (got) sum_partials16(part0, a.part_cols, 0, nseg, mcount, psum);
                }
                __syncwarp();  // lanes polled for different times; converge before tcgen05.ld
            }
            // warp-uniform (and a convergence point) before the warp-wide tcgen05.ld below
            const bool ok = __all_sync(0xffffffffu,
                                       mbar_wait(bar_tfull + 8 * buf, (uint32_t)(seg >> 1) & 1u) &&
                                           *abort_flag == 0u);
            tc_fence_after();
            const uint32_t taddr = tmem + (uint32_t)(buf * NT) + tlane;
            // tcgen05.ld is a warp-wide instruction: every lane of the warp executes it, and
            // only the stores depend on the lane's row (n < N) or on what it collected.
            if (whole) {
                if constexpr (QKV) {
                    // barriers inside: every thread takes every column, whatever `ok`
                    float v[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = 0.f;
                    if (ok) tmem_ld16(taddr, v);
                    // a head finished last has the idle ring to work in; one in the middle of
                    // this CTA's range (whose ring still streams) goes column by column
                    if (u >= u_end)
                        qkv_rope_tile(a, qo, v, mcount, m0, sg.t, row, q, lane, ok,
                                      reinterpret_cast<float*>(gbase));
                    else
                        qkv_rope_columns(a, qo, v, mcount, m0, sg.t, row, q, lane, ok, qk_smem);
                } else if (ok) {
#pragma unroll 1
                    for (int c0 = 16 * half; c0 < NT; c0 += 16 * kHalves) {
                        if (c0 >= mcount) break;  // warp-uniform
                        float v[16];
                        tmem_ld16(taddr + c0, v);
                        if constexpr (AR) {
                            if (n < a.N)
#pragma unroll
                                for (int j = 0; j < 16; ++j)
                                    if (c0 + j < mcount) ar_publish(a, ar_set, m0 + c0 + j, n, v[j]);
                        } else if (store_y && n < a.N) {
#pragma unroll
                            for (int j = 0; j < 16; ++j)
                                if (c0 + j < mcount)
                                    store_out(a, (int64_t)(m0 + c0 + j) * a.ldy + n, v[j]);
                        }
                        if constexpr (AMAX) amax_fold16(a, n < a.N, n, m0 + c0, min(16, mcount - c0), v);
                    }
                }
            } else if (!finisher) {
                // Publish this rank's fp32 partial: as tagged slots (a value and its tag in one
                // 64-bit store, so no fence or count follows), or as plain fp32 followed below
                // by a fence and the tile's count.
                if (ok && !withhold) {
#pragma unroll 1
                    for (int c0 = 16 * half; c0 < NT; c0 += 16 * kHalves) {
                        if (c0 >= mcount) break;  // warp-uniform
                        float v[16];
                        tmem_ld16(taddr + c0, v);
                        const size_t off = ((size_t)rank * a.part_cols + c0) * kTcRows;
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            if (c0 + j < mcount) {
                                if (tagged) st_slot(slot0 + off + (size_t)j * kTcRows, v[j]);
                                else part0[off + (size_t)j * kTcRows] = v[j];
                            }
                    }
                }
            } else {
                // own + (rank 1 + rank 2 + ...): a fixed order, whichever rank is late
                constexpr uint32_t kChunkBytes = 16u * kTcRows * 4u;  // 16 columns of one rank
                constexpr uint32_t kRing = (uint32_t)(STAGES * L::kStage);
                const int partners = nseg - 1;
                const int nchunks = (mcount + 15) / 16;
                // chunk slots in the idle ring: as many chunks in flight as fit (and barriers)
                int slots = partners >= 1 ? (int)(kRing / ((uint32_t)partners * kChunkBytes)) : 0;
                slots = slots < L::kPartBars ? slots : L::kPartBars;
                slots = slots < nchunks ? slots : nchunks;
                const bool bulk = NT != 16 && !tagged && got && slots >= kHalves;
                if (ok && bulk) {
                    // Every MMA of this CTA is done, so the shared-memory ring is idle: pull each
                    // partner's partial columns [16k, 16k + 16) — contiguous fp32, [column][128
                    // rows] — with one bulk copy per rank into slot k % slots of the ring, up to
                    // `slots` chunks in flight, and add them from shared memory.
                    const uint32_t slot_bytes = (uint32_t)partners * kChunkBytes;
                    const float* tile_part =
                        a.part + ((size_t)sg.t * a.segments * a.part_cols) * kTcRows;
                    auto issue = [&](int k) {  // one thread
                        const int h = k % slots;
                        const int cols = min(16, a.part_cols - 16 * k);  // never past the tile
                        const uint32_t bytes = (uint32_t)cols * kTcRows * 4u;
                        mbar_expect_tx(bar_part + 8 * h, (uint32_t)partners * bytes);
                        for (int i = 0; i < partners; ++i)
                            bulk_load(base + h * slot_bytes + (uint32_t)i * kChunkBytes,
                                      tile_part + ((size_t)(1 + i) * a.part_cols + 16 * k) * kTcRows,
                                      bytes, bar_part + 8 * h);
                    };
                    if (ep == 0) {
                        // the partners' stores (acquired above through the generic proxy)
                        // before the async-proxy copies that read them
                        asm volatile("fence.proxy.async.global;" ::: "memory");
                        for (int k = 0; k < slots; ++k) issue(k);
                    }
#pragma unroll 1
                    for (int r0 = 0; r0 < nchunks; r0 += kHalves) {
                        const int k = r0 + half;  // this warp's chunk of the round
                        if (k < nchunks) {
                            const int h = k % slots;
                            const bool arrived = __all_sync(
                                0xffffffffu, mbar_wait(bar_part + 8 * h, (uint32_t)(k / slots) & 1u));
                            float v[16];
                            tmem_ld16(taddr + 16 * k, v);
                            const float* sm =
                                reinterpret_cast<const float*>(gbase + h * slot_bytes) + row;
                            float ps[16];
#pragma unroll
                            for (int j = 0; j < 16; ++j) ps[j] = 0.f;
                            for (int i = 0; i < partners; ++i)
#pragma unroll
                                for (int j = 0; j < 16; ++j) ps[j] += sm[(i * 16 + j) * kTcRows];
#pragma unroll
                            for (int j = 0; j < 16; ++j) v[j] += ps[j];
                            if constexpr (AR) {
                                if (arrived && n < a.N)
#pragma unroll
                                    for (int j = 0; j < 16; ++j)
                                        if (16 * k + j < mcount)
                                            ar_publish(a, ar_set, m0 + 16 * k + j, n, v[j]);
                            } else if (store_y && arrived && n < a.N) {
#pragma unroll
                                for (int j = 0; j < 16; ++j)
                                    if (16 * k + j < mcount)
                                        store_out(a, (int64_t)(m0 + 16 * k + j) * a.ldy + n, v[j]);
                            }
                            if constexpr (AMAX)
                                amax_fold16(a, arrived && n < a.N, n, m0 + 16 * k,
                                            min(16, mcount - 16 * k), v);
                        }
                        // every chunk of the round is done with its slot: refill those slots
                        if (r0 + slots < nchunks) {
                            epi_bar_n<kEpiT>();
                            if (ep == 0) {
                                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                                for (int kk = r0; kk < r0 + kHalves && kk + slots < nchunks; ++kk)
                                    issue(kk + slots);
                            }
                        }
                    }
                } else if (QKV) {
                    // the decode token tile: partners' partials were summed into psum above
                    float v[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = 0.f;
                    if (ok) tmem_ld16(taddr, v);
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] += psum[j];
                    // the finishing segment is this CTA's last: its ring is idle
                    qkv_rope_tile(a, qo, v, mcount, m0, sg.t, row, q, lane, ok && got,
                                  reinterpret_cast<float*>(gbase));
                } else if (ok) {
#pragma unroll 1
                    for (int c0 = 16 * half; c0 < NT; c0 += 16 * kHalves) {
                        if (c0 >= mcount) break;  // warp-uniform
                        if constexpr (NT != 16) {
#pragma unroll
                            for (int j = 0; j < 16; ++j) psum[j] = 0.f;
                            if (tagged) got = collect_rounds<4, 4>(slot0, a.part_cols, c0, nseg, mcount, psum);
                            else if (got) sum_partials16(part0, a.part_cols, c0, nseg, mcount, psum);
                            __syncwarp();  // converge before tcgen05.ld
                        }
                        float v[16];
                        tmem_ld16(taddr + c0, v);
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[j] += psum[j];
                        if constexpr (AR) {
                            if (got && n < a.N)
#pragma unroll
                                for (int j = 0; j < 16; ++j)
                                    if (c0 + j < mcount) ar_publish(a, ar_set, m0 + c0 + j, n, v[j]);
                        } else if (store_y && got && n < a.N) {
#pragma unroll
                            for (int j = 0; j < 16; ++j)
                                if (c0 + j < mcount)
                                    store_out(a, (int64_t)(m0 + c0 + j) * a.ldy + n, v[j]);
                        }
                        if constexpr (AMAX)
                            amax_fold16(a, got && n < a.N, n, m0 + c0, min(16, mcount - c0), v);
                    }
                }
                if (!tagged && ep == 0) a.tickets[sg.t] = 0u;  // re-armed for the next launch
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_tempty + 8 * buf);
            if (!whole && wait_mode && !tagged && rank > 0) {
                // this CTA's partial stores (ordered before the barrier), then one release
                epi_bar_n<kEpiT>();
                if (ep == 0 && !withhold) count_release(a.tickets + sg.t);
            } else if (!whole && !wait_mode) {
                // Without a co-resident grid every rank publishes plain partials (rank 0 above as
                // well) and the CTA whose arrival completes the tile's count sums them, in the
                // same order as the waiting scheme: rank 0 + (rank 1 + rank 2 + ...).
                __threadfence();
                epi_bar_n<kEpiT>();
                if (ep == 0) {
                    const unsigned prev = atomicAdd(a.tickets + sg.t, 1u);
                    *last_flag = (prev == (unsigned)(nseg - 1)) ? 1u : 0u;
                }
                epi_bar_n<kEpiT>();
                if (*last_flag) {
                    __threadfence();
                    const bool live = n < a.N && *abort_flag == 0u;
                    for (int c0 = 16 * half; c0 < mcount; c0 += 16 * kHalves) {
                        float ps[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j) ps[j] = 0.f;
                        if (live) {
                            sum_partials16(part0, a.part_cols, c0, nseg, mcount, ps);
#pragma unroll
                            for (int j = 0; j < 16; ++j)
                                if (c0 + j < mcount) {
                                    ps[j] += __ldcg(part0 + ((size_t)c0 + j) * kTcRows);
                                    if (store_y)
                                        store_out(a, (int64_t)(m0 + c0 + j) * a.ldy + n, ps[j]);
                                }
                        }
                        if constexpr (AMAX)
                            amax_fold16(a, live, n, m0 + c0, min(16, mcount - c0), ps);
                    }
                    if (ep == 0) a.tickets[sg.t] = 0u;  // re-armed for the next launch
                }
                epi_bar_n<kEpiT>();  // last_flag is rewritten by the next partial segment
            }
            if constexpr (AR) {
                if (whole || finisher) {
                    // This rank's values of the tile are in every rank's slot: publish the call
                    // number to every rank, wait (bounded) for every rank's, and store the sum of
                    // the ranks' values in rank order, rounded once to bf16.
                    uint8_t* own = a.ar_buf[a.ar_rank];
                    __threadfence_system();  // this thread's slot stores, before the flags
                    if (ep == 0) *ar_ok = 1u;
                    epi_bar_n<kEpiT>();
                    if (ep < a.ar_world)
                        st_release_sys(ar_flag(a.ar_buf[ep], ar_set, a.ar_rank, sg.t), ar_e);
                    if (ep < a.ar_world) {
                        const unsigned* f = ar_flag(own, ar_set, ep, sg.t);
                        const uint64_t t0 = global_ns();
                        while (ld_acquire_sys(f) != ar_e) {
                            if (global_ns() - t0 > 2000000000ull) {
                                atomicExch(&g_error, NK_ERR_TIMEOUT);
                                *ar_ok = 0u;
                                break;
                            }
                            __nanosleep(64);
                        }
                    }
                    epi_bar_n<kEpiT>();
                    if (*ar_ok && n < a.N) {
                        for (int j = half; j < mcount; j += kHalves) {
                            const size_t off = (size_t)(m0 + j) * a.N + n;
                            float acc =
                                __ldcg(ar_slot(own, ar_set, 0, a.ar_world, a.ar_max_elems) + off);
                            for (int r = 1; r < a.ar_world; ++r)
                                acc += __ldcg(ar_slot(own, ar_set, r, a.ar_world, a.ar_max_elems) + off);
                            a.y[(int64_t)(m0 + j) * a.ldy + n] = __float2bfloat16_rn(acc);
                        }
                    }
                    if (ep == 0) *ar_counter(own, sg.t) = ar_e;
                }
            }
        }
        if constexpr (AMAX) {
            // The CTA whose arrival completes the count turns the keys into indices and
            // leaves keys and count zero for the next call.
            __threadfence();  // this thread's key updates, before the CTA's arrival
            epi_bar_n<kEpiT>();
            if (ep == 0) *last_flag = atomicAdd(a.amax_done, 1u) == gridDim.x - 1 ? 1u : 0u;
            epi_bar_n<kEpiT>();
            if (*last_flag) {
                __threadfence();
                for (int m = ep; m < a.M; m += kEpiT) {
                    const unsigned long long k =
                        atomicExch(a.amax_keys + (size_t)m * (kAmaxKeyStride / 8), 0ull);
                    a.amax_idx[m] = k ? (int64_t)(0xFFFFFFFFu - (uint32_t)k) : (int64_t)-1;
                    if (a.amax_best) a.amax_best[m] = amax_value(k);
                }
                if (ep == 0) atomicExch(a.amax_done, 0u);
            }
        }
    }

    // ---------------- teardown ----------------
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"((uint32_t)L::kTmemCols)
                     : "memory");
    }
}

// ---------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

static int get_encoder() {
    if (g_encode) return NK_OK;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
        return NK_ERR_CUDA;
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    return NK_OK;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix with row stride ld (elements),
// box [box_rows, 64 columns], 128-byte swizzle; out-of-range rows and columns read as zero.
static int make_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, int64_t ld,
                    int box_rows) {
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
    cuuint32_t box[2] = {(cuuint32_t)kTcBox, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims,
                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, (CUtensorMapL2promotion)NK_TC_L2_PROMO,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? NK_OK : NK_ERR_ALIGN;
}

#ifndef NK_TC_MAX_NT
#define NK_TC_MAX_NT 128  // widest token tile a plan may choose
#endif

int tc_token_tile(int M_max) {
    int nt = 256;
    if (M_max <= 16) nt = 16;
    else if (M_max <= 32) nt = 32;
    else if (M_max <= 64) nt = 64;
    else if (M_max <= 128) nt = 128;
    return nt < NK_TC_MAX_NT ? nt : NK_TC_MAX_NT;
}

int tc_stages(int nt) {
    switch (nt) {
        case 16: return TcSmem<16>::kStages;
        case 32: return TcSmem<32>::kStages;
        case 64: return TcSmem<64>::kStages;
        case 128: return TcSmem<128>::kStages;
        default: return TcSmem<256>::kStages;
    }
}

#ifndef NK_TC_GRID_PER_SM
#define NK_TC_GRID_PER_SM 0  // 0: as many CTAs per SM as shared memory allows
#endif

int tc_ctas_per_sm(int nt) {
    if (NK_TC_GRID_PER_SM > 0) return NK_TC_GRID_PER_SM;
    switch (nt) {
        case 16: return TcSmem<16>::kPerSm;
        case 32: return TcSmem<32>::kPerSm;
        case 64: return TcSmem<64>::kPerSm;
        case 128: return TcSmem<128>::kPerSm;
        default: return TcSmem<256>::kPerSm;
    }
}

// CTAs of tc_kernel<NT, MODE> that fit on one SM at once. The runtime's occupancy query answers 1
// for every kernel that executes tcgen05.alloc (on B200 even for a 12-register kernel), but
// the block scheduler places such CTAs by registers, shared memory and threads: 296 CTAs
// that each hold 32 TMEM columns run on 148 SMs as one wave, two overlapping on every SM.
// So the count is made here from those limits, plus the 512 TMEM columns of an SM (so no
// CTA blocks in tcgen05.alloc), and capped at the per-SM count the stage budget assumes.
template <int NT, int MODE>
static int tc_resident_per_sm(int dev) {
    using L = TcSmem<NT, MODE == kModeQkv ? kQkvSmemBytes : 0>;
    cudaFuncAttributes fa;
    int smem_sm = 0, reserved = 0, regs_sm = 0, thr_sm = 0;
    if (cudaFuncGetAttributes(&fa, tc_kernel<NT, MODE>) != cudaSuccess ||
        cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) !=
            cudaSuccess ||
        cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev) !=
            cudaSuccess ||
        cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev) !=
            cudaSuccess ||
        cudaDeviceGetAttribute(&thr_sm, cudaDevAttrMaxThreadsPerMultiProcessor, dev) !=
            cudaSuccess)
        return 0;
    constexpr int kWarps = tc_threads(NT) / 32;
    // registers: 8-register steps per thread, and each of the 4 sub-partitions holds its
    // quarter of the register file for at most ceil(warps / 4) warps of every CTA
    const int regs_warp = ((fa.numRegs + 7) & ~7) * 32;
    const int by_regs = (regs_sm / 4) / (regs_warp * ((kWarps + 3) / 4));
    const int by_smem = smem_sm / (L::kAlloc + (int)fa.sharedSizeBytes + reserved);
    const int by_thr = thr_sm / tc_threads(NT);
    const int by_tmem = 512 / L::kTmemCols;
    int n = L::kPerSm;
    for (int lim : {by_regs, by_smem, by_thr, by_tmem}) n = lim < n ? lim : n;
    return n;
}

// K blocks added to the rank-0 slice of each tile in the tile-aligned schedule. All of a
// tile's CTAs stream equal slices, so they finish together and the partners' publishing, the
// count and rank 0's poll (~2 us at M = 16) all follow the streaming; a longer rank-0 slice
// (taken evenly from the partners) hides them behind rank 0's own streaming. Measured on B200,
// 20 chained launches, us (no lead -> this lead): Qwen3-8B QKV M=1 9.54 -> 9.27, M=8
// 11.13 -> 10.39, M=16 12.39 -> 11.46; o_proj M=8 9.55 -> 9.14, M=16 10.27 -> 9.73; down
// M=16 20.09 -> 19.83; Qwen3-0.6B down M=16 8.14 -> 7.54. Tiles split 7 or more ways (o_proj,
// down) take a longer lead than QKV's 6-way tiles, which lost with it; tiles of fewer than 16
// K blocks (0.6B QKV) lost with any lead, and short tiles lost it under the tagged protocol.
static int tc_lead(int KB, int slices, bool tagged) {
    if (KB >= 32)
        return tagged ? NK_TC_LEAD_TAGGED
                      : (slices >= 7 ? NK_TC_LEAD_COUNTED_WIDE : NK_TC_LEAD_COUNTED);
    if (KB >= 16) return tagged ? 0 : NK_TC_LEAD_COUNTED_SHORT;
    return 0;
}

template <int NT, int MODE>
static int launch_tc_t(const nk_plan& p, GemmArgs& a, const CUtensorMap& mw,
                       const CUtensorMap& mx, cudaStream_t s) {
    using L = TcSmem<NT, MODE == kModeQkv ? kQkvSmemBytes : 0>;
    static int resident[64] = {};  // co-resident CTAs per device (0 = not yet counted)
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return NK_ERR_CUDA;
    if (dev < 0 || dev >= 64) return NK_ERR_DEVICE;
    if (resident[dev] == 0) {
        if (cudaFuncSetAttribute(tc_kernel<NT, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 L::kAlloc) != cudaSuccess ||
            cudaFuncSetAttribute(tc_kernel<NT, MODE>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 (int)cudaSharedmemCarveoutMaxShared) != cudaSuccess)
            return NK_ERR_CUDA;
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return NK_ERR_CUDA;
        const int per_sm = tc_resident_per_sm<NT, MODE>(dev);
        if (per_sm < 1) return NK_ERR_CUDA;
        resident[dev] = per_sm * sms;
    }
    TcPartition& P = a.part_map;
    const int64_t tiles = P.U / P.KB;
    if (p.split_k > 0) {
        P.G = (int)tiles * p.split_k;
        a.seg_max = p.split_k;
    } else if (p.slices > 0 && tiles * p.slices <= resident[dev]) {
        // the tile-aligned schedule: one K slice per CTA, the whole grid resident (every mode
        // takes it, so that the fused forms add the same partials in the same order as the
        // plain launches they replace)
        P.split = p.slices;
        const bool tagged = a.M <= NK_TC_TAG_MAX_M &&
                            a.M * (p.slices - 1) <= 4 * NK_TC_TAG_MAX_M;  // as the epilogue decides
        P.lead = tc_lead(P.KB, p.slices, tagged);
        P.G = (int)(tiles * p.slices);
        a.seg_max = p.slices;
    } else {
        // Keep at least the plan's units per CTA, so no tile is shared by more CTAs than the
        // plan's `segments` (the workspace was sized for that); never more CTAs than can be
        // resident at once.
        const int64_t U_plan = (int64_t)p.n_tiles * p.m_tiles * P.KB;
        const int64_t q = U_plan / p.grid;
        int64_t G = P.U / q;
        if (G > p.grid) G = p.grid;
        if (G > resident[dev]) G = resident[dev];
        if (G < 1) G = 1;
        P.G = (int)G;
        const int64_t qc = P.U / G;  // fewest units a CTA holds
        const int64_t seg = 1 + (P.KB - 1 + qc - 1) / qc;
        a.seg_max = (int)(seg < a.segments ? seg : a.segments);
    }
    a.coresident = P.G <= resident[dev] ? 1 : 0;
    // The fused all-reduce and QKV epilogues finish every tile in the waiting protocol: the
    // whole grid resident.
    if ((MODE == kModeAr || MODE == kModeQkv) && !a.coresident) return NK_ERR_PLAN;
    const int grid = P.G;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(tc_threads(NT), 1, 1);
    cfg.dynamicSmemBytes = L::kAlloc;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = NK_PDL ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, tc_kernel<NT, MODE>, mw, mx, a) == cudaSuccess ? NK_OK
                                                                                      : NK_ERR_CUDA;
}

int launch_tc(const nk_plan& p, const GemmArgs& in, cudaStream_t s) {
    if (get_encoder() != NK_OK) return NK_ERR_CUDA;
    GemmArgs a = in;
    const int nt = p.tile_m;
    const int KB = (a.K + tc_kstep(nt) - 1) / tc_kstep(nt);
    const int m_tiles = (a.M + nt - 1) / nt;  // token tiles of this call (<= the plan's)
    a.n_tiles = p.n_tiles;
    a.segments = p.segments;
    a.part_cols = p.M_max < nt ? p.M_max : nt;
    TcPartition& P = a.part_map;
    P.KB = KB;
    P.U = (int64_t)p.n_tiles * m_tiles * KB;
    P.split = p.split_k;
    P.lead = 0;
    P.G = 1;  // set by launch_tc_t once the device's residency is known
    CUtensorMap mw, mx;
    if (make_map(&mw, a.w, a.N, a.K, a.ldw, kTcRows) != NK_OK) return NK_ERR_ALIGN;
    if (make_map(&mx, a.x, a.M, a.K, a.ldx, nt) != NK_OK) return NK_ERR_ALIGN;
    const int mode = a.amax_keys ? kModeAmax
                   : a.ar_world > 0 ? kModeAr
                   : a.qk_q ? kModeQkv : kModePlain;
    switch (nt * 4 + mode) {
        case 16 * 4 + kModeQkv: return launch_tc_t<16, kModeQkv>(p, a, mw, mx, s);
        case 16 * 4 + kModePlain: return launch_tc_t<16, kModePlain>(p, a, mw, mx, s);
        case 16 * 4 + kModeAmax: return launch_tc_t<16, kModeAmax>(p, a, mw, mx, s);
        case 16 * 4 + kModeAr: return launch_tc_t<16, kModeAr>(p, a, mw, mx, s);
        case 32 * 4 + kModePlain: return launch_tc_t<32, kModePlain>(p, a, mw, mx, s);
        case 32 * 4 + kModeAmax: return launch_tc_t<32, kModeAmax>(p, a, mw, mx, s);
        case 32 * 4 + kModeAr: return launch_tc_t<32, kModeAr>(p, a, mw, mx, s);
        case 64 * 4 + kModePlain: return launch_tc_t<64, kModePlain>(p, a, mw, mx, s);
        case 64 * 4 + kModeAmax: return launch_tc_t<64, kModeAmax>(p, a, mw, mx, s);
        case 64 * 4 + kModeAr: return launch_tc_t<64, kModeAr>(p, a, mw, mx, s);
        case 128 * 4 + kModePlain: return launch_tc_t<128, kModePlain>(p, a, mw, mx, s);
        case 128 * 4 + kModeAmax: return launch_tc_t<128, kModeAmax>(p, a, mw, mx, s);
        case 256 * 4 + kModePlain: return launch_tc_t<256, kModePlain>(p, a, mw, mx, s);
        case 256 * 4 + kModeAmax: return launch_tc_t<256, kModeAmax>(p, a, mw, mx, s);
        default: return NK_ERR_PLAN;  // fused all-reduce: token tiles <= 64; fused QKV: 16
    }
}

}  // namespace nk
