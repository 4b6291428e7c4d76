// Fused non-linear decode kernels that sit between the decode linears (sm_100a).
//
// They replace the reference engine's Triton decode kernels, with the same bf16 cast points:
//   nk_rmsnorm_bf16          <- engine/kernels/rmsnorm.py:12-41   (_norm / norm_out)
//   nk_qk_norm_rope_cache    <- engine/kernels/elementwise.py:27-78 (_qk / qk_rope_cache_out)
//   nk_attention_decode_bf16 <- engine/kernels/attention.py:13-62  (_partial, _merge)
//   nk_silu_mul_bf16         <- engine/kernels/elementwise.py:81-101 (_silu / silu_mul_out)
// Each is one launch (attention: two) with programmatic dependent launch, so that chained
// with the decode GEMMs every launch can start while its predecessor drains; each waits
// (griddepcontrol.wait) before touching data the previous kernel produced.
#include "nk_common.cuh"
#include "../../include/nk_decode.h"

namespace nk {

template <typename Kernel, typename... Args>
static int launch_pdl_smem(Kernel kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                           Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = NK_PDL ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...) == cudaSuccess ? NK_OK : NK_ERR_CUDA;
}

__device__ __forceinline__ float bf16r(float v) {  // round to bf16 and back
    return __bfloat162float(__float2bfloat16_rn(v));
}

// Sum over the block (blockDim.x a multiple of 32, at most 1024). All threads get the sum.
__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();  // red may still be read by a previous call
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = l < nw ? red[l] : 0.f;
    return warp_sum(t);
}

// ---------------------------------------------------------------------------------------
// RMSNorm (+ residual): x <- bf16(x + branch) when branch is given; out = bf16(bf16(x *
// rsqrt(mean(x^2) + eps)) * weight). One CTA of 256 threads per row, 8 elements per chunk.
// ---------------------------------------------------------------------------------------
constexpr int kNormThreads = 256;
constexpr int kNormMaxChunks = 4;  // rows up to 256 * 8 * 4 = 8192 elements

__global__ void __launch_bounds__(kNormThreads)
rmsnorm_kernel(__nv_bfloat16* x, const __nv_bfloat16* branch, const __nv_bfloat16* w,
               __nv_bfloat16* out, int H, float eps) {
    __shared__ float red[32];
    if (threadIdx.x == 0) griddep_launch_dependents();
    griddep_wait();
    const int row = blockIdx.x;
    __nv_bfloat16* xr = x + (int64_t)row * H;
    const __nv_bfloat16* br = branch ? branch + (int64_t)row * H : nullptr;
    float v[kNormMaxChunks][8];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < kNormMaxChunks; ++c) {
        const int i = (c * kNormThreads + threadIdx.x) * 8;
        if (i < H) {
            uint4 xv = *reinterpret_cast<const uint4*>(xr + i);
            if (br) {
                const uint4 bv = *reinterpret_cast<const uint4*>(br + i);
                const uint32_t* xa = &xv.x;
                const uint32_t* ba = &bv.x;
                uint32_t sv[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float lo = bf16lo(xa[k]) + bf16lo(ba[k]);
                    const float hi = bf16hi(xa[k]) + bf16hi(ba[k]);
                    sv[k] = (uint32_t)f32_to_bf16_bits(lo) | ((uint32_t)f32_to_bf16_bits(hi) << 16);
                }
                xv = make_uint4(sv[0], sv[1], sv[2], sv[3]);
                *reinterpret_cast<uint4*>(xr + i) = xv;
            }
            const uint32_t* xa = &xv.x;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                v[c][2 * k] = bf16lo(xa[k]);
                v[c][2 * k + 1] = bf16hi(xa[k]);
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) ss += v[c][k] * v[c][k];
        }
    }
    const float total = block_sum(ss, red);
    const float inv = rsqrtf(total / (float)H + eps);
    __nv_bfloat16* orow = out + (int64_t)row * H;
#pragma unroll
    for (int c = 0; c < kNormMaxChunks; ++c) {
        const int i = (c * kNormThreads + threadIdx.x) * 8;
        if (i < H) {
            const uint4 wv = *reinterpret_cast<const uint4*>(w + i);
            const uint32_t* wa = &wv.x;
            uint32_t o[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float a = bf16r(v[c][2 * k] * inv) * bf16lo(wa[k]);
                const float b = bf16r(v[c][2 * k + 1] * inv) * bf16hi(wa[k]);
                o[k] = (uint32_t)f32_to_bf16_bits(a) | ((uint32_t)f32_to_bf16_bits(b) << 16);
            }
            *reinterpret_cast<uint4*>(orow + i) = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
}

// ---------------------------------------------------------------------------------------
// Per-head Q/K RMSNorm + RoPE at the device-side position + K/V cache write. One CTA of
// 128 threads (one per head element) per (head, sequence); heads [0, Hq) are queries,
// [Hq, Hq + Hkv) keys (whose CTA also copies the matching value head into the cache).
// ---------------------------------------------------------------------------------------
constexpr int kHeadDim = 128;

__global__ void __launch_bounds__(kHeadDim)
qk_norm_rope_cache_kernel(const __nv_bfloat16* qkv, int64_t ld_qkv, const __nv_bfloat16* qn,
                          const __nv_bfloat16* kn, const __nv_bfloat16* cos_t,
                          const __nv_bfloat16* sin_t, const int64_t* position,
                          __nv_bfloat16* q_out, __nv_bfloat16* k_cache, __nv_bfloat16* v_cache,
                          int Hq, int Hkv, int capacity, int64_t cb, int64_t ch, int64_t cs,
                          float eps) {
    __shared__ float red[32];
    __shared__ float xs[kHeadDim];
    if (threadIdx.x == 0) griddep_launch_dependents();
    griddep_wait();
    const int h = blockIdx.x;
    const int b = blockIdx.y;
    const int d = threadIdx.x;
    const int64_t pos = *position;
    if (pos < 0 || pos >= capacity) {  // no cache slot (and no RoPE row) to use
        if (h == 0 && b == 0 && d == 0) atomicExch(&g_error, NK_ERR_RANGE);
        return;
    }
    const bool is_q = h < Hq;
    const __nv_bfloat16* src = qkv + (int64_t)b * ld_qkv + (int64_t)h * kHeadDim;
    const float x = __bfloat162float(src[d]);
    const float ss = block_sum(x * x, red);
    const float inv = rsqrtf(ss / (float)kHeadDim + eps);
    const float wgt = __bfloat162float(is_q ? qn[d] : kn[d]);
    const float xn = bf16r(bf16r(x * inv) * wgt);
    xs[d] = xn;
    __syncthreads();
    const float other = xs[(d + kHeadDim / 2) % kHeadDim];
    const float rotated = d < kHeadDim / 2 ? -other : other;
    const float c = __bfloat162float(cos_t[pos * kHeadDim + d]);
    const float s = __bfloat162float(sin_t[pos * kHeadDim + d]);
    const float y = bf16r(xn * c) + bf16r(rotated * s);  // each product rounded, then the sum
    if (is_q) {
        q_out[((int64_t)b * Hq + h) * kHeadDim + d] = __float2bfloat16_rn(y);
    } else {
        const int kh = h - Hq;
        const int64_t slot = (int64_t)b * cb + (int64_t)kh * ch + pos * cs + d;
        k_cache[slot] = __float2bfloat16_rn(y);
        v_cache[slot] = src[(int64_t)Hkv * kHeadDim + d];  // value head kh follows the keys
    }
}

// ---------------------------------------------------------------------------------------
// Grouped split-KV decode attention. CTA (split, kv head, sequence) covers cache positions
// [split*C, split*C + C) clipped to [0, position] for all G = Hq/Hkv query heads that share
// the KV head, so each K/V row is read once per group.
//
// Decode attention moves a few MB per layer, so its time is DRAM latency unless many loads
// are in flight: every thread first issues its share of the chunk's K rows, then of its V
// rows, as asynchronous copies into shared memory (16 or 8 bytes each; rows past the
// position are zero-filled without a read), so the whole 2 x 16 KB chunk is requested at
// once. Warp w then scores rows [16w, 16w + 16) in two batches of 8: lane l forms the
// partial dot products of elements 4l..4l+3, a recursive-halving reduction leaves each
// (row, head) score on its owner lanes, which alone evaluate the exponentials of the
// online softmax and pass the batch's probabilities to the whole warp through shared
// memory for the V accumulation (lane l again holding elements 4l..4l+3). The warps' states are combined in shared memory
// and the CTA stores (max, sum, unnormalised acc); a merge kernel combines the splits:
// out = sum_s e^(m_s-M) acc_s / sum_s e^(m_s-M) l_s. CTAs whose chunk starts past the
// position store nothing (the merge reads only the splits at or below it).
// ---------------------------------------------------------------------------------------
constexpr int kAttnChunk = 64;
constexpr int kAttnThreads = 128;
constexpr int kAttnMaxGroup = 8;
constexpr int kAttnBatch = 8;                       // rows scored together by a warp
constexpr int kAttnRowBytes = kHeadDim * 2;         // 256 B per cache row
constexpr int kAttnTileBytes = kAttnChunk * kAttnRowBytes;  // 16 KB per K or V chunk

template <int VB>
__device__ __forceinline__ void cp_async(uint32_t dst, const void* src, bool valid) {
    const int n = valid ? VB : 0;  // 0 source bytes: the destination is zero-filled
    if constexpr (VB == 16)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n)
                     : "memory");
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "r"(n)
                     : "memory");
}

// Copies rows [0, C) of one cache chunk into a [C][128] bf16 tile; rows >= valid are zeros.
template <int VB>
__device__ __forceinline__ void attn_load_tile(uint32_t tile, const __nv_bfloat16* rows0,
                                               int64_t cs, int valid) {
    constexpr int kSegs = kAttnRowBytes / VB;  // copies per row
#pragma unroll
    for (int i = 0; i < kAttnChunk * kSegs / kAttnThreads; ++i) {
        const int idx = i * kAttnThreads + threadIdx.x;
        const int row = idx / kSegs, seg = idx - row * kSegs;
        const bool ok = row < valid;
        const __nv_bfloat16* src = rows0 + (int64_t)(ok ? row : 0) * cs + seg * (VB / 2);
        cp_async<VB>(tile + row * kAttnRowBytes + seg * VB, src, ok);
    }
}

// Sums the 8 x G scores of a batch (value i = r * G + g, one partial per lane) across the
// warp by recursive halving: at offset o a lane keeps the half of its values selected by
// bit o of its lane id and adds the partner's copy of that half, so 8G values need 8G - 1
// shuffles instead of 5 * 8G. Afterwards lane l holds the full sums of rows r = l >> 2 and
// heads g = own_head(l, j), j < kOwned (duplicated over the low lane bits when G < 4).
template <int G>
struct AttnOwn {
    static constexpr int kValues = kAttnBatch * G;
    static constexpr int kOwned = G == 8 ? 2 : 1;
    static constexpr int kLog2G = G == 8 ? 3 : G == 4 ? 2 : G == 2 ? 1 : 0;
    __device__ static __forceinline__ int head(int lane, int j) {
        return G == 8 ? 2 * (lane & 3) + j : (lane >> (2 - kLog2G)) & (G - 1);
    }
};

template <int G>
__device__ __forceinline__ void attn_reduce_scores(float (&v)[kAttnBatch * G], int lane) {
    constexpr int NV = kAttnBatch * G;
#pragma unroll
    for (int k = 0; k < 5; ++k) {
        const int o = 16 >> k;
        const int n = NV >> k;  // values still held before this step (constant once unrolled)
        if (n > AttnOwn<G>::kOwned) {
            const bool up = (lane & o) != 0;
#pragma unroll
            for (int j = 0; j < n / 2; ++j) {
                const float send = up ? v[j] : v[j + n / 2];
                const float keep = up ? v[j + n / 2] : v[j];
                v[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
            }
        } else {
#pragma unroll
            for (int j = 0; j < AttnOwn<G>::kOwned; ++j) v[j] += __shfl_xor_sync(0xffffffffu, v[j], o);
        }
    }
}

template <int G, int VB>
__global__ void __launch_bounds__(kAttnThreads)
attn_partial_kernel(const __nv_bfloat16* q, const __nv_bfloat16* k_cache,
                    const __nv_bfloat16* v_cache, const int64_t* position, float* part_acc,
                    float* part_ml, int Hq, int Hkv, int splits, int capacity, int64_t cb,
                    int64_t ch, int64_t cs, float scale) {
    using O = AttnOwn<G>;
    constexpr int NO = O::kOwned;
    // K tile, V tile; after scoring, the K tile holds the warps' accumulators
    __shared__ __align__(128) uint8_t s_tiles[2 * kAttnTileBytes];
    __shared__ __align__(16) float s_p[4][kAttnBatch][G];  // a warp's batch probabilities
    __shared__ __align__(16) float s_c[4][G];              // ... and running-sum rescales
    __shared__ float s_m[4][G], s_l[4][G];
    static_assert(4 * G * kHeadDim * 4 <= kAttnTileBytes, "accumulators must fit the K tile");
    if (threadIdx.x == 0) griddep_launch_dependents();
    griddep_wait();
    const int split = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t pos_in = *position;
    const int64_t pos = min(pos_in, (int64_t)capacity - 1);  // never past the cache
    if ((pos_in < 0 || pos_in >= capacity) && split == 0 && kh == 0 && b == 0 && threadIdx.x == 0)
        atomicExch(&g_error, NK_ERR_RANGE);
    const int j0 = split * kAttnChunk;
    if ((int64_t)j0 > pos) return;  // also every CTA when the position is negative
    const int valid = (int)min((int64_t)kAttnChunk, pos + 1 - j0);

    const uint32_t sk = smem_u32(s_tiles), sv = sk + kAttnTileBytes;
    const int64_t base = (int64_t)b * cb + (int64_t)kh * ch + (int64_t)j0 * cs;
    attn_load_tile<VB>(sk, k_cache + base, cs, valid);
    asm volatile("cp.async.commit_group;" ::: "memory");
    attn_load_tile<VB>(sv, v_cache + base, cs, valid);
    asm volatile("cp.async.commit_group;" ::: "memory");

    float qf[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const __nv_bfloat16* qp = q + ((int64_t)b * Hq + kh * G + g) * kHeadDim + lane * 4;
        const uint2 qv = *reinterpret_cast<const uint2*>(qp);
        qf[g][0] = bf16lo(qv.x); qf[g][1] = bf16hi(qv.x);
        qf[g][2] = bf16lo(qv.y); qf[g][3] = bf16hi(qv.y);
    }
    float acc[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) acc[g][0] = acc[g][1] = acc[g][2] = acc[g][3] = 0.f;
    float m_own[NO], l_own[NO];  // running max and sum of the heads this lane owns
#pragma unroll
    for (int j = 0; j < NO; ++j) { m_own[j] = -INFINITY; l_own[j] = 0.f; }
    const int r_own = lane >> 2;
    const uint8_t* kt = s_tiles + lane * 8;
    const uint8_t* vt = s_tiles + kAttnTileBytes + lane * 8;

    asm volatile("cp.async.wait_group 1;" ::: "memory");  // this thread's K copies landed
    __syncthreads();                                     // ... and everyone's
#pragma unroll
    for (int bt = 0; bt < 2; ++bt) {
        const int r0 = warp * 16 + bt * kAttnBatch;
        float sc[O::kValues];
#pragma unroll
        for (int r = 0; r < kAttnBatch; ++r) {
            const uint2 kv = *reinterpret_cast<const uint2*>(kt + (r0 + r) * kAttnRowBytes);
            const float k0 = bf16lo(kv.x), k1 = bf16hi(kv.x), k2 = bf16lo(kv.y), k3 = bf16hi(kv.y);
#pragma unroll
            for (int g = 0; g < G; ++g)
                sc[r * G + g] = qf[g][0] * k0 + qf[g][1] * k1 + qf[g][2] * k2 + qf[g][3] * k3;
        }
        attn_reduce_scores<G>(sc, lane);
        const bool row_ok = r0 + r_own < valid;
#pragma unroll
        for (int j = 0; j < NO; ++j) {
            const float x = row_ok ? sc[j] * scale : -INFINITY;
            float bm = x;  // batch max over the 8 rows (lane bits 2-4) of this head
            bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 4));
            bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 8));
            bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 16));
            const float mn = fmaxf(m_own[j], bm);
            const bool any = mn != -INFINITY;
            const float corr = any ? expf(m_own[j] - mn) : 1.f;  // 0 while m is still -inf
            const float p = any ? expf(x - mn) : 0.f;            // 0 for rows past the position
            float ps = p;
            ps += __shfl_xor_sync(0xffffffffu, ps, 4);
            ps += __shfl_xor_sync(0xffffffffu, ps, 8);
            ps += __shfl_xor_sync(0xffffffffu, ps, 16);
            l_own[j] = l_own[j] * corr + ps;
            m_own[j] = mn;
            const int g = O::head(lane, j);
            s_p[warp][r_own][g] = p;
            if (r_own == 0) s_c[warp][g] = corr;
        }
        if (bt == 0) {
            asm volatile("cp.async.wait_group 0;" ::: "memory");  // V copies landed
            __syncthreads();
        } else {
            __syncwarp();
        }
        float vr[kAttnBatch][4];
#pragma unroll
        for (int r = 0; r < kAttnBatch; ++r) {
            const uint2 vv = *reinterpret_cast<const uint2*>(vt + (r0 + r) * kAttnRowBytes);
            vr[r][0] = bf16lo(vv.x); vr[r][1] = bf16hi(vv.x);
            vr[r][2] = bf16lo(vv.y); vr[r][3] = bf16hi(vv.y);
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float c = s_c[warp][g];
            float a0 = acc[g][0] * c, a1 = acc[g][1] * c, a2 = acc[g][2] * c, a3 = acc[g][3] * c;
#pragma unroll
            for (int r = 0; r < kAttnBatch; ++r) {
                const float p = s_p[warp][r][g];
                a0 += p * vr[r][0]; a1 += p * vr[r][1]; a2 += p * vr[r][2]; a3 += p * vr[r][3];
            }
            acc[g][0] = a0; acc[g][1] = a1; acc[g][2] = a2; acc[g][3] = a3;
        }
        __syncwarp();  // the next batch overwrites s_p and s_c
    }
    if (r_own == 0) {
#pragma unroll
        for (int j = 0; j < NO; ++j) {
            const int g = O::head(lane, j);
            s_m[warp][g] = m_own[j];
            s_l[warp][g] = l_own[j];
        }
    }
    __syncthreads();  // every warp is done with the K tile
    float* s_acc = reinterpret_cast<float*>(s_tiles);  // [4][G][128]
#pragma unroll
    for (int g = 0; g < G; ++g)
        *reinterpret_cast<float4*>(s_acc + (warp * G + g) * kHeadDim + lane * 4) =
            make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
    __syncthreads();
    // thread t combines element d = t of every query head of the group
    const int d = threadIdx.x;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; ++w) M = fmaxf(M, s_m[w][g]);
        float L = 0.f, A = 0.f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            if (s_m[w][g] == -INFINITY) continue;  // a warp whose rows are all past the position
            const float f = expf(s_m[w][g] - M);
            L += s_l[w][g] * f;
            A += s_acc[(w * G + g) * kHeadDim + d] * f;
        }
        const int64_t hrow = ((int64_t)b * Hq + kh * G + g) * splits + split;
        part_acc[hrow * kHeadDim + d] = A;
        if (d == 0) {
            part_ml[hrow * 2] = M;
            part_ml[hrow * 2 + 1] = L;
        }
    }
}

// One CTA per (sequence, query head); thread d owns output element d. The splits' maxima are
// gathered in parallel (one load per thread per 128 splits) and reduced across the CTA, then
// the weighted sums run over the splits with their loads unrolled.
__global__ void __launch_bounds__(kHeadDim)
attn_merge_kernel(const float* part_acc, const float* part_ml, __nv_bfloat16* out, int splits,
                  int capacity, const int64_t* position) {
    __shared__ float s_max[kHeadDim / 32];
    if (threadIdx.x == 0) griddep_launch_dependents();
    griddep_wait();
    const int64_t hrow = blockIdx.x;  // b * Hq + h
    const int d = threadIdx.x;
    const int64_t pos = min(*position, (int64_t)capacity - 1);
    if (pos < 0) return;  // no partials were written (the partial kernel flagged it)
    const int used = (int)min((int64_t)splits, pos / kAttnChunk + 1);
    const float* ml = part_ml + hrow * splits * 2;
    const float* pa = part_acc + hrow * splits * kHeadDim + d;
    float M = -INFINITY;
    for (int s = d; s < used; s += kHeadDim) M = fmaxf(M, ml[s * 2]);
    M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 16));
    M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 8));
    M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 4));
    M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 2));
    M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 1));
    if ((d & 31) == 0) s_max[d >> 5] = M;
    __syncthreads();
    M = fmaxf(fmaxf(s_max[0], s_max[1]), fmaxf(s_max[2], s_max[3]));
    float L = 0.f, A = 0.f;
#pragma unroll 8
    for (int s = 0; s < used; ++s) {
        const float ms = ml[s * 2];
        const float f = ms == -INFINITY ? 0.f : expf(ms - M);
        L += ml[s * 2 + 1] * f;
        A += pa[(int64_t)s * kHeadDim] * f;
    }
    out[hrow * kHeadDim + d] = __float2bfloat16_rn(A / L);
}

// ---------------------------------------------------------------------------------------
// out = bf16( bf16(g / (1 + exp(-g))) * u ) for gate_up = [g | u] per row.
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
silu_mul_kernel(const __nv_bfloat16* gate_up, __nv_bfloat16* out, int rows, int I) {
    if (threadIdx.x == 0) griddep_launch_dependents();
    griddep_wait();
    const int64_t chunks_per_row = I / 8;
    const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= (int64_t)rows * chunks_per_row) return;
    const int64_t row = c / chunks_per_row;
    const int64_t i = (c - row * chunks_per_row) * 8;
    const __nv_bfloat16* gr = gate_up + row * 2 * I;
    const uint4 gv = *reinterpret_cast<const uint4*>(gr + i);
    const uint4 uv = *reinterpret_cast<const uint4*>(gr + I + i);
    const uint32_t* ga = &gv.x;
    const uint32_t* ua = &uv.x;
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float g0 = bf16lo(ga[k]), g1 = bf16hi(ga[k]);
        const float a0 = bf16r(g0 / (1.f + expf(-g0)));
        const float a1 = bf16r(g1 / (1.f + expf(-g1)));
        o[k] = (uint32_t)f32_to_bf16_bits(a0 * bf16lo(ua[k])) |
               ((uint32_t)f32_to_bf16_bits(a1 * bf16hi(ua[k])) << 16);
    }
    *reinterpret_cast<uint4*>(out + row * I + i) = make_uint4(o[0], o[1], o[2], o[3]);
}

static bool al16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

}  // namespace nk

using namespace nk;

extern "C" int nk_rmsnorm_bf16(void* x, const void* branch, const void* weight, void* out,
                               int rows, int width, float eps, nk_stream_t stream) {
    if (!x || !weight || !out) return NK_ERR_ARG;
    if (rows < 1 || width < 8 || width % 8 || width > kNormThreads * 8 * kNormMaxChunks)
        return NK_ERR_SHAPE;
    if (!al16(x) || !al16(weight) || !al16(out) || (branch && !al16(branch))) return NK_ERR_ALIGN;
    return launch_pdl_smem(rmsnorm_kernel, dim3(rows), dim3(kNormThreads), 0,
                           (cudaStream_t)stream, static_cast<__nv_bfloat16*>(x),
                           static_cast<const __nv_bfloat16*>(branch),
                           static_cast<const __nv_bfloat16*>(weight),
                           static_cast<__nv_bfloat16*>(out), width, eps);
}

extern "C" int nk_qk_norm_rope_cache_bf16(const void* qkv, int64_t ld_qkv, const void* q_norm,
                                          const void* k_norm, const void* cos_table,
                                          const void* sin_table, const int64_t* position,
                                          void* q_out, void* k_cache, void* v_cache, int batch,
                                          int q_heads, int kv_heads, int head_dim, int capacity,
                                          int64_t cache_batch_stride, int64_t cache_head_stride,
                                          int64_t cache_seq_stride, float eps,
                                          nk_stream_t stream) {
    if (!qkv || !q_norm || !k_norm || !cos_table || !sin_table || !position || !q_out ||
        !k_cache || !v_cache)
        return NK_ERR_ARG;
    if (head_dim != kHeadDim || batch < 1 || q_heads < 1 || kv_heads < 1 || capacity < 1 ||
        ld_qkv < (int64_t)(q_heads + 2 * kv_heads) * head_dim || cache_seq_stride < head_dim)
        return NK_ERR_SHAPE;
    return launch_pdl_smem(
        qk_norm_rope_cache_kernel, dim3(q_heads + kv_heads, batch), dim3(kHeadDim), 0,
        (cudaStream_t)stream, static_cast<const __nv_bfloat16*>(qkv), ld_qkv,
        static_cast<const __nv_bfloat16*>(q_norm), static_cast<const __nv_bfloat16*>(k_norm),
        static_cast<const __nv_bfloat16*>(cos_table), static_cast<const __nv_bfloat16*>(sin_table),
        position, static_cast<__nv_bfloat16*>(q_out), static_cast<__nv_bfloat16*>(k_cache),
        static_cast<__nv_bfloat16*>(v_cache), q_heads, kv_heads, capacity, cache_batch_stride,
        cache_head_stride, cache_seq_stride, eps);
}

extern "C" size_t nk_attention_ws_bytes(int batch, int q_heads, int capacity) {
    if (batch < 1 || q_heads < 1 || capacity < 1) return 0;
    const size_t splits = (size_t)(capacity + kAttnChunk - 1) / kAttnChunk;
    return (size_t)batch * q_heads * splits * (kHeadDim + 2) * sizeof(float);
}

extern "C" int nk_attention_decode_bf16(const void* q, const void* k_cache, const void* v_cache,
                                        const int64_t* position, void* out, int batch,
                                        int q_heads, int kv_heads, int head_dim, int capacity,
                                        int64_t cache_batch_stride, int64_t cache_head_stride,
                                        int64_t cache_seq_stride, float scale, void* ws,
                                        size_t ws_bytes, nk_stream_t stream) {
    if (!q || !k_cache || !v_cache || !position || !out) return NK_ERR_ARG;
    if (head_dim != kHeadDim || batch < 1 || kv_heads < 1 || q_heads % kv_heads ||
        capacity < 1 || cache_seq_stride < head_dim)
        return NK_ERR_SHAPE;
    const int G = q_heads / kv_heads;
    if (G > kAttnMaxGroup || (G & (G - 1))) return NK_ERR_SHAPE;
    const size_t need = nk_attention_ws_bytes(batch, q_heads, capacity);
    if (!ws || ws_bytes < need) return NK_ERR_WORKSPACE;
    if (!al16(ws) || ((uintptr_t)q & 7u) || ((uintptr_t)k_cache & 7u) || ((uintptr_t)v_cache & 7u) ||
        (cache_seq_stride % 4) || (cache_head_stride % 4) || (cache_batch_stride % 4))
        return NK_ERR_ALIGN;
    const int splits = (capacity + kAttnChunk - 1) / kAttnChunk;
    float* part_acc = static_cast<float*>(ws);
    float* part_ml = part_acc + (size_t)batch * q_heads * splits * kHeadDim;
    cudaStream_t s = (cudaStream_t)stream;
    const dim3 grid(splits, kv_heads, batch);
    const auto* qq = static_cast<const __nv_bfloat16*>(q);
    const auto* kk = static_cast<const __nv_bfloat16*>(k_cache);
    const auto* vv = static_cast<const __nv_bfloat16*>(v_cache);
    // 16-byte copies when every cache row segment is 16-byte aligned, else 8-byte copies
    const bool wide = al16(k_cache) && al16(v_cache) && cache_seq_stride % 8 == 0 &&
                      cache_head_stride % 8 == 0 && cache_batch_stride % 8 == 0;
    int st;
#define NK_ATTN_LAUNCH(GG, VB)                                                                  \
    launch_pdl_smem(attn_partial_kernel<GG, VB>, grid, dim3(kAttnThreads), 0, s, qq, kk, vv,   \
                    position, part_acc, part_ml, q_heads, kv_heads, splits, capacity,           \
                    cache_batch_stride,                                                       \
                    cache_head_stride, cache_seq_stride, scale)
    switch (G) {
        case 1: st = wide ? NK_ATTN_LAUNCH(1, 16) : NK_ATTN_LAUNCH(1, 8); break;
        case 2: st = wide ? NK_ATTN_LAUNCH(2, 16) : NK_ATTN_LAUNCH(2, 8); break;
        case 4: st = wide ? NK_ATTN_LAUNCH(4, 16) : NK_ATTN_LAUNCH(4, 8); break;
        default: st = wide ? NK_ATTN_LAUNCH(8, 16) : NK_ATTN_LAUNCH(8, 8); break;
    }
#undef NK_ATTN_LAUNCH
    if (st != NK_OK) return st;
    return launch_pdl_smem(attn_merge_kernel, dim3(batch * q_heads), dim3(kHeadDim), 0, s,
                           (const float*)part_acc, (const float*)part_ml,
                           static_cast<__nv_bfloat16*>(out), splits, capacity, position);
}

extern "C" int nk_silu_mul_bf16(const void* gate_up, void* out, int rows, int intermediate,
                                nk_stream_t stream) {
    if (!gate_up || !out) return NK_ERR_ARG;
    if (rows < 1 || intermediate < 8 || intermediate % 8) return NK_ERR_SHAPE;
    if (!al16(gate_up) || !al16(out)) return NK_ERR_ALIGN;
    const int64_t chunks = (int64_t)rows * (intermediate / 8);
    const int blocks = (int)((chunks + 255) / 256);
    return launch_pdl_smem(silu_mul_kernel, dim3(blocks), dim3(256), 0, (cudaStream_t)stream,
                           static_cast<const __nv_bfloat16*>(gate_up),
                           static_cast<__nv_bfloat16*>(out), rows, intermediate);
}
