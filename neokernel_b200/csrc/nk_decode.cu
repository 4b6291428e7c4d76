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
// once. The two contractions then run on the tensor cores (mma.sync m16n8k16, the query
// heads as rows of a 16-row tile), with an fp32 softmax in between (details at the kernel).
// The warps' states are combined in shared memory and the CTA stores (max, sum,
// unnormalised acc); a merge kernel combines the splits:
// out = sum_s e^(m_s-M) acc_s / sum_s e^(m_s-M) l_s. CTAs whose chunk starts past the
// position store nothing (the merge reads only the splits at or below it).
// ---------------------------------------------------------------------------------------
constexpr int kAttnChunk = 64;
constexpr int kAttnThreads = 128;
constexpr int kAttnMaxGroup = 8;
constexpr int kAttnRowBytes = kHeadDim * 2;         // 256 B per cache row

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

// K and V rows sit 16 bytes apart more than their 256 bytes in shared memory, so that the
// fragment loads of 8 consecutive rows hit 8 different bank groups.
constexpr int kAttnPitch = kAttnRowBytes + 16;
constexpr int kAttnPTile = kAttnChunk * kAttnPitch;

template <int VB>
__device__ __forceinline__ void attn_load_tile(uint32_t tile, const __nv_bfloat16* rows0,
                                               int64_t cs, int valid) {
    constexpr int kSegs = kAttnRowBytes / VB;
#pragma unroll
    for (int i = 0; i < kAttnChunk * kSegs / kAttnThreads; ++i) {
        const int idx = i * kAttnThreads + threadIdx.x;
        const int row = idx / kSegs, seg = idx - row * kSegs;
        const bool ok = row < valid;
        const __nv_bfloat16* src = rows0 + (int64_t)(ok ? row : 0) * cs + seg * (VB / 2);
        cp_async<VB>(tile + row * kAttnPitch + seg * VB, src, ok);
    }
}

__device__ __forceinline__ void mma_16816(float (&c)[4], uint32_t a0, uint32_t a2, uint32_t b0,
                                          uint32_t b1) {
    // rows 8..15 of A are zero (at most 8 query heads per KV head). Not volatile: a pure
    // register operation, so the compiler may interleave independent accumulator chains.
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                              uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    return (uint32_t)f32_to_bf16_bits(lo) | ((uint32_t)f32_to_bf16_bits(hi) << 16);
}

// Two pipeline stages, each one chunk's K tile and V tile.
constexpr int kAttnStages = 2;
constexpr int kAttnSmem = kAttnStages * 2 * kAttnPTile;  // 68 KB: 3 CTAs per SM

// CTA (split, kv head, sequence) walks the chunks [c0, c1) of its split (the chunks that
// hold positions 0..pos, divided evenly over the splits), the copies of chunk c+1 in
// flight while chunk c is computed. Warp w owns rows [16w, 16w + 16) of every chunk and
// keeps an online softmax over them (running max m, sum l, unnormalised o).
// Lane (g = lane / 4, t = lane % 4) follows the m16n8k16 fragment layout: query head g
// (rows g >= G are zero), keys 2t, 2t+1, 8+2t, 9+2t of the warp's 16. S = Q K^T (two 8-key
// tiles, eight 16-dim steps) accumulates exact bf16 products in fp32; the softmax is fp32;
// P V uses P = P_hi + P_lo (two bf16 halves, so P keeps ~16 bits) against bf16 V,
// accumulated in fp32 over 16 tiles of 8 dimensions.
template <int G, int VB>
__global__ void __launch_bounds__(kAttnThreads, 3)
attn_partial_kernel(const __nv_bfloat16* q, const __nv_bfloat16* k_cache,
                    const __nv_bfloat16* v_cache, const int64_t* position, float* part_acc,
                    float* part_ml, int Hq, int Hkv, int splits, int capacity, int64_t cb,
                    int64_t ch, int64_t cs, float scale) {
    extern __shared__ __align__(128) uint8_t s_tiles[];  // [stage][K, V][kAttnPTile]
    __shared__ float s_m[4][G], s_l[4][G];
    static_assert(G <= 8, "at most 8 query heads per KV head");
    static_assert(4 * G * kHeadDim * 4 <= kAttnSmem, "accumulators must fit the tiles");
    if (threadIdx.x == 0) griddep_launch_dependents();
    griddep_wait();
    const int split = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int64_t pos_in = *position;
    const int64_t pos = min(pos_in, (int64_t)capacity - 1);  // never past the cache
    if ((pos_in < 0 || pos_in >= capacity) && split == 0 && kh == 0 && b == 0 && threadIdx.x == 0)
        atomicExch(&g_error, NK_ERR_RANGE);
    if (pos < 0) return;
    // chunks [c0, c1) of the n that hold positions 0..pos; with fewer chunks than splits,
    // split s < n takes chunk s and the others store nothing (the merge reads min(n, splits))
    const int n = (int)(pos / kAttnChunk) + 1;
    int c0, c1;
    if (n >= splits) {
        c0 = (int)((int64_t)split * n / splits);
        c1 = (int)((int64_t)(split + 1) * n / splits);
    } else {
        if (split >= n) return;
        c0 = split;
        c1 = split + 1;
    }

    const uint32_t s0 = smem_u32(s_tiles);
    const int64_t base = (int64_t)b * cb + (int64_t)kh * ch;
    auto issue = [&](int c, int stage) {  // K then V of chunk c, one commit group each
        const int j0 = c * kAttnChunk;
        const int valid = (int)min((int64_t)kAttnChunk, pos + 1 - j0);
        const uint32_t sk = s0 + stage * 2 * kAttnPTile;
        attn_load_tile<VB>(sk, k_cache + base + (int64_t)j0 * cs, cs, valid);
        asm volatile("cp.async.commit_group;" ::: "memory");
        attn_load_tile<VB>(sk + kAttnPTile, v_cache + base + (int64_t)j0 * cs, cs, valid);
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    issue(c0, 0);
    if (c0 + 1 < c1) issue(c0 + 1, 1);

    // A fragments of Q: head g, dimensions 16ks + 2t (+1) and 16ks + 8 + 2t (+1)
    uint32_t qa[8][2];
    {
        const __nv_bfloat16* qr = q + ((int64_t)b * Hq + kh * G + (g < G ? g : 0)) * kHeadDim;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            qa[ks][0] = g < G ? *reinterpret_cast<const uint32_t*>(qr + 16 * ks + 2 * t) : 0u;
            qa[ks][1] = g < G ? *reinterpret_cast<const uint32_t*>(qr + 16 * ks + 8 + 2 * t) : 0u;
        }
    }

    float m = -INFINITY, l = 0.f;  // this warp's rows so far, head g (shared by the 4 t lanes)
    float o[16][4];
#pragma unroll
    for (int nn = 0; nn < 16; ++nn) o[nn][0] = o[nn][1] = o[nn][2] = o[nn][3] = 0.f;
    // ldmatrix.trans row addresses: matrix mi = lane / 8 = (keys half mi & 1, dims +8 (mi >> 1))
    const int mi = lane >> 3, mr = lane & 7;
    const int r0 = warp * 16;
    for (int c = c0; c < c1; ++c) {
        const int stage = (c - c0) & 1;
        const bool next = c + 1 < c1;  // chunk c+1's two groups are committed behind this one's
        const uint32_t sk = s0 + stage * 2 * kAttnPTile, sv = sk + kAttnPTile;
        if (next) asm volatile("cp.async.wait_group 3;" ::: "memory");  // K of chunk c landed
        else asm volatile("cp.async.wait_group 1;" ::: "memory");
        __syncthreads();  // ... for every thread
        float sc[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
            sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
            const uint8_t* kr = s_tiles + (sk - s0) + (r0 + nt * 8 + g) * kAttnPitch + 4 * t;
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                const uint32_t b0 = *reinterpret_cast<const uint32_t*>(kr + 32 * ks);
                const uint32_t b1 = *reinterpret_cast<const uint32_t*>(kr + 32 * ks + 16);
                mma_16816(sc[nt], qa[ks][0], qa[ks][1], b0, b1);
            }
        }
        // this lane's scores of head g: keys r0 + 2t, r0 + 2t + 1, r0 + 8 + 2t, r0 + 9 + 2t
        const int valid = (int)min((int64_t)kAttnChunk, pos + 1 - (int64_t)c * kAttnChunk);
        float x[4] = {sc[0][0], sc[0][1], sc[1][0], sc[1][1]};
        const int kk[4] = {r0 + 2 * t, r0 + 2 * t + 1, r0 + 8 + 2 * t, r0 + 9 + 2 * t};
        float mc = -INFINITY;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            x[i] = kk[i] < valid ? x[i] * scale : -INFINITY;
            mc = fmaxf(mc, x[i]);
        }
        mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, 1));
        mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, 2));
        const float mn = fmaxf(m, mc);
        const float alpha = m == mn ? 1.f : expf(m - mn);  // m = mn = -inf keeps o = l = 0
        float p[4], lc = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            p[i] = mn == -INFINITY ? 0.f : expf(x[i] - mn);  // 0 for rows past the position
            lc += p[i];
        }
        lc += __shfl_xor_sync(0xffffffffu, lc, 1);
        lc += __shfl_xor_sync(0xffffffffu, lc, 2);
        l = l * alpha + lc;
        m = mn;
#pragma unroll
        for (int nn = 0; nn < 16; ++nn) {
            o[nn][0] *= alpha;
            o[nn][1] *= alpha;
        }
        // P as A fragments, split into a bf16 high part and the bf16 rounding of the rest
        const uint32_t ph0 = pack_bf16x2(p[0], p[1]), ph2 = pack_bf16x2(p[2], p[3]);
        const uint32_t pl0 = pack_bf16x2(p[0] - bf16lo(ph0), p[1] - bf16hi(ph0));
        const uint32_t pl2 = pack_bf16x2(p[2] - bf16lo(ph2), p[3] - bf16hi(ph2));

        if (next) asm volatile("cp.async.wait_group 2;" ::: "memory");  // V of chunk c landed
        else asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncthreads();
        const uint32_t vrow = sv + (uint32_t)(r0 + (mi & 1) * 8 + mr) * kAttnPitch + (mi >> 1) * 16;
#pragma unroll
        for (int nn = 0; nn < 16; nn += 2) {
            uint32_t b00, b01, b10, b11;
            ldsm_x4_trans(vrow + nn * 16, b00, b01, b10, b11);
            mma_16816(o[nn], ph0, ph2, b00, b01);
            mma_16816(o[nn + 1], ph0, ph2, b10, b11);
            mma_16816(o[nn], pl0, pl2, b00, b01);
            mma_16816(o[nn + 1], pl0, pl2, b10, b11);
        }
        if (c + 2 < c1) {
            __syncthreads();  // every warp is done with this stage
            issue(c + 2, stage);
        }
    }
    __syncthreads();  // every warp is done with the tiles
    float* s_acc = reinterpret_cast<float*>(s_tiles);  // [4][G][128]
    if (g < G) {
#pragma unroll
        for (int nn = 0; nn < 16; ++nn)
            *reinterpret_cast<float2*>(s_acc + (warp * G + g) * kHeadDim + 8 * nn + 2 * t) =
                make_float2(o[nn][0], o[nn][1]);
        if (t == 0) {
            s_m[warp][g] = m;
            s_l[warp][g] = l;
        }
    }
    __syncthreads();
    // thread d combines element d of every query head of the group
    const int d = threadIdx.x;
#pragma unroll
    for (int gg = 0; gg < G; ++gg) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; ++w) M = fmaxf(M, s_m[w][gg]);
        float L = 0.f, A = 0.f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            if (s_m[w][gg] == -INFINITY) continue;  // a warp whose rows are all past the position
            const float f = expf(s_m[w][gg] - M);
            L += s_l[w][gg] * f;
            A += s_acc[(w * G + gg) * kHeadDim + d] * f;
        }
        const int64_t hrow = ((int64_t)b * Hq + kh * G + gg) * splits + split;
        part_acc[hrow * kHeadDim + d] = A;
        if (d == 0) {
            part_ml[hrow * 2] = M;
            part_ml[hrow * 2 + 1] = L;
        }
    }
}

// Splits per (kv head, sequence): as many as keep every CTA of the launch resident at once
// (one wave), at most one per chunk of the cache.
template <int G, int VB>
static int attn_splits(int pairs, int chunks, int* splits) {
    static int slots[64] = {};  // resident CTAs per device (0 = not yet counted)
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return NK_ERR_CUDA;
    if (dev < 0 || dev >= 64) return NK_ERR_DEVICE;
    if (slots[dev] == 0) {
        int sms = 0, per_sm = 0;
        if (cudaFuncSetAttribute(attn_partial_kernel<G, VB>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem) !=
                cudaSuccess ||
            cudaFuncSetAttribute(attn_partial_kernel<G, VB>,
                                 cudaFuncAttributePreferredSharedMemoryCarveout,
                                 (int)cudaSharedmemCarveoutMaxShared) != cudaSuccess ||
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attn_partial_kernel<G, VB>,
                                                          kAttnThreads, kAttnSmem) !=
                cudaSuccess ||
            per_sm < 1)
            return NK_ERR_CUDA;
        slots[dev] = sms * per_sm;
    }
    *splits = max(1, min(chunks, slots[dev] / pairs));
    return NK_OK;
}

// One CTA per (sequence, query head); thread d owns output element d. The splits are read in
// batches of kMergeBatch with every load of a batch in flight at once (the first batch
// together with the position, before the number of used splits is known: entries of
// unused splits are read but ignored). Within a batch the weights use the batch's running
// maximum; across batches the sums are rescaled, so up to kMergeBatch splits the result is
// sum_s e^(m_s - M) acc_s / sum_s e^(m_s - M) l_s with M the maximum over all splits.
constexpr int kMergeBatch = 16;

__global__ void __launch_bounds__(kHeadDim)
attn_merge_kernel(const float* part_acc, const float* part_ml, __nv_bfloat16* out, int splits,
                  int capacity, const int64_t* position) {
    if (threadIdx.x == 0) griddep_launch_dependents();
    griddep_wait();
    const int64_t hrow = blockIdx.x;  // b * Hq + h
    const int d = threadIdx.x;
    const float2* ml = reinterpret_cast<const float2*>(part_ml + hrow * splits * 2);
    const float* pa = part_acc + hrow * splits * kHeadDim + d;
    const int64_t pos_in = *position;
    float2 v[kMergeBatch];
    float acc[kMergeBatch];
#pragma unroll
    for (int j = 0; j < kMergeBatch; ++j) {
        if (j < splits) {
            v[j] = ml[j];
            acc[j] = pa[(int64_t)j * kHeadDim];
        }
    }
    const int64_t pos = min(pos_in, (int64_t)capacity - 1);
    if (pos < 0) return;  // no partials were written (the partial kernel flagged it)
    const int used = (int)min((int64_t)splits, pos / kAttnChunk + 1);
    float M = -INFINITY, L = 0.f, A = 0.f;
    for (int s0 = 0; s0 < used; s0 += kMergeBatch) {
        if (s0 > 0) {
#pragma unroll
            for (int j = 0; j < kMergeBatch; ++j) {
                if (s0 + j < used) {
                    v[j] = ml[s0 + j];
                    acc[j] = pa[(int64_t)(s0 + j) * kHeadDim];
                }
            }
        }
        float Mb = M;
#pragma unroll
        for (int j = 0; j < kMergeBatch; ++j)
            if (s0 + j < used) Mb = fmaxf(Mb, v[j].x);
        const float fo = M == Mb ? 1.f : expf(M - Mb);  // M = -inf: L = A = 0 either way
        L *= fo;
        A *= fo;
#pragma unroll
        for (int j = 0; j < kMergeBatch; ++j) {
            if (s0 + j < used && v[j].x != -INFINITY) {
                const float f = expf(v[j].x - Mb);
                L += v[j].y * f;
                A += acc[j] * f;
            }
        }
        M = Mb;
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

struct AttnArgs {
    const __nv_bfloat16 *q, *k_cache, *v_cache;
    const int64_t* position;
    __nv_bfloat16* out;
    float* ws;
    int batch, q_heads, kv_heads, chunks, capacity;
    int64_t cb, ch, cs;
    float scale;
};

// Partial kernel over `splits` CTAs per (kv head, sequence), then the merge. The partials sit
// in the workspace as acc [batch][q_heads][splits][128], then (max, sum) [..][splits][2];
// splits <= chunks, so they fit the workspace sized for one split per chunk.
template <int G, int VB>
static int launch_attention(const AttnArgs& a, cudaStream_t s) {
    int splits = 0;
    const int st = attn_splits<G, VB>(a.kv_heads * a.batch, a.chunks, &splits);
    if (st != NK_OK) return st;
    float* part_acc = a.ws;
    float* part_ml = part_acc + (size_t)a.batch * a.q_heads * splits * kHeadDim;
    const int rc = launch_pdl_smem(attn_partial_kernel<G, VB>, dim3(splits, a.kv_heads, a.batch),
                                   dim3(kAttnThreads), (size_t)kAttnSmem, s, a.q, a.k_cache,
                                   a.v_cache, a.position, part_acc, part_ml, a.q_heads,
                                   a.kv_heads, splits, a.capacity, a.cb, a.ch, a.cs, a.scale);
    if (rc != NK_OK) return rc;
    return launch_pdl_smem(attn_merge_kernel, dim3(a.batch * a.q_heads), dim3(kHeadDim), 0, s,
                           (const float*)part_acc, (const float*)part_ml, a.out, splits,
                           a.capacity, a.position);
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
    const int chunks = (capacity + kAttnChunk - 1) / kAttnChunk;
    // 16-byte copies when every cache row segment is 16-byte aligned, else 8-byte copies
    const bool wide = al16(k_cache) && al16(v_cache) && cache_seq_stride % 8 == 0 &&
                      cache_head_stride % 8 == 0 && cache_batch_stride % 8 == 0;
    const AttnArgs a{static_cast<const __nv_bfloat16*>(q),
                     static_cast<const __nv_bfloat16*>(k_cache),
                     static_cast<const __nv_bfloat16*>(v_cache), position,
                     static_cast<__nv_bfloat16*>(out), static_cast<float*>(ws), batch, q_heads,
                     kv_heads, chunks, capacity, cache_batch_stride, cache_head_stride,
                     cache_seq_stride, scale};
    cudaStream_t s = (cudaStream_t)stream;
    switch (G) {
        case 1: return wide ? launch_attention<1, 16>(a, s) : launch_attention<1, 8>(a, s);
        case 2: return wide ? launch_attention<2, 16>(a, s) : launch_attention<2, 8>(a, s);
        case 4: return wide ? launch_attention<4, 16>(a, s) : launch_attention<4, 8>(a, s);
        default: return wide ? launch_attention<8, 16>(a, s) : launch_attention<8, 8>(a, s);
    }
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

extern "C" int nk_gemm_bf16_qkv_rope_cache(
    const void* x, int64_t ldx, const void* w, int64_t ldw, int M, int N, int K,
    const nk_plan* p, void* ws, size_t ws_bytes, const void* q_norm, const void* k_norm,
    const void* cos_table, const void* sin_table, const int64_t* position, void* q_out,
    void* k_cache, void* v_cache, int q_heads, int kv_heads, int capacity,
    int64_t cache_batch_stride, int64_t cache_head_stride, int64_t cache_seq_stride, float eps,
    nk_stream_t stream) {
    if (!q_norm || !k_norm || !cos_table || !sin_table || !position || !q_out || !k_cache ||
        !v_cache)
        return NK_ERR_ARG;
    if (q_heads < 1 || kv_heads < 1 || capacity < 1 || !(eps > 0.f) ||
        cache_seq_stride < kHeadDim)
        return NK_ERR_SHAPE;
    if ((int64_t)N != (int64_t)(q_heads + 2 * kv_heads) * kHeadDim) return NK_ERR_SHAPE;
    if (!p || p->magic != NK_PLAN_MAGIC) return NK_ERR_PLAN;
    // decode token tiles in the balanced schedule (whole grid resident)
    if (p->kind != NK_KIND_TC || p->split_k != 0 || p->tile_m != 16) return NK_ERR_PLAN;
    if (((uintptr_t)q_out | (uintptr_t)k_cache | (uintptr_t)v_cache | (uintptr_t)q_norm |
         (uintptr_t)k_norm | (uintptr_t)cos_table | (uintptr_t)sin_table) & 1u)
        return NK_ERR_ALIGN;
    if (((uintptr_t)position & 7u) != 0) return NK_ERR_ALIGN;
    QkvIn qk;
    qk.q_norm = q_norm;
    qk.k_norm = k_norm;
    qk.cos_t = cos_table;
    qk.sin_t = sin_table;
    qk.position = position;
    qk.q_out = q_out;
    qk.k_cache = k_cache;
    qk.v_cache = v_cache;
    qk.hq = q_heads;
    qk.hkv = kv_heads;
    qk.capacity = capacity;
    qk.cb = cache_batch_stride;
    qk.ch = cache_head_stride;
    qk.cs = cache_seq_stride;
    qk.eps = eps;
    return gemm_impl(x, ldx, w, ldw, nullptr, N, false, M, N, K, p, ws, ws_bytes, stream, nullptr,
                     nullptr, &qk);
}

