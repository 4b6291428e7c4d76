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
                          int Hq, int Hkv, int64_t cb, int64_t ch, int64_t cs, float eps) {
    __shared__ float red[32];
    __shared__ float xs[kHeadDim];
    if (threadIdx.x == 0) griddep_launch_dependents();
    griddep_wait();
    const int h = blockIdx.x;
    const int b = blockIdx.y;
    const int d = threadIdx.x;
    const int64_t pos = *position;
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
// the KV head, so each K/V row is read once per group. Four warps take every fourth position
// with an online softmax per query head (lane l holds elements 4l..4l+3); the warps' states
// are combined in shared memory and the CTA stores (max, sum, unnormalised acc). A merge
// kernel combines the splits: out = sum_s e^(m_s-M) acc_s / sum_s e^(m_s-M) l_s.
// ---------------------------------------------------------------------------------------
constexpr int kAttnChunk = 64;
constexpr int kAttnThreads = 128;
constexpr int kAttnMaxGroup = 8;

template <int G>
__global__ void __launch_bounds__(kAttnThreads)
attn_partial_kernel(const __nv_bfloat16* q, const __nv_bfloat16* k_cache,
                    const __nv_bfloat16* v_cache, const int64_t* position, float* part_acc,
                    float* part_ml, int Hq, int Hkv, int splits, int64_t cb, int64_t ch,
                    int64_t cs, float scale) {
    __shared__ float s_m[4][G], s_l[4][G];
    __shared__ float s_acc[4][G][kHeadDim];
    if (threadIdx.x == 0) griddep_launch_dependents();
    griddep_wait();
    const int split = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t pos = *position;
    const int j0 = split * kAttnChunk;
    const int j1 = (int)min((int64_t)j0 + kAttnChunk, pos + 1);

    float qf[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const __nv_bfloat16* qp = q + ((int64_t)b * Hq + kh * G + g) * kHeadDim + lane * 4;
        const uint2 qv = *reinterpret_cast<const uint2*>(qp);
        qf[g][0] = bf16lo(qv.x); qf[g][1] = bf16hi(qv.x);
        qf[g][2] = bf16lo(qv.y); qf[g][3] = bf16hi(qv.y);
    }
    float m[G], l[G], acc[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY; l[g] = 0.f;
        acc[g][0] = acc[g][1] = acc[g][2] = acc[g][3] = 0.f;
    }
    const __nv_bfloat16* kb = k_cache + (int64_t)b * cb + (int64_t)kh * ch + lane * 4;
    const __nv_bfloat16* vb = v_cache + (int64_t)b * cb + (int64_t)kh * ch + lane * 4;
    for (int j = j0 + warp; j < j1; j += 4) {
        const uint2 kv = *reinterpret_cast<const uint2*>(kb + (int64_t)j * cs);
        const uint2 vv = *reinterpret_cast<const uint2*>(vb + (int64_t)j * cs);
        const float k0 = bf16lo(kv.x), k1 = bf16hi(kv.x), k2 = bf16lo(kv.y), k3 = bf16hi(kv.y);
        const float v0 = bf16lo(vv.x), v1 = bf16hi(vv.x), v2 = bf16lo(vv.y), v3 = bf16hi(vv.y);
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float sc = qf[g][0] * k0 + qf[g][1] * k1 + qf[g][2] * k2 + qf[g][3] * k3;
            sc = warp_sum(sc) * scale;
            const float mn = fmaxf(m[g], sc);
            const float corr = expf(m[g] - mn);  // 0 while m is still -inf
            const float p = expf(sc - mn);
            l[g] = l[g] * corr + p;
            acc[g][0] = acc[g][0] * corr + p * v0;
            acc[g][1] = acc[g][1] * corr + p * v1;
            acc[g][2] = acc[g][2] * corr + p * v2;
            acc[g][3] = acc[g][3] * corr + p * v3;
            m[g] = mn;
        }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
        if (lane == 0) { s_m[warp][g] = m[g]; s_l[warp][g] = l[g]; }
#pragma unroll
        for (int e = 0; e < 4; ++e) s_acc[warp][g][lane * 4 + e] = acc[g][e];
    }
    __syncthreads();
    // thread t combines element d = t of every query head of the group
    const int d = threadIdx.x;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; ++w) M = fmaxf(M, s_m[w][g]);
        float L = 0.f, A = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                const float f = expf(s_m[w][g] - M);
                L += s_l[w][g] * f;
                A += s_acc[w][g][d] * f;
            }
        }
        const int64_t hrow = ((int64_t)b * Hq + kh * G + g) * splits + split;
        part_acc[hrow * kHeadDim + d] = A;
        if (d == 0) {
            part_ml[hrow * 2] = M;
            part_ml[hrow * 2 + 1] = L;
        }
    }
}

__global__ void __launch_bounds__(kHeadDim)
attn_merge_kernel(const float* part_acc, const float* part_ml, __nv_bfloat16* out, int splits,
                  const int64_t* position) {
    if (threadIdx.x == 0) griddep_launch_dependents();
    griddep_wait();
    const int64_t hrow = blockIdx.x;  // b * Hq + h
    const int d = threadIdx.x;
    const int used = (int)min((int64_t)splits, *position / kAttnChunk + 1);
    float M = -INFINITY;
    for (int s = 0; s < used; ++s) M = fmaxf(M, part_ml[(hrow * splits + s) * 2]);
    float L = 0.f, A = 0.f;
    for (int s = 0; s < used; ++s) {
        const float ms = part_ml[(hrow * splits + s) * 2];
        if (ms == -INFINITY) continue;
        const float f = expf(ms - M);
        L += part_ml[(hrow * splits + s) * 2 + 1] * f;
        A += part_acc[(hrow * splits + s) * kHeadDim + d] * f;
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
                                          int q_heads, int kv_heads, int head_dim,
                                          int64_t cache_batch_stride, int64_t cache_head_stride,
                                          int64_t cache_seq_stride, float eps,
                                          nk_stream_t stream) {
    if (!qkv || !q_norm || !k_norm || !cos_table || !sin_table || !position || !q_out ||
        !k_cache || !v_cache)
        return NK_ERR_ARG;
    if (head_dim != kHeadDim || batch < 1 || q_heads < 1 || kv_heads < 1 ||
        ld_qkv < (int64_t)(q_heads + 2 * kv_heads) * head_dim || cache_seq_stride < head_dim)
        return NK_ERR_SHAPE;
    return launch_pdl_smem(
        qk_norm_rope_cache_kernel, dim3(q_heads + kv_heads, batch), dim3(kHeadDim), 0,
        (cudaStream_t)stream, static_cast<const __nv_bfloat16*>(qkv), ld_qkv,
        static_cast<const __nv_bfloat16*>(q_norm), static_cast<const __nv_bfloat16*>(k_norm),
        static_cast<const __nv_bfloat16*>(cos_table), static_cast<const __nv_bfloat16*>(sin_table),
        position, static_cast<__nv_bfloat16*>(q_out), static_cast<__nv_bfloat16*>(k_cache),
        static_cast<__nv_bfloat16*>(v_cache), q_heads, kv_heads, cache_batch_stride,
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
    int st;
    switch (G) {
        case 1: st = launch_pdl_smem(attn_partial_kernel<1>, grid, dim3(kAttnThreads), 0, s, qq, kk, vv, position, part_acc, part_ml, q_heads, kv_heads, splits, cache_batch_stride, cache_head_stride, cache_seq_stride, scale); break;
        case 2: st = launch_pdl_smem(attn_partial_kernel<2>, grid, dim3(kAttnThreads), 0, s, qq, kk, vv, position, part_acc, part_ml, q_heads, kv_heads, splits, cache_batch_stride, cache_head_stride, cache_seq_stride, scale); break;
        case 4: st = launch_pdl_smem(attn_partial_kernel<4>, grid, dim3(kAttnThreads), 0, s, qq, kk, vv, position, part_acc, part_ml, q_heads, kv_heads, splits, cache_batch_stride, cache_head_stride, cache_seq_stride, scale); break;
        default: st = launch_pdl_smem(attn_partial_kernel<8>, grid, dim3(kAttnThreads), 0, s, qq, kk, vv, position, part_acc, part_ml, q_heads, kv_heads, splits, cache_batch_stride, cache_head_stride, cache_seq_stride, scale); break;
    }
    if (st != NK_OK) return st;
    return launch_pdl_smem(attn_merge_kernel, dim3(batch * q_heads), dim3(kHeadDim), 0, s,
                           (const float*)part_acc, (const float*)part_ml,
                           static_cast<__nv_bfloat16*>(out), splits, position);
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
