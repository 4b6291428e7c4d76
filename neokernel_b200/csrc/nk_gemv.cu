// CUDA-core weight-streaming GEMV for decode batches M <= 16, and the generic kernel for
// operands whose layout the vectorised kernels cannot take.
//
// Replaces the cuBLAS GEMMs that torch.mm(x, W.t(), out=y) launches at
// engine/kernels/decode.py:54,58,64,66 and engine/engine.py:114 when M is a decode batch.
//
// GEMV data path (one CTA = 8 warps, BN = 8*R weight rows, one K slice):
//   - each warp owns R consecutive weight rows; lane l reads the 16-byte chunk
//     [k + 8l, k + 8l + 8) of every row, so a warp load is 512 contiguous bytes of a row;
//   - U such chunks per row are issued before any is consumed (R*U 128-bit loads in flight
//     per thread) with ld.global.nc.L1::no_allocate, so weight bytes bypass L1;
//   - the activations x[m, k..k+8) are re-read per chunk through the read-only cache
//     (they are tiny and shared by every CTA);
//   - products accumulate in fp32, then a butterfly warp reduction gives the row sums;
//   - with split_k > 1 the CTA stores an fp32 partial and the last CTA of the output tile
//     reduces the slices in a fixed order (nk_common.cuh).
#include "nk_common.cuh"

namespace nk {

template <int MT, int R>
__device__ __forceinline__ void gemv_accumulate(const uint4 (&wv)[R], const __nv_bfloat16* xrow,
                                                int64_t ldx, int k, int mcount,
                                                float (&acc)[R][MT]) {
    float wf[R][8];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        wf[r][0] = bf16lo(wv[r].x); wf[r][1] = bf16hi(wv[r].x);
        wf[r][2] = bf16lo(wv[r].y); wf[r][3] = bf16hi(wv[r].y);
        wf[r][4] = bf16lo(wv[r].z); wf[r][5] = bf16hi(wv[r].z);
        wf[r][6] = bf16lo(wv[r].w); wf[r][7] = bf16hi(wv[r].w);
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        if (m < mcount) {
            const uint4 xv = ld_nc_v4(xrow + (int64_t)m * ldx + k);
            float xf[8];
            xf[0] = bf16lo(xv.x); xf[1] = bf16hi(xv.x);
            xf[2] = bf16lo(xv.y); xf[3] = bf16hi(xv.y);
            xf[4] = bf16lo(xv.z); xf[5] = bf16hi(xv.z);
            xf[6] = bf16lo(xv.w); xf[7] = bf16hi(xv.w);
#pragma unroll
            for (int r = 0; r < R; ++r) {
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[r][m] = fmaf(wf[r][j], xf[j], acc[r][m]);
            }
        }
    }
}

template <int MT, int R, int U>
__global__ void __launch_bounds__(256)
gemv_kernel(GemmArgs a, int k_slice, int splits) {
    constexpr int BN = 8 * R;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int n_tile = blockIdx.x;
    const int s = blockIdx.y;
    const int m_tile = blockIdx.z;
    const int m0 = m_tile * MT;
    const int mcount = min(MT, a.M - m0);
    const int row0 = n_tile * BN + warp * R;
    const int kb = s * k_slice;
    const int ke = min(a.K, kb + k_slice);

    // Rows past N re-read row N-1 (always valid memory); their sums are never stored.
    const __nv_bfloat16* wrow[R];
#pragma unroll
    for (int r = 0; r < R; ++r) wrow[r] = a.w + (int64_t)min(row0 + r, a.N - 1) * a.ldw;
    const __nv_bfloat16* xrow = a.x + (int64_t)m0 * a.ldx;

    float acc[R][MT];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[r][m] = 0.f;

    if (threadIdx.x == 0) griddep_launch_dependents();
    // The first batch of weight loads is issued before waiting for the previous kernel
    // (weights are read-only); activations and outputs are touched only after the wait.
    bool waited = false;
    int kk = kb;
    for (; kk + kGemvKStep * U <= ke; kk += kGemvKStep * U) {
        uint4 wv[U][R];
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
            for (int r = 0; r < R; ++r)
                wv[u][r] = ld_stream_v4(wrow[r] + kk + u * kGemvKStep + lane * 8);
        if (!waited) {
            griddep_wait();
            waited = true;
        }
#pragma unroll
        for (int u = 0; u < U; ++u)
            gemv_accumulate<MT, R>(wv[u], xrow, a.ldx, kk + u * kGemvKStep + lane * 8, mcount, acc);
    }
    if (!waited) griddep_wait();
    for (; kk < ke; kk += kGemvKStep) {
        const int k = kk + lane * 8;
        if (k < ke) {  // K % 8 == 0, so a chunk is either fully inside the slice or outside
            uint4 wv[R];
#pragma unroll
            for (int r = 0; r < R; ++r) wv[r] = ld_stream_v4(wrow[r] + k);
            gemv_accumulate<MT, R>(wv, xrow, a.ldx, k, mcount, acc);
        }
    }

#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[r][m] = warp_sum(acc[r][m]);

    // Every lane now holds every sum; lane (r*MT + m) % 32 stores (row r, token m).
    if (splits == 1) {
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int m = 0; m < MT; ++m)
                if (((r * MT + m) & 31) == lane && m < mcount && row0 + r < a.N)
                    store_out(a, (int64_t)(m0 + m) * a.ldy + row0 + r, acc[r][m]);
        return;
    }

#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int m = 0; m < MT; ++m)
            if (((r * MT + m) & 31) == lane && m < mcount && row0 + r < a.N)
                a.part[((size_t)s * a.M + m0 + m) * a.N + row0 + r] = acc[r][m];

    unsigned* ticket = a.tickets + (size_t)m_tile * gridDim.x + n_tile;
    if (splitk_last_cta(ticket, splits)) {
        if (threadIdx.x == 0) *ticket = 0u;
        splitk_reduce_tile<2>(a, n_tile * BN, BN, m0, mcount, splits);
    }
}

// Generic kernel: any strides, any K, 2-byte aligned operands. One warp per weight row and
// kGenericTokens tokens; lanes stride over K. Correct everywhere, fast nowhere; the plan
// only selects it when the vectorised layout rules are not met.
__global__ void __launch_bounds__(256) generic_kernel(GemmArgs a) {
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int n = blockIdx.x * kGenericRows + warp;
    const int m0 = blockIdx.y * kGenericTokens;
    if (threadIdx.x == 0) griddep_launch_dependents();
    griddep_wait();
    if (n >= a.N) return;
    float acc[kGenericTokens];
#pragma unroll
    for (int j = 0; j < kGenericTokens; ++j) acc[j] = 0.f;
    const __nv_bfloat16* wr = a.w + (int64_t)n * a.ldw;
    for (int k = lane; k < a.K; k += 32) {
        const float wv = __bfloat162float(wr[k]);
#pragma unroll
        for (int j = 0; j < kGenericTokens; ++j)
            if (m0 + j < a.M)
                acc[j] = fmaf(wv, __bfloat162float(a.x[(int64_t)(m0 + j) * a.ldx + k]), acc[j]);
    }
#pragma unroll
    for (int j = 0; j < kGenericTokens; ++j) {
        const float v = warp_sum(acc[j]);
        if (lane == j && m0 + j < a.M) store_out(a, (int64_t)(m0 + j) * a.ldy + n, v);
    }
}

int gemv_token_tile(int M_max) {
    if (M_max <= 1) return 1;
    if (M_max <= 2) return 2;
    if (M_max <= 4) return 4;
    if (M_max <= 8) return 8;
    return 16;
}

int gemv_rows_per_cta(int mt) { return mt <= 2 ? 16 : 32; }

// Launch with programmatic stream serialization (see griddep_wait in nk_common.cuh).
template <typename Kernel, typename... Args>
static int launch_pdl(Kernel kernel, dim3 grid, dim3 block, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = NK_PDL ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...) == cudaSuccess ? NK_OK : NK_ERR_CUDA;
}

int launch_gemv(const nk_plan& p, const GemmArgs& a, cudaStream_t s) {
    const int mt = p.tile_m;
    const dim3 grid(p.n_tiles, p.split_k, (a.M + mt - 1) / mt);
    const dim3 block(256);
    const int ks = p.k_slice;
    const int sp = p.split_k;
    switch (mt) {
        case 1:  return launch_pdl(gemv_kernel<1, 2, 4>, grid, block, s, a, ks, sp);
        case 2:  return launch_pdl(gemv_kernel<2, 2, 4>, grid, block, s, a, ks, sp);
        case 4:  return launch_pdl(gemv_kernel<4, 4, 2>, grid, block, s, a, ks, sp);
        case 8:  return launch_pdl(gemv_kernel<8, 4, 2>, grid, block, s, a, ks, sp);
        case 16: return launch_pdl(gemv_kernel<16, 4, 2>, grid, block, s, a, ks, sp);
        default: return NK_ERR_PLAN;
    }
}

int launch_generic(const nk_plan& p, const GemmArgs& a, cudaStream_t s) {
    (void)p;
    const dim3 grid((a.N + kGenericRows - 1) / kGenericRows,
                    (a.M + kGenericTokens - 1) / kGenericTokens, 1);
    return launch_pdl(generic_kernel, grid, dim3(32 * kGenericRows), s, a);
}

}  // namespace nk
