/*
 * ORACLE — TEST INFRASTRUCTURE ONLY. Nothing in the product (neokernel_b200/) links, loads or
 * calls this file; only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg do,
 * and only as the checker.
 *
 * CPU restatement of the reference's decode linear
 *
 *     torch.mm(x, W.t(), out=y)          engine/kernels/decode.py:54,58,64,66; engine/engine.py:114
 *
 * on bf16 tensors. The arithmetic itself lives in a third-party dependency that is not under
 * the reference tree: PyTorch (the reference pins torch==2.5.1, requirements.txt:9), whose
 * bf16 `mm` widens bf16 operands to fp32, accumulates in fp32 and rounds the result once to
 * bf16 with round-to-nearest-even (cuBLAS on the GPU, ATen/oneDNN on the CPU). This file
 * restates that published algorithm:
 *
 *   - bf16 -> fp32 widening is exact (bf16 is the upper 16 bits of binary32);
 *   - the product of two bf16 values is exact in fp32 (8-bit x 8-bit significands), so the
 *     only roundings are the fp32 additions, done here in ascending k;
 *   - fp32 -> bf16 narrowing is round-to-nearest-even with NaN kept quiet.
 *
 * The summation order of cuBLAS/oneDNN is unpublished, so the oracle agrees with them to
 * within the fp32 re-association error (at most one bf16 ulp after rounding, and rarely);
 * the parity tests state that bound. nko_gemm_f64 gives the exact-order-free reference
 * (double accumulation, no output rounding) used for the north-star tolerance
 * max|y - y_ref| <= 2e-2 * sqrt(K / 1024).
 *
 * Pinned against golden vectors produced by the reference's own packing and call
 * (tests/golden/make_golden.py, run where the reference is importable).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

float nko_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

uint16_t nko_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, sizeof u);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u); /* quiet NaN */
    const uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb; /* ties go to the even neighbour; overflow rounds to infinity */
    return (uint16_t)(u >> 16);
}

/* y[m, n] = bf16( sum_k fp32(x[m, k]) * fp32(w[n, k]) ), k ascending, fp32 accumulator. */
void nko_gemm_bf16(const uint16_t* x, int64_t ldx, const uint16_t* w, int64_t ldw, uint16_t* y,
                   int64_t ldy, int M, int N, int K) {
    for (int n = 0; n < N; ++n) {
        const uint16_t* wr = w + (int64_t)n * ldw;
        for (int m = 0; m < M; ++m) {
            const uint16_t* xr = x + (int64_t)m * ldx;
            float acc = 0.0f;
            for (int k = 0; k < K; ++k) acc += nko_bf16_to_f32(xr[k]) * nko_bf16_to_f32(wr[k]);
            y[(int64_t)m * ldy + n] = nko_f32_to_bf16(acc);
        }
    }
}

/* Same inputs, double accumulation, no rounding of the result (the tolerance reference). */
void nko_gemm_f64(const uint16_t* x, int64_t ldx, const uint16_t* w, int64_t ldw, double* y,
                  int64_t ldy, int M, int N, int K) {
    for (int n = 0; n < N; ++n) {
        const uint16_t* wr = w + (int64_t)n * ldw;
        for (int m = 0; m < M; ++m) {
            const uint16_t* xr = x + (int64_t)m * ldx;
            double acc = 0.0;
            for (int k = 0; k < K; ++k)
                acc += (double)nko_bf16_to_f32(xr[k]) * (double)nko_bf16_to_f32(wr[k]);
            y[(int64_t)m * ldy + n] = acc;
        }
    }
}

/* Element-wise conversions over arrays (used by the tests' rounding known-answer cases). */
void nko_f32_to_bf16_array(const float* f, uint16_t* h, int64_t n) {
    for (int64_t i = 0; i < n; ++i) h[i] = nko_f32_to_bf16(f[i]);
}
