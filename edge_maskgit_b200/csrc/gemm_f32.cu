// gemm_f32.cu -- F32 GEMM with the fused bias/act/residual epilogue (k_mul_mat_t,
// mg-opencl.cpp:57-98).  Used for the MLM head (token_embd, kept F32 by
// tools/convert_to_gguf.py:213-216) and for linears a GGUF stores unquantized.
//
// 128x64 output tile per CTA of 256 threads, 8x4 register micro-tile per thread, K staged
// 16 at a time in shared memory.  Every output accumulates k = 0..K-1 in order with one
// FMA per term, so results equal the sequential reference sum fma by fma.
#include "kernels.h"
#include "ptx.cuh"

namespace mgc {

constexpr int GF_BM = 128, GF_BN = 64, GF_BK = 16, GF_TM = 8, GF_TN = 4;

__device__ __forceinline__ float act_f32(float v, int a) {
    if (a == 1) return 0.5f * v * (1.0f + erff(v * 0.70710678f));
    if (a == 2) return __fdiv_rn(v, 1.0f + expf(-v));
    return v;
}

__global__ void __launch_bounds__(256) gemm_f32_kernel(const float* __restrict__ w, const float* __restrict__ x,
                                                       int M, int N, int K, const float* __restrict__ bias,
                                                       int act, const float* __restrict__ resid,
                                                       float* __restrict__ y) {
    __shared__ float As[GF_BK][GF_BM + 4];   // x slab, As[k][m]
    __shared__ float Bs[GF_BK][GF_BN + 4];   // w slab, Bs[k][n]
    const int tid = threadIdx.x, tm = tid / 16, tn = tid % 16;   // 16 x 16 threads
    const int m0 = blockIdx.y * GF_BM, n0 = blockIdx.x * GF_BN;
    float acc[GF_TM][GF_TN];
#pragma unroll
    for (int i = 0; i < GF_TM; i++)
#pragma unroll
        for (int j = 0; j < GF_TN; j++) acc[i][j] = 0.0f;
    for (int k0 = 0; k0 < K; k0 += GF_BK) {
        for (int l = tid; l < GF_BM * GF_BK; l += 256) {
            const int r = l / GF_BK, kk = l % GF_BK, gm = m0 + r, gk = k0 + kk;
            As[kk][r] = (gm < M && gk < K) ? x[(size_t)gm * K + gk] : 0.0f;
        }
        for (int l = tid; l < GF_BN * GF_BK; l += 256) {
            const int r = l / GF_BK, kk = l % GF_BK, gn = n0 + r, gk = k0 + kk;
            Bs[kk][r] = (gn < N && gk < K) ? w[(size_t)gn * K + gk] : 0.0f;
        }
        __syncthreads();
        const int kn = min(GF_BK, K - k0);
        for (int kk = 0; kk < kn; kk++) {
            float a[GF_TM], bb[GF_TN];
#pragma unroll
            for (int i = 0; i < GF_TM; i++) a[i] = As[kk][tm + 16 * i];
#pragma unroll
            for (int j = 0; j < GF_TN; j++) bb[j] = Bs[kk][tn + 16 * j];
#pragma unroll
            for (int i = 0; i < GF_TM; i++)
#pragma unroll
                for (int j = 0; j < GF_TN; j++) acc[i][j] = __fmaf_rn(bb[j], a[i], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < GF_TM; i++) {
        const int m = m0 + tm + 16 * i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < GF_TN; j++) {
            const int n = n0 + tn + 16 * j;
            if (n >= N) continue;
            float v = acc[i][j];
            if (bias) v = __fadd_rn(v, bias[n]);
            v = act_f32(v, act);
            if (resid) v = __fadd_rn(v, resid[(size_t)m * N + n]);
            y[(size_t)m * N + n] = v;
        }
    }
}

void launch_gemm_f32(const float* w, const float* x, int M, int N, int K, const float* bias, int act,
                     const float* resid, float* y, cudaStream_t st) {
    dim3 grid((N + GF_BN - 1) / GF_BN, (M + GF_BM - 1) / GF_BM);
    gemm_f32_kernel<<<grid, 256, 0, st>>>(w, x, M, N, K, bias, act, resid, y);
}

}  // namespace mgc
