// gemm_f32.cu -- F32 GEMM with the fused bias/act/residual epilogue (k_mul_mat_t,
// mg-opencl.cpp:57-98).  Used for the MLM head (token_embd, kept F32 by
// tools/convert_to_gguf.py:213-216) and for linears a GGUF stores unquantized.
//
// 64x64 output tile per CTA of 256 threads, 4x4 register micro-tile per thread, K staged
// 32 at a time in shared memory.  Every output accumulates k = 0..K-1 in order with one
// FMA per term, so results equal the sequential reference sum fma by fma.
#include "kernels.h"
#include "ptx.cuh"

namespace mgc {

constexpr int GF_BM = 64, GF_BN = 64, GF_BK = 32;   // 256 threads, 4 x 4 outputs each

__device__ __forceinline__ float act_f32(float v, int a) {
    if (a == 1) return 0.5f * v * (1.0f + erff(v * 0.70710678f));
    if (a == 2) return __fdiv_rn(v, 1.0f + expf(-v));
    return v;
}

__global__ void __launch_bounds__(256) gemm_f32_kernel(const float* __restrict__ w, const float* __restrict__ x,
                                                       int M, int N, int K, const float* __restrict__ bias,
                                                       int act, const float* __restrict__ resid,
                                                       float* __restrict__ y) {
    griddep_wait();
    griddep_launch();
    // two slab buffers: the next slab's global loads are in flight while this one is consumed
    __shared__ __align__(16) float As[2][GF_BK][GF_BM + 4];   // x slab, As[k][m]
    __shared__ __align__(16) float Bs[2][GF_BK][GF_BN + 4];   // w slab, Bs[k][n]
    const int tid = threadIdx.x, tm = tid / 16, tn = tid % 16;   // 16 x 16 threads, 4 x 4 each
    const int m0 = blockIdx.y * GF_BM, n0 = blockIdx.x * GF_BN;
    const bool vec = (K % 4) == 0;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;
    // 64 rows x 32 k per operand: 2 float4 per thread, transposed into [k][row]
    float4 xa[2], wb[2];
    auto fetch = [&](int k0) {
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int l = tid + 256 * h, r = l / 8, kq = (l % 8) * 4, gk = k0 + kq;
            const int gm = m0 + r, gn = n0 + r;
            xa[h] = make_float4(0, 0, 0, 0);
            wb[h] = make_float4(0, 0, 0, 0);
            if (vec && gk + 3 < K) {
                if (gm < M) xa[h] = __ldg(reinterpret_cast<const float4*>(x + (size_t)gm * K + gk));
                if (gn < N) wb[h] = __ldg(reinterpret_cast<const float4*>(w + (size_t)gn * K + gk));
            } else {
                float t[4], u[4];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    t[e] = (gm < M && gk + e < K) ? x[(size_t)gm * K + gk + e] : 0.0f;
                    u[e] = (gn < N && gk + e < K) ? w[(size_t)gn * K + gk + e] : 0.0f;
                }
                xa[h] = make_float4(t[0], t[1], t[2], t[3]);
                wb[h] = make_float4(u[0], u[1], u[2], u[3]);
            }
        }
    };
    auto stash = [&](int buf) {
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int l = tid + 256 * h, r = l / 8, kq = (l % 8) * 4;
            As[buf][kq][r] = xa[h].x; As[buf][kq + 1][r] = xa[h].y; As[buf][kq + 2][r] = xa[h].z; As[buf][kq + 3][r] = xa[h].w;
            Bs[buf][kq][r] = wb[h].x; Bs[buf][kq + 1][r] = wb[h].y; Bs[buf][kq + 2][r] = wb[h].z; Bs[buf][kq + 3][r] = wb[h].w;
        }
    };
    fetch(0);
    for (int k0 = 0, buf = 0; k0 < K; k0 += GF_BK, buf ^= 1) {
        stash(buf);
        __syncthreads();   // (one barrier per slab: the buffer written next was last read two slabs ago)
        if (k0 + GF_BK < K) fetch(k0 + GF_BK);
        const int kn = min(GF_BK, K - k0);
        auto step = [&](int kk) {   // k ascending: each output is a sequential fma chain
            const float4 a4 = *reinterpret_cast<const float4*>(&As[buf][kk][tm * 4]);
            const float4 b4 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tn * 4]);
            const float a[4] = {a4.x, a4.y, a4.z, a4.w}, bb[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = __fmaf_rn(bb[j], a[i], acc[i][j]);
        };
        if (kn == GF_BK) {   // full slab: unrolled so the shared-memory loads run ahead of the FMAs
#pragma unroll
            for (int kk = 0; kk < GF_BK; kk++) step(kk);
        } else {
            for (int kk = 0; kk < kn; kk++) step(kk);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int m = m0 + tm * 4 + i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int n = n0 + tn * 4 + j;
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
    ++g_launch_count;
    dim3 grid((N + GF_BN - 1) / GF_BN, (M + GF_BM - 1) / GF_BM);
    launch_k(gemm_f32_kernel, grid, 256, 0, st, w, x, M, N, K, bias, act, resid, y);
}

}  // namespace mgc
