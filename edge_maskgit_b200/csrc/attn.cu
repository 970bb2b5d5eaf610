// attn.cu -- fp16-K/V flash attention (k_flash_attention_h, mg-opencl.cpp:859-937).
//
// Same algorithm and operation order as the reference kernel: Q, K and V are rounded to
// half, keys are visited in tiles of 32, scores / running max / running sum / output are
// f32 with the online-softmax rescale per tile.  The input is the fused QKV projection
// [B*S][3E] (q | k | v, head h at columns h*Dh), the output is written head-merged
// [B*S][E], which is what the reference's permute+cont (mg-transformer.cpp:84) produces.
//
// SIMT kernel: one thread per query row, a CTA = 64 query rows of one (image, head); the
// K/V tile of 32 keys is staged in shared memory (already rounded through half).
#include "kernels.h"
#include "ptx.cuh"
#include <cuda_fp16.h>

namespace mgc {

constexpr int FA_D = 48, FA_BC = 32, FA_ROWS = 64;

__device__ __forceinline__ float rhalf(float x) { return __half2float(__float2half_rn(x)); }

__global__ void __launch_bounds__(FA_ROWS) flash_attn_simt(const float* __restrict__ qkv, int S, int H,
                                                           float scale, float* __restrict__ out) {
    const int E = H * FA_D, W = 3 * E;
    const int h = blockIdx.y, b = blockIdx.z;
    const int row = blockIdx.x * FA_ROWS + threadIdx.x;
    const bool active = row < S;
    __shared__ float Kt[FA_BC * FA_D];
    __shared__ float Vt[FA_BC * FA_D];
    const float* base = qkv + (size_t)b * S * W + h * FA_D;
    float q[FA_D], o[FA_D];
    if (active) {
#pragma unroll
        for (int d = 0; d < FA_D; d++) q[d] = rhalf(base[(size_t)row * W + d]);
    }
#pragma unroll
    for (int d = 0; d < FA_D; d++) o[d] = 0.0f;
    float m_i = -INFINITY, l_i = 0.0f;
    for (int kb = 0; kb < S; kb += FA_BC) {
        __syncthreads();
        for (int idx = threadIdx.x; idx < FA_BC * FA_D; idx += FA_ROWS) {
            const int kc = idx / FA_D, dd = idx % FA_D, t = kb + kc;
            const bool in = t < S;
            Kt[idx] = in ? rhalf(base[(size_t)t * W + E + dd]) : 0.0f;
            Vt[idx] = in ? rhalf(base[(size_t)t * W + 2 * E + dd]) : 0.0f;
        }
        __syncthreads();
        if (!active) continue;
        float sc[FA_BC];
        float m_new = m_i;
#pragma unroll
        for (int kc = 0; kc < FA_BC; kc++) {
            if (kb + kc >= S) { sc[kc] = -INFINITY; continue; }
            float dot = 0.0f;
#pragma unroll
            for (int d = 0; d < FA_D; d++) dot = __fmaf_rn(q[d], Kt[kc * FA_D + d], dot);
            dot = __fmul_rn(dot, scale);
            sc[kc] = dot;
            m_new = fmaxf(m_new, dot);
        }
        const float alpha = expf(m_i - m_new);
        float l_new = __fmul_rn(alpha, l_i);
#pragma unroll
        for (int kc = 0; kc < FA_BC; kc++) {
            const float pk = (sc[kc] == -INFINITY) ? 0.0f : expf(sc[kc] - m_new);
            sc[kc] = pk;
            l_new = __fadd_rn(l_new, pk);
        }
        const int nk = min(FA_BC, S - kb);
#pragma unroll
        for (int d = 0; d < FA_D; d++) {
            float no = __fmul_rn(alpha, o[d]);
            for (int kc = 0; kc < nk; kc++) no = __fmaf_rn(sc[kc], Vt[kc * FA_D + d], no);
            o[d] = no;
        }
        m_i = m_new;
        l_i = l_new;
    }
    if (active) {
        const float inv = __fdiv_rn(1.0f, l_i);
        float* dst = out + ((size_t)b * S + row) * E + h * FA_D;
#pragma unroll
        for (int d = 0; d < FA_D; d++) dst[d] = __fmul_rn(o[d], inv);
    }
}

int launch_flash_attn(const float* qkv, int B, int S, int H, int Dh, float scale, float* out, cudaStream_t st) {
    if (Dh != FA_D) return -2;
    dim3 grid((S + FA_ROWS - 1) / FA_ROWS, H, B);
    flash_attn_simt<<<grid, FA_ROWS, 0, st>>>(qkv, S, H, scale, out);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace mgc
