// act.cu -- activation-side kernels: the per-32-block int8 quantizer, LayerNorm-affine
// (optionally fused with the quantizer of its output) and the token+position embedding.
//
// The quantizer restates k_quantize_q8 (mg-opencl.cpp:424-434) with IEEE operations in
// the same order (amax, d = amax/127, id = 1/d, q = round-half-away(x*id), no clamp), so
// qx and dx are bit-identical to the reference formulas.  LayerNorm restates
// k_norm_affine (mg-opencl.cpp:705-727): the reference's 64 work-items each sum a strided
// slice (d = t, t+64, ...) and then tree-reduce lp[t] += lp[t+k], k = 32..1.  Here one warp
// owns a row and each lane carries the slices of work-items t = lane and t = lane + 32, so
// the tree's first level is a register add and the rest are shuffle-downs in the same order.
#include "kernels.h"
#include "ptx.cuh"

namespace mgc {

// one 32-element block: quantize 32 floats held by one thread
__device__ __forceinline__ void quant_block32(const float* v, int8_t* q, float& d_out, int& sum_out) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(v[i]));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    int s = 0;
#pragma unroll
    for (int i = 0; i < 32; i++) {
        const int qi = (int)roundf(__fmul_rn(v[i], id));
        q[i] = (int8_t)qi;
        s += (int8_t)qi;
    }
    d_out = d;
    sum_out = s;
}

// thread per (row, 32-block)
template <bool TILED>
__global__ void quant_act_kernel(const float* __restrict__ x, int M, int K, int8_t* qx, float* dx,
                                 float* cx, int32_t* sumx, int Mpad) {
    const int nb = K / 32;
    const long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (long)M * nb) return;
    const int m = (int)(t / nb), b = (int)(t % nb);
    float v[32];
    const float4* src = reinterpret_cast<const float4*>(x + (size_t)m * K + b * 32);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const float4 f = src[i];
        v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
    }
    alignas(16) int8_t q[32];
    float d; int s;
    quant_block32(v, q, d, s);
    if (TILED) {
        const int kc = b >> 2, j = b & 3;
        int8_t* row = qx + ((size_t)kc * Mpad + m) * 128;
        const uint32_t c0 = (uint32_t)(2 * j) ^ (uint32_t)(m & 7), c1 = (uint32_t)(2 * j + 1) ^ (uint32_t)(m & 7);
        *reinterpret_cast<int4*>(row + c0 * 16) = *reinterpret_cast<const int4*>(q);
        *reinterpret_cast<int4*>(row + c1 * 16) = *reinterpret_cast<const int4*>(q + 16);
        dx[((size_t)kc * Mpad + m) * 4 + j] = d;
        if (cx) cx[((size_t)kc * Mpad + m) * 4 + j] = __fmul_rn(d, (float)s);
    } else {
        int4* dst = reinterpret_cast<int4*>(qx + (size_t)m * K + b * 32);
        dst[0] = *reinterpret_cast<const int4*>(q);
        dst[1] = *reinterpret_cast<const int4*>(q + 16);
        dx[(size_t)m * nb + b] = d;
        if (sumx) sumx[(size_t)m * nb + b] = s;
    }
}

void launch_quant_act_tiled(const float* x, int M, int K, const ActQ& a, bool want_c, cudaStream_t st) {
    const long n = (long)M * (K / 32);
    quant_act_kernel<true><<<(unsigned)((n + 255) / 256), 256, 0, st>>>(x, M, K, a.q, a.d,
                                                                         want_c ? a.c : nullptr, nullptr, a.Mpad);
}
void launch_quant_act_plain(const float* x, int M, int K, int8_t* qx, float* dx, int32_t* sumx,
                            cudaStream_t st) {
    const long n = (long)M * (K / 32);
    quant_act_kernel<false><<<(unsigned)((n + 255) / 256), 256, 0, st>>>(x, M, K, qx, dx, nullptr, sumx, 0);
}

// ---------------------------------------------------------------- LayerNorm (+ quantizer)
// Lane l holds v[i] = row[l + 32 i], i < NV (NV = D/32 <= 64).  Even i belong to the
// reference's work-item t = l, odd i to t = l + 32.
template <int NV>
__device__ __forceinline__ void ln_row_warp(float (&v)[NV], int D, const float* gamma, const float* beta,
                                            float eps, int lane) {
    float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; i += 2) { s0 = __fadd_rn(s0, v[i]); s1 = __fadd_rn(s1, v[i + 1]); }
    float s = __fadd_rn(s0, s1);
#pragma unroll
    for (int k = 16; k > 0; k >>= 1) s = __fadd_rn(s, __shfl_down_sync(0xffffffffu, s, k));
    s = __shfl_sync(0xffffffffu, s, 0);
    const float mean = __fdiv_rn(s, (float)D);
    float w0 = 0.0f, w1 = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; i += 2) {
        const float u0 = __fsub_rn(v[i], mean), u1 = __fsub_rn(v[i + 1], mean);
        w0 = __fmaf_rn(u0, u0, w0);
        w1 = __fmaf_rn(u1, u1, w1);
    }
    float w = __fadd_rn(w0, w1);
#pragma unroll
    for (int k = 16; k > 0; k >>= 1) w = __fadd_rn(w, __shfl_down_sync(0xffffffffu, w, k));
    w = __shfl_sync(0xffffffffu, w, 0);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(w, (float)D), eps)));
#pragma unroll
    for (int i = 0; i < NV; i++) {
        const int d = lane + 32 * i;
        v[i] = __fmaf_rn(__fmul_rn(__fsub_rn(v[i], mean), inv), __ldg(gamma + d), __ldg(beta + d));
    }
}

// Quantize a row held as v[i] = row[l + 32 i]: block b is v[b] across the warp.
template <int NV>
__device__ __forceinline__ void quant_row_warp(const float (&v)[NV], int m, const ActQ& a, bool want_c, int lane) {
#pragma unroll
    for (int b = 0; b < NV; b++) {
        float amax = fabsf(v[b]);
#pragma unroll
        for (int k = 16; k > 0; k >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, k));
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        const int q = (int)roundf(__fmul_rn(v[b], id));
        const int kc = b >> 2, j = b & 3;
        const uint32_t kb = (uint32_t)(j * 32 + lane);
        a.q[((size_t)kc * a.Mpad + m) * 128 + sw128_off(m & 7, kb) - (uint32_t)(m & 7) * 128u] = (int8_t)q;
        int s = q;
        if (want_c) {
#pragma unroll
            for (int k = 16; k > 0; k >>= 1) s += __shfl_xor_sync(0xffffffffu, s, k);
        }
        if (lane == 0) {
            a.d[((size_t)kc * a.Mpad + m) * 4 + j] = d;
            if (want_c) a.c[((size_t)kc * a.Mpad + m) * 4 + j] = __fmul_rn(d, (float)s);
        }
    }
}

template <int NV>
__global__ void ln_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                          const float* __restrict__ beta, int rows, float eps, float* y, ActQ a,
                          int quant, int want_c) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= rows) return;
    constexpr int D = NV * 32;
    float v[NV];
    const float* r = x + (size_t)warp * D;
#pragma unroll
    for (int i = 0; i < NV; i++) v[i] = r[lane + 32 * i];
    ln_row_warp<NV>(v, D, gamma, beta, eps, lane);
    float* o = y + (size_t)warp * D;
#pragma unroll
    for (int i = 0; i < NV; i++) o[lane + 32 * i] = v[i];
    if (quant) quant_row_warp<NV>(v, warp, a, want_c != 0, lane);
}

template <int NV>
__global__ void embed_ln_kernel(const float* __restrict__ tok, int vocab, const float* __restrict__ pos,
                                const int32_t* __restrict__ tokens, int S, int rows,
                                const float* __restrict__ gamma, const float* __restrict__ beta,
                                float eps, float* y, ActQ a, int do_ln, int quant, int want_c) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= rows) return;
    constexpr int D = NV * 32;
    int id = tokens[warp];
    if (id < 0) id += vocab;   // negative ids wrap (mask token), mg-opencl.cpp:670
    const int s = warp % S;
    float v[NV];
#pragma unroll
    for (int i = 0; i < NV; i++)
        v[i] = __fadd_rn(tok[(size_t)id * D + lane + 32 * i], pos[(size_t)s * D + lane + 32 * i]);
    if (do_ln) ln_row_warp<NV>(v, D, gamma, beta, eps, lane);
    float* o = y + (size_t)warp * D;
#pragma unroll
    for (int i = 0; i < NV; i++) o[lane + 32 * i] = v[i];
    if (quant) quant_row_warp<NV>(v, warp, a, want_c != 0, lane);
}

#define MGC_NV_SWITCH(D, CALL)           \
    switch ((D) / 32) {                  \
        case 2: { constexpr int NV = 2; CALL; } break;   \
        case 4: { constexpr int NV = 4; CALL; } break;   \
        case 8: { constexpr int NV = 8; CALL; } break;   \
        case 12: { constexpr int NV = 12; CALL; } break; \
        case 16: { constexpr int NV = 16; CALL; } break; \
        case 24: { constexpr int NV = 24; CALL; } break; \
        case 32: { constexpr int NV = 32; CALL; } break; \
        case 48: { constexpr int NV = 48; CALL; } break; \
        case 64: { constexpr int NV = 64; CALL; } break; \
        default: break;                  \
    }

void launch_ln(const float* x, const float* gamma, const float* beta, int rows, int D, float eps,
               float* y, const ActQ* a, bool want_c, cudaStream_t st) {
    const ActQ aa = a ? *a : ActQ{};
    const unsigned blocks = (unsigned)((rows + 7) / 8);
    MGC_NV_SWITCH(D, (ln_kernel<NV><<<blocks, 256, 0, st>>>(x, gamma, beta, rows, eps, y, aa, a != nullptr,
                                                            want_c)));
}

void launch_embed(const float* tok, int vocab, const float* pos, int E, const int32_t* tokens, int B,
                  int S, float* y, cudaStream_t st) {
    const int rows = B * S;
    const unsigned blocks = (unsigned)((rows + 7) / 8);
    MGC_NV_SWITCH(E, (embed_ln_kernel<NV><<<blocks, 256, 0, st>>>(tok, vocab, pos, tokens, S, rows, nullptr,
                                                                  nullptr, 0.0f, y, ActQ{}, 0, 0, 0)));
}

void launch_embed_ln(const float* tok, int vocab, const float* pos, int E, const int32_t* tokens, int B,
                     int S, const float* gamma, const float* beta, float eps, float* y, const ActQ* a,
                     bool want_c, cudaStream_t st) {
    const int rows = B * S;
    const ActQ aa = a ? *a : ActQ{};
    const unsigned blocks = (unsigned)((rows + 7) / 8);
    MGC_NV_SWITCH(E, (embed_ln_kernel<NV><<<blocks, 256, 0, st>>>(tok, vocab, pos, tokens, S, rows, gamma,
                                                                  beta, eps, y, aa, 1, a != nullptr, want_c)));
}

}  // namespace mgc
