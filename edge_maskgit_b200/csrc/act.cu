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
#include "rowquant.cuh"

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
__global__ void quant_act_kernel(const float* __restrict__ x, int M, int K, ActQ a, int want_c, int8_t* qx,
                                 float* dx, int32_t* sumx) {
    griddep_wait();
    griddep_launch();
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
        *reinterpret_cast<int4*>(a.q + act_code(a, kc, m, j * 32)) = *reinterpret_cast<const int4*>(q);
        *reinterpret_cast<int4*>(a.q + act_code(a, kc, m, j * 32 + 16)) = *reinterpret_cast<const int4*>(q + 16);
        act_dx(a, kc, m)[j] = d;
        if (want_c) act_cx(a, kc, m)[j] = __fmul_rn(d, (float)s);
    } else {
        int4* dst = reinterpret_cast<int4*>(qx + (size_t)m * K + b * 32);
        dst[0] = *reinterpret_cast<const int4*>(q);
        dst[1] = *reinterpret_cast<const int4*>(q + 16);
        dx[(size_t)m * nb + b] = d;
        if (sumx) sumx[(size_t)m * nb + b] = s;
    }
}

void launch_quant_act_plain(const float* x, int M, int K, int8_t* qx, float* dx, int32_t* sumx,
                            cudaStream_t st) {
    ++g_launch_count;
    const long n = (long)M * (K / 32);
    launch_k(quant_act_kernel<false>, (unsigned)((n + 255) / 256), 256, 0, st, x, M, K, ActQ{}, 0, qx, dx, sumx);
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
        a.q[act_code(a, kc, m, kb)] = (int8_t)q;
        int s = q;
        if (want_c) {
#pragma unroll
            for (int k = 16; k > 0; k >>= 1) s += __shfl_xor_sync(0xffffffffu, s, k);
        }
        if (lane == 0) {
            act_dx(a, kc, m)[j] = d;
            if (want_c) act_cx(a, kc, m)[j] = __fmul_rn(d, (float)s);
        }
    }
}

template <int NV>
__global__ void ln_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                          const float* __restrict__ beta, int rows, float eps, float* y, ActQ a,
                          int quant, int want_c) {
    griddep_wait();
    griddep_launch();
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
    griddep_wait();
    griddep_launch();
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

// ---------------------------------------------------------------- chunked row kernels
// Faster layout for D % 256 == 0: lane l of a row's warp holds, for chunk i, the 8
// contiguous elements 256 i + 8 l .. +7 (two 16-byte loads, a fully coalesced warp access),
// so one 32-element quant block is 4 adjacent lanes and its 32 codes leave as four 8-byte
// stores.  LayerNorm keeps the reference's summation order exactly: the row is staged in
// shared memory and lane l forms the partial sums of work-items t = l and t = l + 32 over
// d = t, t+64, ... before the same shuffle tree as above.
template <int NC>
__device__ __forceinline__ void load_chunks(const float* r, float (&v)[NC][8], int lane) {
#pragma unroll
    for (int i = 0; i < NC; i++) {
        const float4* p = reinterpret_cast<const float4*>(r + 256 * i + 8 * lane);
        const float4 a = p[0], b = p[1];
        v[i][0] = a.x; v[i][1] = a.y; v[i][2] = a.z; v[i][3] = a.w;
        v[i][4] = b.x; v[i][5] = b.y; v[i][6] = b.z; v[i][7] = b.w;
    }
}

// LayerNorm of a row held as chunks; sm = this warp's D-float staging row.
template <int NC>
__device__ __forceinline__ void ln_chunks(float (&v)[NC][8], float* sm, const float* gamma, const float* beta,
                                          float eps, int lane) {
    constexpr int D = NC * 256;
    // gamma / beta do not depend on the row: their loads overlap the reductions
    float4 gb[NC][4];
#pragma unroll
    for (int i = 0; i < NC; i++) {
        const float4* gp = reinterpret_cast<const float4*>(gamma + 256 * i + 8 * lane);
        const float4* bp = reinterpret_cast<const float4*>(beta + 256 * i + 8 * lane);
        gb[i][0] = __ldg(gp); gb[i][1] = __ldg(gp + 1); gb[i][2] = __ldg(bp); gb[i][3] = __ldg(bp + 1);
    }
#pragma unroll
    for (int i = 0; i < NC; i++) {
        float4* p = reinterpret_cast<float4*>(sm + 256 * i + 8 * lane);
        p[0] = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
        p[1] = make_float4(v[i][4], v[i][5], v[i][6], v[i][7]);
    }
    __syncwarp();
    float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
    for (int d = 0; d < D; d += 64) { s0 = __fadd_rn(s0, sm[d + lane]); s1 = __fadd_rn(s1, sm[d + lane + 32]); }
    float s = __fadd_rn(s0, s1);
#pragma unroll
    for (int k = 16; k > 0; k >>= 1) s = __fadd_rn(s, __shfl_down_sync(0xffffffffu, s, k));
    s = __shfl_sync(0xffffffffu, s, 0);
    const float mean = __fdiv_rn(s, (float)D);
    float w0 = 0.0f, w1 = 0.0f;
#pragma unroll
    for (int d = 0; d < D; d += 64) {
        const float u0 = __fsub_rn(sm[d + lane], mean), u1 = __fsub_rn(sm[d + lane + 32], mean);
        w0 = __fmaf_rn(u0, u0, w0);
        w1 = __fmaf_rn(u1, u1, w1);
    }
    float w = __fadd_rn(w0, w1);
#pragma unroll
    for (int k = 16; k > 0; k >>= 1) w = __fadd_rn(w, __shfl_down_sync(0xffffffffu, w, k));
    w = __shfl_sync(0xffffffffu, w, 0);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(w, (float)D), eps)));
#pragma unroll
    for (int i = 0; i < NC; i++) {
        const float4 g0 = gb[i][0], g1 = gb[i][1], b0 = gb[i][2], b1 = gb[i][3];
        const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
        for (int e = 0; e < 8; e++) v[i][e] = __fmaf_rn(__fmul_rn(__fsub_rn(v[i][e], mean), inv), g[e], bb[e]);
    }
}

template <int NC>
__device__ __forceinline__ void store_chunks(float* r, const float (&v)[NC][8], int lane) {
#pragma unroll
    for (int i = 0; i < NC; i++) {
        float4* p = reinterpret_cast<float4*>(r + 256 * i + 8 * lane);
        p[0] = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
        p[1] = make_float4(v[i][4], v[i][5], v[i][6], v[i][7]);
    }
}

// MODE 0: y = LN(x);  MODE 1: y = LN(tok[id] + pos[s]);  MODE 2: quantize x only.
template <int NC, int MODE>
__global__ void __launch_bounds__(128) rows_kernel(const float* __restrict__ x, const float* __restrict__ tok,
                                                   int vocab, const float* __restrict__ pos,
                                                   const int32_t* __restrict__ tokens, int S, int rows,
                                                   const float* __restrict__ gamma, const float* __restrict__ beta,
                                                   float eps, float* y, ActQ a, int quant, int want_c, int xw,
                                                   long long xstride) {
    griddep_wait();
    griddep_launch();
    extern __shared__ float stage[];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m = blockIdx.x * 4 + w;
    if (m >= rows) return;
    constexpr int D = NC * 256;
    float v[NC][8];
    if (MODE == 1) {
        int id = tokens[m];
        if (id < 0) id += vocab;   // negative ids wrap (mask token), mg-opencl.cpp:670
        float p[NC][8];
        load_chunks<NC>(tok + (size_t)id * D, v, lane);
        load_chunks<NC>(pos + (size_t)(m % S) * D, p, lane);
#pragma unroll
        for (int i = 0; i < NC; i++)
#pragma unroll
            for (int e = 0; e < 8; e++) v[i][e] = __fadd_rn(v[i][e], p[i][e]);
    } else if (xw > 0) {
        // column-blocked input (the all-gather layout of a column-split layer): columns
        // [g*xw, (g+1)*xw) of every row sit in block g at x + g*xstride, rows xw apart
#pragma unroll
        for (int i = 0; i < NC; i++) {
            const int k = 256 * i + 8 * lane, g = k / xw;
            const float* src = x + (size_t)g * xstride + (size_t)m * xw + (k - g * xw);
            const float4 u0 = reinterpret_cast<const float4*>(src)[0], u1 = reinterpret_cast<const float4*>(src)[1];
            v[i][0] = u0.x; v[i][1] = u0.y; v[i][2] = u0.z; v[i][3] = u0.w;
            v[i][4] = u1.x; v[i][5] = u1.y; v[i][6] = u1.z; v[i][7] = u1.w;
        }
    } else {
        load_chunks<NC>(x + (size_t)m * D, v, lane);
    }
    if (MODE != 2) {
        ln_chunks<NC>(v, stage + w * D, gamma, beta, eps, lane);
        store_chunks<NC>(y + (size_t)m * D, v, lane);
    }
    if (quant) quant_chunks<NC>(v, m, a, want_c != 0, lane);
}

template <int MODE>
static bool launch_rows(int D, const float* x, const float* tok, int vocab, const float* pos, const int32_t* tokens,
                        int S, int rows, const float* gamma, const float* beta, float eps, float* y, const ActQ* a,
                        bool want_c, cudaStream_t st, int xw = 0, long long xstride = 0) {
    const ActQ aa = a ? *a : ActQ{};
    const unsigned blocks = (unsigned)((rows + 3) / 4);
    const size_t sm = MODE == 2 ? 0 : (size_t)4 * D * sizeof(float);
#define MGC_ROWS(NC)                                                                                       \
    case NC:                                                                                               \
        launch_k(rows_kernel<NC, MODE>, blocks, 128, sm, st, x, tok, vocab, pos, tokens, S, rows, gamma, beta, eps, y, \
                                                       aa, a != nullptr, want_c, xw, xstride);             \
        return true;
    switch (D % 256 == 0 ? D / 256 : 0) {
        MGC_ROWS(1) MGC_ROWS(2) MGC_ROWS(3) MGC_ROWS(4) MGC_ROWS(6) MGC_ROWS(8) MGC_ROWS(12)
        default: return false;
    }
#undef MGC_ROWS
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
    ++g_launch_count;
    if (D <= 2048 && launch_rows<0>(D, x, nullptr, 0, nullptr, nullptr, 1, rows, gamma, beta, eps, y, a, want_c, st))
        return;
    const ActQ aa = a ? *a : ActQ{};
    const unsigned blocks = (unsigned)((rows + 7) / 8);
    MGC_NV_SWITCH(D, (launch_k(ln_kernel<NV>, blocks, 256, 0, st, x, gamma, beta, rows, eps, y, aa, a != nullptr,
                                                            want_c)));
}

void launch_embed(const float* tok, int vocab, const float* pos, int E, const int32_t* tokens, int B,
                  int S, float* y, cudaStream_t st) {
    ++g_launch_count;
    const int rows = B * S;
    const unsigned blocks = (unsigned)((rows + 7) / 8);
    MGC_NV_SWITCH(E, (launch_k(embed_ln_kernel<NV>, blocks, 256, 0, st, tok, vocab, pos, tokens, S, rows, nullptr,
                                                                  nullptr, 0.0f, y, ActQ{}, 0, 0, 0)));
}

void launch_embed_ln(const float* tok, int vocab, const float* pos, int E, const int32_t* tokens, int B,
                     int S, const float* gamma, const float* beta, float eps, float* y, const ActQ* a,
                     bool want_c, cudaStream_t st) {
    ++g_launch_count;
    if (E <= 2048 && launch_rows<1>(E, nullptr, tok, vocab, pos, tokens, S, B * S, gamma, beta, eps, y, a, want_c, st))
        return;
    const int rows = B * S;
    const ActQ aa = a ? *a : ActQ{};
    const unsigned blocks = (unsigned)((rows + 7) / 8);
    MGC_NV_SWITCH(E, (launch_k(embed_ln_kernel<NV>, blocks, 256, 0, st, tok, vocab, pos, tokens, S, rows, gamma,
                                                                  beta, eps, y, aa, 1, a != nullptr, want_c)));
}

bool launch_ln_blocked(const float* x, int xw, long long xstride, const float* gamma, const float* beta, int rows,
                       int D, float eps, float* y, const ActQ* a, bool want_c, cudaStream_t st) {
    ++g_launch_count;
    return D <= 2048 && xw > 0 && xw % 8 == 0 &&
           launch_rows<0>(D, x, nullptr, 0, nullptr, nullptr, 1, rows, gamma, beta, eps, y, a, want_c, st, xw, xstride);
}

bool launch_quant_blocked(const float* x, int xw, long long xstride, int M, int K, const ActQ& a, bool want_c,
                          cudaStream_t st) {
    ++g_launch_count;
    return xw > 0 && xw % 8 == 0 &&
           launch_rows<2>(K, x, nullptr, 0, nullptr, nullptr, 1, M, nullptr, nullptr, 0.0f, nullptr, &a, want_c, st, xw,
                          xstride);
}

void launch_quant_act_tiled(const float* x, int M, int K, const ActQ& a, bool want_c, cudaStream_t st) {
    ++g_launch_count;
    if (launch_rows<2>(K, x, nullptr, 0, nullptr, nullptr, 1, M, nullptr, nullptr, 0.0f, nullptr, &a, want_c, st))
        return;
    const long n = (long)M * (K / 32);
    launch_k(quant_act_kernel<true>, (unsigned)((n + 255) / 256), 256, 0, st, x, M, K, a, want_c ? 1 : 0,
             (int8_t*)nullptr, (float*)nullptr, (int32_t*)nullptr);
}

// ---------------------------------------------------------------- decode-loop sampling
// Per logits row (one warp per row): softmax over the first CB logits and a categorical draw
// with the caller's uniform r, in the arithmetic of generate() (src/mg-generate.cpp:87-100,
// sample_categorical :30-35): mx = max row[v]; e_v = exp(row[v] - mx) (the f32 exponential,
// correctly rounded here by evaluating it in f64); sum = e_0 + e_1 + ... in order (f32);
// p_v = e_v * (1 / sum); the first v with r <= p_0 + ... + p_v (accumulated in f64), else
// CB - 1.  Lanes compute the exponentials, lane 0 runs the two ordered sums.
__global__ void __launch_bounds__(128) sample_codes_kernel(const float* __restrict__ logits, int rows, int vocab,
                                                           int CB, const double* __restrict__ r,
                                                           int32_t* __restrict__ sid, float* __restrict__ psid) {
    griddep_wait();
    griddep_launch();
    extern __shared__ float e_sm[];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, row = blockIdx.x * 4 + w;
    if (row >= rows) return;
    const float* L = logits + (size_t)row * vocab;
    float* e = e_sm + (size_t)w * CB;
    float mx = -INFINITY;
    for (int v = lane; v < CB; v += 32) mx = fmaxf(mx, L[v]);
#pragma unroll
    for (int k = 16; k > 0; k >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, k));
    for (int v = lane; v < CB; v += 32) e[v] = (float)exp((double)__fsub_rn(L[v], mx));
    __syncwarp();
    if (lane == 0) {
        float sum = 0.0f;
        for (int v = 0; v < CB; v++) sum = __fadd_rn(sum, e[v]);
        const float inv = __fdiv_rn(1.0f, sum);
        const double rr = r[row];
        double acc = 0.0;
        int pick = CB - 1;
        for (int v = 0; v < CB; v++) {
            acc = __dadd_rn(acc, (double)__fmul_rn(e[v], inv));
            if (rr <= acc) { pick = v; break; }
        }
        sid[row] = pick;
        psid[row] = __fmul_rn(e[pick], inv);
    }
}

void launch_sample_codes(const float* logits, int rows, int vocab, int CB, const double* r, int32_t* sid, float* psid,
                         cudaStream_t st) {
    ++g_launch_count;
    launch_k(sample_codes_kernel, (unsigned)((rows + 3) / 4), 128, (size_t)4 * CB * sizeof(float), st, logits, rows,
             vocab, CB, r, sid, psid);
}

}  // namespace mgc
