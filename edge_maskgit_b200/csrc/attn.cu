// attn.cu -- fp16-K/V flash attention (k_flash_attention_h, mg-opencl.cpp:859-937) on
// tcgen05 tensor cores.
//
// Semantics follow the reference kernel: Q, K and V are rounded to half, scores are
// accumulated in f32 and scaled by 1/sqrt(Dh) after the dot product, softmax statistics and
// the output accumulator are f32 with the online (flash) rescale per key tile.  Input is the
// fused QKV projection [B*S][3E] (q | k | v, head h at columns h*Dh); the output is written
// head-merged [B*S][E], i.e. what the reference's permute+cont (mg-transformer.cpp:84) makes.
//
// One CTA = 128 query rows of one (image, head), 4 warps, thread = one query row (= one TMEM
// lane).  Per key tile of 128:
//   1. all threads stage K (row-major) and V^T as f16 into 128-byte-swizzled shared memory;
//   2. one thread issues S = Q K^T (M=128, N=128, K=48 as 3 x K16 MMAs) into TMEM;
//   3. each thread reads its score row from TMEM, updates max / sum, and writes P split as
//      P_hi = f16(p), P_lo = f16(p - P_hi) to shared memory (so P keeps ~22 bits, like the
//      reference's f32 P);
//   4. one thread issues O_tile = P_hi V + P_lo V (M=128, N=48, K=128) into TMEM;
//   5. each thread rescales its register accumulator o[48] by alpha and adds O_tile.
#include "kernels.h"
#include "ptx.cuh"
#include "rowquant.cuh"
#include <cuda_fp16.h>

namespace mgc {

namespace fa {
constexpr int D = 48, BM = 128, BC = 128;
constexpr uint32_t Q_BYTES = BM * 128;            // [128 rows][64 halves], cols 48..63 unused
constexpr uint32_t K_BYTES = BC * 128;            // [128 keys][64 halves]
constexpr uint32_t VT_BLK = D * 128;              // V^T atom block: [48 dims][64 keys]
constexpr uint32_t VT_BYTES = 2 * VT_BLK;         // keys 0..63 | 64..127
constexpr uint32_t P_BLK = BM * 128;              // P atom block: [128 rows][64 keys]
constexpr uint32_t P_BYTES = 2 * P_BLK;
constexpr uint32_t OFF_Q = 0, OFF_K = OFF_Q + Q_BYTES, OFF_VT = OFF_K + K_BYTES,
                   OFF_PH = OFF_VT + VT_BYTES, OFF_PL = OFF_PH + P_BYTES, OFF_BAR = OFF_PL + P_BYTES;
constexpr uint32_t SMEM = 1024 + OFF_BAR + 64;
constexpr uint32_t TMEM_COLS = 256;               // S: cols 0..127, O tile: cols 128..175
}  // namespace fa

// store 8 halves (16 bytes) as logical chunk `c` of row `r` in a 128B-swizzled block
__device__ __forceinline__ void st_chunk(uint8_t* blk, int r, int c, const __half2 (&h)[4]) {
    *reinterpret_cast<uint4*>(blk + r * 128 + ((c ^ (r & 7)) << 4)) = *reinterpret_cast<const uint4*>(h);
}
__device__ __forceinline__ void st_half(uint8_t* blk, int r, int k, __half v) {
    *reinterpret_cast<__half*>(blk + sw128_off(r, k * 2)) = v;
}

__global__ void __launch_bounds__(128) flash_attn_tc(const float* __restrict__ qkv, int S, int H, float scale,
                                                     float* __restrict__ out, int nsplit, int tiles_per,
                                                     float* __restrict__ opart, float* __restrict__ mlpart) {
    using namespace fa;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bar_s = (uint64_t*)(sm + OFF_BAR);
    uint64_t* bar_o = bar_s + 1;
    uint32_t* tmem_slot = (uint32_t*)(bar_s + 2);
    volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.y, b = blockIdx.z / nsplit, split = blockIdx.z % nsplit, q0 = blockIdx.x * BM;
    const int E = H * D, W = 3 * E;
    const float* base = qkv + (size_t)b * S * W + h * D;

    if (tid == 0) {
        mbar_init(bar_s, 1);
        mbar_init(bar_o, 1);
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 0) tmem_alloc(tmem_slot, TMEM_COLS);
    griddep_wait();   // qkv comes from the preceding kernel
    griddep_launch();

    // Q tile -> f16, swizzled
    {
        const int r = tid, qr = q0 + r;
        const float4* src = reinterpret_cast<const float4*>(base + (size_t)qr * W);
#pragma unroll
        for (int c = 0; c < D / 8; c++) {
            __half2 hv[4];
            if (qr < S) {
                const float4 a = src[2 * c], bq = src[2 * c + 1];
                hv[0] = __floats2half2_rn(a.x, a.y); hv[1] = __floats2half2_rn(a.z, a.w);
                hv[2] = __floats2half2_rn(bq.x, bq.y); hv[3] = __floats2half2_rn(bq.z, bq.w);
            } else {
                hv[0] = hv[1] = hv[2] = hv[3] = __floats2half2_rn(0.f, 0.f);
            }
            st_chunk(sm + OFF_Q, r, c, hv);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t t_row = tmem + ((uint32_t)(warp * 32) << 16);

    constexpr uint32_t idesc_o = idesc_make(1, 0, 0, BM, D);
    const uint32_t sQ = smem_u32(sm + OFF_Q), sK = smem_u32(sm + OFF_K), sV = smem_u32(sm + OFF_VT),
                   sPh = smem_u32(sm + OFF_PH), sPl = smem_u32(sm + OFF_PL);

    float o[D];
#pragma unroll
    for (int d = 0; d < D; d++) o[d] = 0.0f;
    float m_i = -INFINITY, l_i = 0.0f;
    const int ntiles = (S + BC - 1) / BC;
    const int kt0 = split * tiles_per, kt1 = min(ntiles, kt0 + tiles_per);
    const bool wact = q0 + warp * 32 < S;   // warp-uniform: this warp owns at least one real query row
    bool ok = true;

    for (int kt = kt0; kt < kt1 && ok; kt++) {
        const int kb = kt * BC, ph = (kt - kt0) & 1;
        // a short last tile runs the MMAs at N (and K for P.V) = valid keys rounded up to 16
        const int nvalid = min(BC, S - kb), nmma = (nvalid + 15) & ~15, nch = (nmma + 31) / 32;
        // ---- 1. stage K and V^T (f16)
        {
            const int t = kb + tid;
            const float4* ks = reinterpret_cast<const float4*>(base + (size_t)t * W + E);
            const float4* vs = reinterpret_cast<const float4*>(base + (size_t)t * W + 2 * E);
            uint8_t* vblk = sm + OFF_VT + (tid >> 6) * VT_BLK;
            const int kk = tid & 63;
#pragma unroll
            for (int c = 0; c < D / 8; c++) {
                __half2 hk[4];
                float v8[8];
                if (t < S) {
                    const float4 a = ks[2 * c], bb = ks[2 * c + 1];
                    hk[0] = __floats2half2_rn(a.x, a.y); hk[1] = __floats2half2_rn(a.z, a.w);
                    hk[2] = __floats2half2_rn(bb.x, bb.y); hk[3] = __floats2half2_rn(bb.z, bb.w);
                    const float4 va = vs[2 * c], vb = vs[2 * c + 1];
                    v8[0] = va.x; v8[1] = va.y; v8[2] = va.z; v8[3] = va.w;
                    v8[4] = vb.x; v8[5] = vb.y; v8[6] = vb.z; v8[7] = vb.w;
                } else {
                    hk[0] = hk[1] = hk[2] = hk[3] = __floats2half2_rn(0.f, 0.f);
#pragma unroll
                    for (int i = 0; i < 8; i++) v8[i] = 0.f;
                }
                st_chunk(sm + OFF_K, tid, c, hk);
#pragma unroll
                for (int i = 0; i < 8; i++) st_half(vblk, c * 8 + i, kk, __float2half_rn(v8[i]));
            }
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        // ---- 2. S = Q K^T
        if (tid == 0) {
            tc_fence_after();
#pragma unroll
            const uint32_t idesc_s = idesc_make(1, 0, 0, BM, nmma);
            for (int k = 0; k < D / 16; k++)
                mma_f16(tmem, sdesc_sw128(sQ + 32 * k), sdesc_sw128(sK + 32 * k), idesc_s, k > 0);
            mma_commit(bar_s);
        }
        ok = mbar_wait(bar_s, ph, abort_flag, 21);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; }
        ok = __syncthreads_and(ok);
        if (!ok) break;
        tc_fence_after();
        // ---- 3. softmax row update, P = hi + lo
        float m_new = m_i, alpha = 1.0f;
        if (wact) {
#pragma unroll
        for (int ch = 0; ch < BC / 32; ch++) {
            if (ch >= nch) break;
            uint32_t r[32];
            tmem_ld32(t_row + ch * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; j++)
                if (ch * 32 + j < nvalid) m_new = fmaxf(m_new, __fmul_rn(__uint_as_float(r[j]), scale));
        }
        alpha = expf(m_i - m_new);
        float l_new = __fmul_rn(alpha, l_i);
        const int row = warp * 32 + lane;
#pragma unroll
        for (int ch = 0; ch < BC / 32; ch++) {
            if (ch >= nch) break;
            uint32_t r[32];
            tmem_ld32(t_row + ch * 32, r);
            tmem_ld_wait();
            uint8_t* ph = sm + OFF_PH + (ch >> 1) * P_BLK;
            uint8_t* pl = sm + OFF_PL + (ch >> 1) * P_BLK;
#pragma unroll
            for (int c = 0; c < 4; c++) {
                __half2 hh[4], hl[4];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    float p2[2];
#pragma unroll
                    for (int e = 0; e < 2; e++) {
                        const int j = c * 8 + i * 2 + e;
                        const float s = __fmul_rn(__uint_as_float(r[j]), scale);
                        p2[e] = (ch * 32 + j < nvalid) ? expf(s - m_new) : 0.0f;
                        l_new = __fadd_rn(l_new, p2[e]);
                    }
                    hh[i] = __floats2half2_rn(p2[0], p2[1]);
                    const float2 back = __half22float2(hh[i]);
                    hl[i] = __floats2half2_rn(p2[0] - back.x, p2[1] - back.y);
                }
                // chunk index within the 64-key atom row: (ch & 1) * 4 + c
                st_chunk(ph, row, (ch & 1) * 4 + c, hh);
                st_chunk(pl, row, (ch & 1) * 4 + c, hl);
            }
        }
        m_i = m_new;
        l_i = l_new;
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        // ---- 4. O_tile = P_hi V + P_lo V
        if (tid == 0) {
            tc_fence_after();
#pragma unroll
            for (int part = 0; part < 2; part++) {
                const uint32_t sP = part == 0 ? sPh : sPl;
#pragma unroll
                for (int j = 0; j < nmma / 16; j++) {
                    const uint32_t a = sP + (j >> 2) * P_BLK + (j & 3) * 32;
                    const uint32_t bv = sV + (j >> 2) * VT_BLK + (j & 3) * 32;
                    mma_f16(tmem + BC, sdesc_sw128(a), sdesc_sw128(bv), idesc_o, (part | j) != 0);
                }
            }
            mma_commit(bar_o);
        }
        ok = mbar_wait(bar_o, ph, abort_flag, 22);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; }
        ok = __syncthreads_and(ok);
        if (!ok) break;
        tc_fence_after();
        // ---- 5. o = alpha * o + O_tile
        if (wact) {
            uint32_t r[32], r2[16];
            tmem_ld32(t_row + BC, r);
            tmem_ld16(t_row + BC + 32, r2);
            tmem_ld_wait();
#pragma unroll
            for (int d = 0; d < 32; d++) o[d] = __fmaf_rn(alpha, o[d], __uint_as_float(r[d]));
#pragma unroll
            for (int d = 0; d < 16; d++) o[32 + d] = __fmaf_rn(alpha, o[32 + d], __uint_as_float(r2[d]));
        }
        tc_fence_before();
        __syncthreads();   // K / V / P buffers are rewritten by the next tile
    }

    const int qr = q0 + warp * 32 + lane;
    if (ok && qr < S && nsplit > 1) {   // partial result of this key range, merged by attn_combine
        const size_t R = (size_t)(gridDim.z / nsplit) * S, r = (size_t)split * R + (size_t)b * S + qr;
        float4* dst = reinterpret_cast<float4*>(opart + r * E + h * D);
#pragma unroll
        for (int d = 0; d < D; d += 4) dst[d / 4] = make_float4(o[d], o[d + 1], o[d + 2], o[d + 3]);
        reinterpret_cast<float2*>(mlpart)[r * H + h] = make_float2(m_i, l_i);
    } else if (ok && qr < S) {
        const float inv = __fdiv_rn(1.0f, l_i);
        float4* dst = reinterpret_cast<float4*>(out + ((size_t)b * S + qr) * E + h * D);
#pragma unroll
        for (int d = 0; d < D; d += 4)
            dst[d / 4] = make_float4(__fmul_rn(o[d], inv), __fmul_rn(o[d + 1], inv), __fmul_rn(o[d + 2], inv),
                                     __fmul_rn(o[d + 3], inv));
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, fa::TMEM_COLS);
    }
}

// Merge the key-range partials: m = max m_s, l = sum l_s e^(m_s - m), o = sum o_s e^(m_s - m) / l.
__global__ void attn_combine(const float* __restrict__ opart, const float* __restrict__ mlpart, int nsplit,
                             int R, int H, float* __restrict__ out) {
    griddep_wait();
    griddep_launch();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;   // (row, head, 4-dim group)
    constexpr int G = fa::D / 4;
    if (i >= R * H * G) return;
    const int rh = i / G, d = (i % G) * 4, r = rh / H, h = rh % H, E = H * fa::D;
    const float2* ml = reinterpret_cast<const float2*>(mlpart);
    float m = -INFINITY;
    for (int s = 0; s < nsplit; s++) m = fmaxf(m, ml[(size_t)s * R * H + rh].x);
    float l = 0.0f;
    float4 acc = make_float4(0, 0, 0, 0);
    for (int s = 0; s < nsplit; s++) {
        const float2 v2 = ml[(size_t)s * R * H + rh];
        const float wgt = expf(v2.x - m);
        l = __fmaf_rn(v2.y, wgt, l);
        const float4 v = *reinterpret_cast<const float4*>(opart + ((size_t)s * R + r) * E + h * fa::D + d);
        acc.x = __fmaf_rn(v.x, wgt, acc.x); acc.y = __fmaf_rn(v.y, wgt, acc.y);
        acc.z = __fmaf_rn(v.z, wgt, acc.z); acc.w = __fmaf_rn(v.w, wgt, acc.w);
    }
    const float inv = __fdiv_rn(1.0f, l);
    *reinterpret_cast<float4*>(out + (size_t)r * E + h * fa::D + d) =
        make_float4(__fmul_rn(acc.x, inv), __fmul_rn(acc.y, inv), __fmul_rn(acc.z, inv), __fmul_rn(acc.w, inv));
}

// Same merge as attn_combine, one warp per row over all heads (row held in chunk layout:
// lane l owns elements 256 i + 8 l .. +7, which lie in one head since 48 % 8 == 0), followed by
// the quantizer of the O projection's input.  out may be null (only the quantized row needed).
template <int NC>
__global__ void __launch_bounds__(128) attn_combine_rows(const float* __restrict__ opart, const float* __restrict__ mlpart,
                                                         int nsplit, int R, int H, float* __restrict__ out, ActQ a,
                                                         int want_c) {
    griddep_wait();
    griddep_launch();
    const int lane = threadIdx.x & 31, r = blockIdx.x * 4 + (threadIdx.x >> 5);
    if (r >= R) return;
    constexpr int E = NC * 256;
    const float2* ml = reinterpret_cast<const float2*>(mlpart);
    float v[NC][8];
#pragma unroll
    for (int i = 0; i < NC; i++) {
        const int e0 = 256 * i + 8 * lane, h = e0 / fa::D, rh = r * H + h;
        float m = -INFINITY;
        for (int s = 0; s < nsplit; s++) m = fmaxf(m, ml[(size_t)s * R * H + rh].x);
        float l = 0.0f, acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int s = 0; s < nsplit; s++) {
            const float2 v2 = ml[(size_t)s * R * H + rh];
            const float wgt = expf(v2.x - m);
            l = __fmaf_rn(v2.y, wgt, l);
            const float4* src = reinterpret_cast<const float4*>(opart + ((size_t)s * R + r) * E + e0);
            const float4 x0 = src[0], x1 = src[1];
            const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
            for (int e = 0; e < 8; e++) acc[e] = __fmaf_rn(xs[e], wgt, acc[e]);
        }
        const float inv = __fdiv_rn(1.0f, l);
#pragma unroll
        for (int e = 0; e < 8; e++) v[i][e] = __fmul_rn(acc[e], inv);
        if (out) {
            float4* dst = reinterpret_cast<float4*>(out + (size_t)r * E + e0);
            dst[0] = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
            dst[1] = make_float4(v[i][4], v[i][5], v[i][6], v[i][7]);
        }
    }
    quant_chunks<NC>(v, r, a, want_c != 0, lane);
}

size_t attn_scratch_floats(int B, int S, int H) {
    return (size_t)kAttnMaxSplit * B * S * H * (fa::D + 2);
}

static bool g_attn_ready[64] = {};

int attn_prepare() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    if (cudaFuncSetAttribute(flash_attn_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, fa::SMEM) != cudaSuccess)
        return -1;
    g_attn_ready[dev] = true;
    return 0;
}

int launch_flash_attn(const float* qkv, int B, int S, int H, int Dh, float scale, float* out, float* scratch,
                      size_t scratch_floats, cudaStream_t st, const ActQ* qo, bool qo_c, bool* quantized) {
    if (quantized) *quantized = false;
    if (Dh != fa::D) return -2;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return -1;
    if (!g_attn_ready[dev] && attn_prepare() != 0) return -1;   // runtimes prepare at creation
    // Split the key range over CTAs when (query tiles x heads x images) leaves SMs idle.
    const int qt = (S + fa::BM - 1) / fa::BM, ntiles = (S + fa::BC - 1) / fa::BC;
    const long ctas = (long)qt * H * B;
    int nsplit = 1;
    if (scratch && scratch_floats >= attn_scratch_floats(B, S, H))
        while (nsplit < kAttnMaxSplit && nsplit < ntiles && ctas * (nsplit + 1) <= 2 * 148) nsplit++;
    const int tiles_per = (ntiles + nsplit - 1) / nsplit;
    nsplit = (ntiles + tiles_per - 1) / tiles_per;   // no empty split
    const int R = B * S;
    float* opart = scratch;
    float* mlpart = scratch ? scratch + (size_t)nsplit * R * H * fa::D : nullptr;
    dim3 grid(qt, H, B * nsplit);
    launch_k(flash_attn_tc, grid, 128, fa::SMEM, st, qkv, S, H, scale, out, nsplit, tiles_per, opart, mlpart);
    g_launch_count += nsplit > 1 ? 2 : 1;
    if (nsplit > 1 && qo && H * fa::D == 768) {   // merge + quantize in one pass (warp per row)
        launch_k(attn_combine_rows<3>, (R + 3) / 4, 128, 0, st, opart, mlpart, nsplit, R, H, out, *qo, qo_c ? 1 : 0);
        if (quantized) *quantized = true;
    } else if (nsplit > 1) launch_k(attn_combine, (R * H * (fa::D / 4) + 255) / 256, 256, 0, st, opart, mlpart, nsplit, R, H, out);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace mgc
