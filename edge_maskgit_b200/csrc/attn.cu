// attn.cu -- fp16-K/V flash attention (k_flash_attention_h, mg-opencl.cpp:859-937) on
// tcgen05 tensor cores.
//
// Semantics follow the reference kernel: Q, K and V are rounded to half, scores are
// accumulated in f32 and scaled by 1/sqrt(Dh) after the dot product, softmax statistics and
// the output accumulator are f32 with the online (flash) rescale per key tile.  Input is the
// fused QKV projection [B*S][3E] (q | k | v, head h at columns h*Dh); the output is written
// head-merged [B*S][E], i.e. what the reference's permute+cont (mg-transformer.cpp:84) makes.
// Exponentials run in the base-2 domain (scores pre-scaled by log2 e) with exp2f.
//
// attn_prep converts Q, K, V once to f16 tiles of 128 rows per (image, head), already in the
// 128-byte-swizzled shared-memory layout the MMAs read (Q and K rows of 64 halves, V
// transposed as two [48 dims][64 keys] atom blocks), so the attention kernel streams whole
// tiles with one bulk copy each instead of re-converting every K/V tile in every query-tile CTA.
//
// flash_attn_tc: one CTA = 128 query rows of one (image, head, key range); 8 warps, warps w and
// w+4 share TMEM lanes 32(w%4).. (one query row per lane) and split each tile's 128 scores and
// the 48 output dims in halves.  Per key tile (K/V double-buffered by bulk copies):
//   S = Q K^T (3 x K16 MMAs) in TMEM -> row max / exp / sum in registers (halves exchange max
//   and sum through shared memory) -> P split as P_hi = f16(p), P_lo = f16(p - P_hi) (keeps
//   ~22 bits, like the reference's f32 P) -> O_tile = P_hi V + P_lo V in TMEM -> o = alpha o +
//   O_tile in registers.
#include <cstdlib>

#include "kernels.h"
#include "qgemm_common.cuh"
#include "ptx.cuh"
#include "rowquant.cuh"
#include "attnprep.cuh"

namespace mgc {

// Standalone prep pass: block = 128 positions of one (image, head, part), thread = one position.
// Padding positions (s >= S) are written as zeros so padded keys stay finite in P.V.
__global__ void __launch_bounds__(128) attn_prep(const float* __restrict__ qkv, int S, int H, int nt,
                                                 uint8_t* __restrict__ prep) {
    griddep_wait();
    griddep_launch();
    using namespace fa;
    int x = blockIdx.x;
    const int part = x % 3; x /= 3;
    const int t = x % nt; x /= nt;
    const int h = x % H, b = x / H;
    const int s = t * BM + threadIdx.x, E = H * D;
    const float* src = qkv + ((size_t)b * S + s) * (3 * E) + part * E + h * D;
#pragma unroll
    for (int j = 0; j < D / 16; j++) {
        float v[16];
        if (s < S) {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float4 f = __ldg(reinterpret_cast<const float4*>(src + 16 * j + 4 * i));
                v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 16; i++) v[i] = 0.0f;
        }
        prep_store_at<16>(prep, H, nt, b, s, h, part, 16 * j, v);
    }
}

// Softmax pieces shared by both attention kernels.  A thread holds its query row's scores for
// NCH 32-key chunks, chunk index ch = NCH * part + cc (r[cc][j] = key 32 ch + j, as f32 bits).
// Row max of the raw scores (4 chains), scaled once: rounding is monotonic, so this equals the
// max of the scaled scores.
// FULL: every key of the thread's chunks is valid (all but a key range's last tile), so the
// per-key masking compiles away.
__device__ __forceinline__ float fmax3(float a, float b, float c) {   // one three-input max (sm_100)
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
template <int NCH, bool FULL = false>
__device__ __forceinline__ float tile_row_max(const uint32_t (&r)[NCH][32], int part, int nch, int nvalid, float c1) {
    float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
    for (int cc = 0; cc < NCH; cc++) {
        const int ch = NCH * part + cc;
        if (!FULL && ch >= nch) break;
        if (FULL) {   // two new scores per instruction (the max is exact: same result in any order)
#pragma unroll
            for (int j = 0; j < 32; j += 2)
                mx[(j >> 1) & 3] = fmax3(mx[(j >> 1) & 3], __uint_as_float(r[cc][j]), __uint_as_float(r[cc][j + 1]));
        } else {
#pragma unroll
            for (int j = 0; j < 32; j++)
                if (ch * 32 + j < nvalid) mx[j & 3] = fmaxf(mx[j & 3], __uint_as_float(r[cc][j]));
        }
    }
    return __fmul_rn(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), c1);
}
// p = 2^(s*c1 - m) on pairs (one packed FMA, two MUFU ex2), P_hi = f16(p), P_lo = f16(p - P_hi)
// into the swizzled P blocks of the sets ph / pl (64 keys per block); returns the partial row
// sum of these chunks (packed partials).
template <int NCH, bool FULL = false>
__device__ __forceinline__ float tile_probs(const uint32_t (&r)[NCH][32], int part, int nch, int nvalid, float c1,
                                            float m_new, int row, uint8_t* ph, uint8_t* pl) {
    const uint64_t c1x2 = pack2(c1, c1), nm2 = pack2(-m_new, -m_new), neg1 = pack2(-1.0f, -1.0f);
    uint64_t ls2[2] = {0, 0};
#pragma unroll
    for (int cc = 0; cc < NCH; cc++) {
        const int ch = NCH * part + cc;
        if (!FULL && ch >= nch) break;
        const bool full = FULL || ch * 32 + 32 <= nvalid;
        uint8_t* bh = ph + (ch >> 1) * fa::P_BLK;
        uint8_t* bl = pl + (ch >> 1) * fa::P_BLK;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            __half2 hh[4], hl[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int j = c * 8 + u * 2;
                float t0, t1;
                unpack2(fma2(pack2(__uint_as_float(r[cc][j]), __uint_as_float(r[cc][j + 1])), c1x2, nm2), t0, t1);
                float p0 = ex2_approx(t0), p1 = ex2_approx(t1);
                if (!full) {
                    p0 = ch * 32 + j < nvalid ? p0 : 0.0f;
                    p1 = ch * 32 + j + 1 < nvalid ? p1 : 0.0f;
                }
                const uint64_t p2 = pack2(p0, p1);
                ls2[u & 1] = add2(ls2[u & 1], p2);
                hh[u] = __floats2half2_rn(p0, p1);
                const float2 back = __half22float2(hh[u]);
                float l0, l1;
                unpack2(fma2(pack2(back.x, back.y), neg1, p2), l0, l1);
                hl[u] = __floats2half2_rn(l0, l1);
            }
            st_chunk(bh, row, (ch & 1) * 4 + c, hh);
            st_chunk(bl, row, (ch & 1) * 4 + c, hl);
        }
    }
    float a0, a1, b0, b1;
    unpack2(ls2[0], a0, a1);
    unpack2(ls2[1], b0, b1);
    return (a0 + b0) + (a1 + b1);
}

// Single-key-tile variant (each CTA's key range is one 128-key tile, as for 257 tokens split
// over three CTAs): no pipeline to overlap, so all 8 warps run the one chain
// S -> softmax -> P V, with thread 0 issuing the MMAs; 128-column TMEM, one P buffer.
namespace fa1 {   // shared-memory layout: Q | K | V^T | (P_hi, P_lo) | row max / sum exchange | barriers
constexpr uint32_t OQ = 0, OK = fa::Q_BYTES, OV = OK + fa::K_BYTES, OP = OV + fa::VT_BYTES, OX = OP + fa::P_SET,
                   OBAR = OX + fa::X_SET;
constexpr uint32_t SMEM = 1024 + OBAR + 128, TMEM_COLS = 256;
}  // namespace fa1

__global__ void __launch_bounds__(256) flash_attn_1t(const uint8_t* __restrict__ prep, int S, int H, float scale,
                                                     float* __restrict__ out, int nsplit,
                                                     float* __restrict__ opart, float* __restrict__ mlpart) {
    using namespace fa;
    using fa1::OQ; using fa1::OK; using fa1::OV; using fa1::OP; using fa1::OX; using fa1::OBAR;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align1024_smem(smem_raw);
    uint64_t* bar_in = (uint64_t*)(sm + OBAR);   // Q, K, V landed (tx)
    uint64_t* bar_s = bar_in + 1;
    uint64_t* bar_o = bar_in + 2;
    uint32_t* tmem_slot = (uint32_t*)(bar_in + 3);
    volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
    float* xmax = reinterpret_cast<float*>(sm + OX);   // [2][128]
    float* xsum = xmax + 2 * BM;                           // [2][128]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, half = warp >> 2;
    const int h = blockIdx.y, b = blockIdx.z / nsplit, split = blockIdx.z % nsplit, qti = blockIdx.x, q0 = qti * BM;
    const int E = H * D, nt = (S + BC - 1) / BC, kt = split;   // one key tile per split
    const uint8_t* base = prep_base(const_cast<uint8_t*>(prep), b, h, H, nt);
    if (tid == 0) {
        for (int i = 0; i < 3; i++) mbar_init(bar_in + i, 1);
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 0) tmem_alloc(tmem_slot, fa1::TMEM_COLS);
    griddep_wait();
    griddep_launch();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int nvalid = min(BC, S - kt * BC), nmma = (nvalid + 15) & ~15, nch = (nmma + 31) / 32;
    bool ok = true;
    if (tid == 0) {
        mbar_arrive_expect_tx(bar_in, Q_BYTES + K_BYTES + VT_BYTES);
        bulk_g2s(sm + OQ, base + (size_t)qti * Q_BYTES, Q_BYTES, bar_in);
        bulk_g2s(sm + OK, base + (size_t)nt * Q_BYTES + (size_t)kt * K_BYTES, K_BYTES, bar_in);
        bulk_g2s(sm + OV, base + (size_t)nt * (Q_BYTES + K_BYTES) + (size_t)kt * VT_BYTES, VT_BYTES, bar_in);
        if (mbar_wait(bar_in, 0, abort_flag, 23)) {
            tc_fence_after();
            const uint64_t dq = sdesc_sw128(smem_u32(sm + OQ)), dk = sdesc_sw128(smem_u32(sm + OK));
            const uint32_t idesc_s = idesc_make(1, 0, 0, BM, nmma);
#pragma unroll
            for (int k = 0; k < D / 16; k++) mma_f16(tmem, dq + 2 * k, dk + 2 * k, idesc_s, k > 0);
            mma_commit(bar_s);
        } else {   // let the copies land before the CTA can exit
            volatile int never = 0;
            mbar_wait(bar_in, 0, &never, 12);
        }
    }
    ok = mbar_wait(bar_s, 0, abort_flag, 21);
    ok = __syncthreads_and(ok);
    const int row = (warp & 3) * 32 + lane;
    const uint32_t t_row = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const bool wact = q0 + (warp & 3) * 32 < S;
    const float c1 = scale * LOG2E;
    float m_i = -INFINITY, l_i = 0.0f;
    uint32_t r[2][32];
    if (ok) {
        tc_fence_after();
        float mloc = -INFINITY;
        if (wact) {
#pragma unroll
            for (int cc = 0; cc < 2; cc++)
                if (2 * half + cc < nch) tmem_ld32(t_row + (2 * half + cc) * 32, r[cc]);
            tmem_ld_wait();
            mloc = tile_row_max<2>(r, half, nch, nvalid, c1);
        }
        xmax[half * BM + row] = mloc;
        __syncthreads();
        m_i = fmaxf(xmax[row], xmax[BM + row]);
        float lsum = 0.0f;
        if (wact) {
            lsum = tile_probs<2>(r, half, nch, nvalid, c1, m_i, row, sm + OP, sm + OP + P_BYTES);
        }
        xsum[half * BM + row] = lsum;
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        l_i = __fadd_rn(xsum[row], xsum[BM + row]);
        if (tid == 0) {   // O = P_hi V + P_lo V
            tc_fence_after();
            constexpr uint32_t idesc_o = idesc_make(1, 0, 0, BM, D);
            const uint64_t dv = sdesc_sw128(smem_u32(sm + OV));
#pragma unroll
            for (int part = 0; part < 2; part++) {
                const uint64_t dp = sdesc_sw128(smem_u32(sm + OP + part * P_BYTES));
                if (nmma == BC) {
#pragma unroll
                    for (int t = 0; t < BC / 16; t++)
                        mma_f16(tmem + BC, dp + (t >> 2) * (P_BLK >> 4) + (t & 3) * 2,
                                dv + (t >> 2) * (VT_BLK >> 4) + (t & 3) * 2, idesc_o, (part | t) != 0);
                } else {
                    for (int t = 0; t < nmma / 16; t++)
                        mma_f16(tmem + BC, dp + (t >> 2) * (P_BLK >> 4) + (t & 3) * 2,
                                dv + (t >> 2) * (VT_BLK >> 4) + (t & 3) * 2, idesc_o, (part | t) != 0);
                }
            }
            mma_commit(bar_o);
        }
        ok = mbar_wait(bar_o, 0, abort_flag, 22);
        ok = __syncthreads_and(ok);
    }
    float o[D / 2];
    if (ok && wact) {
        tc_fence_after();
        uint32_t a16[16], a8[8];
        if (half == 0) { tmem_ld16(t_row + BC, a16); tmem_ld8(t_row + BC + 16, a8); }
        else { tmem_ld8(t_row + BC + 24, a8); tmem_ld16(t_row + BC + 32, a16); }
        tmem_ld_wait();
        if (half == 0) {
#pragma unroll
            for (int d = 0; d < 16; d++) o[d] = __uint_as_float(a16[d]);
#pragma unroll
            for (int d = 0; d < 8; d++) o[16 + d] = __uint_as_float(a8[d]);
        } else {
#pragma unroll
            for (int d = 0; d < 8; d++) o[d] = __uint_as_float(a8[d]);
#pragma unroll
            for (int d = 0; d < 16; d++) o[8 + d] = __uint_as_float(a16[d]);
        }
        const int qr = q0 + row, d0 = half * (D / 2);
        if (qr < S && nsplit > 1) {
            const size_t R = (size_t)(gridDim.z / nsplit) * S, rr = (size_t)split * R + (size_t)b * S + qr;
            float4* dst = reinterpret_cast<float4*>(opart + rr * E + h * D + d0);
#pragma unroll
            for (int d = 0; d < D / 2; d += 4) dst[d / 4] = make_float4(o[d], o[d + 1], o[d + 2], o[d + 3]);
            if (half == 0) reinterpret_cast<float2*>(mlpart)[rr * H + h] = make_float2(m_i, l_i);
        } else if (qr < S) {
            const float inv = __fdiv_rn(1.0f, l_i);
            float4* dst = reinterpret_cast<float4*>(out + ((size_t)b * S + qr) * E + h * D + d0);
#pragma unroll
            for (int d = 0; d < D / 2; d += 4)
                dst[d / 4] = make_float4(__fmul_rn(o[d], inv), __fmul_rn(o[d + 1], inv), __fmul_rn(o[d + 2], inv),
                                         __fmul_rn(o[d + 3], inv));
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, fa1::TMEM_COLS);
    }
}

__global__ void __launch_bounds__(fa::THREADS, 1) flash_attn_tc(const uint8_t* __restrict__ prep, int S, int H,
                                                               float scale, float* __restrict__ out, int nsplit,
                                                               int tiles_per, float* __restrict__ opart,
                                                               float* __restrict__ mlpart) {
    using namespace fa;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align1024_smem(smem_raw);
    uint64_t* bars = (uint64_t*)(sm + OFF_BAR);
    uint64_t* bar_q = bars;            // Q landed (tx)
    uint64_t* k_full = bars + 1;       // [2] K tile landed (tx)
    uint64_t* v_full = bars + 3;       // [2] V^T tile landed (tx)
    uint64_t* s_full = bars + 5;       // [2] S = Q K^T in TMEM (MMA commit)
    uint64_t* p_full = bars + 7;       // [2] P written to shared memory (16 softmax warps)
    uint64_t* o_full = bars + 9;       // [2] O tile = P V in TMEM (MMA commit)
    uint64_t* o_free = bars + 11;      // [2] O tile read back (16 softmax warps)
    uint64_t* v_free = bars + 13;      // [2] V^T buffer no longer read (MMA commit)
    uint32_t* tmem_slot = (uint32_t*)(bars + 15);
    volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

    constexpr int MMA_WARP = 16;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, part = (warp >> 2) & 3;
    const int h = blockIdx.y, b = blockIdx.z / nsplit, split = blockIdx.z % nsplit, qti = blockIdx.x, q0 = qti * BM;
    const int E = H * D, nt = (S + BC - 1) / BC;
    const int kt0 = split * tiles_per, kt1 = min(nt, kt0 + tiles_per), n = max(0, kt1 - kt0);
    const uint8_t* base = prep_base(const_cast<uint8_t*>(prep), b, h, H, nt);
    const uint8_t* gq = base + (size_t)qti * Q_BYTES;
    const uint8_t* gk = base + (size_t)nt * Q_BYTES;
    const uint8_t* gv = base + (size_t)nt * (Q_BYTES + K_BYTES);
    auto nvalid_of = [&](int i) { return min(BC, S - (kt0 + i) * BC); };

    if (tid == 0) {
        mbar_init(bar_q, 1);
        for (int j = 0; j < 2; j++) {
            mbar_init(k_full + j, 1); mbar_init(v_full + j, 1); mbar_init(s_full + j, 1);
            mbar_init(p_full + j, 16); mbar_init(o_full + j, 1); mbar_init(o_free + j, 16); mbar_init(v_free + j, 1);
        }
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == MMA_WARP) tmem_alloc(tmem_slot, TMEM_COLS);
    griddep_wait();   // prep / qkv come from the preceding kernel
    griddep_launch();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const float c1 = scale * LOG2E;   // scores in the base-2 domain

    if (warp == MMA_WARP) {
        // ------------------------------------------------------------------ MMA + copy warp
        // per step i: S(i) = Q K(i)^T; then, once softmax(i-1) has written P(i-1),
        // O(i-1) = P_hi V + P_lo V.  K(i+1) reuses the buffer S(i-1) read; V(i+1) the one PV(i-1) read.
        if (lane == 0 && n > 0) {
            auto load_k = [&](int i) {
                mbar_arrive_expect_tx(k_full + (i & 1), K_BYTES);
                bulk_g2s(sm + OFF_K + (i & 1) * K_BYTES, gk + (size_t)(kt0 + i) * K_BYTES, K_BYTES, k_full + (i & 1));
            };
            auto load_v = [&](int i) {
                mbar_arrive_expect_tx(v_full + (i & 1), VT_BYTES);
                bulk_g2s(sm + OFF_V + (i & 1) * VT_BYTES, gv + (size_t)(kt0 + i) * VT_BYTES, VT_BYTES, v_full + (i & 1));
            };
            mbar_arrive_expect_tx(bar_q, Q_BYTES);
            bulk_g2s(sm + OFF_Q, gq, Q_BYTES, bar_q);
            int nk = 0, nv = 0;   // tiles whose K / V copies were issued
            load_k(nk++);         // S(0) needs Q and K(0); V(0) follows at once (a one-tile CTA
            load_v(nv++);         // needs it right after its softmax), the second tile after S(0)
            auto more_loads = [&] {
                for (; nv < 2 && nv < n; nv++) load_v(nv);
                for (; nk < 2 && nk < n; nk++) load_k(nk);
            };
            const uint64_t dq = sdesc_sw128(smem_u32(sm + OFF_Q));
            constexpr uint32_t idesc_o = idesc_make(1, 0, 0, BM, D);
            bool ok = mbar_wait(bar_q, 0, abort_flag, 23);
            for (int i = 0; ok && i <= n; i++) {
                if (i < n) {
                    const int nmma = (nvalid_of(i) + 15) & ~15;
                    if (!(ok = mbar_wait(k_full + (i & 1), (i >> 1) & 1, abort_flag, 24))) break;
                    tc_fence_after();
                    const uint64_t dk = sdesc_sw128(smem_u32(sm + OFF_K + (i & 1) * K_BYTES));
                    const uint32_t idesc_s = idesc_make(1, 0, 0, BM, nmma);
#pragma unroll
                    for (int k = 0; k < D / 16; k++) mma_f16(tmem + (i & 1) * BC, dq + 2 * k, dk + 2 * k, idesc_s, k > 0);
                    mma_commit(s_full + (i & 1));
                    if (i == 0) more_loads();
                }
                if (i >= 1) {
                    const int j = i - 1, nmma = (nvalid_of(j) + 15) & ~15;
                    if (!(ok = mbar_wait(p_full + (j & 1), (j >> 1) & 1, abort_flag, 25))) break;
                    if (nk < n) load_k(nk++);   // S(j) has completed: its K buffer is free
                    if (!(ok = mbar_wait(v_full + (j & 1), (j >> 1) & 1, abort_flag, 26))) break;
                    if (j >= 2 && !(ok = mbar_wait(o_free + (j & 1), ((j - 2) >> 1) & 1, abort_flag, 27))) break;
                    tc_fence_after();
                    const uint64_t dv = sdesc_sw128(smem_u32(sm + OFF_V + (j & 1) * VT_BYTES));
                    const uint32_t tO = tmem + TM_O + (j & 1) * D;
#pragma unroll
                    for (int part = 0; part < 2; part++) {
                        const uint64_t dp = sdesc_sw128(smem_u32(sm + OFF_P + (j & 1) * P_SET + part * P_BYTES));
                        if (nmma == BC) {
#pragma unroll
                            for (int t = 0; t < BC / 16; t++)
                                mma_f16(tO, dp + (t >> 2) * (P_BLK >> 4) + (t & 3) * 2,
                                        dv + (t >> 2) * (VT_BLK >> 4) + (t & 3) * 2, idesc_o, (part | t) != 0);
                        } else {
                            for (int t = 0; t < nmma / 16; t++)
                                mma_f16(tO, dp + (t >> 2) * (P_BLK >> 4) + (t & 3) * 2,
                                        dv + (t >> 2) * (VT_BLK >> 4) + (t & 3) * 2, idesc_o, (part | t) != 0);
                        }
                    }
                    mma_commit(o_full + (j & 1));
                    mma_commit(v_free + (j & 1));
                    if (nv < n) {   // V(j+2) into the buffer PV(j) read
                        if (!(ok = mbar_wait(v_free + (j & 1), (j >> 1) & 1, abort_flag, 28))) break;
                        load_v(nv++);
                    }
                }
            }
            // let every issued copy land before the CTA can exit
            volatile int never = 0;
            mbar_wait(bar_q, 0, &never, 12);
            for (int t = (nk > 2 ? nk - 2 : 0); t < nk; t++) mbar_wait(k_full + (t & 1), (t >> 1) & 1, &never, 13);
            for (int t = (nv > 2 ? nv - 2 : 0); t < nv; t++) mbar_wait(v_full + (t & 1), (t >> 1) & 1, &never, 14);
        }
    } else {
        // ------------------------------------------------------------------ softmax warps
        // warps w, w+4, w+8, w+12 share TMEM lanes 32(w%4).. (query row per lane); warp part p
        // = w / 4 owns keys [32p, 32p+32) of each tile and output dims [12p, 12p+12).  Only the
        // four warps of a row quarter exchange the row max and sum, so each quarter synchronises
        // on its own named barrier and the quarters run independently.
        const int row = (warp & 3) * 32 + lane;
        const uint32_t t_row = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        const bool wact = q0 + (warp & 3) * 32 < S;   // warp-uniform: owns at least one real query row
        constexpr int DP = D / 4;
        float o[DP];
#pragma unroll
        for (int d = 0; d < DP; d++) o[d] = 0.0f;
        float m_i = -INFINITY, l_i = 0.0f, alpha_prev = 1.0f;
        bool ok = true;
        // O(j) accumulation: o = alpha_j o + O(j)
        auto accumulate = [&](int j, float alpha) {
            ok = ok && mbar_wait(o_full + (j & 1), (j >> 1) & 1, abort_flag, 22);
            ok = __all_sync(0xffffffffu, ok);
            if (ok && wact) {
                tc_fence_after();
                const uint32_t tO = t_row + TM_O + (j & 1) * D + part * DP;
                // each load starts at a multiple of its own width: 8 + 4 columns for even parts,
                // 4 + 8 for odd ones
                uint32_t a8[8], a4[4];
                const bool even = (part & 1) == 0;
                tmem_ld8(tO + (even ? 0 : 4), a8);
                tmem_ld4(tO + (even ? 8 : 0), a4);
                tmem_ld_wait();
                if (even) {
#pragma unroll
                    for (int d = 0; d < 8; d++) o[d] = __fmaf_rn(alpha, o[d], __uint_as_float(a8[d]));
#pragma unroll
                    for (int d = 0; d < 4; d++) o[8 + d] = __fmaf_rn(alpha, o[8 + d], __uint_as_float(a4[d]));
                } else {
#pragma unroll
                    for (int d = 0; d < 4; d++) o[d] = __fmaf_rn(alpha, o[d], __uint_as_float(a4[d]));
#pragma unroll
                    for (int d = 0; d < 8; d++) o[4 + d] = __fmaf_rn(alpha, o[4 + d], __uint_as_float(a8[d]));
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(o_free + (j & 1));
        };
        for (int i = 0; i < n; i++) {
            const int nvalid = nvalid_of(i), nmma = (nvalid + 15) & ~15, nch = (nmma + 31) / 32;
            float* xmax = reinterpret_cast<float*>(sm + OFF_X + (i & 1) * X_SET);   // [4][128]
            float* xsum = xmax + 4 * BM;                                             // [4][128]
            ok = ok && mbar_wait(s_full + (i & 1), (i >> 1) & 1, abort_flag, 21);
            ok = __all_sync(0xffffffffu, ok);
            tc_fence_after();
            float alpha = 1.0f, mloc = -INFINITY;
            uint32_t r[1][32];
            if (ok && wact) {
                if (part < nch) tmem_ld32(t_row + (i & 1) * BC + part * 32, r[0]);
                tmem_ld_wait();
                mloc = nvalid == BC ? tile_row_max<1, true>(r, part, nch, nvalid, c1)
                                    : tile_row_max<1>(r, part, nch, nvalid, c1);
            }
            xmax[part * BM + row] = mloc;
            named_bar_sync(2 + (warp & 3), 128);   // the 4 warps of this query-row quarter
            const float m_new = fmaxf(fmaxf(m_i, fmaxf(xmax[row], xmax[BM + row])),
                                      fmaxf(xmax[2 * BM + row], xmax[3 * BM + row]));
            float lsum = 0.0f;
            if (ok && wact) {
                alpha = exp2f(m_i - m_new);
                uint8_t* ps = sm + OFF_P + (i & 1) * P_SET;
                lsum = nvalid == BC ? tile_probs<1, true>(r, part, nch, nvalid, c1, m_new, row, ps, ps + P_BYTES)
                                    : tile_probs<1>(r, part, nch, nvalid, c1, m_new, row, ps, ps + P_BYTES);
            }
            fence_async_smem();   // P is read by the tensor core
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full + (i & 1));
            xsum[part * BM + row] = lsum;
            named_bar_sync(2 + (warp & 3), 128);   // the 4 warps of this query-row quarter
            if (ok && wact) {
                l_i = __fadd_rn(__fmul_rn(alpha, l_i), __fadd_rn(__fadd_rn(xsum[row], xsum[BM + row]),
                                                                 __fadd_rn(xsum[2 * BM + row], xsum[3 * BM + row])));
                m_i = m_new;
            }
            if (i >= 1) accumulate(i - 1, alpha_prev);
            alpha_prev = alpha;
        }
        if (n >= 1) accumulate(n - 1, alpha_prev);

        const int qr = q0 + row, d0 = part * DP;
        if (ok && qr < S && nsplit > 1) {   // partial result of this key range, merged by the combine pass
            const size_t R = (size_t)(gridDim.z / nsplit) * S, rr = (size_t)split * R + (size_t)b * S + qr;
            float4* dst = reinterpret_cast<float4*>(opart + rr * E + h * D + d0);
#pragma unroll
            for (int d = 0; d < DP; d += 4) dst[d / 4] = make_float4(o[d], o[d + 1], o[d + 2], o[d + 3]);
            if (part == 0) reinterpret_cast<float2*>(mlpart)[rr * H + h] = make_float2(m_i, l_i);
        } else if (ok && qr < S) {
            const float inv = __fdiv_rn(1.0f, l_i);
            float4* dst = reinterpret_cast<float4*>(out + ((size_t)b * S + qr) * E + h * D + d0);
#pragma unroll
            for (int d = 0; d < DP; d += 4)
                dst[d / 4] = make_float4(__fmul_rn(o[d], inv), __fmul_rn(o[d + 1], inv), __fmul_rn(o[d + 2], inv),
                                         __fmul_rn(o[d + 3], inv));
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == MMA_WARP) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

// Merge the key-range partials (m in the base-2 domain): m = max m_s, l = sum l_s 2^(m_s - m),
// o = sum o_s 2^(m_s - m) / l.
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
        const float wgt = exp2f(v2.x - m);
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
// NS (the number of key ranges) is a template parameter so every load of a row is issued before
// the first one is used.
template <int NC, int NS>
__global__ void __launch_bounds__(128) attn_combine_rows(const float* __restrict__ opart, const float* __restrict__ mlpart,
                                                         int R, int H, float* __restrict__ out, ActQ a, int want_c) {
    griddep_wait();
    griddep_launch();
    const int lane = threadIdx.x & 31, r = blockIdx.x * 4 + (threadIdx.x >> 5);
    if (r >= R) return;
    constexpr int E = NC * 256;
    const float2* ml = reinterpret_cast<const float2*>(mlpart);
    float2 mls[NC][NS];
    float4 xs[NC][NS][2];
#pragma unroll
    for (int i = 0; i < NC; i++) {
        const int e0 = 256 * i + 8 * lane, rh = r * H + e0 / fa::D;
#pragma unroll
        for (int s = 0; s < NS; s++) {
            mls[i][s] = __ldcg(ml + (size_t)s * R * H + rh);
            const float4* src = reinterpret_cast<const float4*>(opart + ((size_t)s * R + r) * E + e0);
            xs[i][s][0] = __ldcg(src);
            xs[i][s][1] = __ldcg(src + 1);
        }
    }
    float v[NC][8];
#pragma unroll
    for (int i = 0; i < NC; i++) {
        float m = -INFINITY;
#pragma unroll
        for (int s = 0; s < NS; s++) m = fmaxf(m, mls[i][s].x);
        float l = 0.0f, acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
        for (int s = 0; s < NS; s++) {
            const float wgt = exp2f(mls[i][s].x - m);
            l = __fmaf_rn(mls[i][s].y, wgt, l);
            const float x8[8] = {xs[i][s][0].x, xs[i][s][0].y, xs[i][s][0].z, xs[i][s][0].w,
                                 xs[i][s][1].x, xs[i][s][1].y, xs[i][s][1].z, xs[i][s][1].w};
#pragma unroll
            for (int e = 0; e < 8; e++) acc[e] = __fmaf_rn(x8[e], wgt, acc[e]);
        }
        const float inv = __fdiv_rn(1.0f, l);
#pragma unroll
        for (int e = 0; e < 8; e++) v[i][e] = __fmul_rn(acc[e], inv);
        if (out) {
            float4* dst = reinterpret_cast<float4*>(out + (size_t)r * E + 256 * i + 8 * lane);
            dst[0] = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
            dst[1] = make_float4(v[i][4], v[i][5], v[i][6], v[i][7]);
        }
    }
    quant_chunks<NC>(v, r, a, want_c != 0, lane);
}

size_t attn_prep_floats(int B, int S, int H) {
    const size_t nt = (size_t)(S + fa::BC - 1) / fa::BC;
    return (size_t)B * H * nt * 128 * fa::PREP_ROW / 4;
}

AttnPrepOut attn_prep_out(float* scratch, int B, int S, int H) {
    (void)B;
    return AttnPrepOut{reinterpret_cast<uint8_t*>(scratch), S, H, (S + fa::BC - 1) / fa::BC};
}

size_t attn_scratch_floats(int B, int S, int H) {
    return attn_prep_floats(B, S, H) + (size_t)kAttnMaxSplit * B * S * H * (fa::D + 2);
}

static bool g_attn_ready[64] = {};


int attn_prepare() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    if (cudaFuncSetAttribute(flash_attn_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, fa::SMEM) != cudaSuccess ||
        cudaFuncSetAttribute(flash_attn_1t, cudaFuncAttributeMaxDynamicSharedMemorySize, fa1::SMEM) != cudaSuccess)
        return -1;
    g_attn_ready[dev] = true;
    return 0;
}

int launch_flash_attn(const float* qkv, int B, int S, int H, int Dh, float scale, float* out, float* scratch,
                      size_t scratch_floats, cudaStream_t st, const ActQ* qo, bool qo_c, bool* quantized,
                      bool prepped, long split_ctas) {
    if (quantized) *quantized = false;
    if (Dh != fa::D) return -2;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return -1;
    if (!g_attn_ready[dev] && attn_prepare() != 0) return -1;   // runtimes prepare at creation
    const size_t prep_n = attn_prep_floats(B, S, H);
    if (!scratch || scratch_floats < prep_n) return -3;
    // Split the key range over CTAs when (query tiles x heads x images) leaves SMs idle.
    const int qt = (S + fa::BM - 1) / fa::BM, ntiles = (S + fa::BC - 1) / fa::BC;
    const long ctas = split_ctas > 0 ? split_ctas : (long)qt * H * B;
    int nsplit = 1;
    static const int max_split = [] {   // MGC_ATTN_MAXSPLIT caps the key split (measurement knob)
        const char* e = std::getenv("MGC_ATTN_MAXSPLIT");
        const int v = e ? std::atoi(e) : kAttnMaxSplit;
        return v < 1 ? 1 : v > kAttnMaxSplit ? kAttnMaxSplit : v;
    }();
    if (scratch_floats >= attn_scratch_floats(B, S, H))
        while (nsplit < max_split && nsplit < ntiles && ctas * (nsplit + 1) <= 2 * sm_count()) nsplit++;
    const int tiles_per = (ntiles + nsplit - 1) / nsplit;
    nsplit = (ntiles + tiles_per - 1) / tiles_per;   // no empty split
    const int R = B * S;
    uint8_t* prep = reinterpret_cast<uint8_t*>(scratch);
    float* opart = scratch + prep_n;
    float* mlpart = opart + (size_t)nsplit * R * H * fa::D;
    if (!prepped) launch_k(attn_prep, B * H * ntiles * 3, 128, 0, st, qkv, S, H, ntiles, prep);
    dim3 grid(qt, H, B * nsplit);
    if (tiles_per == 1)   // one key tile per CTA: nothing to pipeline
        launch_k(flash_attn_1t, grid, 256, fa1::SMEM, st, (const uint8_t*)prep, S, H, scale, out, nsplit, opart, mlpart);
    else
        launch_k(flash_attn_tc, grid, fa::THREADS, fa::SMEM, st, (const uint8_t*)prep, S, H, scale, out, nsplit,
                 tiles_per, opart, mlpart);
    g_launch_count += (nsplit > 1 ? 2 : 1) + (prepped ? 0 : 1);
    if (nsplit > 1 && qo && H * fa::D == 768) {   // merge + quantize in one pass (warp per row)
        auto kern = nsplit == 2 ? attn_combine_rows<3, 2> : nsplit == 3 ? attn_combine_rows<3, 3> : attn_combine_rows<3, 4>;
        launch_k(kern, (R + 3) / 4, 128, 0, st, opart, mlpart, R, H, out, *qo, qo_c ? 1 : 0);
        if (quantized) *quantized = true;
    } else if (nsplit > 1) launch_k(attn_combine, (R * H * (fa::D / 4) + 255) / 256, 256, 0, st, opart, mlpart, nsplit, R, H, out);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace mgc
