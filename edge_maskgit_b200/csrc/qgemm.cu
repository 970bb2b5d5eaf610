// qgemm.cu -- Q8_0 / Q4_K int8-dot GEMM on Blackwell tensor cores (tcgen05, kind::i8).
//
// Computes, for every output (m, n), exactly the reference's per-block accumulation
// (k_mul_mat_q8_i8 mg-opencl.cpp:440-494, k_mul_mat_q4k_i8 :504-590):
//     idot_b = sum_{i<32} qw[n, 32b+i] * qx[m, 32b+i]            (exact int32)
//     Q8_0:  acc = fma(dw[n,b] * dx[m,b], idot_b, acc)
//     Q4_K:  acc = fma(scl[n,b] * dx[m,b], idot_b, acc); acc = fma(-mnl[n,b], dx*sumx, acc)
// over b ascending, then y = act(acc + bias[n]) + resid[m,n].
//
// One CTA owns a 128 x BN output tile.  Warp roles:
//   warp 0       producer: one cp.async.bulk per operand tile per 4-block K-chunk into a
//                4-stage shared-memory ring (the operands are stored pre-swizzled in HBM,
//                so a linear bulk copy lands them in the tcgen05 128-byte-swizzle layout)
//   warp 1       MMA issuer: one tcgen05.mma (M=128, N=BN, K=32 = one quant block) per
//                block into a ring of 4 TMEM accumulators, without accumulation, so each
//                TMEM buffer holds one block's exact int32 dot products
//   warps 2..    "promotion": tcgen05.ld a block's int32 tile, release the TMEM buffer,
//                convert exactly to f32 and apply the per-block scales with FMAs into
//                register accumulators (thread = one output row, CW columns); then the
//                fused bias / activation / residual epilogue.
#include "kernels.h"
#include "ptx.cuh"

#include <cstdio>
#include <cstdlib>

namespace mgc {

struct QGemmArgs {
    const int8_t* aq; const float* adx; const float* acx; int Mpad;
    const int8_t* wq; const float* wsa; const float* wsb; int Npad;
    int M, N, K;
    const float* bias; const float* resid; float* y; int act;
};

// exact int32 -> f32 for |v| < 2^22: place v in the mantissa of 1.5 * 2^23 and subtract.
__device__ __forceinline__ float i2f_exact(uint32_t v) {
    return __int_as_float((int)(v + 0x4B400000u)) - 12582912.0f;
}

__device__ __forceinline__ float act_apply(float v, int a) {
    if (a == 1) return 0.5f * v * (1.0f + erff(v * 0.70710678f));
    if (a == 2) return __fdiv_rn(v, 1.0f + expf(-v));
    return v;
}

template <int BN, int CG, bool Q4K>
struct QGemmCfg {
    static constexpr int NST = 4, NBUF = 4, NPW = 4 * CG, CW = BN / CG;
    static constexpr int THREADS = 64 + 32 * NPW;
    static constexpr uint32_t A_BYTES = 128 * 128, B_BYTES = BN * 128, DX_BYTES = 128 * 16,
                              DW_BYTES = 16 * BN;
    static constexpr uint32_t OFF_B = A_BYTES, OFF_DX = OFF_B + B_BYTES, OFF_DW = OFF_DX + DX_BYTES,
                              OFF_MN = OFF_DW + DW_BYTES, OFF_CX = OFF_MN + (Q4K ? DW_BYTES : 0),
                              STAGE_RAW = OFF_CX + (Q4K ? DX_BYTES : 0),
                              STAGE = (STAGE_RAW + 1023) & ~1023u;
    static constexpr uint32_t TX_BYTES = A_BYTES + B_BYTES + DX_BYTES + DW_BYTES +
                                         (Q4K ? DW_BYTES + DX_BYTES : 0);
    static constexpr uint32_t SMEM = 1024 + NST * STAGE + 256;
    static constexpr uint32_t TMEM_COLS = BN * NBUF;
};

template <int BN, int CG, bool Q4K>
__global__ void __launch_bounds__(QGemmCfg<BN, CG, Q4K>::THREADS, 1)
qgemm_kernel(const QGemmArgs p) {
    using C = QGemmCfg<BN, CG, Q4K>;
    constexpr int NST = C::NST, NBUF = C::NBUF, CW = C::CW;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* full = (uint64_t*)(smem + NST * C::STAGE);
    uint64_t* empty = full + NST;
    uint64_t* tfull = empty + NST;
    uint64_t* tempty = tfull + NBUF;
    uint32_t* tmem_slot = (uint32_t*)(tempty + NBUF);
    volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * 128;
    const int nb = p.K / 32, nkc = p.K / 128;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NST; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1 + C::NPW); }
        for (int b = 0; b < NBUF; b++) { mbar_init(&tfull[b], 1); mbar_init(&tempty[b], C::NPW); }
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            int last_it[NST];
            for (int s = 0; s < NST; s++) last_it[s] = -1;
            for (int kc = 0; kc < nkc; kc++) {
                const int s = kc % NST, it = kc / NST;
                if (!mbar_wait(&empty[s], (it & 1) ^ 1, abort_flag, 1)) break;
                uint8_t* st = smem + s * C::STAGE;
                mbar_arrive_expect_tx(&full[s], C::TX_BYTES);
                bulk_g2s(st, p.aq + ((size_t)kc * p.Mpad + m0) * 128, C::A_BYTES, &full[s]);
                bulk_g2s(st + C::OFF_B, p.wq + ((size_t)kc * p.Npad + n0) * 128, C::B_BYTES, &full[s]);
                bulk_g2s(st + C::OFF_DX, p.adx + ((size_t)kc * p.Mpad + m0) * 4, C::DX_BYTES, &full[s]);
#pragma unroll
                for (int j = 0; j < 4; j++)
                    bulk_g2s(st + C::OFF_DW + j * BN * 4, p.wsa + (size_t)(kc * 4 + j) * p.Npad + n0,
                             BN * 4, &full[s]);
                if constexpr (Q4K) {
#pragma unroll
                    for (int j = 0; j < 4; j++)
                        bulk_g2s(st + C::OFF_MN + j * BN * 4, p.wsb + (size_t)(kc * 4 + j) * p.Npad + n0,
                                 BN * 4, &full[s]);
                    bulk_g2s(st + C::OFF_CX, p.acx + ((size_t)kc * p.Mpad + m0) * 4, C::DX_BYTES, &full[s]);
                }
                last_it[s] = it;
            }
            if (*abort_flag) {   // let copies already in flight land before the CTA exits
                volatile int never = 0;
                for (int s = 0; s < NST; s++)
                    if (last_it[s] >= 0) mbar_wait(&full[s], last_it[s] & 1, &never, 11);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_make(2, 1, Q4K ? 0 : 1, 128, BN);
            bool ok = true;
            for (int kc = 0; kc < nkc && ok; kc++) {
                const int s = kc % NST, it = kc / NST;
                if (!mbar_wait(&full[s], it & 1, abort_flag, 2)) break;
                tc_fence_after();
                const uint32_t a_base = smem_u32(smem + s * C::STAGE), b_base = a_base + C::OFF_B;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int b = kc * 4 + j, buf = b % NBUF, u = b / NBUF;
                    if (!mbar_wait(&tempty[buf], (u & 1) ^ 1, abort_flag, 3)) { ok = false; break; }
                    tc_fence_after();
                    mma_i8(tmem + buf * BN, sdesc_sw128(a_base + 32 * j), sdesc_sw128(b_base + 32 * j),
                           idesc, 0);
                    mma_commit(&tfull[buf]);
                }
                if (ok) mma_commit(&empty[s]);
            }
        }
    } else {
        const int pw = warp - 2, q = warp & 3, cg = pw >> 2;
        const int row = q * 32 + lane, m = m0 + row, c0 = cg * CW;
        const bool active = (m0 + q * 32) < p.M;   // warp-uniform
        float acc[CW];
#pragma unroll
        for (int c = 0; c < CW; c++) acc[c] = 0.0f;
        float4 dxv = make_float4(0, 0, 0, 0), cxv = make_float4(0, 0, 0, 0);
        const uint32_t t_lane = tmem + ((uint32_t)(q * 32) << 16) + c0;
        for (int b = 0; b < nb; b++) {
            const int kc = b >> 2, j = b & 3, s = kc % NST;
            const uint8_t* st = smem + s * C::STAGE;
            if (j == 0) {
                bool ok = mbar_wait(&full[s], (kc / NST) & 1, abort_flag, 4);
                if (!__all_sync(0xffffffffu, ok)) break;
                dxv = reinterpret_cast<const float4*>(st + C::OFF_DX)[row];
                if constexpr (Q4K) cxv = reinterpret_cast<const float4*>(st + C::OFF_CX)[row];
            }
            const int buf = b % NBUF, u = b / NBUF;
            bool ok = mbar_wait(&tfull[buf], u & 1, abort_flag, 5);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            uint32_t I[CW];
#pragma unroll
            for (int t = 0; t < CW / 32; t++)
                tmem_ld32(t_lane + buf * BN + t * 32, *reinterpret_cast<uint32_t(*)[32]>(&I[t * 32]));
            tmem_ld_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
            if (active) {
                const float dxj = j == 0 ? dxv.x : j == 1 ? dxv.y : j == 2 ? dxv.z : dxv.w;
                const float* dw = reinterpret_cast<const float*>(st + C::OFF_DW) + j * BN + c0;
#pragma unroll
                for (int c = 0; c < CW; c += 4) {
                    const float4 w4 = *reinterpret_cast<const float4*>(dw + c);
                    acc[c + 0] = __fmaf_rn(__fmul_rn(w4.x, dxj), i2f_exact(I[c + 0]), acc[c + 0]);
                    acc[c + 1] = __fmaf_rn(__fmul_rn(w4.y, dxj), i2f_exact(I[c + 1]), acc[c + 1]);
                    acc[c + 2] = __fmaf_rn(__fmul_rn(w4.z, dxj), i2f_exact(I[c + 2]), acc[c + 2]);
                    acc[c + 3] = __fmaf_rn(__fmul_rn(w4.w, dxj), i2f_exact(I[c + 3]), acc[c + 3]);
                }
                if constexpr (Q4K) {
                    const float cxj = j == 0 ? cxv.x : j == 1 ? cxv.y : j == 2 ? cxv.z : cxv.w;
                    const float* mn = reinterpret_cast<const float*>(st + C::OFF_MN) + j * BN + c0;
#pragma unroll
                    for (int c = 0; c < CW; c += 4) {
                        const float4 n4 = *reinterpret_cast<const float4*>(mn + c);
                        acc[c + 0] = __fmaf_rn(-n4.x, cxj, acc[c + 0]);
                        acc[c + 1] = __fmaf_rn(-n4.y, cxj, acc[c + 1]);
                        acc[c + 2] = __fmaf_rn(-n4.z, cxj, acc[c + 2]);
                        acc[c + 3] = __fmaf_rn(-n4.w, cxj, acc[c + 3]);
                    }
                }
            }
            if (j == 3) {
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
            }
        }
        // epilogue: bias -> act -> residual (mg-opencl.cpp:481-493)
        if (m < p.M && !*abort_flag) {
            const int nbase = n0 + c0;
            const bool vec = (p.N % 4) == 0;
#pragma unroll
            for (int c = 0; c < CW; c += 4) {
                const int n = nbase + c;
                if (n >= p.N) break;
                float v[4] = {acc[c], acc[c + 1], acc[c + 2], acc[c + 3]};
                if (vec) {
                    if (p.bias) {
                        const float4 b4 = __ldg(reinterpret_cast<const float4*>(p.bias + n));
                        v[0] = __fadd_rn(v[0], b4.x); v[1] = __fadd_rn(v[1], b4.y);
                        v[2] = __fadd_rn(v[2], b4.z); v[3] = __fadd_rn(v[3], b4.w);
                    }
#pragma unroll
                    for (int i = 0; i < 4; i++) v[i] = act_apply(v[i], p.act);
                    if (p.resid) {
                        const float4 r4 = *reinterpret_cast<const float4*>(p.resid + (size_t)m * p.N + n);
                        v[0] = __fadd_rn(v[0], r4.x); v[1] = __fadd_rn(v[1], r4.y);
                        v[2] = __fadd_rn(v[2], r4.z); v[3] = __fadd_rn(v[3], r4.w);
                    }
                    *reinterpret_cast<float4*>(p.y + (size_t)m * p.N + n) = make_float4(v[0], v[1], v[2], v[3]);
                } else {
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        if (n + i >= p.N) break;
                        float x = v[i];
                        if (p.bias) x = __fadd_rn(x, p.bias[n + i]);
                        x = act_apply(x, p.act);
                        if (p.resid) x = __fadd_rn(x, p.resid[(size_t)m * p.N + n + i]);
                        p.y[(size_t)m * p.N + n + i] = x;
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

template <int BN, int CG, bool Q4K>
static int set_smem_attr() {
    using C = QGemmCfg<BN, CG, Q4K>;
    return cudaFuncSetAttribute(qgemm_kernel<BN, CG, Q4K>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                C::SMEM) == cudaSuccess ? 0 : -1;
}

// Sets the dynamic shared-memory limit of every instantiation on the current device.  Must
// run once per device before the first launch (the runtime does it at creation, outside any
// stream capture).
int qgemm_prepare() {
    int rc = 0;
    rc |= set_smem_attr<128, 2, false>(); rc |= set_smem_attr<128, 2, true>();
    rc |= set_smem_attr<64, 2, false>();  rc |= set_smem_attr<64, 2, true>();
    rc |= set_smem_attr<32, 1, false>();  rc |= set_smem_attr<32, 1, true>();
    return rc;
}

template <int BN, int CG, bool Q4K>
static int run_qgemm(const QGemmArgs& a, cudaStream_t st) {
    using C = QGemmCfg<BN, CG, Q4K>;
    dim3 grid((a.N + BN - 1) / BN, (a.M + 127) / 128);
    qgemm_kernel<BN, CG, Q4K><<<grid, C::THREADS, C::SMEM, st>>>(a);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

// Tile width: the widest BN that still gives >= ~one CTA per SM; MGC_QGEMM_BN overrides.
static int pick_bn(int M, int N) {
    static int forced = -1;
    if (forced < 0) {
        const char* e = std::getenv("MGC_QGEMM_BN");
        forced = e ? std::atoi(e) : 0;
    }
    if (forced == 32 || forced == 64 || forced == 128) return forced;
    const int mt = (M + 127) / 128;
    for (int bn : {128, 64}) if ((long)mt * ((N + bn - 1) / bn) >= 140) return bn;
    return 32;
}

int launch_qgemm(const QWeight& w, const ActQ& a, int M, const float* bias, int act,
                 const float* resid, float* y, cudaStream_t st) {
    if (w.K % 128 != 0 || M <= 0 || M > a.Mpad) return -2;
    QGemmArgs p{a.q, a.d, a.c, a.Mpad, w.q, w.sa, w.sb, w.Npad, M, w.N, w.K, bias, resid, y, act};
    const int bn = pick_bn(M, w.N);
    const bool q4 = w.wtype == 12;
    if (bn == 128) return q4 ? run_qgemm<128, 2, true>(p, st) : run_qgemm<128, 2, false>(p, st);
    if (bn == 64) return q4 ? run_qgemm<64, 2, true>(p, st) : run_qgemm<64, 2, false>(p, st);
    return q4 ? run_qgemm<32, 1, true>(p, st) : run_qgemm<32, 1, false>(p, st);
}

}  // namespace mgc
