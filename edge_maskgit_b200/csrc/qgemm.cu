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
#include "attnprep.cuh"
#include "qgemm_common.cuh"

#include <cstdio>
#include <cstdlib>
#include <algorithm>
#include <atomic>

#ifndef MGC_QGEMM_MINB
#define MGC_QGEMM_MINB 1     // CTAs per SM the register budget is sized for
#endif
#ifndef MGC_QGEMM_IREGS
#define MGC_QGEMM_IREGS 64   // int32 dot values a promotion thread loads per TMEM batch
#endif



namespace mgc {

template <int BN, int CG, bool Q4K, int CB>
struct QGemmCfg {
    // CB: 32-blocks per pipeline chunk (4 or 8); a chunk is SUB = CB/4 activation tiles of 128 K
    static constexpr int NPW = 4 * CG, CW = BN / CG;
    // NGRP: TMEM ring of chunk groups (CB * BN columns each), at most 256 columns by default
    static constexpr int SUB = CB / 4;
#ifdef MGC_NGRP   // upper bound; the ring never exceeds the 512 TMEM columns
    static constexpr int NGRP = MGC_NGRP * CB * BN <= 512 ? MGC_NGRP : 512 / (CB * BN);
#else
    // (one CTA per SM -- the ring's shared memory allows no more -- so the whole 512 columns
    // are available; with MGC_QGEMM_MINB=2 each CTA keeps to 256)
    static constexpr int NGRP = (MGC_QGEMM_MINB == 1 ? 512 : 256) / (CB * BN) >= 2 ? 2 : 1;
#endif
    static constexpr int THREADS = 64 + 32 * NPW;
    // stage = [SUB activation tiles: codes | dx | (dx*sumx)] [SUB weight code tiles] [SUB scale tiles]
    static constexpr uint32_t T = Q4K ? 2 : 1;
    static constexpr uint32_t A_BYTES = Q4K ? 20480 : 18432, B_BYTES = BN * 128, S_BYTES = BN * 16 * T;
    // Q4_K: the packed weight bytes land in a raw area (BN x 64 nibble bytes, BN x 16 scale
    // bytes per 128-K tile) and the MMA warp unpacks them into the code and scale tiles
    static constexpr uint32_t R_BYTES = Q4K ? BN * 80 : 0;
    static constexpr uint32_t OFF_DX = 16384, OFF_CX = 18432, OFF_B = SUB * A_BYTES, OFF_S = OFF_B + SUB * B_BYTES,
                              OFF_R = OFF_S + SUB * S_BYTES, STAGE = (OFF_R + SUB * R_BYTES + 1023) & ~1023u;
    static constexpr uint32_t TX_BYTES = Q4K ? SUB * (A_BYTES + R_BYTES) : SUB * (A_BYTES + B_BYTES + S_BYTES);
#ifdef MGC_NST
    static constexpr int NST = MGC_NST;
#else
    // ~190 KB ring for 4-block chunks (deeper measured faster); 8-block chunks fill what fits
    static constexpr int NST_PREF = CB == 4 ? (BN <= 32 ? 8 : BN <= 64 ? 6 : 4) : 8;
    static constexpr int NST_FIT = (232448 - 1024 - 320 - 2 * NPW * 32 * 4) / STAGE;   // what fits
    static constexpr int NST = NST_PREF < NST_FIT ? NST_PREF : NST_FIT;
#endif
    static constexpr uint32_t XCHG = NST * STAGE + 320;   // (barriers, then) epilogue exchange: [2][NPW][32] f32
    static constexpr uint32_t SMEM = 1024 + XCHG + 2 * NPW * 32 * 4;
    // allocation is a power of two >= 32 columns
    static constexpr uint32_t TMEM_NEED = CB * BN * NGRP,
                              TMEM_COLS = TMEM_NEED <= 32 ? 32 : TMEM_NEED <= 64 ? 64 : TMEM_NEED <= 128 ? 128
                                        : TMEM_NEED <= 256 ? 256 : 512;
    static_assert(NGRP >= 1 && TMEM_NEED <= 512, "TMEM ring exceeds 512 columns");
    static_assert(SMEM <= 232448, "shared memory beyond the opt-in limit");
    static_assert((3 * NST + 2 * NGRP) * 8 + 8 <= 320, "barrier area");
};

template <int BN, int CG, bool Q4K, int CB, bool PERSIST>
__global__ void __launch_bounds__(QGemmCfg<BN, CG, Q4K, CB>::THREADS, MGC_QGEMM_MINB)
qgemm_kernel(const QGemmArgs p) {
    using C = QGemmCfg<BN, CG, Q4K, CB>;
    constexpr int SUB = C::SUB;
    // int32 dot values per TMEM batch: 64 registers, 32 when the CTA is too wide for that
    constexpr int IREGS = C::THREADS > 448 ? 32 : MGC_QGEMM_IREGS;
    constexpr int NST = C::NST, NGRP = C::NGRP, CW = C::CW, BATCH = CW >= IREGS ? 1 : IREGS / CW > 4 ? 4 : IREGS / CW;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align1024_smem(smem_raw);
    uint64_t* full = (uint64_t*)(smem + NST * C::STAGE);
    uint64_t* empty = full + NST;
    uint64_t* tfull = empty + NST;
    uint64_t* tempty = tfull + NGRP;
    uint64_t* unpk = tempty + NGRP;   // Q4_K: stage s unpacked (the MMA warp's lane 0 arrives)
    uint32_t* tmem_slot = (uint32_t*)(unpk + NST);
    volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr bool persist = PERSIST;   // (p.tiles_n > 0)
    const int my_tiles = persist ? (p.tiles_n * p.tiles_m - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 1;
    auto tile_of = [&](int ti, int& n0_, int& mt_) {   // ti-th tile of this CTA: n offset, m-tile index
        if (persist) {
            const int t = blockIdx.x + ti * gridDim.x;
            n0_ = (t % p.tiles_n) * BN;
            mt_ = t / p.tiles_n;
        } else {
            n0_ = blockIdx.x * BN;
            mt_ = blockIdx.y;
        }
    };
    const int nkc = p.K / (32 * CB);
    const int kz = blockIdx.z, kc0 = kz * p.cps, nloc = max(0, min(nkc, kc0 + p.cps) - kc0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < NST; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1 + C::NPW); }
        for (int g = 0; g < NGRP; g++) { mbar_init(&tfull[g], 1); mbar_init(&tempty[g], C::NPW); }
        for (int s = 0; s < NST; s++) mbar_init(&unpk[s], 1);
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
    // With programmatic dependent launch this prologue, and the weight copies of the first
    // stages (weights do not depend on the preceding kernel), overlap the preceding kernel's
    // tail: only the activation copies and the epilogue wait for it (griddep_wait below).
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (warp == 0) {
        if (lane == 0) {
            int last_it[NST];
            for (int s = 0; s < NST; s++) last_it[s] = -1;
            // three copies per 128-K tile: activation tile (+ its scales), weight codes, weight scales
            // (i: chunk within the tile; gc: running chunk index of this CTA, which picks the stage)
            int n0, mt;
            auto copy_w = [&](int i, int gc) {
                const int kc = kc0 + i, s = gc % NST;
                uint8_t* st = smem + s * C::STAGE;
#pragma unroll
                for (int u = 0; u < SUB; u++) {
                    const size_t kk = (size_t)kc * SUB + u;
                    if constexpr (Q4K) {   // packed nibbles + compact scales into the raw area
                        uint8_t* raw = st + C::OFF_R + u * C::R_BYTES;
                        bulk_g2s(raw, p.wq + (kk * p.Npad + n0) * 64, BN * 64, &full[s]);
                        bulk_g2s(raw + BN * 64, reinterpret_cast<const uint8_t*>(p.ws) + (kk * p.Npad + n0) * 16, BN * 16,
                                 &full[s]);
                    } else {
                        bulk_g2s(st + C::OFF_B + u * C::B_BYTES, p.wq + (kk * p.Npad + n0) * 128, C::B_BYTES, &full[s]);
                        bulk_g2s(st + C::OFF_S + u * C::S_BYTES, p.ws + (kk * (p.Npad / 4) + n0 / 4) * 16, C::S_BYTES,
                                 &full[s]);
                    }
                }
            };
            // Rows of the m-tile that hold data, rounded up to the 8-row swizzle atom: a partial
            // last m-tile (M=257 leaves one row in the third) copies only those rows of codes,
            // dx (and dx*sumx) -- rows past M are never stored, so the MMA may read whatever the
            // stage held.  Every CTA of an m-tile re-reads its activation slab from L2, and that
            // ingest is what bounds these kernels at small M.
            auto a_rows = [&]() { const int r = p.M - mt * 128; return r >= 128 ? 128 : (r + 7) & ~7; };
            auto tx_bytes = [&]() {
                const int r = a_rows();
                return r == 128 ? C::TX_BYTES : C::TX_BYTES - SUB * (C::A_BYTES - (uint32_t)r * (Q4K ? 160u : 144u));
            };
            auto copy_a = [&](int i, int gc) {
                const int kc = kc0 + i, s = gc % NST, r = a_rows();
                uint8_t* st = smem + s * C::STAGE;
#pragma unroll
                for (int u = 0; u < SUB; u++) {
                    const size_t kk = (size_t)kc * SUB + u;   // 128-K activation tile index
                    const int8_t* src = p.aq + (kk * (p.Mpad / 128) + mt) * kActTile;
                    uint8_t* dst = st + u * C::A_BYTES;
                    if (r == 128) {
                        bulk_g2s(dst, src, C::A_BYTES, &full[s]);
                    } else {
                        bulk_g2s(dst, src, (uint32_t)r * 128u, &full[s]);
                        bulk_g2s(dst + C::OFF_DX, src + C::OFF_DX, (uint32_t)r * 16u, &full[s]);
                        if constexpr (Q4K) bulk_g2s(dst + C::OFF_CX, src + C::OFF_CX, (uint32_t)r * 16u, &full[s]);
                    }
                }
            };
            // the first stages are free: their weights go out before the wait on the preceding kernel
            const int npre = nloc < NST ? nloc : NST;
            tile_of(0, n0, mt);
            for (int i = 0; i < npre; i++) {
                mbar_arrive_expect_tx(&full[i], tx_bytes());
                copy_w(i, i);
                last_it[i] = 0;
            }
            griddep_wait();   // the activation tiles come from the preceding kernel
            for (int i = 0; i < npre; i++) copy_a(i, i);
            bool go = true;
            for (int ti = 0; go && ti < my_tiles; ti++) {
                tile_of(ti, n0, mt);
                for (int i = ti == 0 ? npre : 0; i < nloc; i++) {
                    const int gc = ti * nloc + i, s = gc % NST, it = gc / NST;
                    if (!(go = mbar_wait(&empty[s], (it & 1) ^ 1, abort_flag, 1))) break;
                    mbar_arrive_expect_tx(&full[s], tx_bytes());
                    copy_w(i, gc);
                    copy_a(i, gc);
                    last_it[s] = it;
                }
            }
            if (*abort_flag) {   // let copies already in flight land before the CTA exits
                volatile int never = 0;
                for (int s = 0; s < NST; s++)
                    if (last_it[s] >= 0) mbar_wait(&full[s], last_it[s] & 1, &never, 11);
            }
        }
        griddep_launch();   // this CTA's loads are all issued: the next kernel may start its prologue
    } else if (warp == 1) {
        // lane 0 issues the MMAs; for Q4_K the whole warp first unpacks the stage
        constexpr uint32_t idesc = idesc_make(2, 1, Q4K ? 0 : 1, 128, BN);
        for (int kc = 0; kc < my_tiles * nloc; kc++) {   // running chunk index over this CTA's tiles
            const int s = kc % NST, it = kc / NST, g = kc % NGRP, ug = kc / NGRP;
            bool go = true;
            if constexpr (Q4K) {
                if (!__all_sync(0xffffffffu, mbar_wait(&full[s], it & 1, abort_flag, 2))) break;
                uint8_t* st = smem + s * C::STAGE;
#pragma unroll
                for (int u = 0; u < SUB; u++)
                    unpack_q4k_stage<BN>(st + C::OFF_R + u * C::R_BYTES, st + C::OFF_B + u * C::B_BYTES,
                                         reinterpret_cast<float*>(st + C::OFF_S + u * C::S_BYTES), lane);
                __syncwarp();
                if (lane == 0) mbar_arrive(&unpk[s]);   // the promotion warps may read the scale tile
            } else if (lane == 0) {
                go = mbar_wait(&full[s], it & 1, abort_flag, 2);
            }
            if (lane == 0 && go) go = mbar_wait(&tempty[g], (ug & 1) ^ 1, abort_flag, 3);
            if (lane == 0 && go) {
                tc_fence_after();
                const uint32_t a_base = smem_u32(smem + s * C::STAGE), b_base = a_base + C::OFF_B;
                // one MMA per 32-block, each into its own TMEM buffer (no accumulation)
#pragma unroll
                for (int j = 0; j < CB; j++) {
                    const uint32_t u = j / 4, jj = j % 4;
                    mma_i8(tmem + (g * CB + j) * BN, sdesc_sw128(a_base + u * C::A_BYTES + 32 * jj),
                           sdesc_sw128(b_base + u * C::B_BYTES + 32 * jj), idesc, 0);
                }
                mma_commit(&tfull[g]);   // the chunk's dot tiles are ready
                mma_commit(&empty[s]);   // its shared-memory operands may be overwritten
            }
            if (!__shfl_sync(0xffffffffu, go ? 1 : 0, 0)) break;   // the whole warp leaves together
        }
        griddep_launch();
    } else {
        const int pw = warp - 2, q = warp & 3, cg = pw >> 2;
        const int row = q * 32 + lane, c0 = cg * CW;
        int n0, mt;
        tile_of(0, n0, mt);
        int m0 = mt * 128, m = m0 + row;
        bool active = (m0 + q * 32) < p.M;   // warp-uniform
        uint64_t acc2[CW / 2];   // column pairs (2c, 2c+1), packed for f32x2 math
        const uint32_t t_lane = tmem + ((uint32_t)(q * 32) << 16) + c0;
        // Work unit = a batch of BATCH blocks (BATCH*CW int32 per thread, one TMEM-load wait
        // per batch); BPC batches per 4-block chunk.  (Overlapping batch t+1's loads with batch
        // t's math measured slower: it forces smaller batches, and the waits dominate.)
        constexpr int BPC = CB / BATCH;
        const int nbatch = nloc * BPC;   // chunk indices below are local to this K split
        bool ok = true;
        // wait for a chunk's operands + dot tiles, then issue the batch's TMEM loads
        auto issue = [&](uint32_t (&I)[BATCH][CW], int t) {
            const int kc = t / BPC, jb = t % BPC, g = kc % NGRP;
            if (jb == 0) {
                bool w = mbar_wait(&full[kc % NST], (kc / NST) & 1, abort_flag, 4) &&
                         (!Q4K || mbar_wait(&unpk[kc % NST], (kc / NST) & 1, abort_flag, 6)) &&
                         mbar_wait(&tfull[g], (kc / NGRP) & 1, abort_flag, 5);
                ok = __all_sync(0xffffffffu, w);
                if (!ok) return;
                tc_fence_after();
            }
#pragma unroll
            for (int jj = 0; jj < BATCH; jj++) {
                const uint32_t ta = t_lane + (g * CB + jb * BATCH + jj) * BN;
                if constexpr (CW % 32 == 0) {
#pragma unroll
                    for (int u = 0; u < CW / 32; u++)
                        tmem_ld32(ta + u * 32, *reinterpret_cast<uint32_t(*)[32]>(&I[jj][u * 32]));
                } else if constexpr (CW == 16) {
                    tmem_ld16(ta, I[jj]);
                } else if constexpr (CW == 8) {
                    tmem_ld8(ta, I[jj]);
                } else {
                    static_assert(CW == 4, "promotion warps own 4, 8, 16 or a multiple of 32 columns");
                    tmem_ld4(ta, I[jj]);
                }
            }
        };
        // wait for batch t's loads, pin the registers after the wait, release the TMEM group
        auto landed = [&](uint32_t (&I)[BATCH][CW], int t) {
            tmem_ld_wait();
#pragma unroll
            for (int jj = 0; jj < BATCH; jj++)
#pragma unroll
                for (int c = 0; c < CW; c++) asm volatile("" : "+r"(I[jj][c]));
            if (t % BPC == BPC - 1) {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[(t / BPC) % NGRP]);
            }
        };
        auto promote = [&](const uint32_t (&I)[BATCH][CW], int t) {
            const int kc = t / BPC, jb = t % BPC, s = kc % NST;
            // this batch's blocks lie in one 128-K tile u of the chunk (BATCH divides 4)
            const int u = (jb * BATCH) / 4;
            const uint8_t* st = smem + s * C::STAGE;
            if (active) {
                const float4 dxv = reinterpret_cast<const float4*>(st + u * C::A_BYTES + C::OFF_DX)[row];
                const float dxa[4] = {dxv.x, dxv.y, dxv.z, dxv.w};
                float cxa[4] = {0, 0, 0, 0};
                if constexpr (Q4K) {
                    const float4 cxv = reinterpret_cast<const float4*>(st + u * C::A_BYTES + C::OFF_CX)[row];
                    cxa[0] = cxv.x; cxa[1] = cxv.y; cxa[2] = cxv.z; cxa[3] = cxv.w;
                }
#pragma unroll
                for (int jj = 0; jj < BATCH; jj++) {   // blocks in ascending order: b = 4 kc + j
                    const int j = (jb * BATCH + jj) % 4;
                    const uint64_t dx2 = pack2(dxa[j], dxa[j]);
                    // scale tile: [BN/4 column quads][T][4 blocks][4 columns]
                    const float* sq = reinterpret_cast<const float*>(st + C::OFF_S + u * C::S_BYTES) + (c0 / 4) * 16 * C::T + j * 4;
#pragma unroll
                    for (int c = 0; c < CW; c += 4) {
                        const float4 w4 = *reinterpret_cast<const float4*>(sq + (c / 4) * 16 * C::T);
                        // exact int32 -> f32: bits(v + 0x4B400000) = 1.5*2^23 + v, minus 1.5*2^23
                        const uint64_t f01 = add2(pack2(__uint_as_float(I[jj][c] + 0x4B400000u),
                                                        __uint_as_float(I[jj][c + 1] + 0x4B400000u)), kMagicNeg2);
                        const uint64_t f23 = add2(pack2(__uint_as_float(I[jj][c + 2] + 0x4B400000u),
                                                        __uint_as_float(I[jj][c + 3] + 0x4B400000u)), kMagicNeg2);
                        acc2[c / 2] = fma2(mul2(pack2(w4.x, w4.y), dx2), f01, acc2[c / 2]);
                        acc2[c / 2 + 1] = fma2(mul2(pack2(w4.z, w4.w), dx2), f23, acc2[c / 2 + 1]);
                    }
                    if constexpr (Q4K) {
                        const uint64_t cx2 = pack2(cxa[j], cxa[j]);
#pragma unroll
                        for (int c = 0; c < CW; c += 4) {
                            const float4 n4 = *reinterpret_cast<const float4*>(sq + (c / 4) * 16 * C::T + 16);
                            acc2[c / 2] = fma2(pack2(-n4.x, -n4.y), cx2, acc2[c / 2]);
                            acc2[c / 2 + 1] = fma2(pack2(-n4.z, -n4.w), cx2, acc2[c / 2 + 1]);
                        }
                    }
                }
            }
            if (jb == BPC - 1) {   // chunk done: its shared-memory stage may be refilled
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
            }
        };
        for (int ti = 0; ok && ti < my_tiles; ti++) {
        if (ti > 0) {
            tile_of(ti, n0, mt);
            m0 = mt * 128;
            m = m0 + row;
            active = (m0 + q * 32) < p.M;
        }
#pragma unroll
        for (int c = 0; c < CW / 2; c++) acc2[c] = 0;
        for (int t = ti * nbatch; ok && t < (ti + 1) * nbatch; t++) {   // running batch index
            uint32_t I[BATCH][CW];
            issue(I, t);
            if (!ok) break;
            landed(I, t);
            promote(I, t);
        }
        griddep_launch();
        griddep_wait();   // the residual and the output buffers belong to the preceding kernels' chain
        // epilogue: bias -> act -> residual (mg-opencl.cpp:481-493)
        float acc[CW];
#pragma unroll
        for (int c = 0; c < CW / 2; c++) unpack2(acc2[c], acc[2 * c], acc[2 * c + 1]);
        if (p.nsplit > 1) {
            // split-K: publish this split's partial, then the last CTA of the tile sums all
            // partials in split order (deterministic) and runs the epilogue below
            const bool vecp = (p.N % 4) == 0;
            if (m < p.M && !*abort_flag) {
                float* dst = p.part + ((size_t)kz * p.M + m) * p.N;
#pragma unroll
                for (int c = 0; c < CW; c += 4) {
                    const int n = n0 + c0 + c;
                    if (n >= p.N) break;
                    if (vecp) *reinterpret_cast<float4*>(dst + n) = make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);
                    else for (int i = 0; i < 4 && n + i < p.N; i++) dst[n + i] = acc[c + i];
                }
            }
            __threadfence();
            asm volatile("bar.sync 1, %0;" ::"r"(C::NPW * 32) : "memory");
            volatile int* last_flag = (volatile int*)(tmem_slot + 2);
            int* ctr = p.counters + blockIdx.y * gridDim.x + blockIdx.x;   // (split-K is never persistent)
            if (threadIdx.x == 64) {
                const int prev = atomicAdd(ctr, 1);
                *last_flag = prev == p.nsplit - 1;
                if (prev == p.nsplit - 1) *ctr = 0;   // every split has arrived: re-arm for the next call
            }
            asm volatile("bar.sync 1, %0;" ::"r"(C::NPW * 32) : "memory");
            if (!*last_flag) goto done;
            __threadfence();
            if (m < p.M) {
#pragma unroll
                for (int c = 0; c < CW; c++) {
                    const int n = n0 + c0 + c;
                    if (n >= p.N) break;
                    float v = 0.0f;
                    for (int z = 0; z < p.nsplit; z++) {
                        const float pz = z == kz ? acc[c] : __ldcg(p.part + ((size_t)z * p.M + m) * p.N + n);
                        v = z == 0 ? pz : __fadd_rn(v, pz);
                    }
                    acc[c] = v;
                }
            }
        }
        const bool store = m < p.M && !*abort_flag;
        const int nbase = n0 + c0;
        float vals[CW];
        if (store) {
            const bool vec = (p.N % 4) == 0;
#pragma unroll
            for (int c = 0; c < CW; c += 4) {
                const int n = nbase + c;
                float v[4] = {acc[c], acc[c + 1], acc[c + 2], acc[c + 3]};
                if (n + 3 < p.N && vec) {
                    if (p.bias) {
                        const float4 b4 = __ldg(reinterpret_cast<const float4*>(p.bias + n));
                        v[0] = __fadd_rn(v[0], b4.x); v[1] = __fadd_rn(v[1], b4.y);
                        v[2] = __fadd_rn(v[2], b4.z); v[3] = __fadd_rn(v[3], b4.w);
                    }
#pragma unroll
                    for (int i = 0; i < 4; i++) v[i] = act_apply(v[i], p.act);
                    if (p.resid) {
                        const float4 r4 = *reinterpret_cast<const float4*>(p.resid + (size_t)m * p.resid_ld + n);
                        v[0] = __fadd_rn(v[0], r4.x); v[1] = __fadd_rn(v[1], r4.y);
                        v[2] = __fadd_rn(v[2], r4.z); v[3] = __fadd_rn(v[3], r4.w);
                    }
                    if (p.y) *reinterpret_cast<float4*>(p.y + (size_t)m * p.N + n) = make_float4(v[0], v[1], v[2], v[3]);
                } else {
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        if (n + i >= p.N) { v[i] = 0.0f; continue; }
                        float x = v[i];
                        if (p.bias) x = __fadd_rn(x, p.bias[n + i]);
                        x = act_apply(x, p.act);
                        if (p.resid) x = __fadd_rn(x, p.resid[(size_t)m * p.resid_ld + n + i]);
                        if (p.y) p.y[(size_t)m * p.N + n + i] = x;
                        v[i] = x;
                    }
                }
#pragma unroll
                for (int i = 0; i < 4; i++) vals[c + i] = v[i];
            }
        } else {
#pragma unroll
            for (int c = 0; c < CW; c++) vals[c] = 0.0f;
        }
        if constexpr (CW == 8 || CW == 16) {
            if (p.ap && store) prep_store<CW>(p.ap, p.ap_S, p.ap_H, p.ap_nt, m, nbase, vals);
        }
        if constexpr (CW == 16) {
            if (p.qo) {
                // The 32-block of columns [32k, 32k+32) is split between this warp (16 columns) and
                // the warp of the neighbouring column group (same rows): exchange amax and sum.
                float* xa = reinterpret_cast<float*>(smem + C::XCHG);
                int* xs = reinterpret_cast<int*>(xa + C::NPW * 32);
                float amax = 0.0f;
#pragma unroll
                for (int c = 0; c < CW; c++) amax = fmaxf(amax, fabsf(vals[c]));
                xa[pw * 32 + lane] = amax;
                asm volatile("bar.sync 1, %0;" ::"r"(C::NPW * 32) : "memory");
                amax = fmaxf(amax, xa[(pw ^ 4) * 32 + lane]);
                const float d = __fdiv_rn(amax, 127.0f);
                const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
                alignas(16) int8_t qv[16];
                int sum = 0;
#pragma unroll
                for (int c = 0; c < 16; c++) {
                    const int qi = (int)roundf(__fmul_rn(vals[c], id));
                    qv[c] = (int8_t)qi;
                    sum += qi;
                }
                if (p.qo_c) {
                    xs[pw * 32 + lane] = sum;
                    asm volatile("bar.sync 1, %0;" ::"r"(C::NPW * 32) : "memory");
                    sum += xs[(pw ^ 4) * 32 + lane];
                }
                if (store) {
                    ActQ qa;
                    qa.q = p.qo;
                    qa.Mpad = p.qo_Mpad;
                    const int gn = p.qo_n0 + nbase, kc = gn >> 7, j = (gn >> 5) & 3;
                    *reinterpret_cast<int4*>(qa.q + act_code(qa, kc, m, gn & 127)) = *reinterpret_cast<const int4*>(qv);
                    if (((gn >> 4) & 1) == 0) {   // the lower half writes the block's scales
                        act_dx(qa, kc, m)[j] = d;
                        if (p.qo_c) act_cx(qa, kc, m)[j] = __fmul_rn(d, (float)sum);
                    }
                }
            }
        }
        }   // tiles
    }

done:
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

template <int BN, int CG, bool Q4K, int CB>
static int set_smem_attr() {
    using C = QGemmCfg<BN, CG, Q4K, CB>;
    const bool a = cudaFuncSetAttribute(qgemm_kernel<BN, CG, Q4K, CB, false>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) == cudaSuccess;
    const bool b = cudaFuncSetAttribute(qgemm_kernel<BN, CG, Q4K, CB, true>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) == cudaSuccess;
    return a && b ? 0 : -1;
}

// Sets the dynamic shared-memory limit of every instantiation on the current device.  Must
// run once per device before the first launch (the runtime does it at creation, outside any
// stream capture).
// (BN, CG, CB): tile width, column groups, 32-blocks per pipeline chunk
#define MGC_QGEMM_CONFIGS(X) X(16, 1, 4) X(16, 1, 8) X(16, 2, 4) X(16, 2, 8) X(16, 4, 4) X(16, 4, 8) X(32, 1, 4) X(32, 2, 4) X(32, 2, 8) X(32, 4, 4) X(32, 4, 8) X(48, 3, 4) \
    X(48, 6, 4) \
    X(64, 2, 4) X(64, 4, 4)

int qgemm_prepare() {
    int rc = 0;
#define X(BN, CG, CB) rc |= set_smem_attr<BN, CG, false, CB>(); rc |= set_smem_attr<BN, CG, true, CB>();
    MGC_QGEMM_CONFIGS(X)
#undef X
    return rc;
}

int sm_count() {   // SMs of the current device (cached per device; concurrent first calls agree)
    static std::atomic<int> n[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    int v = n[dev].load(std::memory_order_relaxed);
    if (v == 0) {
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
        n[dev].store(v, std::memory_order_relaxed);
    }
    return v;
}

template <int BN, int CG, bool Q4K, int CB>
static int run_qgemm(QGemmArgs a, cudaStream_t st) {
    ++g_launch_count;
    using C = QGemmCfg<BN, CG, Q4K, CB>;
    const int tiles_n = (a.N + BN - 1) / BN, tiles_m = (a.M + 127) / 128, ctas = sm_count() * MGC_QGEMM_MINB;
    if (a.nsplit == 1 && tiles_n * tiles_m > ctas) {   // more tiles than one wave: persistent CTAs
        a.tiles_n = tiles_n;
        a.tiles_m = tiles_m;
        launch_k(qgemm_kernel<BN, CG, Q4K, CB, true>, dim3(ctas, 1, 1), C::THREADS, C::SMEM, st, a);
        return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
    }
    dim3 grid(tiles_n, tiles_m, a.nsplit);
    launch_k(qgemm_kernel<BN, CG, Q4K, CB, false>, grid, C::THREADS, C::SMEM, st, a);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

// Tile shape (BN columns, CG column groups of promotion warps, CB 32-blocks per chunk).
// MGC_QGEMM_CFG="BN,CG[,CB]" overrides the heuristic (used to sweep shapes); MGC_QGEMM_CB=4
// keeps 4-block chunks everywhere.
static void pick_cfg(int M, int N, int K, bool q4k, bool fused_quant, bool prep, int& bn, int& cg, int& cb) {
    struct Overrides { int fbn = 0, fcg = 0, fcb = 0, cb_max = 8; };
    static const Overrides ov = [] {   // read once (thread-safe static initialisation)
        Overrides o;
        if (const char* e = std::getenv("MGC_QGEMM_CFG")) std::sscanf(e, "%d,%d,%d", &o.fbn, &o.fcg, &o.fcb);
        if (const char* e = std::getenv("MGC_QGEMM_CB")) o.cb_max = std::atoi(e) == 4 ? 4 : 8;
        return o;
    }();
    const int fbn = ov.fbn, fcg = ov.fcg, fcb = ov.fcb, cb_max = ov.cb_max;
    const long wave = (long)sm_count() * MGC_QGEMM_MINB;   // CTAs of one wave (the persistent grid)
    // 8-block chunks (half the pipeline hand-offs per block) where instantiated and K allows
    auto chunk = [&](int b, int g) { return cb_max == 8 && K % 256 == 0 && (b == 16 || (b == 32 && g >= 2)) ? 8 : 4; };
    if (fbn && (!fused_quant || (fbn % 32 == 0 && fbn / fcg == 16)) && (!prep || fbn / fcg == 8 || fbn / fcg == 16)) {
        bn = fbn; cg = fcg; cb = fcb ? fcb : chunk(bn, cg);
        return;
    }
    // Pick the width whose tile grid fills the SMs in the fewest waves, weighing a wave by
    // its per-CTA work (BN) plus a fixed per-chunk cost (~16 columns' worth).  Promotion warps
    // own 4-8 columns (several warps per SM sub-partition hide each other's latency), 16 where
    // the epilogue quantizes (a 32-block split over two warps).  Widths whose last tile would
    // run past the padded weight rows are skipped.
    const int mt = (M + 127) / 128, npad = round_up(N, 128);
    // (16-wide tiles run four 4-column warps, except when the epilogue stores attention tiles,
    // which take 8 or 16 columns per warp)
    static const int cand8[4][2] = {{16, 4}, {32, 4}, {48, 6}, {64, 4}}, cand8p[4][2] = {{16, 2}, {32, 4}, {48, 6}, {64, 4}},
                     cand16[4][2] = {{16, 1}, {32, 2}, {48, 3}, {64, 4}};
    const auto& cand = fused_quant ? cand16 : prep ? cand8p : cand8;
    // Many waves (the CTAs will run persistent): the wave count no longer separates the widths.
    // Measured at M = 4097 and 16388 (768 <-> 3072 shapes): Q8_0 runs fastest with 48-wide tiles
    // of three 16-column groups and 4-block chunks (87.8 vs 92.7 us for 4097 x 768 -> 3072 with
    // 32-wide tiles), Q4_K with 32-wide tiles of two 16-column groups and 8-block chunks (125.6
    // vs 130.0 us); both keep the activation re-reads per promotion below the 16- and 32-wide
    // tiles with more column groups, which are bound by the L2 ingest of those re-reads.
    if (!fused_quant && (long)((N + 63) / 64) * mt > wave && K % 256 == 0) {
        if (q4k) { bn = 32; cg = 2; cb = chunk(bn, cg); }
        else { bn = 48; cg = 3; cb = 4; }
        if ((long)((N + bn - 1) / bn) * bn <= npad) return;
        bn = 32; cg = 4; cb = chunk(bn, cg);   // (48 would read past the padded weight rows)
        return;
    }
    long best = -1;
    for (const auto& c : cand) {
        const int tiles_n = (N + c[0] - 1) / c[0];
        if (tiles_n * c[0] > npad) continue;
        if (fused_quant && c[0] % 32 != 0) continue;   // both halves of a 32-block in one CTA
        const long waves = ((long)tiles_n * mt + wave - 1) / wave;
        const long cost = waves * (c[0] + 16);
        if (best < 0 || cost < best) { best = cost; bn = c[0]; cg = c[1]; }
    }
    cb = chunk(bn, cg);
}

int launch_qgemm(const QWeight& w, const ActQ& a, int M, const float* bias, int act,
                 const float* resid, float* y, cudaStream_t st, const SplitK* sk, const ActQ* qo, bool qo_c,
                 const AttnPrepOut* ap, int resid_ld, int qo_n0) {
    if (w.K % 128 != 0 || M <= 0 || M > a.Mpad) return -2;
    if (ap && (w.N != 3 * ap->H * fa::D || M % ap->S != 0)) return -2;
    if (qo && (w.N % 128 != 0 || qo_n0 % 128 != 0 || M > qo->Mpad)) return -2;
    const bool q4 = w.wtype == 12;
    int bn, cg, cb;
    pick_cfg(M, w.N, w.K, w.wtype == 12, qo != nullptr, ap != nullptr, bn, cg, cb);
    if (w.K % (32 * cb) != 0) return -2;
    // Split-K (MGC_QGEMM_SPLITK=<n>) is off by default: on the config-1 shapes it measured
    // slower than one CTA per tile (ncu: attn_o 11 -> 26 us with 3 splits, ffn_down 22 -> 38 us
    // with 4), so the library only splits when asked.
    const int nkc = w.K / (32 * cb), tiles = ((w.N + bn - 1) / bn) * ((M + 127) / 128);
    int nsplit = 1;
    if (sk && sk->part && sk->counters) {
        if (const char* e = std::getenv("MGC_QGEMM_SPLITK")) nsplit = std::max(1, std::atoi(e));
        nsplit = std::min(nsplit, nkc);
        if ((size_t)nsplit * M * w.N > sk->part_floats || tiles > sk->n_counters) nsplit = 1;
    }
    const int cps = (nkc + nsplit - 1) / nsplit;
    nsplit = (nkc + cps - 1) / cps;   // no empty split
    QGemmArgs p{a.q, a.Mpad, w.q, w.s, w.Npad, M, w.N, w.K, bias, resid, y, act,
                sk ? sk->part : nullptr, sk ? sk->counters : nullptr, nsplit, cps,
                qo ? qo->q : nullptr, qo ? qo->Mpad : 0, qo_c ? 1 : 0, qo_n0, resid_ld > 0 ? resid_ld : w.N,
                ap ? ap->buf : nullptr, ap ? ap->S : 1, ap ? ap->H : 1, ap ? ap->nt : 1, 0, 0};
#define X(BN, CG, CB) \
    if (bn == BN && cg == CG && cb == CB) return q4 ? run_qgemm<BN, CG, true, CB>(p, st) : run_qgemm<BN, CG, false, CB>(p, st);
    MGC_QGEMM_CONFIGS(X)
#undef X
    return -2;
}

}  // namespace mgc
