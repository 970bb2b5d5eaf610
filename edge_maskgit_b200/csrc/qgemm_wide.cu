// qgemm_wide.cu -- the Q8_0 / Q4_K int8-dot GEMM for large M (config 2's M >= 1025, the
// 16388-row config-5 step): wide persistent tiles and a ring of per-block TMEM slots.
//
// Same arithmetic as qgemm.cu (k_mul_mat_q8_i8 / k_mul_mat_q4k_i8, mg-opencl.cpp:440-590):
// per output (m, n) and 32-block b ascending, idot_b on the tensor core (exact int32), then
//     Q8_0:  acc = fma(dw*dx, idot_b, acc)
//     Q4_K:  acc = fma(scl*dx, idot_b, acc); acc = fma(-mnl, dx*sumx, acc)
// and the fused bias -> act -> residual epilogue.  Results are bit-identical to qgemm.cu.
//
// Structure (one CTA per SM, persistent over 128 x BN tiles, BN = 32, 64 or 128):
//   warp 0      producer: per 128-K chunk, three cp.async.bulk copies (activation tile with its
//               scales, weight codes, weight scales) into an up-to-8-stage shared-memory ring
//   warp 1      MMA issuer: one tcgen05.mma.kind::i8 (M=128, N=BN, K=32) per 32-block into the
//               next free TMEM slot (512/BN slots of BN columns), each slot with its own
//               full / empty mbarrier -- so the tensor core runs up to 512/BN blocks ahead of
//               the promotion, across chunk and tile boundaries
//   warps 2..   promotion, 4*BN/32 warps: thread = one row x 32 columns.  Per block: tcgen05.ld
//               the 32 dots, re-arm the slot and release it at once, then promote in registers.
// Pre-biased accumulators: every slot holds the int32 bit pattern of 1.5*2^23 before its MMA,
// which accumulates onto it, so a slot comes back as the f32 bit pattern of 1.5*2^23 + idot
// (|idot| <= 32*127*128 < 2^22): one packed f32x2 subtraction converts two dots exactly.  The
// promotion warp writes the bias back (tcgen05.st) before it releases the slot.
#include "qgemm_common.cuh"
#include "attnprep.cuh"

#include <algorithm>
#include <cstdio>
#include <cstdlib>

namespace mgc {

template <int BN, bool Q4K>
struct WideCfg {
    // promotion threads own one row x 32 columns; BN/32 column groups of 4 warps (one per SM
    // sub-partition / TMEM lane quarter)
    static constexpr int CG = BN / 32, NPW = 4 * CG, THREADS = 64 + 32 * NPW;
    static constexpr int NSLOT = 512 / BN > 16 ? 16 : 512 / BN;
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr uint32_t T = Q4K ? 2 : 1;
    // stage = [activation tile: codes | dx | (dx*sumx)] [weight code tile] [weight scale tile]
    static constexpr uint32_t A_BYTES = Q4K ? 20480 : 18432, B_BYTES = BN * 128, S_BYTES = BN * 16 * T;
    static constexpr uint32_t OFF_DX = 16384, OFF_CX = 18432, OFF_B = A_BYTES, OFF_S = OFF_B + B_BYTES;
    static constexpr uint32_t STAGE = (OFF_S + S_BYTES + 1023) & ~1023u;
    static constexpr uint32_t TX_BYTES = A_BYTES + B_BYTES + S_BYTES;
    // epilogue staging: a 32 x 32 f32 tile per promotion warp
    static constexpr uint32_t EPI_BYTES = NPW * 32 * 32 * 4;
    static constexpr uint32_t RING_MAX = 232448 - 1024 - 512 - EPI_BYTES;   // opt-in limit - slack - barriers - staging
    static constexpr int NST = RING_MAX / STAGE > 8 ? 8 : (int)(RING_MAX / STAGE);
    static constexpr uint32_t OFF_EPI = NST * STAGE, BAR_OFF = OFF_EPI + EPI_BYTES;
    static constexpr uint32_t SMEM = 1024 + BAR_OFF + 512;
    static_assert(BN == 32 || BN == 64, "tile width");
    static_assert((2 * NST + 2 * NSLOT) * 8 + 8 <= 512, "barrier area");
};

constexpr uint32_t kBias = 0x4B400000u;   // int32 bits of 1.5 * 2^23

template <int BN, bool Q4K>
__global__ void __launch_bounds__(WideCfg<BN, Q4K>::THREADS, 1) qgemm_wide_kernel(const QGemmArgs p) {
    using C = WideCfg<BN, Q4K>;
    constexpr int NST = C::NST, NSLOT = C::NSLOT;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* full = (uint64_t*)(smem + C::BAR_OFF);
    uint64_t* empty = full + NST;
    uint64_t* tfull = empty + NST;
    uint64_t* tempty = tfull + NSLOT;
    uint32_t* tmem_slot = (uint32_t*)(tempty + NSLOT);
    volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = p.tiles_n * p.tiles_m, nkc = p.K / 128;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NST; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1 + C::NPW); }
        for (int s = 0; s < NSLOT; s++) { mbar_init(&tfull[s], 1); mbar_init(&tempty[s], C::NPW); }
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // promotion warp (q, cg): TMEM lanes 32q.. (its sub-partition), columns 32cg.. of every slot
    const int pw = warp - 2, q = warp & 3, cg = pw >> 2;
    const uint32_t t_lane = tmem + ((uint32_t)(q * 32) << 16) + cg * 32;
    const bool prebias = p.wide_prebias != 0;
    if (warp >= 2 && prebias) {
        for (int s = 0; s < NSLOT; s++) tmem_st32_fill(t_lane + s * BN, kBias);
        tmem_st_wait();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    griddep_wait();   // the activation tiles and the residual come from the preceding kernels

    if (warp == 0) {
        if (lane == 0) {
            int gc = 0;
            bool go = true;
            for (int t = blockIdx.x; go && t < ntiles; t += gridDim.x) {
                const int n0 = (t % p.tiles_n) * BN, mt = t / p.tiles_n;
                for (int kc = 0; kc < nkc; kc++, gc++) {
                    const int s = gc % NST, it = gc / NST;
                    if (it > 0 && !(go = mbar_wait(&empty[s], (it - 1) & 1, abort_flag, 21))) break;
                    uint8_t* st = smem + s * C::STAGE;
                    mbar_arrive_expect_tx(&full[s], C::TX_BYTES);
                    bulk_g2s(st, p.aq + ((size_t)kc * (p.Mpad / 128) + mt) * kActTile, C::A_BYTES, &full[s]);
                    bulk_g2s(st + C::OFF_B, p.wq + ((size_t)kc * p.Npad + n0) * 128, C::B_BYTES, &full[s]);
                    bulk_g2s(st + C::OFF_S, p.ws + ((size_t)kc * (p.Npad / 4) + n0 / 4) * 16 * C::T, C::S_BYTES,
                             &full[s]);
                }
            }
            if (*abort_flag) {   // let the copies already in flight land before the CTA exits
                volatile int never = 0;
                for (int s = 0; s < NST && s < gc; s++) {
                    const int g = gc - 1 - ((gc - 1 - s) % NST);   // last chunk issued into stage s
                    mbar_wait(&full[s], (g / NST) & 1, &never, 11);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_make(2, 1, Q4K ? 0 : 1, 128, BN);
            int gc = 0, gb = 0;
            bool go = true;
            for (int t = blockIdx.x; go && t < ntiles; t += gridDim.x) {
                for (int kc = 0; go && kc < nkc; kc++, gc++) {
                    const int s = gc % NST;
                    if (!(go = mbar_wait(&full[s], (gc / NST) & 1, abort_flag, 22))) break;
                    tc_fence_after();
                    const uint32_t a_base = smem_u32(smem + s * C::STAGE), b_base = a_base + C::OFF_B;
#pragma unroll
                    for (int j = 0; j < 4; j++, gb++) {
                        const int sl = gb % NSLOT, u = gb / NSLOT;
                        if (u > 0 && !(go = mbar_wait(&tempty[sl], (u - 1) & 1, abort_flag, 23))) break;
                        tc_fence_after();
                        // accumulate onto the slot's 1.5*2^23 bias (see the header)
                        mma_i8(tmem + sl * BN, sdesc_sw128(a_base + 32 * j), sdesc_sw128(b_base + 32 * j), idesc,
                               prebias ? 1u : 0u);
                        mma_commit(&tfull[sl]);
                    }
                    if (go) mma_commit(&empty[s]);   // the chunk's operands may be overwritten
                }
            }
        }
    } else {
        const int row = q * 32 + lane, c0 = cg * 32;
        float* stg = reinterpret_cast<float*>(smem + C::OFF_EPI) + pw * 32 * 32;   // this warp's staging tile
        int gc = 0, gb = 0;
        bool ok = true;
        for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x) {
            const int n0 = (t % p.tiles_n) * BN, mt = t / p.tiles_n;
            const bool active = (mt * 128 + q * 32) < p.M;   // warp-uniform
            uint64_t acc2[16];
#pragma unroll
            for (int c = 0; c < 16; c++) acc2[c] = 0;
            const int nblk = 4 * nkc, gc0 = gc;
            // Software pipeline over the tile's blocks: block i's dots sit in registers (cur)
            // while block i+1's TMEM load (nxt) is in flight behind block i's promotion; the
            // slot's re-arm store is waited for only after the promotion.
            uint32_t IA[32], IB[32];
            auto wait_slot = [&](int b) {
                return __all_sync(0xffffffffu, mbar_wait(&tfull[b % NSLOT], (b / NSLOT) & 1, abort_flag, 25));
            };
            auto step = [&](uint32_t (&cur)[32], uint32_t (&nxt)[32], int i) {
                const int b = gb + i, sl = b % NSLOT, j = i & 3, s = (gc0 + (i >> 2)) % NST;
                if (j == 0) {   // the chunk's dx / scales: observe its arrival on this thread too
                    ok = __all_sync(0xffffffffu, mbar_wait(&full[s], ((gc0 + (i >> 2)) / NST) & 1, abort_flag, 24));
                    if (!ok) return;
                }
                tmem_ld_wait();
#pragma unroll
                for (int c = 0; c < 32; c++) asm volatile("" : "+r"(cur[c]));   // pin after the wait
                if (prebias) tmem_st32_fill(t_lane + sl * BN, kBias);   // re-arm the slot
                else {
#pragma unroll
                    for (int c = 0; c < 32; c++) cur[c] += kBias;   // plain dots: bias here
                }
                if (i + 1 < nblk) {
                    if (!(ok = wait_slot(b + 1))) return;
                    tc_fence_after();
                    tmem_ld32(t_lane + ((b + 1) % NSLOT) * BN, nxt);
                }
                if (active) {
                    const uint8_t* st = smem + s * C::STAGE;
                    const float dj = reinterpret_cast<const float*>(st + C::OFF_DX)[row * 4 + j];
                    const uint64_t dx2 = pack2(dj, dj);
                    // scale tile: [BN/4 column quads][T][4 blocks][4 columns]
                    const float* sq = reinterpret_cast<const float*>(st + C::OFF_S) + (c0 / 4) * 16 * C::T + j * 4;
#pragma unroll
                    for (int c = 0; c < 32; c += 4) {
                        const float4 w4 = *reinterpret_cast<const float4*>(sq + (c / 4) * 16 * C::T);
                        const uint64_t f01 = add2(pack2(__uint_as_float(cur[c]), __uint_as_float(cur[c + 1])), kMagicNeg2);
                        const uint64_t f23 = add2(pack2(__uint_as_float(cur[c + 2]), __uint_as_float(cur[c + 3])), kMagicNeg2);
                        acc2[c / 2] = fma2(mul2(pack2(w4.x, w4.y), dx2), f01, acc2[c / 2]);
                        acc2[c / 2 + 1] = fma2(mul2(pack2(w4.z, w4.w), dx2), f23, acc2[c / 2 + 1]);
                    }
                    if constexpr (Q4K) {
                        const float cj = reinterpret_cast<const float*>(st + C::OFF_CX)[row * 4 + j];
                        const uint64_t cx2 = pack2(cj, cj);
#pragma unroll
                        for (int c = 0; c < 32; c += 4) {
                            const float4 n4 = *reinterpret_cast<const float4*>(sq + (c / 4) * 16 * C::T + 16);
                            acc2[c / 2] = fma2(pack2(-n4.x, -n4.y), cx2, acc2[c / 2]);
                            acc2[c / 2 + 1] = fma2(pack2(-n4.z, -n4.w), cx2, acc2[c / 2 + 1]);
                        }
                    }
                }
                if (prebias) tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&tempty[sl]);                  // the slot may take its next block
                    if (j == 3) mbar_arrive(&empty[s]);        // the chunk's dx / scales are consumed
                }
            };
            if (!(ok = wait_slot(gb))) break;
            tc_fence_after();
            tmem_ld32(t_lane + (gb % NSLOT) * BN, IA);
            for (int i = 0; ok && i < nblk; i += 2) {   // nblk is a multiple of 4
                step(IA, IB, i);
                if (ok) step(IB, IA, i + 1);
            }
            gb += nblk;
            gc += nkc;
            if (!ok) break;
            // ---- epilogue: bias -> act -> residual (mg-opencl.cpp:481-493), then the optional
            // fused consumers (attention prep tiles, next layer's quantizer).  The raw sums go
            // through a per-warp shared-memory tile so that global stores are row-contiguous:
            // lane l then owns row 4k + l/8 and columns 4(l%8)..+3 of the warp's 32 x 32 block.
            {
                float acc[32];
#pragma unroll
                for (int c = 0; c < 16; c++) unpack2(acc2[c], acc[2 * c], acc[2 * c + 1]);
#pragma unroll
                for (int c4 = 0; c4 < 8; c4++)   // 16-byte chunks XOR-swizzled by row % 8
                    *reinterpret_cast<float4*>(stg + lane * 32 + ((c4 ^ (lane & 7)) * 4)) =
                        make_float4(acc[4 * c4], acc[4 * c4 + 1], acc[4 * c4 + 2], acc[4 * c4 + 3]);
            }
            __syncwarp();
            const int cl = (lane & 7) * 4, nb = n0 + c0, n = nb + cl;
            const bool full4 = (p.N % 4) == 0 && n + 3 < p.N;
            float4 b4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (p.bias) {
                if (full4) b4 = __ldg(reinterpret_cast<const float4*>(p.bias + n));
                else {
                    b4.x = n < p.N ? p.bias[n] : 0.f; b4.y = n + 1 < p.N ? p.bias[n + 1] : 0.f;
                    b4.z = n + 2 < p.N ? p.bias[n + 2] : 0.f; b4.w = n + 3 < p.N ? p.bias[n + 3] : 0.f;
                }
            }
            const bool no_abort = !*abort_flag;
#pragma unroll 2
            for (int k = 0; k < 8; k++) {
                const int r = 4 * k + (lane >> 3), m = mt * 128 + q * 32 + r;
                const float4 a4 = *reinterpret_cast<const float4*>(stg + r * 32 + (((lane & 7) ^ (r & 7)) * 4));
                float v[4] = {a4.x, a4.y, a4.z, a4.w};
                const bool row_ok = m < p.M && no_abort;
                if (p.bias) { v[0] = __fadd_rn(v[0], b4.x); v[1] = __fadd_rn(v[1], b4.y); v[2] = __fadd_rn(v[2], b4.z); v[3] = __fadd_rn(v[3], b4.w); }
#pragma unroll
                for (int e = 0; e < 4; e++) v[e] = act_apply(v[e], p.act);
                if (row_ok) {
                    if (full4) {
                        if (p.resid) {
                            const float4 r4 = *reinterpret_cast<const float4*>(p.resid + (size_t)m * p.N + n);
                            v[0] = __fadd_rn(v[0], r4.x); v[1] = __fadd_rn(v[1], r4.y);
                            v[2] = __fadd_rn(v[2], r4.z); v[3] = __fadd_rn(v[3], r4.w);
                        }
                        if (p.y) *reinterpret_cast<float4*>(p.y + (size_t)m * p.N + n) = make_float4(v[0], v[1], v[2], v[3]);
                    } else {
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            if (n + e >= p.N) { v[e] = 0.0f; continue; }
                            if (p.resid) v[e] = __fadd_rn(v[e], p.resid[(size_t)m * p.N + n + e]);
                            if (p.y) p.y[(size_t)m * p.N + n + e] = v[e];
                        }
                    }
                    if (p.ap) prep_store<4>(p.ap, p.ap_S, p.ap_H, p.ap_nt, m, n, v);
                }
                if (p.qo) {
                    // the warp's 32 columns are one 32-block of the next layer's input, held by the
                    // 8 lanes of a row: k_quantize_q8 (mg-opencl.cpp:424-434) as launch_quant_act_tiled
                    float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
                    // (the same maximum as a sequential scan: max is exact and order-free)
                    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
                    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
                    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
                    const float d = __fdiv_rn(amax, 127.0f);
                    const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
                    uint32_t packed = 0;
                    int sum = 0;
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const int qi = (int)roundf(__fmul_rn(v[e], id));
                        sum += qi;
                        packed |= (uint32_t)(qi & 0xFF) << (8 * e);
                    }
                    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
                    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
                    sum += __shfl_xor_sync(0xffffffffu, sum, 4);
                    if (row_ok) {
                        ActQ qa;
                        qa.q = p.qo;
                        qa.Mpad = p.qo_Mpad;
                        const int kc = nb >> 7, j = (nb >> 5) & 3;
                        *reinterpret_cast<uint32_t*>(qa.q + act_code(qa, kc, m, (nb & 127) + cl)) = packed;
                        if ((lane & 7) == 0) {
                            act_dx(qa, kc, m)[j] = d;
                            if (p.qo_c) act_cx(qa, kc, m)[j] = __fmul_rn(d, (float)sum);
                        }
                    }
                }
            }
            __syncwarp();   // the staging tile is reused by the next tile
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

template <int BN, bool Q4K>
static int wide_attr() {
    return cudaFuncSetAttribute(qgemm_wide_kernel<BN, Q4K>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                WideCfg<BN, Q4K>::SMEM) == cudaSuccess ? 0 : -1;
}

int wide_prepare() {
    return wide_attr<32, false>() | wide_attr<32, true>() | wide_attr<64, false>() | wide_attr<64, true>();
}

template <int BN, bool Q4K>
static int run_wide(QGemmArgs p, cudaStream_t st) {
    using C = WideCfg<BN, Q4K>;
    ++g_launch_count;
    p.tiles_n = (p.N + BN - 1) / BN;
    p.tiles_m = (p.M + 127) / 128;
    const int tiles = p.tiles_n * p.tiles_m;
    const int grid = std::min(tiles, sm_count());
    launch_k(qgemm_wide_kernel<BN, Q4K>, dim3(grid, 1, 1), C::THREADS, C::SMEM, st, p);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

int launch_qgemm_wide(const QGemmArgs& p, bool q4k, int bn, cudaStream_t st) {
    if (p.K % 128 != 0 || p.nsplit > 1 || p.M <= 0) return -2;
    if (p.qo && p.N % 128 != 0) return -2;
    if (bn == 32) return q4k ? run_wide<32, true>(p, st) : run_wide<32, false>(p, st);
    if (bn == 64) return q4k ? run_wide<64, true>(p, st) : run_wide<64, false>(p, st);
    return -2;
}

// Tile width for the wide kernel, or 0 to keep the narrow kernel.  MGC_QGEMM_WIDE=0 turns the
// wide kernel off, =32|64|128 forces that width wherever it applies.  Default: the wide kernel
// once the narrow tile grid would need more than one wave; its width minimises an estimate of
// waves x per-tile time (per 32-block: ~70 SM cycles of MMA issue for a 32-wide tile, ~128 /
// ~250 cycles of promotion for 64 / 128-wide tiles; ~1500 cycles of fill + epilogue per tile).
int pick_wide(int M, int N, int K, bool fused_quant, bool prep) {
    const char* fe = std::getenv("MGC_QGEMM_WIDE");   // read per call (tests switch it)
    const int force = fe ? std::atoi(fe) : -1;
    if (K % 128 != 0 || force == 0) return 0;
    if (fused_quant && N % 128 != 0) return 0;
    if (prep && N % 32 != 0) return 0;
    const int npad = (N + 127) / 128 * 128;
    if (force == 32 || force == 64) return force;
    if (force < 0) return 0;   // (default off until it outruns the narrow kernel at large M)
    const long sms = sm_count();
    const long mt = (M + 127) / 128;
    if (mt * ((N + 63) / 64) <= sms) return 0;   // one narrow wave: the narrow kernel's latency wins
    long best = -1;
    int bn = 0;
    for (int c : {64, 32}) {
        const long tn = (N + c - 1) / c;
        if (tn * c > npad) continue;
        const long tiles = tn * mt, waves = (tiles + sms - 1) / sms;
        const long per_block = c == 64 ? 200 : 150;
        const long cost = waves * ((long)(K / 32) * per_block + 1500);
        if (best < 0 || cost < best) { best = cost; bn = c; }
    }
    return bn;
}

}  // namespace mgc
