// vqgan.cu -- the MaskGIT VQGAN decoder on the GPU: the graph of src/mg-vqgan.cpp:67-108
// (codebook lookup, conv_in, ResBlocks with the shortcut conv applied to the processed tensor,
// nearest 2x upsampling + conv, GroupNorm(32) + affine + SiLU, conv_out) run as a fixed program of
// kernels over one or more token grids, captured once per image count as a CUDA graph.
//
// Layout.  Activations are NHWC, [image][y][x][channel]: a pixel's channels are one contiguous
// run, so the codebook lookup is a row copy, a 3x3 conv is an implicit GEMM whose K dimension
// (tap, channel) reads contiguous channel runs of shifted pixels, and the last conv (3 output
// channels) writes the HWC image of the VqganFwd callback (include/mg-generate.hpp:17)
// directly.  Every conv writes f32; every conv READS a pair of bf16 tensors (hi, lo) with
// hi = bf16(v), lo = bf16(v - hi), so hi + lo carries v to ~2^-17 relative.  GroupNorm writes
// that pair directly; a split kernel makes it (with the nearest 2x upsample folded in) for the
// up-convs and the shortcut conv.
//
// Convs.  The tensor-core conv (conv_tc_kernel) computes out = sum over (tap, channel) of
// x * w as three bf16 MMAs per K step -- hi*hi + hi*lo + lo*hi -- into an f32 TMEM accumulator
// (tcgen05.mma kind::f16, M = 128 pixels, N = 128 / 256 output channels); the dropped lo*lo
// term and the two roundings leave ~2^-16 relative per product, far inside the decoder gate.
// Its A operand (128 pixels x 64 channels of one tap) is one 4-D TMA load from the (hi or lo)
// activation tensor at the tap's shifted pixel origin: the zero padding of the conv is the
// TMA's out-of-bounds fill.  B (weights) is pre-tiled on load so a (k-block, n-tile) is one
// contiguous 128-byte-swizzled run moved by one bulk copy.  Shapes it does not tile (channel
// counts not multiples of 64 / 128, images narrower than 16 pixels) run on a SIMT f32
// implicit GEMM; MGC_VQGAN_SIMT=1 at create time forces that path for every conv.
//
// Numerics follow mg-cpu (src/mg-cpu/mg-cpu.cpp): GroupNorm statistics in double
// (:124-147, variance as E[x^2] - mean^2 over per-chunk double sums; where the tensor-core conv
// epilogue supplies them, each chunk is a warp's 32 pixels summed in f32 first), inv = 1/sqrt((float)var +
// eps) as there; the apply computes xn = (x - mean) * (gamma * inv) + beta in f32 with one fused
// multiply-add (mg-cpu: (float)(x - mean) * inv, then * gamma + beta, :265-276; a few ulp apart)
// and xn / (1 + exp(-xn)); convs accumulate in f32 in another order.
#include "../../include/mgc.h"
#include "gguf.h"
#include "kernels.h"
#include "ptx.cuh"
#include "qgemm_common.cuh"

#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

namespace mgc {
namespace {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ float2 bf2_to_f2(uint32_t v) {
    return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xFFFF0000u));
}
// 4 consecutive channels of (hi, lo) -> f32
__device__ __forceinline__ float4 load_pair4(const bf16* hi, const bf16* lo, size_t off) {
    const uint2 h = __ldg(reinterpret_cast<const uint2*>(hi + off));
    const uint2 l = __ldg(reinterpret_cast<const uint2*>(lo + off));
    const float2 h0 = bf2_to_f2(h.x), h1 = bf2_to_f2(h.y), l0 = bf2_to_f2(l.x), l1 = bf2_to_f2(l.y);
    return make_float4(h0.x + l0.x, h0.y + l0.y, h1.x + l1.x, h1.y + l1.y);
}
__device__ __forceinline__ void split_store4(bf16* hi, bf16* lo, size_t off, const float (&v)[4]) {
    __align__(8) bf16 h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        h[j] = __float2bfloat16_rn(v[j]);
        l[j] = __float2bfloat16_rn(v[j] - __bfloat162float(h[j]));
    }
    *reinterpret_cast<uint2*>(hi + off) = *reinterpret_cast<const uint2*>(h);
    *reinterpret_cast<uint2*>(lo + off) = *reinterpret_cast<const uint2*>(l);
}

// ------------------------------------------------------------------------------------------
// SIMT implicit-GEMM conv (f32 FMA).  Rows = output pixels (M = images * H * W), columns =
// output channels, K = taps * IC (IC a multiple of 8, OC of 4).  CTA tile 128 x 128 x 8, 256
// threads, 8 x 8 outputs a thread, register-prefetched double buffer.
struct ConvArgs {
    const bf16* xh;       // [N][H][W][IC] hi
    const bf16* xl;       //               lo
    const float* w;       // [T][IC][OC] f32
    const float* bias;    // [OC] or null
    const float* resid;   // [M][OC] or null (added after the conv)
    float* y;             // [M][OC]
    float* part;          // [nsplit][M][OC] when nsplit > 1
    int H, W, IC, OC, ks, M;
    int kper;             // K iterations (8 channels of one tap) per split
    int kiters;
};

constexpr int CBM = 128, CBN = 128, CBK = 8, CPAD = 4;

__global__ void __launch_bounds__(256, 2) conv_simt_kernel(ConvArgs a) {
    griddep_wait();   // inputs come from the preceding kernel (no-op without PDL)
    __shared__ __align__(16) float As[2][CBK][CBM + CPAD];
    __shared__ __align__(16) float Bs[2][CBK][CBN];
    const int tid = threadIdx.x;
    const int m0 = blockIdx.x * CBM, n0 = blockIdx.y * CBN;
    const int it0 = blockIdx.z * a.kper, it1 = min(a.kiters, it0 + a.kper);
    const int icg = a.IC / CBK;
    const int pr = tid >> 1, cq = (tid & 1) * 4;   // this thread's A row (pixel) and channel quad
    const int m = m0 + pr;
    const int HW = a.H * a.W;
    const int img = m / HW, rem = m - img * HW, py = rem / a.W, px = rem - py * a.W;
    const size_t xbase = (size_t)img * HW * a.IC + cq;
    const int br = tid >> 5, bc = (tid & 31) * 4;
    const int half = a.ks >> 1;

    auto load_a = [&](int it) -> float4 {
        const int tap = it / icg, c0 = (it - tap * icg) * CBK;
        const int yy = py + tap / a.ks - half, xx = px + tap % a.ks - half;
        if (m >= a.M || yy < 0 || yy >= a.H || xx < 0 || xx >= a.W) return make_float4(0.f, 0.f, 0.f, 0.f);
        return load_pair4(a.xh, a.xl, xbase + ((size_t)yy * a.W + xx) * a.IC + c0);
    };
    auto load_b = [&](int it) -> float4 {
        const int tap = it / icg, c0 = (it - tap * icg) * CBK;
        if (n0 + bc >= a.OC) return make_float4(0.f, 0.f, 0.f, 0.f);
        return __ldg(reinterpret_cast<const float4*>(a.w + ((size_t)tap * a.IC + c0 + br) * a.OC + n0 + bc));
    };
    auto store = [&](int buf, float4 av, float4 bv) {
        As[buf][cq + 0][pr] = av.x; As[buf][cq + 1][pr] = av.y;
        As[buf][cq + 2][pr] = av.z; As[buf][cq + 3][pr] = av.w;
        *reinterpret_cast<float4*>(&Bs[buf][br][bc]) = bv;
    };

    const int ty = tid >> 4, tx = tid & 15;
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0.f;

    if (it0 < it1) {
        store(0, load_a(it0), load_b(it0));
        __syncthreads();
        int buf = 0;
        for (int it = it0; it < it1; it++) {
            float4 na = make_float4(0.f, 0.f, 0.f, 0.f), nb = na;
            const bool more = it + 1 < it1;
            if (more) { na = load_a(it + 1); nb = load_b(it + 1); }
#pragma unroll
            for (int k = 0; k < CBK; k++) {
                const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][k][ty * 4]);
                const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][k][64 + ty * 4]);
                const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][k][tx * 4]);
                const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][k][64 + tx * 4]);
                const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                for (int i = 0; i < 8; i++)
#pragma unroll
                    for (int j = 0; j < 8; j++) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
            }
            if (more) {
                store(buf ^ 1, na, nb);
                __syncthreads();
                buf ^= 1;
            }
        }
    }
    const bool split = gridDim.z > 1;
    float* dst = split ? a.part + (size_t)blockIdx.z * a.M * a.OC : a.y;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int row = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
        if (row >= a.M) continue;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int col = n0 + h * 64 + tx * 4;
            if (col >= a.OC) continue;
            float4 v = make_float4(acc[i][h * 4], acc[i][h * 4 + 1], acc[i][h * 4 + 2], acc[i][h * 4 + 3]);
            if (!split) {
                if (a.bias) {
                    const float4 b = *reinterpret_cast<const float4*>(a.bias + col);
                    v.x += b.x; v.y += b.y; v.z += b.z; v.w += b.w;
                }
                if (a.resid) {
                    const float4 r = *reinterpret_cast<const float4*>(a.resid + (size_t)row * a.OC + col);
                    v.x += r.x; v.y += r.y; v.z += r.z; v.w += r.w;
                }
            }
            *reinterpret_cast<float4*>(dst + (size_t)row * a.OC + col) = v;
        }
    }
}

// Sum of the split-K partials in split order, then + bias, + residual.
__global__ void conv_splitk_reduce_kernel(const float* __restrict__ part, int nsplit, size_t n4, int OC,
                                          const float* __restrict__ bias, const float* __restrict__ resid,
                                          float* __restrict__ y) {
    griddep_wait();   // inputs come from the preceding kernel (no-op without PDL)
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n4) return;
    const float4* p = reinterpret_cast<const float4*>(part);
    float4 v = p[i];
    for (int s = 1; s < nsplit; s++) {
        const float4 q = p[(size_t)s * n4 + i];
        v.x += q.x; v.y += q.y; v.z += q.z; v.w += q.w;
    }
    if (bias) {
        const float4 b = *reinterpret_cast<const float4*>(bias + (i * 4) % OC);
        v.x += b.x; v.y += b.y; v.z += b.z; v.w += b.w;
    }
    if (resid) {
        const float4 r = reinterpret_cast<const float4*>(resid)[i];
        v.x += r.x; v.y += r.y; v.z += r.z; v.w += r.w;
    }
    reinterpret_cast<float4*>(y)[i] = v;
}

// Conv with few output channels (conv_out: 3x3, OC <= 4).  A block computes a 32 x 32 pixel
// tile of one image, 256 threads, 4 vertically adjacent pixels a thread.  Input channels go in
// chunks of 8: the (34 x 34)-pixel haloed tile of the chunk is staged in shared memory as f32
// (hi + lo, zeros outside the image, 9-float pixel stride: conflict-free), then each thread
// runs the chunk's 9 taps x 8 channels on its 4 pixels with the weights ([tap][IC][4], read as
// one broadcast float4) from shared memory.
constexpr int kSmallOC = 4;
constexpr int kCoTile = 32, kCoHalo = kCoTile + 2, kCoCh = 8, kCoPix = kCoHalo * kCoHalo, kCoStride = kCoCh + 1;
__global__ void __launch_bounds__(256) conv_small_oc_kernel(const bf16* __restrict__ xh, const bf16* __restrict__ xl,
                                                            const float* __restrict__ w,
                                                            const float* __restrict__ bias, float* __restrict__ y,
                                                            int H, int W, int IC, int OC) {
    griddep_wait();   // inputs come from the preceding kernel (no-op without PDL)
    extern __shared__ float sm[];
    float* ws = sm;                           // [9][IC][4]
    float* xs = sm + 9 * IC * kSmallOC;       // [kCoPix][kCoStride]
    for (int i = threadIdx.x; i < 9 * IC * kSmallOC; i += blockDim.x) {
        const int o = i % kSmallOC, r = i / kSmallOC;
        ws[i] = o < OC ? w[(size_t)r * OC + o] : 0.f;
    }
    const int img = blockIdx.z, x0 = blockIdx.x * kCoTile, y0 = blockIdx.y * kCoTile;
    const int tx = threadIdx.x & 31, ty = (threadIdx.x >> 5) * 4;   // pixels (x0+tx, y0+ty .. +3)
    float acc[4][kSmallOC];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int o = 0; o < kSmallOC; o++) acc[i][o] = 0.f;
    const size_t img_base = (size_t)img * H * W;
    for (int c0 = 0; c0 < IC; c0 += kCoCh) {
        __syncthreads();   // the previous chunk's reads are done (and, first time, the weights are in)
        for (int p = threadIdx.x; p < kCoPix; p += blockDim.x) {
            const int gy = y0 + p / kCoHalo - 1, gx = x0 + p % kCoHalo - 1;
            float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            if (gy >= 0 && gy < H && gx >= 0 && gx < W) {
                const size_t off = (img_base + (size_t)gy * W + gx) * IC + c0;
                const uint4 h = __ldg(reinterpret_cast<const uint4*>(xh + off));
                const uint4 l = __ldg(reinterpret_cast<const uint4*>(xl + off));
                const uint32_t hw[4] = {h.x, h.y, h.z, h.w}, lw[4] = {l.x, l.y, l.z, l.w};
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const float2 hf = bf2_to_f2(hw[q]), lf = bf2_to_f2(lw[q]);
                    v[2 * q] = hf.x + lf.x;
                    v[2 * q + 1] = hf.y + lf.y;
                }
            }
#pragma unroll
            for (int c = 0; c < kCoCh; c++) xs[p * kCoStride + c] = v[c];
        }
        __syncthreads();
#pragma unroll
        for (int kx = 0; kx < 3; kx++)
#pragma unroll 2
            for (int c = 0; c < kCoCh; c++) {
                float col[6];
#pragma unroll
                for (int r = 0; r < 6; r++) col[r] = xs[((ty + r) * kCoHalo + tx + kx) * kCoStride + c];
#pragma unroll
                for (int ky = 0; ky < 3; ky++) {
                    const float4 wv = *reinterpret_cast<const float4*>(ws + ((size_t)(ky * 3 + kx) * IC + c0 + c) * 4);
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const float xv = col[i + ky];
                        acc[i][0] = fmaf(xv, wv.x, acc[i][0]); acc[i][1] = fmaf(xv, wv.y, acc[i][1]);
                        acc[i][2] = fmaf(xv, wv.z, acc[i][2]); acc[i][3] = fmaf(xv, wv.w, acc[i][3]);
                    }
                }
            }
    }
    const int gx = x0 + tx;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int gy = y0 + ty + i;
        if (gx >= W || gy >= H) continue;
        float* o = y + (img_base + (size_t)gy * W + gx) * OC;
        for (int k = 0; k < OC; k++) o[k] = acc[i][k] + (bias ? bias[k] : 0.f);
    }
}

// ------------------------------------------------------------------------------------------
// Tensor-core conv.  Persistent CTAs (one per SM, 192 KB of stages), warp roles:
//   warp 0 lane 0  producer: per k-block (one tap, 64 input channels) two 4-D TMA loads (A hi,
//                  A lo: 128 pixels x 128 B, 128-byte swizzle) and two bulk copies (B hi, B lo)
//   warp 1 lane 0  MMA issuer: 4 K steps x 3 MMAs per k-block into a TMEM accumulator
//   warps 2..5     epilogue: TMEM -> registers -> (+ bias, + residual) -> f32 out (or the
//                  split-K partials); TMEM accumulators are double-buffered so a tile's
//                  epilogue overlaps the next tile's MMAs.
// Work unit = (m-tile, n-tile, K split), m-tile fastest so concurrent CTAs share weight tiles
// in L2.  An m-tile is a BH x BW pixel rectangle of one image (BW = min(W, 128)); TMEM lane r
// of the accumulator is pixel (y0 + r / BW, x0 + r % BW), the row order of the TMA box.
constexpr int TC_BM = 128, TC_BK = 64;
constexpr int TC_A_BYTES = TC_BM * 128;

template <int BN>
struct TcCfg {
    static constexpr int B_BYTES = BN * 128;
    static constexpr int STAGE = 2 * TC_A_BYTES + 2 * B_BYTES;
    static constexpr int NST = BN == 256 ? 2 : 3;
    static constexpr int BAR_BYTES = 256;
    static constexpr int SMEM = 1024 + NST * STAGE + BAR_BYTES;
    static constexpr int TMEM_COLS = 2 * BN;
    static_assert(SMEM <= 232448, "shared memory");
    static_assert(TMEM_COLS <= 512, "tmem");
    static_assert((2 * NST + 4) * 8 + 8 <= BAR_BYTES, "barrier area");
};

struct TcArgs {
    const uint8_t* wh;    // pre-tiled B hi: [OC/BN][kblocks][BN rows x 128 B swizzled]
    const uint8_t* wl;    // lo
    const float* bias;
    const float* resid;
    float* y;
    float* part;
    double* stats;        // GroupNorm partials of the output or null: [img][tiles_per_img * 4][OC][2]
    int H, W, IC, OC, ks, M;
    int BW, BH, tiles_x, tiles_per_img;
    int m_tiles, n_tiles, kblocks, kper, nsplit, n_units;
};

// Column sums of a warp's 32 x 32 register block: lane l holds row l's 32 values in a[]; after
// 31 shuffles lane l holds the sum over the 32 rows of column l in a[0] (fixed order).
__device__ __forceinline__ void warp_colsum32(float (&a)[32], int lane) {
#pragma unroll
    for (int w = 16; w >= 1; w >>= 1) {
        const bool up = lane & w;
#pragma unroll
        for (int j = 0; j < w; j++) {
            const float send = up ? a[j] : a[j + w];
            const float keep = up ? a[j + w] : a[j];
            a[j] = keep + __shfl_xor_sync(0xffffffffu, send, w);
        }
    }
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
          "r"(smem_u32(bar)) : "memory");
}

template <int BN>
__global__ void __launch_bounds__(192, 1) conv_tc_kernel(const __grid_constant__ CUtensorMap map_hi,
                                                          const __grid_constant__ CUtensorMap map_lo, TcArgs p) {
    using C = TcCfg<BN>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = align1024_smem(smem_raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::NST * C::STAGE);
    uint64_t* empty = full + C::NST;
    uint64_t* afull = empty + C::NST;    // [2]
    uint64_t* aempty = afull + 2;        // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(aempty + 2);
    volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::NST; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int a = 0; a < 2; a++) { mbar_init(&afull[a], 1); mbar_init(&aempty[a], 128); }
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
    griddep_wait();   // activations / residual come from the preceding kernel (no-op without PDL)
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int icb = p.IC / TC_BK, half = p.ks >> 1;

    auto unit_of = [&](int u, int& mt, int& nt, int& ks) {
        mt = u % p.m_tiles;
        const int r = u / p.m_tiles;
        nt = r % p.n_tiles;
        ks = r / p.n_tiles;
    };

    if (warp == 0) {
        if (lane == 0) {
            int gc = 0;
            int last_it[C::NST];
            for (int s = 0; s < C::NST; s++) last_it[s] = -1;
            bool go = true;
            for (int u = blockIdx.x; go && u < p.n_units; u += gridDim.x) {
                int mt, nt, ks;
                unit_of(u, mt, nt, ks);
                const int img = mt / p.tiles_per_img, r = mt % p.tiles_per_img;
                const int y0 = (r / p.tiles_x) * p.BH, x0 = (r % p.tiles_x) * p.BW;
                const int kb0 = ks * p.kper, kb1 = min(p.kblocks, kb0 + p.kper);
                for (int kb = kb0; kb < kb1; kb++, gc++) {
                    const int s = gc % C::NST, it = gc / C::NST;
                    if (!(go = mbar_wait(&empty[s], (it & 1) ^ 1, abort_flag, 21))) break;
                    uint8_t* st = smem + s * C::STAGE;
                    const int tap = kb / icb, c0 = (kb - tap * icb) * TC_BK;
                    const int dy = tap / p.ks - half, dx = tap % p.ks - half;
                    mbar_arrive_expect_tx(&full[s], C::STAGE);
                    // x (innermost) = channel c0, a multiple of 64: 128-byte aligned
                    tma_load_4d(st, &map_hi, c0, x0 + dx, y0 + dy, img, &full[s]);
                    tma_load_4d(st + TC_A_BYTES, &map_lo, c0, x0 + dx, y0 + dy, img, &full[s]);
                    const size_t boff = ((size_t)nt * p.kblocks + kb) * C::B_BYTES;
                    bulk_g2s(st + 2 * TC_A_BYTES, p.wh + boff, C::B_BYTES, &full[s]);
                    bulk_g2s(st + 2 * TC_A_BYTES + C::B_BYTES, p.wl + boff, C::B_BYTES, &full[s]);
                    last_it[s] = it;
                }
            }
            if (*abort_flag) {   // let copies already in flight land before the CTA exits
                volatile int never = 0;
                for (int s = 0; s < C::NST; s++)
                    if (last_it[s] >= 0) mbar_wait(&full[s], last_it[s] & 1, &never, 29);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_make(1, 1, 1, TC_BM, BN);
            int gc = 0, i = 0;
            bool go = true;
            for (int u = blockIdx.x; go && u < p.n_units; u += gridDim.x, i++) {
                int mt, nt, ks;
                unit_of(u, mt, nt, ks);
                const int kb0 = ks * p.kper, kb1 = min(p.kblocks, kb0 + p.kper);
                const int a = i & 1;
                if (!(go = mbar_wait(&aempty[a], ((i >> 1) & 1) ^ 1, abort_flag, 22))) break;
                tc_fence_after();
                const uint32_t d = tmem + a * BN;
                for (int kb = kb0; kb < kb1; kb++, gc++) {
                    const int s = gc % C::NST, it = gc / C::NST;
                    if (!(go = mbar_wait(&full[s], it & 1, abort_flag, 23))) break;
                    tc_fence_after();
                    const uint32_t ah = smem_u32(smem + s * C::STAGE), al = ah + TC_A_BYTES;
                    const uint32_t bh = ah + 2 * TC_A_BYTES, bl = bh + C::B_BYTES;
#pragma unroll
                    for (int k = 0; k < TC_BK / 16; k++) {
                        const uint32_t acc = (kb == kb0 && k == 0) ? 0u : 1u;
                        mma_f16(d, sdesc_sw128(ah + 32 * k), sdesc_sw128(bh + 32 * k), idesc, acc);
                        mma_f16(d, sdesc_sw128(ah + 32 * k), sdesc_sw128(bl + 32 * k), idesc, 1);
                        mma_f16(d, sdesc_sw128(al + 32 * k), sdesc_sw128(bh + 32 * k), idesc, 1);
                    }
                    mma_commit(&empty[s]);   // the stage may be refilled once these MMAs are done
                }
                if (go) mma_commit(&afull[a]);   // the accumulator is complete
            }
        }
    } else {
        // epilogue: warp w reads TMEM lanes 32*(w%4) .. +31 (one pixel a thread)
        const int q = warp & 3, row = q * 32 + lane;
        int i = 0;
        for (int u = blockIdx.x; u < p.n_units; u += gridDim.x, i++) {
            int mt, nt, ks;
            unit_of(u, mt, nt, ks);
            const int a = i & 1;
            if (!mbar_wait(&afull[a], (i >> 1) & 1, abort_flag, 24)) break;
            tc_fence_after();
            const int img = mt / p.tiles_per_img, r = mt % p.tiles_per_img;
            const int y = (r / p.tiles_x) * p.BH + row / p.BW, x = (r % p.tiles_x) * p.BW + row % p.BW;
            const size_t m = ((size_t)img * p.H + y) * p.W + x;
            const bool split = p.nsplit > 1;
            float* dst = split ? p.part + (size_t)ks * p.M * p.OC : p.y;
            const uint32_t t_row = tmem + a * BN + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
            for (int c = 0; c < BN / 32; c++) {
                uint32_t v[32];
                tmem_ld32(t_row + c * 32, v);
                tmem_ld_wait();
                const int col = nt * BN + c * 32;
                float* o = dst + m * p.OC + col;
                float sa[32], sq[32];
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    float4 f = make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]),
                                           __uint_as_float(v[j + 2]), __uint_as_float(v[j + 3]));
                    if (!split) {
                        if (p.bias) {
                            const float4 b = __ldg(reinterpret_cast<const float4*>(p.bias + col + j));
                            f.x += b.x; f.y += b.y; f.z += b.z; f.w += b.w;
                        }
                        if (p.resid) {
                            const float4 rr = __ldg(reinterpret_cast<const float4*>(p.resid + m * p.OC + col + j));
                            f.x += rr.x; f.y += rr.y; f.z += rr.z; f.w += rr.w;
                        }
                    }
                    *reinterpret_cast<float4*>(o + j) = f;
                    sa[j] = f.x; sa[j + 1] = f.y; sa[j + 2] = f.z; sa[j + 3] = f.w;
                }
                if (p.stats) {   // this warp's 32 pixels: per-channel sum and sum of squares
#pragma unroll
                    for (int j = 0; j < 32; j++) sq[j] = sa[j] * sa[j];
                    warp_colsum32(sa, lane);
                    warp_colsum32(sq, lane);
                    double* st = p.stats + ((((size_t)img * p.tiles_per_img + r) * 4 + q) * p.OC + col + lane) * 2;
                    st[0] = (double)sa[0];
                    st[1] = (double)sq[0];
                }
            }
            tc_fence_before();
            mbar_arrive(&aempty[a]);   // the MMA warp may reuse this accumulator
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// ------------------------------------------------------------------------------------------
// GroupNorm + affine + SiLU over NHWC.  Pass 1: per (image, pixel chunk) per-channel double
// sums of x and x^2 (fixed-order reductions, so the result is deterministic).  Pass 2: per
// (image, group) mean and 1/sqrt(var + eps).  Pass 3: the elementwise apply, writing the
// (hi, lo) pair the next conv reads.
constexpr int kGnThreads = 256;

__global__ void __launch_bounds__(kGnThreads) gn_partial_kernel(const float* __restrict__ x, int HW, int C,
                                                                int pix_per_chunk, double* __restrict__ part) {
    griddep_wait();   // inputs come from the preceding kernel (no-op without PDL)
    __shared__ double red[kGnThreads * 8];
    const int chunk = blockIdx.x, img = blockIdx.y, nch = gridDim.x;
    const int C4 = C / 4, rows = kGnThreads / C4;   // C4 divides kGnThreads (host checks)
    const int q = threadIdx.x % C4, r = threadIdx.x / C4;
    const int p0 = chunk * pix_per_chunk, p1 = min(HW, p0 + pix_per_chunk);
    double s[4] = {0, 0, 0, 0}, ss[4] = {0, 0, 0, 0};
    const float4* xb = reinterpret_cast<const float4*>(x + (size_t)img * HW * C) + q;
    for (int p = p0 + r; p < p1; p += rows) {
        const float4 v = __ldg(xb + (size_t)p * C4);
        const double d[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; j++) { s[j] += d[j]; ss[j] += d[j] * d[j]; }
    }
#pragma unroll
    for (int j = 0; j < 4; j++) { red[threadIdx.x * 8 + j] = s[j]; red[threadIdx.x * 8 + 4 + j] = ss[j]; }
    __syncthreads();
    for (int c = threadIdx.x; c < C; c += kGnThreads) {
        const int cq4 = c / 4, j = c % 4;
        double ts = 0, tss = 0;
        for (int rr = 0; rr < rows; rr++) {
            const int t = rr * C4 + cq4;
            ts += red[t * 8 + j];
            tss += red[t * 8 + 4 + j];
        }
        double* o = part + (((size_t)img * nch + chunk) * C + c) * 2;
        o[0] = ts; o[1] = tss;
    }
}

// Pass 2: one block per (group, image); the chunk x channel partials are summed by a fixed
// strided split and a fixed tree (deterministic).  Writes, per (image, channel), the group's
// mean (rounded to f32) and a = gamma * inv, inv = 1 / sqrt(var + eps) as mg-cpu rounds it.
constexpr int kGnFinThreads = 128;
__global__ void __launch_bounds__(kGnFinThreads) gn_finalize_kernel(const double* __restrict__ part, int nch, int C,
                                                                    int G, int HW, float eps,
                                                                    const float* __restrict__ gamma,
                                                                    float* __restrict__ mean_c, float* __restrict__ a_c) {
    griddep_wait();   // inputs come from the preceding kernel (no-op without PDL)
    __shared__ double rs[kGnFinThreads], rss[kGnFinThreads];
    const int g = blockIdx.x, img = blockIdx.y, cpg = C / G, n_items = nch * cpg;
    double s = 0, ss = 0;
    for (int i = threadIdx.x; i < n_items; i += kGnFinThreads) {
        const int k = i / cpg, c = g * cpg + i % cpg;
        const double* p = part + (((size_t)img * nch + k) * C + c) * 2;
        s += p[0]; ss += p[1];
    }
    rs[threadIdx.x] = s; rss[threadIdx.x] = ss;
    __syncthreads();
    for (int w = kGnFinThreads / 2; w > 0; w >>= 1) {
        if (threadIdx.x < w) { rs[threadIdx.x] += rs[threadIdx.x + w]; rss[threadIdx.x] += rss[threadIdx.x + w]; }
        __syncthreads();
    }
    const double cnt = (double)HW * cpg;
    const double mean = rs[0] / cnt;
    const double var = fmax(rss[0] / cnt - mean * mean, 0.0);
    const float inv = 1.0f / sqrtf((float)var + eps);
    for (int j = threadIdx.x; j < cpg; j += kGnFinThreads) {
        const int c = g * cpg + j;
        mean_c[(size_t)img * C + c] = (float)mean;
        a_c[(size_t)img * C + c] = __fmul_rn(inv, gamma[c]);
    }
}

// Pass 3: y = silu((x - mean) * a + beta), 8 channels a thread, written as the (hi, lo) pair.
__global__ void gn_apply_silu_kernel(const float* __restrict__ x, const float* __restrict__ mean_c,
                                     const float* __restrict__ a_c, const float* __restrict__ beta, int HW, int C,
                                     size_t n8, bf16* __restrict__ yh, bf16* __restrict__ yl) {
    griddep_wait();   // inputs come from the preceding kernel (no-op without PDL)
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n8) return;
    const size_t e = i * 8;
    const int c0 = (int)(e % C);
    const size_t img = e / ((size_t)HW * C);
    const float4* xp = reinterpret_cast<const float4*>(x + e);
    const float4 v0 = __ldg(xp), v1 = __ldg(xp + 1);
    const float xv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    const float* mc = mean_c + img * C + c0;
    const float* ac = a_c + img * C + c0;
    __align__(16) bf16 h[8], l[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const float xn = fmaf(xv[j] - mc[j], ac[j], beta[c0 + j]);
        const float o = xn / (1.0f + expf(-xn));
        h[j] = __float2bfloat16_rn(o);
        l[j] = __float2bfloat16_rn(o - __bfloat162float(h[j]));
    }
    *reinterpret_cast<uint4*>(yh + e) = *reinterpret_cast<const uint4*>(h);
    *reinterpret_cast<uint4*>(yl + e) = *reinterpret_cast<const uint4*>(l);
}

// f32 NHWC -> (hi, lo) pair, optionally nearest-upsampled 2x (mg-cpu.cpp:190-196): output
// pixel (y, x) reads input (y / 2, x / 2).  H, W: the input's size.
__global__ void split_kernel(const float* __restrict__ x, int H, int W, int C, int up, size_t n4,
                             bf16* __restrict__ yh, bf16* __restrict__ yl) {
    griddep_wait();   // inputs come from the preceding kernel (no-op without PDL)
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n4) return;
    const int C4 = C / 4;
    const int c = (int)(i % C4) * 4;
    const size_t pix = i / C4;   // output pixel
    size_t src = pix;
    if (up) {
        const int Wo = W * 2, Ho = H * 2;
        const size_t img = pix / ((size_t)Ho * Wo);
        const int r = (int)(pix - img * Ho * Wo), yo = r / Wo, xo = r - yo * Wo;
        src = (img * H + (yo >> 1)) * W + (xo >> 1);
    }
    const float4 v = __ldg(reinterpret_cast<const float4*>(x + src * C + c));
    const float o[4] = {v.x, v.y, v.z, v.w};
    split_store4(yh, yl, i * 4, o);
}

// Codebook lookup (get_rows, mg-vqgan.cpp:79-81): pixel p of image n is token grid[n][p]
// (p = y * L + x), its channels the codebook row, written as the (hi, lo) pair.  Ids outside
// [0, codebook) decode as zeros.
__global__ void vq_gather_kernel(const int32_t* __restrict__ grid, const float* __restrict__ cb, int n_codes, int E,
                                 size_t n4, bf16* __restrict__ yh, bf16* __restrict__ yl) {
    griddep_wait();   // inputs come from the preceding kernel (no-op without PDL)
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n4) return;
    const int E4 = E / 4;
    const size_t pix = i / E4;
    const int c4 = (int)(i % E4);
    const int id = grid[pix];
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (id >= 0 && id < n_codes) v = __ldg(reinterpret_cast<const float4*>(cb + (size_t)id * E) + c4);
    const float o[4] = {v.x, v.y, v.z, v.w};
    split_store4(yh, yl, i * 4, o);
}

// The bytes of mg::Image (mg-generate.cpp:141-144): v = min(max(x, 0), 1) * 255 + 0.5, truncated.
__global__ void rgb8_kernel(const float* __restrict__ img, size_t n, uint8_t* __restrict__ out) {
    griddep_wait();   // inputs come from the preceding kernel (no-op without PDL)
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float v = __fadd_rn(__fmul_rn(fminf(fmaxf(img[i], 0.f), 1.f), 255.f), 0.5f);
    out[i] = (uint8_t)__float2uint_rz(v);
}

// ------------------------------------------------------------------------------------------
// Host side.
void ck(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

template <class T>
T* dalloc(size_t n) {
    void* p = nullptr;
    ck(cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)), "cudaMalloc");
    return (T*)p;
}

// f32 -> bf16 bits, round to nearest even (finite inputs)
uint16_t bf16_bits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
float bf16_float(uint16_t b) {
    const uint32_t u = (uint32_t)b << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    });
    if (!fn) throw std::runtime_error("vqgan: cuTensorMapEncodeTiled is not available");
    return fn;
}

// 4-D map over an NHWC bf16 tensor [N][H][W][C]: box = 64 channels x BW x BH x 1, 128-byte
// swizzle, zero fill outside the tensor (the conv's padding).
CUtensorMap make_act_map(const bf16* base, int N, int H, int W, int C, int BW, int BH) {
    CUtensorMap m;
    const cuuint64_t dims[4] = {(cuuint64_t)C, (cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)N};
    const cuuint64_t strides[3] = {(cuuint64_t)C * 2, (cuuint64_t)W * C * 2, (cuuint64_t)H * W * C * 2};
    const cuuint32_t box[4] = {(cuuint32_t)TC_BK, (cuuint32_t)BW, (cuuint32_t)BH, 1};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<bf16*>(base), dims, strides,
                                   box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("vqgan: cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    return m;
}

struct Conv {
    int ic = 0, oc = 0, ks = 0;
    float* w = nullptr;       // [T][IC][OC] f32 (SIMT and small-OC convs)
    float* b = nullptr;
    int bn = 0;               // tensor-core n-tile (128 / 256); 0 = channels not tensor-core shaped
    uint8_t* wh = nullptr;    // pre-tiled bf16 hi / lo (tensor-core convs)
    uint8_t* wl = nullptr;
};
struct Norm { int c = 0; float* g = nullptr; float* b = nullptr; };

// One step of the decoder program.  F32 buffers: 0 = x (the running tensor), 2 = u, 3 = h;
// every conv reads the (hi, lo) pair.
struct Step {
    enum Kind { Gather, GnSilu, Split, ConvOp, ConvOut, SwapXH } kind;
    int src = 0, dst = 0, resid = -1;   // f32 buffer ids (resid -1 = none)
    int conv = -1, norm = -1;
    int H = 0, W = 0, C = 0;            // output spatial size; channels of the step's input
    bool up = false;
    // bound by reserve():
    const float* p_src = nullptr;
    float* p_dst = nullptr;
    const float* p_res = nullptr;
    bool tc = false;
    bool feeds_gn = false;   // the next step (past swaps) is a GroupNorm of this conv's output
    CUtensorMap mh{}, ml{};
};

}  // namespace
}  // namespace mgc

using namespace mgc;

struct mgc_vqgan {
    int device = 0, max_images = 0;
    int n_tokens = 0, L = 0, R = 0, E = 0, n_codes = 0, groups = 32;
    bool simt_only = false;
    cudaStream_t st = nullptr;
    float* codebook = nullptr;
    std::vector<Conv> convs;
    std::vector<Norm> norms;
    std::vector<Step> prog;
    size_t buf_floats = 0;       // per image
    float* buf[4] = {nullptr, nullptr, nullptr, nullptr};
    bf16* ph = nullptr;          // the conv-input pair
    bf16* pl = nullptr;
    float* part = nullptr;       // split-K partials
    int gn_chunks = 0;
    double* gn_part = nullptr;
    float* gn_mean = nullptr;    // [n][C] per-channel group mean
    float* gn_a = nullptr;       // [n][C] gamma * inv
    int32_t* d_grid = nullptr;
    float* d_img = nullptr;
    uint8_t* d_rgb = nullptr;
    std::map<int, cudaGraphExec_t> graphs;   // per image count
    int launches = 0;                         // kernels one decode launches

    ~mgc_vqgan() {
        for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
        for (auto& c : convs) { cudaFree(c.w); cudaFree(c.b); cudaFree(c.wh); cudaFree(c.wl); }
        for (auto& n : norms) { cudaFree(n.g); cudaFree(n.b); }
        for (float* b : buf) cudaFree(b);
        cudaFree(ph); cudaFree(pl);
        cudaFree(codebook); cudaFree(part); cudaFree(gn_part); cudaFree(gn_mean); cudaFree(gn_a); cudaFree(d_grid); cudaFree(d_img);
        cudaFree(d_rgb);
        if (st) cudaStreamDestroy(st);
    }

    // ---- split-K choices (deterministic functions of the shape and image count)
    int simt_split(int M, int OC, int kiters) const {
        const int tiles = ((M + CBM - 1) / CBM) * ((OC + CBN - 1) / CBN);
        const int target = 2 * sm_count();
        if (tiles >= target) return 1;
        return std::max(1, std::min((target + tiles - 1) / tiles, kiters / 4));
    }
    int tc_split(int tiles, int kblocks) const {
        const int target = sm_count();
        if (tiles >= target) return 1;
        return std::max(1, std::min((target + tiles - 1) / tiles, kblocks / 2));
    }
    static bool tc_shape_ok(const Conv& c, int H, int W) {
        if (!c.bn) return false;
        const int BW = std::min(W, 128);
        if (BW < 16 || (BW & (BW - 1)) || W % BW) return false;
        return H % (TC_BM / BW) == 0;
    }

    void load(const char* path) {
        simt_only = [] { const char* e = std::getenv("MGC_VQGAN_SIMT"); return e && e[0] == '1'; }();
        Gguf g;
        g.open(path);
        n_tokens = g.geti("maskgit.n_tokens", 256);
        L = 1;
        while (L * L < n_tokens) L++;
        if (L * L != n_tokens) throw std::runtime_error("vqgan: n_tokens is not a square grid");
        E = g.geti("maskgit.vqgan.embedding_dim", 0);
        const int filters = g.geti("maskgit.vqgan.filters", 0);
        const int nrb = g.geti("maskgit.vqgan.num_res_blocks", 0);
        groups = g.geti("maskgit.vqgan.group_norm_groups", 32);
        auto it = g.int_arrays.find("maskgit.vqgan.channel_multipliers");
        if (E <= 0 || filters <= 0 || nrb <= 0 || it == g.int_arrays.end() || it->second.empty())
            throw std::runtime_error("vqgan: the GGUF has no VQGAN decoder hyperparameters");
        if (E % 8) throw std::runtime_error("vqgan: embedding_dim must be a multiple of 8");
        const std::vector<int64_t> mult = it->second;
        const int nb = (int)mult.size();
        R = L << (nb - 1);
        const int res = g.geti("maskgit.resolution", R);
        if (res != R) throw std::runtime_error("vqgan: maskgit.resolution does not match the decoder");

        const GgufTensor& cbt = g.req("vqgan.quantizer.codebook.weight");
        if (cbt.type != 0 || cbt.ne[0] != E) throw std::runtime_error("vqgan: codebook must be F32 [codes][embedding_dim]");
        n_codes = (int)cbt.ne[1];
        codebook = dalloc<float>((size_t)n_codes * E);
        ck(cudaMemcpy(codebook, cbt.data, (size_t)n_codes * E * 4, cudaMemcpyHostToDevice), "upload codebook");

        auto add_conv = [&](const std::string& name, int ic, int oc, int ks, bool bias) {
            const GgufTensor& t = g.req(name + ".weight");
            if (t.type != 0 || t.ne[0] != ks || t.ne[1] != ks || t.ne[2] != ic || t.ne[3] != oc)
                throw std::runtime_error("vqgan: unexpected shape or type of " + name + ".weight");
            const float* src = (const float*)t.data;   // [OC][IC][KH][KW]
            const int T = ks * ks;
            Conv c;
            c.ic = ic; c.oc = oc; c.ks = ks;
            {   // [tap][IC][OC] f32
                std::vector<float> w((size_t)T * ic * oc);
                for (int o = 0; o < oc; o++)
                    for (int i = 0; i < ic; i++)
                        for (int k = 0; k < T; k++) w[((size_t)k * ic + i) * oc + o] = src[((size_t)o * ic + i) * T + k];
                c.w = dalloc<float>(w.size());
                ck(cudaMemcpy(c.w, w.data(), w.size() * 4, cudaMemcpyHostToDevice), "upload conv");
            }
            c.bn = (ic % TC_BK == 0) ? (oc % 256 == 0 ? 256 : oc % 128 == 0 ? 128 : 0) : 0;
            if (c.bn) {   // pre-tiled bf16 pair: [OC/BN][T * IC/64][BN rows x 64 bf16, 128-byte swizzle]
                const int kbl = T * ic / TC_BK, ntl = oc / c.bn;
                const size_t bytes = (size_t)ntl * kbl * c.bn * 128;
                std::vector<uint8_t> hi(bytes), lo(bytes);
                for (int nt = 0; nt < ntl; nt++)
                    for (int kb = 0; kb < kbl; kb++) {
                        const int tap = kb / (ic / TC_BK), c0 = (kb % (ic / TC_BK)) * TC_BK;
                        uint8_t* th = hi.data() + ((size_t)nt * kbl + kb) * c.bn * 128;
                        uint8_t* tl = lo.data() + ((size_t)nt * kbl + kb) * c.bn * 128;
                        for (int r = 0; r < c.bn; r++)
                            for (int j = 0; j < TC_BK; j++) {
                                const float v = src[((size_t)(nt * c.bn + r) * ic + c0 + j) * T + tap];
                                const uint16_t h = bf16_bits(v), l = bf16_bits(v - bf16_float(h));
                                const uint32_t off = sw128_off(r, j * 2);
                                std::memcpy(th + off, &h, 2);
                                std::memcpy(tl + off, &l, 2);
                            }
                    }
                c.wh = dalloc<uint8_t>(bytes);
                c.wl = dalloc<uint8_t>(bytes);
                ck(cudaMemcpy(c.wh, hi.data(), bytes, cudaMemcpyHostToDevice), "upload conv");
                ck(cudaMemcpy(c.wl, lo.data(), bytes, cudaMemcpyHostToDevice), "upload conv");
            }
            if (bias) {
                const GgufTensor& b = g.req(name + ".bias");
                if (b.type != 0 || b.ne[0] != oc) throw std::runtime_error("vqgan: bad " + name + ".bias");
                c.b = dalloc<float>(oc);
                ck(cudaMemcpy(c.b, b.data, (size_t)oc * 4, cudaMemcpyHostToDevice), "upload bias");
            }
            convs.push_back(c);
            return (int)convs.size() - 1;
        };
        auto add_norm = [&](const std::string& name, int c) {
            const GgufTensor& w = g.req(name + ".weight");
            const GgufTensor& b = g.req(name + ".bias");
            if (w.type != 0 || b.type != 0 || w.ne[0] != c || b.ne[0] != c)
                throw std::runtime_error("vqgan: bad GroupNorm " + name);
            if (c % groups || c % 8 || kGnThreads % (c / 4)) throw std::runtime_error("vqgan: unsupported channel count");
            Norm n;
            n.c = c;
            n.g = dalloc<float>(c);
            n.b = dalloc<float>(c);
            ck(cudaMemcpy(n.g, w.data, (size_t)c * 4, cudaMemcpyHostToDevice), "upload gn");
            ck(cudaMemcpy(n.b, b.data, (size_t)c * 4, cudaMemcpyHostToDevice), "upload gn");
            norms.push_back(n);
            return (int)norms.size() - 1;
        };
        auto step = [&](Step::Kind k, int src, int dst, int resid, int conv, int norm, int H, int W, int C, bool up) {
            Step s{};
            s.kind = k; s.src = src; s.dst = dst; s.resid = resid; s.conv = conv; s.norm = norm;
            s.H = H; s.W = W; s.C = C; s.up = up;
            prog.push_back(s);
        };

        // the program (mg-vqgan.cpp:67-108)
        int H = L, W = L, cur = (int)(filters * mult[nb - 1]);
        size_t maxf = (size_t)H * W * E;
        auto note = [&](int c) { maxf = std::max(maxf, (size_t)H * W * c); };
        step(Step::Gather, -1, -1, -1, -1, -1, H, W, E, false);
        step(Step::ConvOp, -1, 0, -1, add_conv("vqgan.decoder.conv_in", E, cur, 3, true), -1, H, W, E, false);
        note(cur);
        auto resblock = [&](const std::string& pfx, int cin, int cout) {
            step(Step::GnSilu, 0, -1, -1, -1, add_norm(pfx + "norm0", cin), H, W, cin, false);
            step(Step::ConvOp, -1, 2, -1, add_conv(pfx + "conv0", cin, cout, 3, false), -1, H, W, cin, false);
            step(Step::GnSilu, 2, -1, -1, -1, add_norm(pfx + "norm1", cout), H, W, cout, false);
            if (cin == cout) {
                step(Step::ConvOp, -1, 3, 0, add_conv(pfx + "conv1", cout, cout, 3, false), -1, H, W, cout, false);
            } else {   // the shortcut conv reads the processed h (mg-vqgan.cpp:57-60)
                step(Step::ConvOp, -1, 2, -1, add_conv(pfx + "conv1", cout, cout, 3, false), -1, H, W, cout, false);
                step(Step::Split, 2, -1, -1, -1, -1, H, W, cout, false);
                step(Step::ConvOp, -1, 3, 2, add_conv(pfx + "conv_res", cout, cout, 1, false), -1, H, W, cout, false);
            }
            note(cin); note(cout);
            step(Step::SwapXH, -1, -1, -1, -1, -1, H, W, cout, false);
        };
        for (int l = 0; l < nrb; l++) resblock("vqgan.decoder.res_blocks.0." + std::to_string(l) + ".", cur, cur);
        int prev = cur, bi = 1;
        for (int i = nb - 1; i >= 0; i--, bi++) {
            cur = (int)(filters * mult[i]);
            for (int l = 0; l < nrb; l++) {
                resblock("vqgan.decoder.res_blocks." + std::to_string(bi) + "." + std::to_string(l) + ".", prev, cur);
                prev = cur;
            }
            if (i > 0) {
                H *= 2; W *= 2;
                note(cur);
                const int c = add_conv("vqgan.decoder.res_blocks." + std::to_string(bi) + "." + std::to_string(nrb + 1),
                                       cur, cur, 3, true);
                step(Step::Split, 0, -1, -1, -1, -1, H, W, cur, true);
                step(Step::ConvOp, -1, 3, -1, c, -1, H, W, cur, false);
                step(Step::SwapXH, -1, -1, -1, -1, -1, H, W, cur, false);
            }
        }
        step(Step::GnSilu, 0, -1, -1, -1, add_norm("vqgan.decoder.norm_out", cur), H, W, cur, false);
        const GgufTensor& co = g.req("vqgan.decoder.conv_out.weight");
        if (co.ne[3] > kSmallOC || co.ne[0] != 3) throw std::runtime_error("vqgan: conv_out must be 3x3 with at most 4 outputs");
        step(Step::ConvOut, -1, -1, -1, add_conv("vqgan.decoder.conv_out", cur, (int)co.ne[3], 3, true), -1, H, W, cur,
             false);
        if (co_smem(cur) > 200 * 1024 || cur % kCoCh) throw std::runtime_error("vqgan: unsupported conv_out input channels");
        ck(cudaFuncSetAttribute(conv_small_oc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)co_smem(cur)),
           "conv_out smem");
        ck(cudaFuncSetAttribute(conv_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<128>::SMEM),
           "conv smem");
        ck(cudaFuncSetAttribute(conv_tc_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<256>::SMEM),
           "conv smem");
        for (size_t i = 0; i < prog.size(); i++) {
            if (prog[i].kind != Step::ConvOp) continue;
            size_t j = i + 1;
            while (j < prog.size() && prog[j].kind == Step::SwapXH) j++;
            prog[i].feeds_gn = j < prog.size() && prog[j].kind == Step::GnSilu;
        }
        for (const Conv& c : convs)
            if (c.oc > kSmallOC && (c.oc % 4 || c.ic % CBK))
                throw std::runtime_error("vqgan: conv channel counts must be multiples of 4 (out) and 8 (in)");
        buf_floats = maxf;
    }

    static size_t co_smem(int ic) { return ((size_t)9 * ic * kSmallOC + (size_t)kCoPix * kCoStride) * 4; }

    int chunks_for(int n, int HW) const {
        const int want = std::max(1, (2 * sm_count() + n - 1) / n);
        return std::max(1, std::min(want, HW / 64));
    }

    // Device buffers for n images; binds every step to its buffers and tensor maps.
    void reserve(int n) {
        for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
        graphs.clear();
        for (float*& b : buf) { cudaFree(b); b = nullptr; }
        for (int i : {0, 2, 3}) buf[i] = dalloc<float>(buf_floats * n);
        cudaFree(ph); ph = dalloc<bf16>(buf_floats * n);
        cudaFree(pl); pl = dalloc<bf16>(buf_floats * n);
        size_t pf = 0;
        gn_chunks = 0;
        size_t gn_need = 0;
        float* b[4] = {buf[0], buf[1], buf[2], buf[3]};
        for (Step& s : prog) {
            if (s.kind == Step::SwapXH) { std::swap(b[0], b[3]); continue; }
            s.p_src = s.src >= 0 ? b[s.src] : nullptr;
            s.p_dst = s.dst >= 0 ? b[s.dst] : nullptr;
            s.p_res = s.resid >= 0 ? b[s.resid] : nullptr;
            if (s.kind != Step::ConvOp) continue;
            const Conv& c = convs[s.conv];
            s.tc = !simt_only && tc_shape_ok(c, s.H, s.W);
            if (s.tc) {
                const int BW = std::min(s.W, 128), BH = TC_BM / BW;
                s.mh = make_act_map(ph, n, s.H, s.W, c.ic, BW, BH);
                s.ml = make_act_map(pl, n, s.H, s.W, c.ic, BW, BH);
            }
        }
        // split-K partials and GroupNorm partials: the largest over every image count <= n
        for (int k = 1; k <= n; k++)
            for (const Step& s : prog) {
                if (s.kind == Step::GnSilu) {
                    const int nch = chunks_for(k, s.H * s.W);
                    gn_chunks = std::max(gn_chunks, nch);
                    gn_need = std::max(gn_need, (size_t)k * nch * s.C * 2);
                }
                if (s.kind != Step::ConvOp) continue;
                const Conv& c = convs[s.conv];
                const int M = k * s.H * s.W;
                int kit, ns;
                if (s.tc) {
                    kit = c.ks * c.ks * c.ic / TC_BK;
                    ns = tc_split((M / TC_BM) * (c.oc / c.bn), kit);
                } else {
                    kit = c.ks * c.ks * c.ic / CBK;
                    ns = simt_split(M, c.oc, kit);
                }
                const int kper = (kit + ns - 1) / ns, nsu = (kit + kper - 1) / kper;
                if (nsu > 1) pf = std::max(pf, (size_t)nsu * M * c.oc);
                if (s.tc && nsu == 1 && s.feeds_gn)   // epilogue GroupNorm partials: 4 per 128-pixel tile
                    gn_need = std::max(gn_need, (size_t)M / TC_BM * 4 * c.oc * 2);
            }
        cudaFree(part); part = dalloc<float>(pf);
        cudaFree(gn_part); gn_part = dalloc<double>(gn_need);
        int maxc = 0;
        for (const Step& s : prog)
            if (s.kind == Step::GnSilu) maxc = std::max(maxc, s.C);
        cudaFree(gn_mean); gn_mean = dalloc<float>((size_t)n * maxc);
        cudaFree(gn_a); gn_a = dalloc<float>((size_t)n * maxc);
        cudaFree(d_grid); d_grid = dalloc<int32_t>((size_t)n * n_tokens);
        cudaFree(d_img); d_img = dalloc<float>((size_t)n * R * R * 3);
        cudaFree(d_rgb); d_rgb = dalloc<uint8_t>((size_t)n * R * R * 3);
        max_images = n;
    }

    // Enqueue the decoder on `s` for n <= max_images images: grid (device, [n][n_tokens]) ->
    // out (device, [n][R][R][3]).  Returns the number of kernels launched.
    enum OpBit { kGather = 1, kGn = 2, kSplit = 4, kConvTc = 8, kConvSimt = 16, kReduce = 32, kConvOut = 64,
                 kAll = 127 };
    int enqueue(const int32_t* grid, int n, float* out, cudaStream_t s, int mask = kAll) {
        int nl = 0;
        int fused_nch = 0;   // > 0: the preceding conv wrote the GroupNorm partials (that many chunks)
        for (const Step& stp : prog) {
            const int HW = stp.H * stp.W;
            if (stp.kind != Step::SwapXH && stp.kind != Step::GnSilu) fused_nch = 0;
            switch (stp.kind) {
            case Step::SwapXH:
                break;
            case Step::Gather: {
                if (!(mask & kGather)) break;
                const size_t n4 = (size_t)n * HW * E / 4;
                launch_k(vq_gather_kernel, (unsigned)((n4 + 255) / 256), 256, 0, s, grid, (const float*)codebook,
                         n_codes, E, n4, ph, pl);
                nl++;
                break;
            }
            case Step::Split: {
                if (!(mask & kSplit)) break;
                const size_t n4 = (size_t)n * HW * stp.C / 4;
                const int Hs = stp.up ? stp.H / 2 : stp.H, Ws = stp.up ? stp.W / 2 : stp.W;
                launch_k(split_kernel, (unsigned)((n4 + 255) / 256), 256, 0, s, stp.p_src, Hs, Ws, stp.C,
                         stp.up ? 1 : 0, n4, ph, pl);
                nl++;
                break;
            }
            case Step::GnSilu: {
                if (!(mask & kGn)) break;
                const Norm& nm = norms[stp.norm];
                int nch = fused_nch;
                fused_nch = 0;
                if (!nch) {
                    nch = chunks_for(n, HW);
                    const int ppc = (HW + nch - 1) / nch;
                    launch_k(gn_partial_kernel, dim3(nch, n), kGnThreads, 0, s, stp.p_src, HW, nm.c, ppc, gn_part);
                    nl++;
                }
                launch_k(gn_finalize_kernel, dim3(groups, n), kGnFinThreads, 0, s, (const double*)gn_part, nch, nm.c,
                         groups, HW, 1e-5f, (const float*)nm.g, gn_mean, gn_a);
                const size_t n8 = (size_t)n * HW * nm.c / 8;
                launch_k(gn_apply_silu_kernel, (unsigned)((n8 + 255) / 256), 256, 0, s, stp.p_src,
                         (const float*)gn_mean, (const float*)gn_a, (const float*)nm.b, HW, nm.c, n8, ph, pl);
                nl += 2;
                break;
            }
            case Step::ConvOp: {
                const Conv& c = convs[stp.conv];
                const int M = n * HW;
                int nsu = 1;
                const bool run_conv = mask & (stp.tc ? kConvTc : kConvSimt);
                if (!run_conv) {
                    // (only the split count is needed, for the reduce below)
                    const int kit = stp.tc ? c.ks * c.ks * c.ic / TC_BK : c.ks * c.ks * c.ic / CBK;
                    const int ns = stp.tc ? tc_split((M / TC_BM) * (c.oc / c.bn), kit) : simt_split(M, c.oc, kit);
                    const int kper = (kit + ns - 1) / ns;
                    nsu = (kit + kper - 1) / kper;
                    if (stp.tc && nsu == 1 && stp.feeds_gn && (mask & kGn)) {
                        const int BW = std::min(stp.W, 128);
                        fused_nch = (stp.W / BW) * (stp.H / (TC_BM / BW)) * 4;
                    }
                } else if (stp.tc) {
                    TcArgs a{};
                    a.wh = c.wh; a.wl = c.wl; a.bias = c.b; a.resid = stp.p_res; a.y = stp.p_dst; a.part = part;
                    a.H = stp.H; a.W = stp.W; a.IC = c.ic; a.OC = c.oc; a.ks = c.ks; a.M = M;
                    a.BW = std::min(stp.W, 128);
                    a.BH = TC_BM / a.BW;
                    a.tiles_x = stp.W / a.BW;
                    a.tiles_per_img = a.tiles_x * (stp.H / a.BH);
                    a.m_tiles = n * a.tiles_per_img;
                    a.n_tiles = c.oc / c.bn;
                    a.kblocks = c.ks * c.ks * c.ic / TC_BK;
                    const int ns = tc_split(a.m_tiles * a.n_tiles, a.kblocks);
                    a.kper = (a.kblocks + ns - 1) / ns;
                    nsu = (a.kblocks + a.kper - 1) / a.kper;
                    a.nsplit = nsu;
                    a.n_units = a.m_tiles * a.n_tiles * nsu;
                    if (nsu == 1 && stp.feeds_gn && (mask & kGn)) {   // the GroupNorm partials come from the epilogue
                        a.stats = gn_part;
                        fused_nch = a.tiles_per_img * 4;
                    }
                    const int grid_x = std::min(a.n_units, sm_count());
                    if (c.bn == 256)
                        launch_k(conv_tc_kernel<256>, grid_x, 192, TcCfg<256>::SMEM, s, stp.mh, stp.ml, a);
                    else
                        launch_k(conv_tc_kernel<128>, grid_x, 192, TcCfg<128>::SMEM, s, stp.mh, stp.ml, a);
                } else {
                    ConvArgs a{};
                    a.xh = ph; a.xl = pl; a.w = c.w; a.bias = c.b; a.resid = stp.p_res;
                    a.y = stp.p_dst; a.part = part;
                    a.H = stp.H; a.W = stp.W; a.IC = c.ic; a.OC = c.oc; a.ks = c.ks; a.M = M;
                    a.kiters = c.ks * c.ks * c.ic / CBK;
                    const int ns = simt_split(M, c.oc, a.kiters);
                    a.kper = (a.kiters + ns - 1) / ns;
                    nsu = (a.kiters + a.kper - 1) / a.kper;
                    dim3 gr((M + CBM - 1) / CBM, (c.oc + CBN - 1) / CBN, nsu);
                    launch_k(conv_simt_kernel, gr, 256, 0, s, a);
                }
                if (run_conv) nl++;
                if (nsu > 1 && (mask & kReduce)) {
                    const size_t n4 = (size_t)M * c.oc / 4;
                    launch_k(conv_splitk_reduce_kernel, (unsigned)((n4 + 255) / 256), 256, 0, s, (const float*)part, nsu,
                             n4, c.oc, (const float*)c.b, stp.p_res, stp.p_dst);
                    nl++;
                }
                break;
            }
            case Step::ConvOut: {
                if (!(mask & kConvOut)) break;
                const Conv& c = convs[stp.conv];
                dim3 gr((stp.W + kCoTile - 1) / kCoTile, (stp.H + kCoTile - 1) / kCoTile, n);
                launch_k(conv_small_oc_kernel, gr, 256, co_smem(c.ic), s, (const bf16*)ph, (const bf16*)pl,
                         (const float*)c.w, (const float*)c.b, out, stp.H, stp.W, c.ic, c.oc);
                nl++;
                break;
            }
            }
        }
        return nl;
    }

    // Mean milliseconds of one replay of a graph holding only the launches of `mask` for n images
    // (on the decoder's buffers, whatever they hold), replayed `iters` times between CUDA events.
    float time_mask(int mask, int n, int iters, int* nl) {
        cudaStream_t cap = nullptr;
        ck(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking), "stream");
        cudaGraph_t gph = nullptr;
        ck(cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal), "capture");
        *nl = enqueue(d_grid, n, d_img, cap, mask);
        const cudaError_t e = cudaStreamEndCapture(cap, &gph);
        cudaStreamDestroy(cap);
        ck(e, "end capture");
        cudaGraphExec_t ex = nullptr;
        const cudaError_t ei = cudaGraphInstantiate(&ex, gph, 0);
        cudaGraphDestroy(gph);
        ck(ei, "instantiate");
        cudaEvent_t e0, e1;
        ck(cudaEventCreate(&e0), "event");
        ck(cudaEventCreate(&e1), "event");
        ck(cudaGraphLaunch(ex, st), "graph launch");   // warm-up
        ck(cudaEventRecord(e0, st), "event");
        for (int i = 0; i < iters; i++) ck(cudaGraphLaunch(ex, st), "graph launch");
        ck(cudaEventRecord(e1, st), "event");
        ck(cudaEventSynchronize(e1), "sync");
        float ms = 0.f;
        ck(cudaEventElapsedTime(&ms, e0, e1), "elapsed");
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        cudaGraphExecDestroy(ex);
        return ms / iters;
    }

    // Decode d_grid -> d_img through a CUDA graph captured once per image count.
    void run(int n, cudaStream_t s) {
        auto it = graphs.find(n);
        if (it == graphs.end()) {
            cudaStream_t cap = nullptr;
            ck(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking), "stream");
            cudaGraph_t gph = nullptr;
            ck(cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal), "capture");
            launches = enqueue(d_grid, n, d_img, cap);
            const cudaError_t e = cudaStreamEndCapture(cap, &gph);
            cudaStreamDestroy(cap);
            ck(e, "end capture");
            cudaGraphExec_t ex = nullptr;
            const cudaError_t ei = cudaGraphInstantiate(&ex, gph, 0);
            cudaGraphDestroy(gph);
            ck(ei, "instantiate");
            it = graphs.emplace(n, ex).first;
        }
        ck(cudaGraphLaunch(it->second, s), "graph launch");
    }
};

namespace {
// After a synchronous decode: a bounded wait inside a conv that timed out left a code in the
// device error word (the kernel returned early); report it and clear the word.
void check_vq_dev_error() {
    int v = 0;
    ck(cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(int)), "device error word");
    if (v != 0) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(int));
        throw std::runtime_error("vqgan: a kernel gave up waiting (device error code " + std::to_string(v) + ")");
    }
}

template <class F>
int vq_guard(F&& f) {
    try { f(); return 0; }
    catch (const std::exception& e) { set_last_error(e.what()); return -1; }
}
}  // namespace

extern "C" {

int mgc_vqgan_create(const char* gguf_path, int max_images, int device, mgc_vqgan** out) {
    return vq_guard([&] {
        if (!gguf_path || !out) throw std::runtime_error("mgc_vqgan_create: null argument");
        if (max_images <= 0) throw std::runtime_error("mgc_vqgan_create: max_images must be positive");
        *out = nullptr;
        ck(cudaSetDevice(device), "cudaSetDevice");
        std::unique_ptr<mgc_vqgan> v(new mgc_vqgan);
        v->device = device;
        ck(cudaStreamCreateWithFlags(&v->st, cudaStreamNonBlocking), "stream");
        v->load(gguf_path);
        v->reserve(max_images);
        *out = v.release();
    });
}

int mgc_vqgan_info(const mgc_vqgan* v, int* n_tokens, int* resolution, int* codebook_size) {
    return vq_guard([&] {
        if (!v) throw std::runtime_error("mgc_vqgan_info: null handle");
        if (n_tokens) *n_tokens = v->n_tokens;
        if (resolution) *resolution = v->R;
        if (codebook_size) *codebook_size = v->n_codes;
    });
}

int mgc_vqgan_decode(mgc_vqgan* v, const int32_t* grid, int n_images, float* image_hwc) {
    return vq_guard([&] {
        if (!v || !grid || !image_hwc) throw std::runtime_error("mgc_vqgan_decode: null argument");
        if (n_images <= 0 || n_images > v->max_images)
            throw std::runtime_error("mgc_vqgan_decode: n_images must be in [1, max_images]");
        const size_t nt = (size_t)n_images * v->n_tokens;
        for (size_t i = 0; i < nt; i++)
            if (grid[i] < 0 || grid[i] >= v->n_codes) throw std::runtime_error("mgc_vqgan_decode: token id out of range");
        ck(cudaSetDevice(v->device), "cudaSetDevice");
        ck(cudaMemcpyAsync(v->d_grid, grid, nt * 4, cudaMemcpyHostToDevice, v->st), "copy grid");
        v->run(n_images, v->st);
        const size_t no = (size_t)n_images * v->R * v->R * 3;
        ck(cudaMemcpyAsync(image_hwc, v->d_img, no * 4, cudaMemcpyDeviceToHost, v->st), "copy image");
        ck(cudaStreamSynchronize(v->st), "decode");
        check_vq_dev_error();
    });
}

int mgc_vqgan_decode_rgb8(mgc_vqgan* v, const int32_t* grid, int n_images, uint8_t* rgb) {
    return vq_guard([&] {
        if (!v || !grid || !rgb) throw std::runtime_error("mgc_vqgan_decode_rgb8: null argument");
        if (n_images <= 0 || n_images > v->max_images)
            throw std::runtime_error("mgc_vqgan_decode_rgb8: n_images must be in [1, max_images]");
        const size_t nt = (size_t)n_images * v->n_tokens;
        for (size_t i = 0; i < nt; i++)
            if (grid[i] < 0 || grid[i] >= v->n_codes) throw std::runtime_error("mgc_vqgan_decode_rgb8: token id out of range");
        ck(cudaSetDevice(v->device), "cudaSetDevice");
        ck(cudaMemcpyAsync(v->d_grid, grid, nt * 4, cudaMemcpyHostToDevice, v->st), "copy grid");
        v->run(n_images, v->st);
        const size_t no = (size_t)n_images * v->R * v->R * 3;
        launch_k(rgb8_kernel, (unsigned)((no + 255) / 256), 256, 0, v->st, (const float*)v->d_img, no, v->d_rgb);
        ck(cudaMemcpyAsync(rgb, v->d_rgb, no, cudaMemcpyDeviceToHost, v->st), "copy image");
        ck(cudaStreamSynchronize(v->st), "decode");
        check_vq_dev_error();
    });
}

int mgc_generate_images(mgc_runtime* rt, mgc_vqgan* v, int B, const int32_t* class_ids, const uint64_t* seeds,
                        int steps, float temperature, uint8_t* rgb, int32_t* tokens_out) {
    if (!v || !rt || B <= 0 || !rgb) { set_last_error("mgc_generate_images: bad arguments"); return -1; }
    const int S = v->n_tokens + 1;
    std::vector<int32_t> tokens((size_t)B * S);
    if (mgc_generate(rt, B, class_ids, seeds, steps, temperature, tokens.data()) != 0) return -1;
    if (tokens_out) std::memcpy(tokens_out, tokens.data(), tokens.size() * sizeof(int32_t));
    // the final grids (class token dropped, mg-generate.cpp:131-140), decoded in batches
    std::vector<int32_t> grids((size_t)B * v->n_tokens);
    for (int i = 0; i < B; i++)
        std::memcpy(grids.data() + (size_t)i * v->n_tokens, tokens.data() + (size_t)i * S + 1,
                    sizeof(int32_t) * v->n_tokens);
    const size_t img_bytes = (size_t)v->R * v->R * 3;
    for (int i0 = 0; i0 < B; i0 += v->max_images) {
        const int n = std::min(v->max_images, B - i0);
        if (mgc_vqgan_decode_rgb8(v, grids.data() + (size_t)i0 * v->n_tokens, n, rgb + (size_t)i0 * img_bytes) != 0)
            return -1;
    }
    return 0;
}

int mgc_vqgan_decode_device(mgc_vqgan* v, const int32_t* grid_dev, int n_images, float* image_dev, void* stream) {
    return vq_guard([&] {
        if (!v || !grid_dev || !image_dev) throw std::runtime_error("mgc_vqgan_decode_device: null argument");
        if (n_images <= 0 || n_images > v->max_images)
            throw std::runtime_error("mgc_vqgan_decode_device: n_images must be in [1, max_images]");
        ck(cudaSetDevice(v->device), "cudaSetDevice");
        v->launches = v->enqueue(grid_dev, n_images, image_dev, (cudaStream_t)stream);
        ck(cudaPeekAtLastError(), "decode launch");
    });
}

int mgc_vqgan_time_op(mgc_vqgan* v, const char* op, int n_images, int iters, float* ms_per_replay, int* launches) {
    return vq_guard([&] {
        if (!v || !op || !ms_per_replay) throw std::runtime_error("mgc_vqgan_time_op: null argument");
        if (n_images <= 0 || n_images > v->max_images || iters <= 0)
            throw std::runtime_error("mgc_vqgan_time_op: n_images must be in [1, max_images], iters positive");
        static const std::map<std::string, int> ops = {
            {"gather", mgc_vqgan::kGather}, {"groupnorm", mgc_vqgan::kGn}, {"split", mgc_vqgan::kSplit},
            {"conv_tc", mgc_vqgan::kConvTc}, {"conv_simt", mgc_vqgan::kConvSimt},
            {"splitk_reduce", mgc_vqgan::kReduce}, {"conv_out", mgc_vqgan::kConvOut}, {"all", mgc_vqgan::kAll}};
        auto it = ops.find(op);
        if (it == ops.end()) throw std::runtime_error(std::string("mgc_vqgan_time_op: unknown op ") + op);
        ck(cudaSetDevice(v->device), "cudaSetDevice");
        int nl = 0;
        *ms_per_replay = v->time_mask(it->second, n_images, iters, &nl);
        if (launches) *launches = nl;
    });
}

int mgc_vqgan_launches(const mgc_vqgan* v) { return v ? v->launches : -1; }

void mgc_vqgan_destroy(mgc_vqgan* v) { delete v; }

}  // extern "C"
