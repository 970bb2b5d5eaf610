// attnprep.cuh -- the f16 tile layout the attention kernel streams (see attn.cu), and the
// store helpers shared by the standalone prep pass and the fused QKV-GEMM epilogue.
#pragma once
#include "ptx.cuh"
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
constexpr uint32_t PREP_ROW = Q_BYTES / BM + K_BYTES / BC + VT_BYTES / BC;   // 352 bytes per row
// attention kernel shared memory: Q | K x2 | V^T x2 | (P_hi, P_lo) x2 | row max / sum exchange x2 | barriers
constexpr uint32_t OFF_Q = 0, OFF_K = OFF_Q + Q_BYTES, OFF_V = OFF_K + 2 * K_BYTES, OFF_P = OFF_V + 2 * VT_BYTES,
                   P_SET = 2 * P_BYTES, OFF_X = OFF_P + 2 * P_SET, X_SET = 8 * BM * 4, OFF_BAR = OFF_X + 2 * X_SET;
constexpr uint32_t SMEM = 1024 + OFF_BAR + 256;
// TMEM: S x2 (128 columns each) at 0 / 128, O tile x2 (48 columns each) at 256 / 304
constexpr uint32_t TMEM_COLS = 512, TM_O = 256;
constexpr int THREADS = 544;   // 16 softmax warps + 1 MMA / copy warp
constexpr float LOG2E = 1.4426950408889634f;
}  // namespace fa

// store 8 halves (16 bytes) as logical chunk `c` of row `r` in a 128B-swizzled block
__device__ __forceinline__ void st_chunk(uint8_t* blk, int r, int c, const __half2 (&h)[4]) {
    *reinterpret_cast<uint4*>(blk + r * 128 + ((c ^ (r & 7)) << 4)) = *reinterpret_cast<const uint4*>(h);
}
__device__ __forceinline__ void st_half(uint8_t* blk, int r, int k, __half v) {
    *reinterpret_cast<__half*>(blk + sw128_off(r, k * 2)) = v;
}

// prep layout per (image b, head h), nt = ceil(S/128) tiles: [nt x Q tile][nt x K tile][nt x V^T tile]
__device__ __forceinline__ uint8_t* prep_base(uint8_t* prep, int b, int h, int H, int nt) {
    return prep + ((size_t)b * H + h) * nt * (size_t)(128 * fa::PREP_ROW);
}

// Store NC (4, 8 or 16) columns [n, n+NC) (n % NC == 0) of QKV row (image b, position s) as f16
// into the prep tiles: part 0/1/2 = q/k/v, head h, first dim d0.  NC columns never straddle a
// head (48 = 3 x 16 = 6 x 8) nor the q | k | v boundary (E = 48 H).
template <int NC>
__device__ __forceinline__ void prep_store_at(uint8_t* prep, int H, int nt, int b, int s, int h, int part, int d0,
                                              const float* v) {
    using namespace fa;
    const int t = s >> 7, r = s & 127;
    uint8_t* base = prep_base(prep, b, h, H, nt);
    if (part < 2) {
        uint8_t* blk = base + (part == 0 ? (size_t)t * Q_BYTES : (size_t)nt * Q_BYTES + (size_t)t * K_BYTES);
        if constexpr (NC == 4) {   // 4 halves: the upper or lower half of one 16-byte chunk
            const __half2 h0 = __floats2half2_rn(v[0], v[1]), h1 = __floats2half2_rn(v[2], v[3]);
            uint2 u;
            u.x = *reinterpret_cast<const uint32_t*>(&h0);
            u.y = *reinterpret_cast<const uint32_t*>(&h1);
            *reinterpret_cast<uint2*>(blk + sw128_off(r, d0 * 2)) = u;
            return;
        }
#pragma unroll
        for (int c = 0; c < NC / 8; c++) {
            __half2 hh[4];
#pragma unroll
            for (int u = 0; u < 4; u++) hh[u] = __floats2half2_rn(v[8 * c + 2 * u], v[8 * c + 2 * u + 1]);
            st_chunk(blk, r, d0 / 8 + c, hh);
        }
    } else {
        uint8_t* blk = base + (size_t)nt * (Q_BYTES + K_BYTES) + (size_t)t * VT_BYTES + (r >> 6) * VT_BLK;
#pragma unroll
        for (int i = 0; i < NC; i++) st_half(blk, d0 + i, r & 63, __float2half_rn(v[i]));
    }
}
// the same for QKV row m = b * S + s and column n
template <int NC>
__device__ __forceinline__ void prep_store(uint8_t* prep, int S, int H, int nt, int m, int n, const float* v) {
    const int E = H * fa::D, part = n / E, rem = n - part * E, h = rem / fa::D, d0 = rem - h * fa::D;
    const int b = m / S, s = m - b * S;
    prep_store_at<NC>(prep, H, nt, b, s, h, part, d0, v);
}

}  // namespace mgc
