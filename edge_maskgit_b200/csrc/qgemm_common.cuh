// qgemm_common.cuh -- pieces of the int8-dot GEMM (qgemm.cu): the argument block, the
// activation functions of the epilogue, the exact int32 -> f32 conversion constant and the
// shared-memory unpack of packed Q4_K stages.
#pragma once
#include "kernels.h"
#include "ptx.cuh"
#include <cuda_fp16.h>

namespace mgc {

struct QGemmArgs {
    const int8_t* aq; int Mpad;      // activation tiles (kernels.h ActQ)
    const int8_t* wq; const float* ws; int Npad;   // weight codes / scale tiles
    int M, N, K;
    const float* bias; const float* resid; float* y; int act;
    // split-K: CTA z of gridDim.z handles K chunks [z*cps, (z+1)*cps); partials go to
    // part [nsplit][M][N], the last CTA of a tile (counters[tile] reaches nsplit) reduces them
    float* part; int* counters; int nsplit, cps;
    // fused output quantizer (optional): quantize y per 32-block into ActQ tiles qo (the next
    // layer's activation); y may then be null.  Needs CW == 16 and BN % 32 == 0.
    int8_t* qo; int qo_Mpad; int qo_c;
    int qo_n0;     // global column of output column 0 inside qo (column-split layers)
    int resid_ld;  // row stride of resid
    // fused attention prep (optional): also store y as the f16 Q/K/V tiles of attnprep.cuh
    uint8_t* ap; int ap_S, ap_H, ap_nt;
    // persistent mode (tiles_n > 0): a 1-D grid of CTAs walks the tiles t = blockIdx.x, +gridDim.x,
    // ... (tile t = n-tile t % tiles_n of m-tile t / tiles_n); the pipeline runs on across tiles
    int tiles_n, tiles_m;
};

// (-1.5 * 2^23, -1.5 * 2^23): |v| < 2^22 always holds (32 * 127 * 128 < 2^22)
constexpr uint64_t kMagicNeg2 = 0xCB400000CB400000ull;

__device__ __forceinline__ float act_apply(float v, int a) {
    if (a == 1) return 0.5f * v * (1.0f + erff(v * 0.70710678f));
    if (a == 2) return __fdiv_rn(v, 1.0f + expf(-v));
    return v;
}



// SMs of the current device.
int sm_count();

}  // namespace mgc

namespace mgc {

// Q4_K stage unpack (run by the 32 lanes of the MMA warp once the stage's
// bulk copies have landed): the raw packed tile -- BN rows x 64 nibble bytes, then BN rows x
// 16 scale bytes (kernels.h) -- becomes the u8 code tile the MMA reads (BN rows x 128 bytes,
// 16-byte chunks XOR-swizzled by row % 8) and the f32 scale tile [BN/4][2][4 blocks][4 cols].
// Nibbles (convert_to_gguf.py:97-99, unpacked as mg-opencl.cpp:521-530): byte l of group g of
// the chunk holds k = 64g + l (low nibble) and k = 64g + 32 + l (high nibble).
template <int BN>
__device__ __forceinline__ void unpack_q4k_stage(const uint8_t* raw, uint8_t* btile, float* stile, int lane) {
#pragma unroll
    for (int idx = lane; idx < BN * 4; idx += 32) {   // (row, 16-byte packed segment)
        const int r = idx >> 2, sg = idx & 3;
        const uint4 v = *reinterpret_cast<const uint4*>(raw + r * 64 + sg * 16);
        const uint4 lo = make_uint4(v.x & 0x0F0F0F0Fu, v.y & 0x0F0F0F0Fu, v.z & 0x0F0F0F0Fu, v.w & 0x0F0F0F0Fu);
        const uint4 hi = make_uint4((v.x >> 4) & 0x0F0F0F0Fu, (v.y >> 4) & 0x0F0F0F0Fu, (v.z >> 4) & 0x0F0F0F0Fu,
                                    (v.w >> 4) & 0x0F0F0F0Fu);
        const int c_lo = 4 * (sg >> 1) + (sg & 1), c_hi = c_lo + 2;
        *reinterpret_cast<uint4*>(btile + r * 128 + ((c_lo ^ (r & 7)) << 4)) = lo;
        *reinterpret_cast<uint4*>(btile + r * 128 + ((c_hi ^ (r & 7)) << 4)) = hi;
    }
    const uint8_t* sraw = raw + BN * 64;
#pragma unroll
    for (int r = lane; r < BN; r += 32) {
        const uint4 v = *reinterpret_cast<const uint4*>(sraw + r * 16);
        const float d = __half2float(__ushort_as_half((unsigned short)(v.x & 0xFFFFu)));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(v.x >> 16)));
        float* sq = stile + (r >> 2) * 32 + (r & 3);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            sq[j * 4] = __fmul_rn(d, (float)((v.y >> (8 * j)) & 0xFFu));          // scl = d * sc_j
            sq[16 + j * 4] = __fmul_rn(dmin, (float)((v.z >> (8 * j)) & 0xFFu));   // mnl = dmin * m_j
        }
    }
    fence_async_smem();   // the code tile is read by the tensor core (async proxy)
}

}  // namespace mgc
