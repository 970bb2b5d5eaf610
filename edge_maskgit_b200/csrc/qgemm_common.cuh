// qgemm_common.cuh -- what the two int8-dot GEMM kernels (qgemm.cu: narrow tiles for small M;
// qgemm_wide.cu: wide persistent tiles for large M) share: the argument block, the activation
// functions of the epilogue and the exact int32 -> f32 conversion constant.
#pragma once
#include "kernels.h"
#include "ptx.cuh"

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
    // fused attention prep (optional): also store y as the f16 Q/K/V tiles of attnprep.cuh
    uint8_t* ap; int ap_S, ap_H, ap_nt;
    // persistent mode (tiles_n > 0): a 1-D grid of CTAs walks the tiles t = blockIdx.x, +gridDim.x,
    // ... (tile t = n-tile t % tiles_n of m-tile t / tiles_n); the pipeline runs on across tiles
    int tiles_n, tiles_m;
    // wide kernel: 1 = MMAs accumulate onto TMEM pre-filled with the 1.5*2^23 bias pattern,
    // 0 = plain int32 dots and an integer add per dot in the promotion
    int wide_prebias;
};

// (-1.5 * 2^23, -1.5 * 2^23): |v| < 2^22 always holds (32 * 127 * 128 < 2^22)
constexpr uint64_t kMagicNeg2 = 0xCB400000CB400000ull;

__device__ __forceinline__ float act_apply(float v, int a) {
    if (a == 1) return 0.5f * v * (1.0f + erff(v * 0.70710678f));
    if (a == 2) return __fdiv_rn(v, 1.0f + expf(-v));
    return v;
}



// The wide kernel (qgemm_wide.cu).  Returns -2 when it does not take the shape / options
// (the caller then uses the narrow kernel), 0 on a successful launch, -1 on a launch error.
int launch_qgemm_wide(const QGemmArgs& p, bool q4k, int bn, cudaStream_t st);
// Tile width the wide kernel would use for this GEMM, or 0 if the narrow kernel is the better
// fit (fused split-K is never wide).
int pick_wide(int M, int N, int K, bool fused_quant, bool prep);
int wide_prepare();
int sm_count();

}  // namespace mgc
