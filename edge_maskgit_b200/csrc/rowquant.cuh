// rowquant.cuh -- the per-32-block activation quantizer (k_quantize_q8, mg-opencl.cpp:424-434)
// applied to a row held by one warp in "chunk" layout: lane l holds, for chunk i, the 8
// contiguous elements 256 i + 8 l .. +7, so a 32-block is 4 adjacent lanes.  Shared by the
// LayerNorm / embedding / quantizer rows kernels and the attention combine.
#pragma once
#include "kernels.h"

namespace mgc {

template <int NC>
__device__ __forceinline__ void quant_chunks(const float (&v)[NC][8], int m, const ActQ& a, bool want_c, int lane) {
#pragma unroll
    for (int i = 0; i < NC; i++) {
        float amax = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; e++) amax = fmaxf(amax, fabsf(v[i][e]));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        uint32_t lo = 0, hi = 0;
        int sum = 0;
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const int q = (int)roundf(__fmul_rn(v[i][e], id));
            sum += q;
            const uint32_t byte = (uint32_t)(q & 0xFF);
            if (e < 4) lo |= byte << (8 * e); else hi |= byte << (8 * (e - 4));
        }
        const int b = 8 * i + (lane >> 2), kc = b >> 2, j = b & 3;
        const uint32_t kb = (uint32_t)(j * 32 + (lane & 3) * 8);
        *reinterpret_cast<uint2*>(a.q + act_code(a, kc, m, kb)) = make_uint2(lo, hi);
        if (want_c) {
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        }
        if ((lane & 3) == 0) {
            act_dx(a, kc, m)[j] = d;
            if (want_c) act_cx(a, kc, m)[j] = __fmul_rn(d, (float)sum);
        }
    }
}

}  // namespace mgc
