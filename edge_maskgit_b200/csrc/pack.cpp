// pack.cpp -- host-side ggml block formats: the Q8_0 / Q4_K packers of the reference's
// converter (tools/convert_to_gguf.py:68-124), the dequant formulas of its OpenCL path
// (mg-opencl.cpp:252-262, 386-387), and the lossless repack of GGUF blocks into the
// device streaming layout documented in kernels.h.
#include "pack.h"

#include <algorithm>
#include <cmath>
#include <cstring>

namespace mgc {

uint16_t f32_to_f16(float f) {   // IEEE binary16, round to nearest even
    uint32_t u; std::memcpy(&u, &f, 4);
    const uint32_t sign = (u >> 16) & 0x8000u, a = u & 0x7fffffffu;
    if (a >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (a > 0x7f800000u ? 0x200u : 0u));
    if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);
    if (a < 0x38800000u) {
        if (a < 0x33000000u) return (uint16_t)sign;
        const uint32_t e = a >> 23, mant = (a & 0x7fffffu) | 0x800000u, sh = 126 - e;
        uint32_t r = mant >> sh;
        const uint32_t rem = mant & ((1u << sh) - 1), half = 1u << (sh - 1);
        r += (rem > half || (rem == half && (r & 1u))) ? 1u : 0u;
        return (uint16_t)(sign | r);
    }
    uint32_t r = (a - 0x38000000u) >> 13;
    const uint32_t rem = a & 0x1fffu;
    r += (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) ? 1u : 0u;
    return (uint16_t)(sign | r);
}

float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    int e = (h >> 10) & 31;
    uint32_t mant = h & 1023u, u;
    if (e == 31) u = sign | 0x7f800000u | (mant << 13);
    else if (e != 0) u = sign | ((uint32_t)(e + 112) << 23) | (mant << 13);
    else if (mant == 0) u = sign;
    else {
        e = 113;
        while (!(mant & 1024u)) { mant <<= 1; --e; }
        u = sign | ((uint32_t)e << 23) | ((mant & 1023u) << 13);
    }
    float f; std::memcpy(&f, &u, 4);
    return f;
}

static inline float rdh(const uint8_t* p) { uint16_t h; std::memcpy(&h, p, 2); return f16_to_f32(h); }

void q4k_get_scale_min(const uint8_t* s12, int j, int* sc, int* mn) {
    if (j < 4) { *sc = s12[j] & 63; *mn = s12[j + 4] & 63; return; }
    *sc = (s12[j + 4] & 0x0F) | ((s12[j - 4] >> 6) << 4);
    *mn = (s12[j + 4] >> 4) | ((s12[j] >> 6) << 4);
}

// Q8_0: per 32-block d = amax/127 (f32), q = clip(rint(w/d), +-127), d stored as fp16.
void pack_q8_0(const float* w, int64_t N, int64_t K, uint8_t* out) {
    const int64_t blocks = N * (K / 32);
    for (int64_t blk = 0; blk < blocks; ++blk) {
        const float* v = w + blk * 32;
        uint8_t* o = out + blk * 34;
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) amax = std::max(amax, std::fabs(v[i]));
        const float d = amax / 127.0f;
        const float div = d > 0.0f ? d : 1.0f;
        const uint16_t hd = f32_to_f16(d);
        std::memcpy(o, &hd, 2);
        for (int i = 0; i < 32; ++i) {
            const float q = std::clamp(std::nearbyint(v[i] / div), -127.0f, 127.0f);
            o[2 + i] = (uint8_t)(int8_t)q;
        }
    }
}

// Q4_K: 256-weight super-blocks of 8 sub-blocks; per sub-block scale (max+min)/15 and
// min -min; super-block d = max scale / 63, dmin = max min / 63; 6-bit codes, nibbles.
void pack_q4_k(const float* w, int64_t N, int64_t K, uint8_t* out) {
    const int64_t sbs = N * (K / 256);
    for (int64_t sb = 0; sb < sbs; ++sb) {
        const float* v = w + sb * 256;
        float scale[8], mins[8];
        for (int j = 0; j < 8; ++j) {
            const float* s = v + 32 * j;
            float lo = s[0], hi = s[0];
            for (int i = 1; i < 32; ++i) { lo = std::min(lo, s[i]); hi = std::max(hi, s[i]); }
            mins[j] = std::max(0.0f, -lo);
            const float span = hi + mins[j];
            scale[j] = span > 0.0f ? span / 15.0f : 0.0f;
        }
        const float smax = *std::max_element(scale, scale + 8), mmax = *std::max_element(mins, mins + 8);
        const float d = smax > 0.0f ? smax / 63.0f : 0.0f;
        const float dmin = mmax > 0.0f ? mmax / 63.0f : 0.0f;
        uint8_t* o = out + sb * 144;
        const uint16_t hd = f32_to_f16(d), hm = f32_to_f16(dmin);
        std::memcpy(o, &hd, 2);
        std::memcpy(o + 2, &hm, 2);
        uint8_t sc6[8], mn6[8];
        for (int j = 0; j < 8; ++j) {
            sc6[j] = (uint8_t)std::clamp(std::nearbyint(d > 0.0f ? scale[j] / d : 0.0f), 0.0f, 63.0f);
            mn6[j] = (uint8_t)std::clamp(std::nearbyint(dmin > 0.0f ? mins[j] / dmin : 0.0f), 0.0f, 63.0f);
        }
        uint8_t* s12 = o + 4;
        for (int j = 0; j < 4; ++j) {
            s12[j] = (uint8_t)((sc6[j] & 63) | (((sc6[j + 4] >> 4) & 3) << 6));
            s12[j + 4] = (uint8_t)((mn6[j] & 63) | (((mn6[j + 4] >> 4) & 3) << 6));
            s12[j + 8] = (uint8_t)((sc6[j + 4] & 0xF) | ((mn6[j + 4] & 0xF) << 4));
        }
        uint8_t* qs = o + 16;
        for (int j = 0; j < 8; ++j) {
            const float rs = d * (float)sc6[j], rm = dmin * (float)mn6[j];
            const float div = rs > 0.0f ? rs : 1.0f;
            for (int i = 0; i < 32; ++i) {
                const uint8_t q = (uint8_t)std::clamp(std::nearbyint((v[32 * j + i] + rm) / div), 0.0f, 15.0f);
                uint8_t& byte = qs[(j >> 1) * 32 + i];
                byte = (j & 1) ? (uint8_t)((byte & 0x0F) | (q << 4)) : q;
            }
        }
    }
}

void dequant(int wtype, const uint8_t* w, int64_t N, int64_t K, float* out) {
    if (wtype == 8) {
        for (int64_t blk = 0; blk < N * (K / 32); ++blk) {
            const uint8_t* b = w + blk * 34;
            const float d = rdh(b);
            for (int i = 0; i < 32; ++i) out[blk * 32 + i] = d * (float)(int8_t)b[2 + i];
        }
        return;
    }
    for (int64_t sb = 0; sb < N * (K / 256); ++sb) {
        const uint8_t* b = w + sb * 144;
        const float d = rdh(b), dmin = rdh(b + 2);
        for (int j = 0; j < 8; ++j) {
            int sc, mn;
            q4k_get_scale_min(b + 4, j, &sc, &mn);
            for (int i = 0; i < 32; ++i) {
                const uint8_t byte = b[16 + (j >> 1) * 32 + i];
                const float q = (float)((j & 1) ? (byte >> 4) : (byte & 0xF));
                out[sb * 256 + 32 * j + i] = d * (float)sc * q - dmin * (float)mn;
            }
        }
    }
}

// GGUF blocks -> device streaming layout (see kernels.h).  Lossless.
//  Q8_0: int8 codes, 128-byte-swizzled K-major rows, and exact f32 scales (fp16 -> f32).
//  Q4_K: the packed nibbles stay packed -- each row's 64 bytes per 128-K chunk are the GGUF
//        bytes of that half super-block unchanged -- plus 16 bytes per row and chunk: d and
//        dmin (fp16 bits) and the four decoded 6-bit scales and mins of the chunk's
//        sub-blocks (q4k_get_scale_min, mg-opencl.cpp:544-550), so the kernel forms the exact
//        f32 products d*sc and dmin*m (11-bit x 6-bit significands).
void repack(int wtype, const uint8_t* w, int N, int K, int Npad, std::vector<int8_t>& q, std::vector<float>& sc) {
    const int nb = K / 32;
    if (wtype == 12) {
        const int nkc = K / 128;
        q.assign((size_t)nkc * Npad * kQ4Row, 0);
        sc.assign((size_t)nkc * Npad * kQ4Scl / sizeof(float), 0.0f);
        uint8_t* s8 = reinterpret_cast<uint8_t*>(sc.data());
        for (int n = 0; n < N; ++n)
            for (int kc = 0; kc < nkc; ++kc) {
                const uint8_t* blk = w + ((size_t)n * (K / 256) + kc / 2) * 144;
                const int h = kc & 1;   // which half (sub-blocks 4h .. 4h+3) of the super-block
                std::memcpy(q.data() + ((size_t)kc * Npad + n) * kQ4Row, blk + 16 + h * 64, 64);
                uint8_t* o = s8 + ((size_t)kc * Npad + n) * kQ4Scl;
                std::memcpy(o, blk, 4);   // d, dmin
                for (int j = 0; j < 4; ++j) {
                    int s6, m6;
                    q4k_get_scale_min(blk + 4, 4 * h + j, &s6, &m6);
                    o[4 + j] = (uint8_t)s6;
                    o[8 + j] = (uint8_t)m6;
                }
            }
        return;
    }
    q.assign((size_t)K * Npad, 0);
    sc.assign((size_t)nb * Npad, 0.0f);
    for (int n = 0; n < N; ++n)
        for (int b = 0; b < nb; ++b) {
            const int kc = b >> 2, j = b & 3;
            float* tile = sc.data() + ((size_t)kc * (Npad / 4) + n / 4) * 16;
            const uint8_t* blk = w + ((size_t)n * nb + b) * 34;
            tile[j * 4 + (n & 3)] = rdh(blk);
            int8_t* row = q.data() + ((size_t)kc * Npad + n) * 128;
            for (int i = 0; i < 32; ++i) {
                const int k = j * 32 + i;
                row[((((k >> 4) ^ (n & 7)) << 4) | (k & 15))] = (int8_t)blk[2 + i];
            }
        }
}

}  // namespace mgc
