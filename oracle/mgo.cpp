// mgo.cpp -- CPU restatement of edge_maskgit's quantized transformer hot path.
//
// TEST INFRASTRUCTURE ONLY: this is the checker the CUDA library is compared against.  It
// is never linked into, loaded by, or called from the shipped library.  Each function
// cites the reference (chenxugz/edge_maskgit) file:line it restates.  Build with
// -ffp-contract=off so that only the explicit fmaf() calls fuse.
#include "mgo.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <random>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace {

thread_local std::string g_err;

// ---------------------------------------------------------------- fp16 (IEEE binary16)
inline float h2f(uint16_t h) {
    uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31, m = h & 1023, u;
    if (e == 0) {
        if (m == 0) u = s;
        else {  // subnormal: normalise
            int sh = 0;
            while (!(m & 1024)) { m <<= 1; sh++; }
            m &= 1023;
            u = s | ((uint32_t)(127 - 15 + 1 - sh) << 23) | (m << 13);
        }
    } else if (e == 31) u = s | 0x7f800000u | (m << 13);
    else u = s | ((e + 112) << 23) | (m << 13);
    float f; std::memcpy(&f, &u, 4); return f;
}
inline uint16_t f2h(float f) {  // round to nearest even, like numpy astype(float16)
    uint32_t u; std::memcpy(&u, &f, 4);
    uint32_t s = (u >> 16) & 0x8000u;
    uint32_t a = u & 0x7fffffffu;
    if (a >= 0x7f800000u) return (uint16_t)(s | 0x7c00u | (a > 0x7f800000u ? 0x200u : 0));
    if (a >= 0x477ff000u) return (uint16_t)(s | 0x7c00u);           // overflow -> inf
    if (a < 0x38800000u) {                                         // subnormal / zero
        if (a < 0x33000000u) return (uint16_t)s;                    // < 2^-25 -> 0
        uint32_t e = a >> 23, m = (a & 0x7fffffu) | 0x800000u;
        uint32_t shift = 126 - e;                                   // 14..24
        uint32_t r = m >> shift, rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (r & 1))) r++;
        return (uint16_t)(s | r);
    }
    uint32_t r = ((a - 0x38000000u) >> 13);
    uint32_t rem = a & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1))) r++;
    return (uint16_t)(s | r);
}
inline float rd_f16(const uint8_t* p) { uint16_t h; std::memcpy(&h, p, 2); return h2f(h); }

// ggml get_scale_min_k4, as inlined in k_mul_mat_q4k_i8 (mg-opencl.cpp:544-550).
inline void q4k_scale_min(const uint8_t* sc, int j, int& dq, int& mq) {
    if (j < 4) { dq = sc[j] & 63; mq = sc[j + 4] & 63; }
    else {
        dq = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
        mq = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
}

inline float act_fn(float v, int a) {   // mg_act, mg-opencl.cpp:36-40
    if (a == 1) return 0.5f * v * (1.0f + std::erf(v * 0.70710678f));
    if (a == 2) return v / (1.0f + std::exp(-v));
    return v;
}

}  // namespace

extern "C" {

const char* mgo_last_error(void) { return g_err.c_str(); }
float mgo_f16_to_f32(uint16_t h) { return h2f(h); }
uint16_t mgo_f32_to_f16(float f) { return f2h(f); }

// tools/convert_to_gguf.py:109-124 (quant_q8_0).  numpy evaluates every step in float32
// (python scalars are "weak"): d = amax/127, q = clip(rint(w/d), -127, 127), d -> fp16.
void mgo_pack_q8_0(const float* w, int64_t N, int64_t K, uint8_t* out) {
    const int64_t nb = K / 32;
    for (int64_t n = 0; n < N; n++)
        for (int64_t b = 0; b < nb; b++) {
            const float* x = w + n * K + b * 32;
            uint8_t* o = out + (n * nb + b) * 34;
            float amax = 0.0f;
            for (int i = 0; i < 32; i++) amax = std::max(amax, std::fabs(x[i]));
            float d = amax / 127.0f;
            float ds = d > 0.0f ? d : 1.0f;
            uint16_t h = f2h(d);
            std::memcpy(o, &h, 2);
            for (int i = 0; i < 32; i++) {
                float q = std::nearbyint(x[i] / ds);
                q = std::min(127.0f, std::max(-127.0f, q));
                o[2 + i] = (uint8_t)(int8_t)q;
            }
        }
}

// tools/convert_to_gguf.py:68-106 (quant_q4_k): min/max sub-block quantisation, 6-bit
// scales/mins packed by the inverse of get_scale_min_k4, nibble groups g = sub-blocks
// (2g, 2g+1) in (low, high) nibbles.  All arithmetic float32, np.round = half to even.
void mgo_pack_q4_k(const float* w, int64_t N, int64_t K, uint8_t* out) {
    const int64_t nsb_row = K / 256, NSB = N * nsb_row;
    for (int64_t s = 0; s < NSB; s++) {
        const float* x = w + s * 256;   // rows are contiguous, so super-blocks are too
        float sc[8], minv[8];
        for (int j = 0; j < 8; j++) {
            float mn = x[j * 32], mx = x[j * 32];
            for (int i = 1; i < 32; i++) { mn = std::min(mn, x[j * 32 + i]); mx = std::max(mx, x[j * 32 + i]); }
            minv[j] = std::max(0.0f, -mn);
            float t = mx + minv[j];
            sc[j] = t > 0.0f ? t / 15.0f : 0.0f;
        }
        float scmax = sc[0], mnmax = minv[0];
        for (int j = 1; j < 8; j++) { scmax = std::max(scmax, sc[j]); mnmax = std::max(mnmax, minv[j]); }
        float d = scmax > 0.0f ? scmax / 63.0f : 0.0f;
        float dmn = mnmax > 0.0f ? mnmax / 63.0f : 0.0f;
        uint8_t scq[8], mq[8], q[8][32];
        for (int j = 0; j < 8; j++) {
            float a = d > 0.0f ? sc[j] / d : 0.0f;
            float b = dmn > 0.0f ? minv[j] / dmn : 0.0f;
            scq[j] = (uint8_t)std::min(63.0f, std::max(0.0f, std::nearbyint(a)));
            mq[j] = (uint8_t)std::min(63.0f, std::max(0.0f, std::nearbyint(b)));
            float asc = d * (float)scq[j], amin = dmn * (float)mq[j];
            float safe = asc > 0.0f ? asc : 1.0f;
            for (int i = 0; i < 32; i++) {
                float v = std::nearbyint((x[j * 32 + i] + amin) / safe);
                q[j][i] = (uint8_t)std::min(15.0f, std::max(0.0f, v));
            }
        }
        uint8_t* o = out + s * 144;
        uint16_t hd = f2h(d), hm = f2h(dmn);
        std::memcpy(o, &hd, 2); std::memcpy(o + 2, &hm, 2);
        uint8_t* S = o + 4;
        for (int j = 0; j < 4; j++) { S[j] = scq[j] & 63; S[j + 4] = mq[j] & 63; }
        for (int j = 0; j < 4; j++) S[8 + j] = (uint8_t)((scq[4 + j] & 0xF) | ((mq[4 + j] & 0xF) << 4));
        for (int j = 0; j < 4; j++) {
            S[j] |= (uint8_t)(((scq[4 + j] >> 4) & 3) << 6);
            S[j + 4] |= (uint8_t)(((mq[4 + j] >> 4) & 3) << 6);
        }
        for (int g = 0; g < 4; g++)
            for (int i = 0; i < 32; i++)
                o[16 + g * 32 + i] = (uint8_t)((q[2 * g][i] & 0xF) | ((q[2 * g + 1][i] & 0xF) << 4));
    }
}

// DEQ_Q8 (mg-opencl.cpp:386-387): fp16 d * int8 q.  deq_q4k_elem (:252-262):
// d*sc*q - dmin*m, evaluated left to right in float32.
void mgo_dequant(int wtype, const uint8_t* w, int64_t N, int64_t K, float* out) {
    if (wtype == 8) {
        const int64_t nb = K / 32;
        for (int64_t n = 0; n < N; n++)
            for (int64_t k = 0; k < K; k++) {
                const uint8_t* blk = w + (n * nb + k / 32) * 34;
                out[n * K + k] = rd_f16(blk) * (float)(int8_t)blk[2 + (k & 31)];
            }
    } else {
        const int64_t nsb = K / 256;
        for (int64_t n = 0; n < N; n++)
            for (int64_t k = 0; k < K; k++) {
                const uint8_t* blk = w + (n * nsb + k / 256) * 144;
                int r = (int)(k & 255), sub = r >> 5, j = r & 31, dq, mq;
                q4k_scale_min(blk + 4, sub, dq, mq);
                uint8_t qb = blk[16 + (sub >> 1) * 32 + j];
                float q = (float)((sub & 1) ? (qb >> 4) : (qb & 0xF));
                out[n * K + k] = rd_f16(blk) * (float)dq * q - rd_f16(blk + 2) * (float)mq;
            }
    }
}

// k_quantize_q8 (mg-opencl.cpp:424-434): amax over the 32-block, d = amax/127,
// id = 1/d (0 when d == 0), q = (char)round(x*id) -- round half away from zero, no clamp.
void mgo_quantize_act(const float* x, int64_t M, int64_t K, int8_t* qx, float* dx, int32_t* sumx) {
    const int64_t nb = K / 32;
    for (int64_t m = 0; m < M; m++)
        for (int64_t b = 0; b < nb; b++) {
            const float* r = x + m * K + b * 32;
            float amax = 0.0f;
            for (int i = 0; i < 32; i++) amax = std::fmax(amax, std::fabs(r[i]));
            float d = amax / 127.0f, id = d > 0.0f ? 1.0f / d : 0.0f;
            dx[m * nb + b] = d;
            int s = 0;
            for (int i = 0; i < 32; i++) {
                int q = (int)std::round(r[i] * id);
                qx[m * K + b * 32 + i] = (int8_t)q;
                s += (int8_t)q;
            }
            if (sumx) sumx[m * nb + b] = s;
        }
}

// k_mul_mat_q8_i8 (mg-opencl.cpp:440-494) and k_mul_mat_q4k_i8 (:504-590).  One output at
// a time, blocks b ascending, exact int32 block dot, then the fused epilogue
// bias -> act -> residual (mg-opencl.cpp:481-493).
static void qgemm_impl(int wtype, const uint8_t* w, const int8_t* qx, const float* dx,
                       const int32_t* sumx, int64_t M, int64_t N, int64_t K,
                       const float* bias, int act, const float* resid, float* y, int32_t* idot_out,
                       bool q4k_ref_order) {
    const int64_t nb = K / 32, nsb = K / 256;
    // decode per-(n,b) weight scales once
    std::vector<float> sA((size_t)N * nb), sB((size_t)N * nb);
    std::vector<int8_t> wq((size_t)N * K);
    for (int64_t n = 0; n < N; n++)
        for (int64_t b = 0; b < nb; b++) {
            if (wtype == 8) {
                const uint8_t* blk = w + (n * nb + b) * 34;
                sA[n * nb + b] = rd_f16(blk);
                for (int i = 0; i < 32; i++) wq[n * K + b * 32 + i] = (int8_t)blk[2 + i];
            } else {
                const uint8_t* blk = w + (n * nsb + b / 8) * 144;
                int j = (int)(b & 7), g = j >> 1, hi = j & 1, dq, mq;
                q4k_scale_min(blk + 4, j, dq, mq);
                sA[n * nb + b] = rd_f16(blk) * (float)dq;      // scl, mg-opencl.cpp:551
                sB[n * nb + b] = rd_f16(blk + 2) * (float)mq;  // mnl, mg-opencl.cpp:552
                for (int i = 0; i < 32; i++) {
                    uint8_t v = blk[16 + g * 32 + i];
                    wq[n * K + b * 32 + i] = (int8_t)(hi ? (v >> 4) : (v & 0xF));
                }
            }
        }
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; m++) {
        for (int64_t n = 0; n < N; n++) {
            float acc = 0.0f;
            for (int64_t b = 0; b < nb; b++) {
                const int8_t* a = qx + m * K + b * 32;
                const int8_t* q = wq.data() + n * K + b * 32;
                int idot = 0;
                for (int i = 0; i < 32; i++) idot += (int)a[i] * (int)q[i];
                if (idot_out) idot_out[(m * N + n) * nb + b] = idot;
                float d = dx[m * nb + b];
                if (wtype == 8) {
                    acc = std::fmaf(sA[n * nb + b] * d, (float)idot, acc);
                } else if (q4k_ref_order) {
                    // mg-opencl.cpp:572  acc += scl*dxm*(float)idot - mnl*dxm*(float)sum_x:
                    // the difference is formed first (the first product contracted into it,
                    // as the Q8_0 line contracts into acc), then added to acc.
                    const float t2 = (sB[n * nb + b] * d) * (float)sumx[m * nb + b];
                    const float t = std::fmaf(sA[n * nb + b] * d, (float)idot, -t2);
                    acc = acc + t;
                } else {
                    // the CUDA kernel's order: two fused multiply-adds into acc
                    acc = std::fmaf(sA[n * nb + b] * d, (float)idot, acc);
                    acc = std::fmaf(-sB[n * nb + b], d * (float)sumx[m * nb + b], acc);
                }
            }
            float v = acc;
            if (bias) v = v + bias[n];
            v = act_fn(v, act);
            if (resid) v = v + resid[m * N + n];
            y[m * N + n] = v;
        }
    }
}

void mgo_qgemm(int wtype, const uint8_t* w, const int8_t* qx, const float* dx,
               const int32_t* sumx, int64_t M, int64_t N, int64_t K,
               const float* bias, int act, const float* resid, float* y, int32_t* idot_out) {
    qgemm_impl(wtype, w, qx, dx, sumx, M, N, K, bias, act, resid, y, idot_out, true);
}

void mgo_qgemm_fused(int wtype, const uint8_t* w, const int8_t* qx, const float* dx,
                     const int32_t* sumx, int64_t M, int64_t N, int64_t K,
                     const float* bias, int act, const float* resid, float* y, int32_t* idot_out) {
    qgemm_impl(wtype, w, qx, dx, sumx, M, N, K, bias, act, resid, y, idot_out, false);
}

// k_mul_mat_t (mg-opencl.cpp:57-98): F32 GEMM, k ascending, same epilogue.
void mgo_gemm_f32(const float* w, const float* x, int64_t M, int64_t N, int64_t K,
                  const float* bias, int act, const float* resid, float* y) {
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; m++)
        for (int64_t n = 0; n < N; n++) {
            float acc = 0.0f;
            const float* a = x + m * K;
            const float* b = w + n * K;
            for (int64_t k = 0; k < K; k++) acc = std::fmaf(b[k], a[k], acc);
            float v = acc;
            if (bias) v = v + bias[n];
            v = act_fn(v, act);
            if (resid) v = v + resid[m * N + n];
            y[m * N + n] = v;
        }
}

// k_norm_affine (mg-opencl.cpp:705-727): 64 lanes, lane t sums d = t, t+64, ...; tree
// lp[t] += lp[t+k] for k = 32..1; mean = sum/D; var the same over (x-mean)^2;
// inv = 1/sqrt(var/D + eps); y = fmaf((x-mean)*inv, gamma, beta).
void mgo_layernorm_affine(const float* x, const float* gamma, const float* beta,
                          int64_t rows, int64_t D, float eps, float* y) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        const float* a = x + r * D;
        float lp[64];
        for (int t = 0; t < 64; t++) { float s = 0.0f; for (int64_t d = t; d < D; d += 64) s += a[d]; lp[t] = s; }
        for (int k = 32; k > 0; k >>= 1) for (int t = 0; t < k; t++) lp[t] += lp[t + k];
        float mean = lp[0] / (float)D;
        for (int t = 0; t < 64; t++) {
            float v = 0.0f;
            for (int64_t d = t; d < D; d += 64) { float u = a[d] - mean; v = std::fmaf(u, u, v); }
            lp[t] = v;
        }
        for (int k = 32; k > 0; k >>= 1) for (int t = 0; t < k; t++) lp[t] += lp[t + k];
        float inv = 1.0f / std::sqrt(lp[0] / (float)D + eps);
        for (int64_t d = 0; d < D; d++) y[r * D + d] = std::fmaf((a[d] - mean) * inv, gamma[d], beta[d]);
    }
}

// k_flash_attention_h (mg-opencl.cpp:859-937): per query row, Q/K/V rounded to half,
// keys in tiles of 32, online softmax with f32 stats and accumulator.
void mgo_flash_attn(const float* qkv, int64_t B, int64_t S, int64_t H, int64_t Dh,
                    float scale, float* out) {
    const int64_t E = H * Dh, W = 3 * E;
    auto rh = [](float f) { return h2f(f2h(f)); };
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t b = 0; b < B; b++)
        for (int64_t h = 0; h < H; h++) {
            std::vector<float> K_((size_t)S * Dh), V_((size_t)S * Dh);
            for (int64_t t = 0; t < S; t++)
                for (int64_t d = 0; d < Dh; d++) {
                    K_[t * Dh + d] = rh(qkv[(b * S + t) * W + E + h * Dh + d]);
                    V_[t * Dh + d] = rh(qkv[(b * S + t) * W + 2 * E + h * Dh + d]);
                }
            std::vector<float> q(Dh), o(Dh);
            for (int64_t s = 0; s < S; s++) {
                for (int64_t d = 0; d < Dh; d++) q[d] = rh(qkv[(b * S + s) * W + h * Dh + d]);
                float m_i = -INFINITY, l_i = 0.0f;
                std::fill(o.begin(), o.end(), 0.0f);
                for (int64_t kb = 0; kb < S; kb += 32) {
                    float sc[32];
                    float m_new = m_i;
                    for (int kc = 0; kc < 32; kc++) {
                        int64_t t = kb + kc;
                        if (t >= S) { sc[kc] = -INFINITY; continue; }
                        float dot = 0.0f;
                        for (int64_t d = 0; d < Dh; d++) dot = std::fmaf(q[d], K_[t * Dh + d], dot);
                        dot *= scale;
                        sc[kc] = dot;
                        m_new = std::fmax(m_new, dot);
                    }
                    float alpha = std::exp(m_i - m_new);
                    float l_new = alpha * l_i;
                    for (int kc = 0; kc < 32; kc++) {
                        float p = (sc[kc] == -INFINITY) ? 0.0f : std::exp(sc[kc] - m_new);
                        sc[kc] = p;
                        l_new += p;
                    }
                    for (int64_t d = 0; d < Dh; d++) {
                        float no = alpha * o[d];
                        for (int kc = 0; kc < 32 && kb + kc < S; kc++) no = std::fmaf(sc[kc], V_[(kb + kc) * Dh + d], no);
                        o[d] = no;
                    }
                    m_i = m_new; l_i = l_new;
                }
                float inv = 1.0f / l_i;
                for (int64_t d = 0; d < Dh; d++) out[(b * S + s) * E + h * Dh + d] = o[d] * inv;
            }
        }
}

// get_rows (negative ids wrap, mg-opencl.cpp:667-672) + pos add (mg-transformer.cpp:41-44)
void mgo_embed(const float* tok_embd, int64_t vocab, const float* pos_embd, int64_t E,
               const int32_t* tokens, int64_t B, int64_t S, float* out) {
    for (int64_t b = 0; b < B; b++)
        for (int64_t s = 0; s < S; s++) {
            int64_t id = tokens[b * S + s];
            if (id < 0) id += vocab;
            for (int64_t e = 0; e < E; e++)
                out[(b * S + s) * E + e] = tok_embd[id * E + e] + pos_embd[s * E + e];
        }
}

}  // extern "C"

// ------------------------------------------------------------------ whole model oracle
namespace {

struct OTensor { uint32_t type; int64_t ne[4]; const uint8_t* data; };

// GGUF v3 reader restating Model::load (mg-model.cpp:139-201): metadata keys of
// mg-model.cpp:65-103, tensor data aligned to general.alignment (default 32).
struct Gguf {
    std::vector<uint8_t> buf;
    std::unordered_map<std::string, OTensor> t;
    int n_layer = 0, n_head = 0, n_embd = 0, n_ffn = 0, head_dim = 0, vocab = 0, n_tokens = 0;
    int mask_id = -1, codebook = 0;
    float ln_eps = 1e-12f, choice_temp = 4.5f;
    size_t p = 0;
    template <class T> T rd() {
        if (p + sizeof(T) > buf.size()) throw std::runtime_error("gguf: unexpected EOF");
        T v; std::memcpy(&v, buf.data() + p, sizeof(T)); p += sizeof(T); return v;
    }
    std::string str() {
        uint64_t n = rd<uint64_t>();
        if (p + n > buf.size()) throw std::runtime_error("gguf: bad string");
        std::string s((const char*)buf.data() + p, n); p += n; return s;
    }
    static size_t vsize(uint32_t vt) {
        switch (vt) { case 0: case 1: case 7: return 1; case 2: case 3: return 2;
                      case 4: case 5: case 6: return 4; case 10: case 11: case 12: return 8; }
        return 0;
    }
    void load(const char* path) {
        std::ifstream f(path, std::ios::binary);
        if (!f) throw std::runtime_error(std::string("cannot open ") + path);
        buf.assign(std::istreambuf_iterator<char>(f), {});
        if (rd<uint32_t>() != 0x46554747u) throw std::runtime_error("not a GGUF file");
        if (rd<uint32_t>() != 3) throw std::runtime_error("unsupported GGUF version");
        uint64_t nt = rd<uint64_t>(), nkv = rd<uint64_t>();
        uint32_t align = 32;
        for (uint64_t i = 0; i < nkv; i++) {
            std::string k = str();
            uint32_t vt = rd<uint32_t>();
            if (vt == 8) { str(); continue; }
            if (vt == 9) {
                uint32_t sub = rd<uint32_t>(); uint64_t n = rd<uint64_t>();
                if (sub == 8) { for (uint64_t j = 0; j < n; j++) str(); }
                else p += vsize(sub) * n;
                continue;
            }
            if (vt == 6) {
                float v = rd<float>();
                if (k == "maskgit.layernorm_eps") ln_eps = v;
                else if (k == "maskgit.sampling.choice_temperature") choice_temp = v;
                continue;
            }
            int64_t v;
            switch (vt) {
                case 4: v = rd<uint32_t>(); break; case 5: v = rd<int32_t>(); break;
                case 10: v = (int64_t)rd<uint64_t>(); break; case 11: v = rd<int64_t>(); break;
                case 0: case 7: v = rd<uint8_t>(); break;
                default: p += vsize(vt); continue;
            }
            if (k == "general.alignment") align = (uint32_t)v;
            else if (k == "maskgit.n_layer") n_layer = (int)v;
            else if (k == "maskgit.n_head") n_head = (int)v;
            else if (k == "maskgit.n_embd") n_embd = (int)v;
            else if (k == "maskgit.n_ffn") n_ffn = (int)v;
            else if (k == "maskgit.head_dim") head_dim = (int)v;
            else if (k == "maskgit.vocab_size") vocab = (int)v;
            else if (k == "maskgit.n_tokens") n_tokens = (int)v;
            else if (k == "maskgit.mask_token_id") mask_id = (int)v;
            else if (k == "maskgit.vqgan.codebook_size") codebook = (int)v;
        }
        struct Info { std::string name; OTensor t; uint64_t off; };
        std::vector<Info> infos;
        for (uint64_t i = 0; i < nt; i++) {
            Info in; in.name = str();
            uint32_t nd = rd<uint32_t>();
            for (int d = 0; d < 4; d++) in.t.ne[d] = 1;
            for (uint32_t d = 0; d < nd; d++) in.t.ne[d] = (int64_t)rd<uint64_t>();
            in.t.type = rd<uint32_t>();
            in.off = rd<uint64_t>();
            infos.push_back(in);
        }
        size_t ds = (p + align - 1) / align * align;
        for (auto& in : infos) { in.t.data = buf.data() + ds + in.off; t[in.name] = in.t; }
    }
    const OTensor& req(const std::string& n) const {
        auto it = t.find(n);
        if (it == t.end()) throw std::runtime_error("gguf: missing required tensor '" + n + "'");
        return it->second;
    }
    const float* f32(const std::string& n) const {
        const OTensor& x = req(n);
        if (x.type != 0) throw std::runtime_error("tensor '" + n + "' is not F32");
        return (const float*)x.data;
    }
};

}  // namespace

struct mgo_model { Gguf g; };

extern "C" {

mgo_model* mgo_model_load(const char* path) {
    try { auto* m = new mgo_model(); m->g.load(path); return m; }
    catch (const std::exception& e) { g_err = e.what(); return nullptr; }
}
void mgo_model_free(mgo_model* m) { delete m; }
void mgo_model_hparams(const mgo_model* m, int32_t o[10]) {
    const Gguf& g = m->g;
    int wt = -1;
    auto it = g.t.find("blk.0.attn_q.weight");
    if (it != g.t.end()) wt = (int)it->second.type;
    int v[10] = {g.n_layer, g.n_head, g.n_embd, g.n_ffn, g.head_dim, g.vocab, g.n_tokens,
                 g.mask_id, g.codebook, wt};
    for (int i = 0; i < 10; i++) o[i] = v[i];
}

// build_transformer (mg-transformer.cpp:32-111) evaluated directly.  Linear layers stored
// F32 use mgo_gemm_f32; Q8_0/Q4_K use quantize_act + qgemm (the dispatch of
// mg-opencl.cpp:1381-1399).
int mgo_forward(mgo_model* mm, const int32_t* tokens, int B, int S, float* logits, float* dump) {
    try {
        const Gguf& g = mm->g;
        const int64_t E = g.n_embd, F = g.n_ffn, R = (int64_t)B * S, V = g.vocab;
        std::vector<float> x(R * E), qkv(R * 3 * E), att(R * E), ff(R * F), tmp(R * E);
        std::vector<int8_t> qx(R * std::max(E, F));
        std::vector<float> dx(R * std::max(E, F) / 32);
        std::vector<int32_t> sx(R * std::max(E, F) / 32);
        int64_t doff = 0;
        auto put = [&](const float* a, int64_t w) {
            if (dump) { std::memcpy(dump + doff, a, sizeof(float) * R * w); doff += R * w; }
        };
        auto linear = [&](const std::string& wn, const std::string& bn, const float* in, int64_t K,
                          int act, const float* resid, float* out) {
            const OTensor& w = g.req(wn);
            const int64_t N = w.ne[1];
            const float* bias = bn.empty() ? nullptr : g.f32(bn);
            if (w.type == 0) { mgo_gemm_f32((const float*)w.data, in, R, N, K, bias, act, resid, out); return; }
            mgo_quantize_act(in, R, K, qx.data(), dx.data(), sx.data());
            mgo_qgemm((int)w.type, w.data, qx.data(), dx.data(), sx.data(), R, N, K, bias, act, resid, out, nullptr);
        };
        const float eps = g.ln_eps;
        std::vector<float> e0(R * E);
        mgo_embed(g.f32("token_embd.weight"), V, g.f32("pos_embd.weight"), E, tokens, B, S, e0.data());
        mgo_layernorm_affine(e0.data(), g.f32("token_embd_norm.weight"), g.f32("token_embd_norm.bias"), R, E, eps, x.data());
        put(x.data(), E);
        const float scale = 1.0f / std::sqrt((float)g.head_dim);
        std::vector<float> t1(R * E);
        for (int i = 0; i < g.n_layer; i++) {
            std::string p = "blk." + std::to_string(i) + ".";
            // q, k, v as three linears writing the column blocks of qkv
            for (int j = 0; j < 3; j++) {
                const char* nm = j == 0 ? "q" : j == 1 ? "k" : "v";
                linear(p + "attn_" + nm + ".weight", p + "attn_" + nm + ".bias", x.data(), E, 0, nullptr, t1.data());
                for (int64_t r = 0; r < R; r++) std::memcpy(&qkv[r * 3 * E + j * E], &t1[r * E], sizeof(float) * E);
            }
            mgo_flash_attn(qkv.data(), B, S, g.n_head, g.head_dim, scale, att.data());
            linear(p + "attn_o.weight", p + "attn_o.bias", att.data(), E, 0, x.data(), tmp.data());
            mgo_layernorm_affine(tmp.data(), g.f32(p + "attn_norm.weight"), g.f32(p + "attn_norm.bias"), R, E, eps, x.data());
            put(x.data(), E);
            linear(p + "ffn_up.weight", p + "ffn_up.bias", x.data(), E, 1, nullptr, ff.data());
            linear(p + "ffn_down.weight", p + "ffn_down.bias", ff.data(), F, 0, x.data(), tmp.data());
            mgo_layernorm_affine(tmp.data(), g.f32(p + "ffn_norm.weight"), g.f32(p + "ffn_norm.bias"), R, E, eps, x.data());
            put(x.data(), E);
        }
        linear("output_proj.weight", "output_proj.bias", x.data(), E, 1, nullptr, tmp.data());
        mgo_layernorm_affine(tmp.data(), g.f32("output_norm.weight"), g.f32("output_norm.bias"), R, E, eps, x.data());
        put(x.data(), E);
        mgo_gemm_f32(g.f32("token_embd.weight"), x.data(), R, V, E, g.f32("output.bias"), 0, nullptr, logits);
        put(logits, V);
        return 0;
    } catch (const std::exception& e) { g_err = e.what(); return -1; }
}

int mgo_forward_cb(void* user, const int32_t* tokens, int B, int S, float* logits) {
    return mgo_forward((mgo_model*)user, tokens, B, S, logits, nullptr);
}

// generate() sampling loop, mg-generate.cpp:24-35 (gumbel, sample_categorical) and
// :53-123 (cosine schedule, confidence, nth_element re-mask), for B independent images
// whose forwards are batched into one callback.
int mgo_generate(const mgo_model* mm, mgo_fwd_fn fwd, void* user, int B,
                 const int32_t* class_ids, const uint64_t* seeds, int steps,
                 float temperature, int32_t* tokens_out) {
    const Gguf& g = mm->g;
    const int CB = g.codebook, MASK = g.mask_id, S = g.n_tokens + 1;
    const int64_t vocab = g.vocab;
    const float choice_temp = temperature < 0 ? g.choice_temp : temperature;
    std::vector<std::mt19937_64> rng;
    for (int i = 0; i < B; i++) rng.emplace_back(seeds[i]);
    std::vector<int32_t> tokens((size_t)B * S, MASK), sampled(S), result((size_t)B * S);
    for (int i = 0; i < B; i++) tokens[(size_t)i * S] = class_ids[i] + CB;
    std::vector<float> L((size_t)B * S * vocab), selp(S), conf(S), probs(CB);
    const int unknown_begin = g.n_tokens;
    for (int step = 0; step < steps; step++) {
        if (fwd(user, tokens.data(), B, S, L.data()) != 0) return -1;
        for (int i = 0; i < B; i++) {
            std::mt19937_64& r = rng[i];
            int32_t* tk = tokens.data() + (size_t)i * S;
            for (int s = 0; s < S; s++) {
                const float* row = L.data() + ((size_t)i * S + s) * vocab;
                float mx = -INFINITY;
                for (int v = 0; v < CB; v++) mx = std::fmax(mx, row[v]);
                float sum = 0.f;
                for (int v = 0; v < CB; v++) { float e = std::exp(row[v] - mx); probs[v] = e; sum += e; }
                float inv = 1.f / sum;
                for (int v = 0; v < CB; v++) probs[v] *= inv;
                std::uniform_real_distribution<double> u(0.0, 1.0);
                double rr = u(r), acc = 0.0;
                int sid = CB - 1;
                for (int v = 0; v < CB; v++) { acc += probs[v]; if (rr <= acc) { sid = v; break; } }
                bool unknown = (tk[s] == MASK);
                sampled[s] = unknown ? sid : tk[s];
                selp[s] = unknown ? probs[sid] : INFINITY;
            }
            std::memcpy(result.data() + (size_t)i * S, sampled.data(), sizeof(int32_t) * S);
            float ratio = (float)(step + 1) / steps;
            float mask_ratio = std::cos((float)M_PI / 2.f * ratio);
            int n_unknown_now = 0;
            for (int s = 0; s < S; s++) n_unknown_now += (tk[s] == MASK);
            int mask_len = (int)std::floor(unknown_begin * mask_ratio);
            mask_len = std::max(1, std::min(mask_len, n_unknown_now - 1));
            float temp = choice_temp * (1.f - ratio);
            for (int s = 0; s < S; s++) {
                std::uniform_real_distribution<double> u(1e-12, 1.0);
                float gmb = (float)(-std::log(-std::log(u(r))));
                conf[s] = std::log(selp[s]) + temp * gmb;
            }
            std::vector<float> sorted(conf);
            std::nth_element(sorted.begin(), sorted.begin() + mask_len, sorted.end());
            float cutoff = sorted[mask_len];
            for (int s = 0; s < S; s++) tk[s] = (conf[s] < cutoff) ? MASK : sampled[s];
        }
    }
    std::memcpy(tokens_out, result.data(), sizeof(int32_t) * B * S);
    return 0;
}

}  // extern "C"
