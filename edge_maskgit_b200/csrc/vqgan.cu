// vqgan.cu -- the MaskGIT VQGAN decoder on the GPU: the graph of src/mg-vqgan.cpp:67-108
// (codebook lookup, conv_in, ResBlocks with the shortcut conv applied to the processed tensor,
// nearest 2x upsampling + conv, GroupNorm(32) + affine + SiLU, conv_out) run as a fixed program of
// kernels over one or more token grids.
//
// Layout.  Activations are NHWC f32, [image][y][x][channel]: a pixel's channels are one
// contiguous run, so the codebook lookup is a row copy, a 3x3 conv is an implicit GEMM whose
// K dimension (tap, channel) reads contiguous channel runs of shifted pixels, and the last conv
// (3 output channels) writes the HWC image of the VqganFwd callback (include/mg-generate.hpp:17)
// directly.  Conv weights are re-laid on load from GGUF [OC][IC][KH][KW] to [tap][IC][OC].
//
// Numerics follow mg-cpu (src/mg-cpu/mg-cpu.cpp): GroupNorm statistics in double
// (:124-147, variance as E[x^2] - mean^2 over per-chunk double sums), normalisation
// (float)(x - mean) * inv, then xn = o * gamma + beta and xn / (1 + exp(-xn)) (:265-276) with
// separately rounded multiply and add; convs accumulate in f32 (tap-major instead of
// (ic, kh, kw), the only reordering).
#include "../../include/mgc.h"
#include "gguf.h"
#include "kernels.h"
#include "qgemm_common.cuh"

#include <algorithm>
#include <cmath>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace mgc {
namespace {

// ------------------------------------------------------------------------------------------
// Implicit-GEMM 3x3 / 1x1 conv, SIMT f32.  Rows = output pixels (M = images * H * W), columns =
// output channels, K = taps * IC (IC a multiple of 8, OC of 4).  CTA tile 128 x 128 x 8, 256 threads, 8 x 8 outputs a thread,
// register-prefetched double buffer.  With UP the input is the half-resolution tensor and the
// nearest 2x upsample (mg-cpu.cpp:190-196) is folded into the pixel address.
struct ConvArgs {
    const float* x;       // [N][Hin][Win][IC]
    const float* w;       // [T][IC][OC]
    const float* bias;    // [OC] or null
    const float* resid;   // [M][OC] or null (added after the conv)
    float* y;             // [M][OC]
    float* part;          // [nsplit][M][OC] when nsplit > 1
    int H, W, IC, OC, ks, up, M;
    int kper;             // K iterations (8 channels of one tap) per split
    int kiters;
};

constexpr int CBM = 128, CBN = 128, CBK = 8, CPAD = 4;

template <bool UP>
__global__ void __launch_bounds__(256, 2) conv_simt_kernel(ConvArgs a) {
    __shared__ __align__(16) float As[2][CBK][CBM + CPAD];
    __shared__ __align__(16) float Bs[2][CBK][CBN];
    const int tid = threadIdx.x;
    const int m0 = blockIdx.x * CBM, n0 = blockIdx.y * CBN;
    const int it0 = blockIdx.z * a.kper, it1 = min(a.kiters, it0 + a.kper);
    const int icg = a.IC / CBK;
    // this thread's A row (pixel) and channel quad
    const int pr = tid >> 1, cq = (tid & 1) * 4;
    const int m = m0 + pr;
    const int HW = a.H * a.W;
    const int img = m / HW, rem = m - img * HW, py = rem / a.W, px = rem - py * a.W;
    const int Hin = UP ? a.H >> 1 : a.H, Win = UP ? a.W >> 1 : a.W;
    const float* xbase = a.x + (size_t)img * Hin * Win * a.IC + cq;
    const int br = tid >> 5, bc = (tid & 31) * 4;
    const int half = a.ks >> 1;

    auto load_a = [&](int it) -> float4 {
        const int tap = it / icg, c0 = (it - tap * icg) * CBK;
        const int yy = py + tap / a.ks - half, xx = px + tap % a.ks - half;
        if (m >= a.M || yy < 0 || yy >= a.H || xx < 0 || xx >= a.W) return make_float4(0.f, 0.f, 0.f, 0.f);
        const int sy = UP ? yy >> 1 : yy, sx = UP ? xx >> 1 : xx;
        return __ldg(reinterpret_cast<const float4*>(xbase + ((size_t)sy * Win + sx) * a.IC + c0));
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

// Conv with few output channels (conv_out, OC = 3): one thread a pixel, weights in shared
// memory as [tap][IC][4].
constexpr int kSmallOC = 4;
__global__ void __launch_bounds__(128) conv_small_oc_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                            const float* __restrict__ bias, float* __restrict__ y,
                                                            int M, int H, int W, int IC, int OC, int ks) {
    extern __shared__ float ws[];   // [T][IC][4]
    const int T = ks * ks;
    for (int i = threadIdx.x; i < T * IC * kSmallOC; i += blockDim.x) {
        const int o = i % kSmallOC, r = i / kSmallOC;
        ws[i] = o < OC ? w[(size_t)r * OC + o] : 0.f;
    }
    __syncthreads();
    const int m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m >= M) return;
    const int HW = H * W, img = m / HW, rem = m - img * HW, py = rem / W, px = rem - py * W;
    const int half = ks >> 1;
    float acc[kSmallOC] = {0.f, 0.f, 0.f, 0.f};
    for (int tap = 0; tap < T; tap++) {
        const int yy = py + tap / ks - half, xx = px + tap % ks - half;
        if (yy < 0 || yy >= H || xx < 0 || xx >= W) continue;
        const float4* src = reinterpret_cast<const float4*>(x + ((size_t)(img * H + yy) * W + xx) * IC);
        const float4* wt = reinterpret_cast<const float4*>(ws + (size_t)tap * IC * kSmallOC);
        for (int c4 = 0; c4 < IC / 4; c4++) {
            const float4 v = __ldg(src + c4);
            const float xv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float4 wv = wt[c4 * 4 + j];
                acc[0] = fmaf(xv[j], wv.x, acc[0]); acc[1] = fmaf(xv[j], wv.y, acc[1]);
                acc[2] = fmaf(xv[j], wv.z, acc[2]); acc[3] = fmaf(xv[j], wv.w, acc[3]);
            }
        }
    }
    for (int o = 0; o < OC; o++) y[(size_t)m * OC + o] = acc[o] + (bias ? bias[o] : 0.f);
}

// ------------------------------------------------------------------------------------------
// GroupNorm + affine + SiLU over NHWC.  Pass 1: per (image, pixel chunk) per-channel double
// sums of x and x^2 (fixed-order reductions, so the result is deterministic).  Pass 2: per
// (image, group) mean and 1/sqrt(var + eps).  Pass 3: the elementwise apply.
constexpr int kGnThreads = 256;

__global__ void __launch_bounds__(kGnThreads) gn_partial_kernel(const float* __restrict__ x, int HW, int C,
                                                                int pix_per_chunk, double* __restrict__ part) {
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

struct GnStat { double mean; float inv; float pad; };

__global__ void gn_finalize_kernel(const double* __restrict__ part, int nch, int C, int G, int HW, float eps,
                                   GnStat* __restrict__ st) {
    const int img = blockIdx.x, g = threadIdx.x;
    if (g >= G) return;
    const int cpg = C / G;
    double s = 0, ss = 0;
    for (int k = 0; k < nch; k++)
        for (int c = g * cpg; c < (g + 1) * cpg; c++) {
            const double* p = part + (((size_t)img * nch + k) * C + c) * 2;
            s += p[0]; ss += p[1];
        }
    const double cnt = (double)HW * cpg;
    const double mean = s / cnt;
    const double var = fmax(ss / cnt - mean * mean, 0.0);
    st[img * G + g] = GnStat{mean, 1.0f / sqrtf((float)var + eps), 0.f};
}

__global__ void gn_apply_silu_kernel(const float* __restrict__ x, const GnStat* __restrict__ st,
                                     const float* __restrict__ gamma, const float* __restrict__ beta, int HW, int C,
                                     int G, size_t n4, float* __restrict__ y) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n4) return;
    const size_t e = i * 4;
    const int c0 = (int)(e % C);
    const int img = (int)(e / ((size_t)HW * C));
    const int cpg = C / G;
    const float4 v = reinterpret_cast<const float4*>(x)[i];
    const float xv[4] = {v.x, v.y, v.z, v.w};
    float o[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const int c = c0 + j;
        const GnStat s = st[img * G + c / cpg];
        const float nrm = __fmul_rn((float)((double)xv[j] - s.mean), s.inv);
        const float xn = __fadd_rn(__fmul_rn(nrm, gamma[c]), beta[c]);
        o[j] = xn / (1.0f + expf(-xn));
    }
    reinterpret_cast<float4*>(y)[i] = make_float4(o[0], o[1], o[2], o[3]);
}

// Codebook lookup (get_rows, mg-vqgan.cpp:79-81): pixel p of image n is token grid[n][p]
// (p = y * L + x), its channels the codebook row.  Ids outside [0, codebook) decode as zeros.
__global__ void vq_gather_kernel(const int32_t* __restrict__ grid, const float* __restrict__ cb, int n_codes, int E,
                                 size_t n4, float* __restrict__ y) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n4) return;
    const int E4 = E / 4;
    const size_t pix = i / E4;
    const int c4 = (int)(i % E4);
    const int id = grid[pix];
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (id >= 0 && id < n_codes) v = reinterpret_cast<const float4*>(cb + (size_t)id * E)[c4];
    reinterpret_cast<float4*>(y)[i] = v;
}

// ------------------------------------------------------------------------------------------
// Host side.
struct Conv { int ic = 0, oc = 0, ks = 0; float* w = nullptr; float* b = nullptr; };
struct Norm { int c = 0; float* g = nullptr; float* b = nullptr; };

// One step of the decoder program.  Buffers: 0 = x (stream), 1 = t (normed), 2 = u, 3 = h.
struct Step {
    enum Kind { Gather, GnSilu, ConvOp, ConvOut, SwapXH } kind;
    int src = 0, dst = 0, resid = -1;   // buffer ids (resid -1 = none)
    int conv = -1, norm = -1;
    int H = 0, W = 0, C = 0;            // output spatial size; channels of the step's input
    bool up = false;
};

void ck(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

template <class T>
T* dalloc(size_t n) {
    void* p = nullptr;
    ck(cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)), "cudaMalloc");
    return (T*)p;
}

}  // namespace
}  // namespace mgc

using namespace mgc;

struct mgc_vqgan {
    int device = 0, max_images = 0;
    int n_tokens = 0, L = 0, R = 0, E = 0, n_codes = 0, groups = 32;
    cudaStream_t st = nullptr;
    float* codebook = nullptr;
    std::vector<Conv> convs;
    std::vector<Norm> norms;
    std::vector<Step> prog;
    size_t buf_floats = 0;       // per image
    float* buf[4] = {nullptr, nullptr, nullptr, nullptr};
    size_t part_floats = 0;      // split-K partials, all images
    float* part = nullptr;
    int gn_chunks = 0;
    double* gn_part = nullptr;
    GnStat* gn_stat = nullptr;
    int32_t* d_grid = nullptr;
    float* d_img = nullptr;
    std::map<int, cudaGraphExec_t> graphs;   // per image count
    int launches = 0;                         // kernels one decode launches

    ~mgc_vqgan() {
        for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
        for (auto& c : convs) { cudaFree(c.w); cudaFree(c.b); }
        for (auto& n : norms) { cudaFree(n.g); cudaFree(n.b); }
        for (float* b : buf) cudaFree(b);
        cudaFree(codebook); cudaFree(part); cudaFree(gn_part); cudaFree(gn_stat); cudaFree(d_grid); cudaFree(d_img);
        if (st) cudaStreamDestroy(st);
    }

    int conv_split(int M, int OC, int kiters) const {
        const int tiles = ((M + CBM - 1) / CBM) * ((OC + CBN - 1) / CBN);
        const int target = 2 * sm_count();
        if (tiles >= target) return 1;
        int s = (target + tiles - 1) / tiles;
        return std::max(1, std::min(s, kiters / 4));
    }

    void load(const char* path) {
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
            // [OC][IC][KH][KW] -> [tap][IC][OC]
            const float* src = (const float*)t.data;
            const int T = ks * ks;
            std::vector<float> w((size_t)T * ic * oc);
            for (int o = 0; o < oc; o++)
                for (int i = 0; i < ic; i++)
                    for (int k = 0; k < T; k++) w[((size_t)k * ic + i) * oc + o] = src[((size_t)o * ic + i) * T + k];
            Conv c;
            c.ic = ic; c.oc = oc; c.ks = ks;
            c.w = dalloc<float>(w.size());
            ck(cudaMemcpy(c.w, w.data(), w.size() * 4, cudaMemcpyHostToDevice), "upload conv");
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
            if (c % groups || c % 4 || kGnThreads % (c / 4)) throw std::runtime_error("vqgan: unsupported channel count");
            Norm n;
            n.c = c;
            n.g = dalloc<float>(c);
            n.b = dalloc<float>(c);
            ck(cudaMemcpy(n.g, w.data, (size_t)c * 4, cudaMemcpyHostToDevice), "upload gn");
            ck(cudaMemcpy(n.b, b.data, (size_t)c * 4, cudaMemcpyHostToDevice), "upload gn");
            norms.push_back(n);
            return (int)norms.size() - 1;
        };

        // the program (mg-vqgan.cpp:67-108); buffers 0 = x, 1 = t, 2 = u, 3 = h
        int H = L, W = L, cur = (int)(filters * mult[nb - 1]);
        size_t maxf = (size_t)H * W * E;
        auto note = [&](int c) { maxf = std::max(maxf, (size_t)H * W * c); };
        prog.push_back(Step{Step::Gather, -1, 1, -1, -1, -1, H, W, E, false});
        prog.push_back(Step{Step::ConvOp, 1, 0, -1, add_conv("vqgan.decoder.conv_in", E, cur, 3, true), -1, H, W, E, false});
        note(cur);
        auto resblock = [&](const std::string& pfx, int cin, int cout) {
            prog.push_back(Step{Step::GnSilu, 0, 1, -1, -1, add_norm(pfx + "norm0", cin), H, W, cin, false});
            prog.push_back(Step{Step::ConvOp, 1, 2, -1, add_conv(pfx + "conv0", cin, cout, 3, false), -1, H, W, cin, false});
            prog.push_back(Step{Step::GnSilu, 2, 1, -1, -1, add_norm(pfx + "norm1", cout), H, W, cout, false});
            if (cin == cout) {
                prog.push_back(Step{Step::ConvOp, 1, 3, 0, add_conv(pfx + "conv1", cout, cout, 3, false), -1, H, W, cout, false});
            } else {   // the shortcut conv reads the processed h (mg-vqgan.cpp:57-60)
                prog.push_back(Step{Step::ConvOp, 1, 2, -1, add_conv(pfx + "conv1", cout, cout, 3, false), -1, H, W, cout, false});
                prog.push_back(Step{Step::ConvOp, 2, 3, 2, add_conv(pfx + "conv_res", cout, cout, 1, false), -1, H, W, cout, false});
            }
            note(cin); note(cout);
            prog.push_back(Step{Step::SwapXH});
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
                prog.push_back(Step{Step::ConvOp, 0, 3, -1, c, -1, H, W, cur, true});
                prog.push_back(Step{Step::SwapXH});
            }
        }
        prog.push_back(Step{Step::GnSilu, 0, 1, -1, -1, add_norm("vqgan.decoder.norm_out", cur), H, W, cur, false});
        const GgufTensor& co = g.req("vqgan.decoder.conv_out.weight");
        if (co.ne[3] > kSmallOC) throw std::runtime_error("vqgan: conv_out must have at most 4 output channels");
        prog.push_back(Step{Step::ConvOut, 1, -1, -1, add_conv("vqgan.decoder.conv_out", cur, (int)co.ne[3], 3, true), -1,
                            H, W, cur, false});
        const size_t co_smem = (size_t)9 * cur * kSmallOC * 4;
        if (co_smem > 200 * 1024) throw std::runtime_error("vqgan: conv_out input has too many channels");
        ck(cudaFuncSetAttribute(conv_small_oc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)co_smem),
           "conv_out smem");
        for (const Conv& c : convs)
            if (c.oc > kSmallOC && (c.oc % 4 || c.ic % CBK))
                throw std::runtime_error("vqgan: conv channel counts must be multiples of 4 (out) and 8 (in)");
        buf_floats = maxf;
    }

    // device buffers for n images (grown on demand)
    void reserve(int n) {
        if (n <= max_images) return;
        for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
        graphs.clear();
        for (float*& b : buf) { cudaFree(b); b = dalloc<float>(buf_floats * n); }
        // split-K partials: the largest over the conv steps at n images
        size_t pf = 0;
        int maxc = 0;
        for (const Step& s : prog) {
            if (s.kind == Step::GnSilu) maxc = std::max(maxc, s.C);
            if (s.kind != Step::ConvOp) continue;
            const Conv& c = convs[s.conv];
            const int M = n * s.H * s.W, kit = c.ks * c.ks * c.ic / CBK;
            const int ns = conv_split(M, c.oc, kit);
            if (ns > 1) pf = std::max(pf, (size_t)ns * M * c.oc);
        }
        cudaFree(part); part = dalloc<float>(pf);
        part_floats = pf;
        gn_chunks = 0;
        for (const Step& s : prog)
            if (s.kind == Step::GnSilu) gn_chunks = std::max(gn_chunks, chunks_for(n, s.H * s.W));
        cudaFree(gn_part); gn_part = dalloc<double>((size_t)n * gn_chunks * maxc * 2);
        cudaFree(gn_stat); gn_stat = dalloc<GnStat>((size_t)n * groups);
        cudaFree(d_grid); d_grid = dalloc<int32_t>((size_t)n * n_tokens);
        cudaFree(d_img); d_img = dalloc<float>((size_t)n * R * R * 3);
        max_images = n;
    }

    int chunks_for(int n, int HW) const {
        const int want = std::max(1, (2 * sm_count() + n - 1) / n);
        return std::max(1, std::min(want, HW / 64));
    }

    // Enqueue the decoder on `s` for n images: grid (device, [n][n_tokens]) -> out (device,
    // [n][R][R][3]).  Returns the number of kernels launched.
    int enqueue(const int32_t* grid, int n, float* out, cudaStream_t s) {
        int nl = 0;
        float* b[4] = {buf[0], buf[1], buf[2], buf[3]};
        for (const Step& stp : prog) {
            const int HW = stp.H * stp.W;
            switch (stp.kind) {
            case Step::Gather: {
                const size_t n4 = (size_t)n * HW * E / 4;
                launch_k(vq_gather_kernel, (unsigned)((n4 + 255) / 256), 256, 0, s, grid, codebook, n_codes, E, n4,
                         b[stp.dst]);
                nl++;
                break;
            }
            case Step::SwapXH:
                std::swap(b[0], b[3]);
                break;
            case Step::GnSilu: {
                const Norm& nm = norms[stp.norm];
                const int nch = chunks_for(n, HW), ppc = (HW + nch - 1) / nch;
                launch_k(gn_partial_kernel, dim3(nch, n), kGnThreads, 0, s, b[stp.src], HW, nm.c, ppc, gn_part);
                launch_k(gn_finalize_kernel, n, std::max(32, groups), 0, s, gn_part, nch, nm.c, groups, HW, 1e-5f,
                         gn_stat);
                const size_t n4 = (size_t)n * HW * nm.c / 4;
                launch_k(gn_apply_silu_kernel, (unsigned)((n4 + 255) / 256), 256, 0, s, b[stp.src], gn_stat, nm.g, nm.b,
                         HW, nm.c, groups, n4, b[stp.dst]);
                nl += 3;
                break;
            }
            case Step::ConvOp: {
                const Conv& c = convs[stp.conv];
                ConvArgs a{};
                a.x = b[stp.src]; a.w = c.w; a.bias = c.b; a.resid = stp.resid >= 0 ? b[stp.resid] : nullptr;
                a.y = b[stp.dst]; a.part = part;
                a.H = stp.H; a.W = stp.W; a.IC = c.ic; a.OC = c.oc; a.ks = c.ks; a.up = stp.up;
                a.M = n * HW;
                a.kiters = c.ks * c.ks * c.ic / CBK;
                const int ns = conv_split(a.M, c.oc, a.kiters);
                a.kper = (a.kiters + ns - 1) / ns;
                const int nsu = (a.kiters + a.kper - 1) / a.kper;
                dim3 gr((a.M + CBM - 1) / CBM, (c.oc + CBN - 1) / CBN, nsu);
                if (stp.up) launch_k(conv_simt_kernel<true>, gr, 256, 0, s, a);
                else launch_k(conv_simt_kernel<false>, gr, 256, 0, s, a);
                nl++;
                if (nsu > 1) {
                    const size_t n4 = (size_t)a.M * c.oc / 4;
                    launch_k(conv_splitk_reduce_kernel, (unsigned)((n4 + 255) / 256), 256, 0, s, part, nsu, n4, c.oc,
                             c.b, a.resid, a.y);
                    nl++;
                }
                break;
            }
            case Step::ConvOut: {
                const Conv& c = convs[stp.conv];
                const int M = n * HW;
                const size_t smem = (size_t)c.ks * c.ks * c.ic * kSmallOC * 4;
                launch_k(conv_small_oc_kernel, (unsigned)((M + 127) / 128), 128, smem, s, b[stp.src], c.w, c.b, out, M,
                         stp.H, stp.W, c.ic, c.oc, c.ks);
                nl++;
                break;
            }
            }
        }
        return nl;
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
            ck(cudaStreamEndCapture(cap, &gph), "end capture");
            cudaGraphExec_t ex = nullptr;
            ck(cudaGraphInstantiate(&ex, gph, 0), "instantiate");
            cudaGraphDestroy(gph);
            cudaStreamDestroy(cap);
            it = graphs.emplace(n, ex).first;
        }
        ck(cudaGraphLaunch(it->second, s), "graph launch");
    }
};

namespace {
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
    });
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

int mgc_vqgan_launches(const mgc_vqgan* v) { return v ? v->launches : -1; }

void mgc_vqgan_destroy(mgc_vqgan* v) { delete v; }

}  // extern "C"
