// kernels.h -- internal launch interface between the runtime and the CUDA kernels.
//
// Device layouts.  Every operand a qGEMM CTA needs for one 4-block K chunk is one contiguous,
// 16-byte aligned run that a single cp.async.bulk moves into shared memory already in the
// tcgen05 128-byte-swizzle layout (three copies per chunk):
//
//   ActQ  quantized activation of an [M][K] f32 tensor, rows padded to Mpad (multiple of 128),
//         as tiles of (128-column K chunk kc, 128-row m-tile mt), tile (kc, mt) at byte
//         ((kc * Mpad/128) + mt) * kActTile:
//     [0, 16384)       int8 codes, row r's 128 bytes at r*128 with 16-byte groups XOR-swizzled
//                      by (r % 8)
//     [16384, 18432)   dx  f32 [128 rows][4 blocks]
//     [18432, 20480)   dx * sum(qx) f32 [128][4] (written only for Q4_K consumers)
//
//   QWeight  quantized [N][K] weight, rows padded to Npad (multiple of 128)
//     Q8_0  q : int8 codes [K/128][Npad][128], same swizzle as the activation codes
//           s : f32 scale tiles [K/128][Npad/4][4 blocks][4 columns] (d) -- BN*4 floats a tile
//     Q4_K  q : packed nibbles [K/128][Npad][64]: the GGUF bytes of each half super-block
//               unchanged (0.5 byte per weight in HBM)
//           s : 16 bytes per row and 128-K chunk, [K/128][Npad][16]: d, dmin (fp16 bits), the
//               chunk's four 6-bit scales, its four 6-bit mins, 4 bytes pad
//           The GEMM kernels unpack a stage in shared memory into the same operand layouts as
//           Q8_0: u8 code tile (128-byte swizzle) and f32 scale tile [BN/4][2][4][4] holding
//           scl = d*sc_j then mnl = dmin*m_j (exact products)
//     f32: for wtype 0 the weight itself, [N][K] row-major
#pragma once
#include <cstdint>
#include <cstdlib>
#include <utility>
#include <cuda_runtime.h>

namespace mgc {

constexpr int kActTile = 20480;

struct ActQ {
    int8_t* q = nullptr;   // tiles as above; Mpad * K * 5/4 bytes
    int Mpad = 0;
};

__host__ __device__ inline size_t act_tile(const ActQ& a, int kc, int m) {
    return ((size_t)kc * (a.Mpad / 128) + (m >> 7)) * kActTile;
}
// byte offset of code k (0..127 within chunk kc) of row m
__host__ __device__ inline size_t act_code(const ActQ& a, int kc, int m, uint32_t k) {
    const uint32_t r = m & 127;
    return act_tile(a, kc, m) + r * 128u + ((((k >> 4) ^ (r & 7u)) << 4) | (k & 15u));
}
__host__ __device__ inline float* act_dx(const ActQ& a, int kc, int m) {   // 4 floats (blocks of kc)
    return reinterpret_cast<float*>(a.q + act_tile(a, kc, m) + 16384 + (m & 127) * 16);
}
__host__ __device__ inline float* act_cx(const ActQ& a, int kc, int m) {
    return reinterpret_cast<float*>(a.q + act_tile(a, kc, m) + 18432 + (m & 127) * 16);
}

struct QWeight {
    int wtype = 0, N = 0, K = 0, Npad = 0;
    int8_t* q = nullptr;
    float* s = nullptr;
    float* f32 = nullptr;
};

inline int round_up(int x, int m) { return (x + m - 1) / m * m; }

// Launch with programmatic dependent launch (the kernel overlaps its prologue with the tail of
// the previous kernel in the stream; every kernel here calls griddep_wait() before reading
// inputs).  Off unless MGC_PDL=1: on the config-1 step it measured slower (408 vs 428 steps/s),
// the step being bound by kernel bodies rather than launch gaps.
inline bool pdl_enabled() {
    static const bool on = [] { const char* e = std::getenv("MGC_PDL"); return e && e[0] == '1'; }();
    return on;
}
// Every kernel runs with the max-shared carveout so consecutive kernels never reconfigure the
// SM's L1 / shared-memory split (set once per kernel and device, on its first launch).
void set_max_shared_carveout(const void* kernel);

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Args&&... args) {
    set_max_shared_carveout((const void*)kernel);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Kernels this library has launched (host-side count, for the runtime's launch report).
extern int g_launch_count;
// A bounded busy-wait kernel of ~`cycles` SM clocks (profiling: lets the host run ahead).
void launch_spin(long long cycles, cudaStream_t st);

// decode-loop sampling: per logits row, softmax over the first CB logits and a categorical draw
// with uniform r[row] (generate(), mg-generate.cpp:87-100) -> sid[row], its probability psid[row]
void launch_sample_codes(const float* logits, int rows, int vocab, int CB, const double* r, int32_t* sid, float* psid,
                         cudaStream_t st);
// quantizer: x [M][K] f32 -> tiled ActQ (want_c: also write the Q4_K correction term)
void launch_quant_act_tiled(const float* x, int M, int K, const ActQ& a, bool want_c, cudaStream_t st);
// LayerNorm (+quantizer) and quantizer over a column-blocked input -- the layout an all-gather
// of column slices produces: columns [g*xw, (g+1)*xw) of row m at x[g*xstride + m*xw + ...].
// false: unsupported width (D <= 2048 for LayerNorm, D % 256 == 0, xw % 8 == 0).
bool launch_ln_blocked(const float* x, int xw, long long xstride, const float* gamma, const float* beta, int rows,
                       int D, float eps, float* y, const ActQ* a, bool want_c, cudaStream_t st);
bool launch_quant_blocked(const float* x, int xw, long long xstride, int M, int K, const ActQ& a, bool want_c,
                          cudaStream_t st);
// quantizer with plain outputs (kernel-level C ABI)
void launch_quant_act_plain(const float* x, int M, int K, int8_t* qx, float* dx, int32_t* sumx,
                            cudaStream_t st);
// LayerNorm-affine over D, optionally fused with the quantizer of its output.
void launch_ln(const float* x, const float* gamma, const float* beta, int rows, int D, float eps,
               float* y, const ActQ* a, bool want_c, cudaStream_t st);
// token + position embedding, optionally followed by LayerNorm-affine (+quantizer).
void launch_embed(const float* tok, int vocab, const float* pos, int E, const int32_t* tokens,
                  int B, int S, float* y, cudaStream_t st);
void launch_embed_ln(const float* tok, int vocab, const float* pos, int E, const int32_t* tokens,
                     int B, int S, const float* gamma, const float* beta, float eps, float* y,
                     const ActQ* a, bool want_c, cudaStream_t st);
// Split-K scratch: partial sums (part_floats floats) and per-tile arrival counters
// (n_counters ints, zero-initialised once; the kernel leaves them at zero again).
struct SplitK {
    float* part = nullptr;
    size_t part_floats = 0;
    int* counters = nullptr;
    int n_counters = 0;
};
// int8-dot GEMM on tcgen05: y = act(W . x + bias) + resid.  sk == nullptr: no split-K.
// qo != nullptr: also quantize y into qo (the quantizer of the next linear layer, bit-identical
// to launch_quant_act_tiled on y; qo_c: write the Q4_K term); y may then be null.
// destination of the attention prep tiles (f16 Q/K/V of B = M/S images, H heads, nt = ceil(S/128))
struct AttnPrepOut { uint8_t* buf; int S, H, nt; };
// resid_ld: row stride of resid (0 = N; a column slice of a wider matrix in tensor-parallel
// layers); qo_n0: global column of this GEMM's first output column inside qo (its K).
int launch_qgemm(const QWeight& w, const ActQ& a, int M, const float* bias, int act,
                 const float* resid, float* y, cudaStream_t st, const SplitK* sk = nullptr,
                 const ActQ* qo = nullptr, bool qo_c = false, const AttnPrepOut* ap = nullptr,
                 int resid_ld = 0, int qo_n0 = 0);
// set the kernels' shared-memory limits on the current device (once per device)
int qgemm_prepare();
int attn_prepare();
// F32 GEMM (SIMT), same epilogue
void launch_gemm_f32(const float* w, const float* x, int M, int N, int K, const float* bias, int act,
                     const float* resid, float* y, cudaStream_t st);
// fp16-K/V flash attention, qkv [B*S][3E] -> out [B*S][E]
// scratch holds the f16 tiles of the prep pass (attn_prep_floats(), required) followed by the
// key-split partials (splitting is used when scratch_floats >= attn_scratch_floats()).
// split_ctas > 0: decide the key split as for a launch of that many CTAs (query tiles x heads x
// images) -- a tensor-parallel rank passes the single-GPU count so its heads split the same way.
constexpr int kAttnMaxSplit = 4;
size_t attn_prep_floats(int B, int S, int H);
size_t attn_scratch_floats(int B, int S, int H);
// qo (optional): when the key range is split, the merge pass also quantizes the output rows
// into qo (*quantized = true); otherwise the caller quantizes.
int launch_flash_attn(const float* qkv, int B, int S, int H, int Dh, float scale, float* out, float* scratch,
                      size_t scratch_floats, cudaStream_t st, const ActQ* qo = nullptr, bool qo_c = false,
                      bool* quantized = nullptr, bool prepped = false,
                      long split_ctas = 0);
// where launch_flash_attn expects the prep tiles inside `scratch` (fill them with a fused
// QKV-GEMM epilogue, then launch with prepped = true)
AttnPrepOut attn_prep_out(float* scratch, int B, int S, int H);

}  // namespace mgc

namespace mgc {
// Set the message mgc_last_error() returns on this thread.
void set_last_error(const char* msg);
}  // namespace mgc

// Handle behind the C ABI's opaque mgc_qweight (include/mgc.h).
struct mgc_qweight { mgc::QWeight w; };
