// kernels.h -- internal launch interface between the runtime and the CUDA kernels.
//
// Device layouts (all chosen so every tile a CTA needs is one contiguous, 16-byte aligned
// run that a single cp.async.bulk can move into shared memory in its MMA layout):
//
//   ActQ  quantized activation of an [M][K] f32 tensor, rows padded to Mpad (multiple of 128)
//     q : int8 [K/128][Mpad][128]  -- row r's 128-byte K-chunk, 16-byte groups XOR-swizzled
//                                     by (r % 8) (the tcgen05 128-byte swizzle)
//     d : f32  [K/128][Mpad][4]    -- dx of the 4 32-blocks of each chunk
//     c : f32  [K/128][Mpad][4]    -- dx * sum(qx) per block (only for Q4_K consumers)
//
//   QWeight  quantized [N][K] weight, rows padded to Npad (multiple of 128)
//     q  : int8 (Q8_0) or u8 nibble values 0..15 (Q4_K), [K/128][Npad][128], same swizzle
//     sa : f32 [K/32][Npad]   Q8_0: d (fp16 -> f32);  Q4_K: scl = d * sc_j
//     sb : f32 [K/32][Npad]   Q4_K only: mnl = dmin * m_j
//     f32: for wtype 0 the weight itself, [N][K] row-major
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace mgc {

struct ActQ {
    int8_t* q = nullptr;
    float* d = nullptr;
    float* c = nullptr;
    int Mpad = 0;
};

struct QWeight {
    int wtype = 0, N = 0, K = 0, Npad = 0;
    int8_t* q = nullptr;
    float* sa = nullptr;
    float* sb = nullptr;
    float* f32 = nullptr;
};

inline int round_up(int x, int m) { return (x + m - 1) / m * m; }

// Kernels this library has launched (host-side count, for the runtime's launch report).
extern int g_launch_count;
// A bounded busy-wait kernel of ~`cycles` SM clocks (profiling: lets the host run ahead).
void launch_spin(long long cycles, cudaStream_t st);

// quantizer: x [M][K] f32 -> tiled ActQ (want_c: also write the Q4_K correction term)
void launch_quant_act_tiled(const float* x, int M, int K, const ActQ& a, bool want_c, cudaStream_t st);
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
int launch_qgemm(const QWeight& w, const ActQ& a, int M, const float* bias, int act,
                 const float* resid, float* y, cudaStream_t st, const SplitK* sk = nullptr);
// set the kernels' shared-memory limits on the current device (once per device)
int qgemm_prepare();
int attn_prepare();
// F32 GEMM (SIMT), same epilogue
void launch_gemm_f32(const float* w, const float* x, int M, int N, int K, const float* bias, int act,
                     const float* resid, float* y, cudaStream_t st);
// fp16-K/V flash attention, qkv [B*S][3E] -> out [B*S][E]
// scratch (optional) holds the key-split partials: attn_scratch_floats() floats.
constexpr int kAttnMaxSplit = 4;
size_t attn_scratch_floats(int B, int S, int H);
int launch_flash_attn(const float* qkv, int B, int S, int H, int Dh, float scale, float* out, float* scratch,
                      size_t scratch_floats, cudaStream_t st);

}  // namespace mgc

namespace mgc {
// Set the message mgc_last_error() returns on this thread.
void set_last_error(const char* msg);
}  // namespace mgc

// Handle behind the C ABI's opaque mgc_qweight (include/mgc.h).
struct mgc_qweight { mgc::QWeight w; };
