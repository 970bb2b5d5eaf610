/* mgc.h -- C ABI of libmgcuda.so, the B200 (sm_100a) backend for edge_maskgit's quantized
 * MaskGIT transformer.
 *
 * Conventions
 *   - Every entry point returns int: 0 on success, <0 on error; mgc_last_error() then
 *     returns a message (thread-local, valid until the next call on that thread).
 *   - "dev" pointers are CUDA device pointers; "host" pointers are ordinary host memory.
 *   - stream is a cudaStream_t passed as void* (NULL = the legacy default stream).
 *   - Layouts follow the reference's row-major activation convention x[m*K + k]
 *     (ggml ne = {K, M}); weight bytes are the GGUF Q8_0 / Q4_K blocks unchanged.
 *   - wtype codes are GGML's: 0 = F32, 8 = Q8_0, 12 = Q4_K.
 */
#ifndef MGC_H
#define MGC_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MGC_F32 0
#define MGC_Q8_0 8
#define MGC_Q4_K 12

const char* mgc_last_error(void);
/* Reads and clears the device-side error word written by bounded waits inside kernels
 * (0 = none).  A non-zero value means a kernel gave up waiting and returned early. */
int mgc_device_error(void);
/* Self-test of that path: one kernel waits on an mbarrier nothing arrives on, gives up after
 * the wait limit (~2 s), records `code` (> 0) in the device error word and returns; the call
 * syncs `stream`.  mgc_device_error() then returns `code`, and the context stays usable. */
int mgc_selftest_wait_timeout(int code, void* stream);

/* ------------------------------------------------------------------ weight packing (host)
 * Replaces tools/convert_to_gguf.py quant_q8_0 (:109-124) and quant_q4_k (:68-106):
 * w [N][K] f32 row-major -> GGUF block bytes (N*K/32*34 or N*K/256*144 bytes). */
int mgc_pack_q8_0(const float* w_host, int64_t N, int64_t K, uint8_t* out_host);
int mgc_pack_q4_k(const float* w_host, int64_t N, int64_t K, uint8_t* out_host);
/* Dequantise GGUF blocks to f32 with the reference formulas DEQ_Q8 / deq_q4k_elem
 * (src/mg-opencl/mg-opencl.cpp:386-387, :252-262). */
int mgc_dequant(int wtype, const uint8_t* w_host, int64_t N, int64_t K, float* out_host);

/* ------------------------------------------------------------------ kernel-level ops
 * Replaces k_quantize_q8 (mg-opencl.cpp:424-434, dispatched at :1386-1389):
 * x dev [M][K] f32 -> qx dev [M][K] int8, dx dev [M][K/32] f32, sumx dev [M][K/32] int32
 * (sumx may be NULL). */
int mgc_quantize_act(const float* x_dev, int M, int K, int8_t* qx_dev, float* dx_dev,
                     int32_t* sumx_dev, void* stream);

/* A quantized weight resident on the device in the GEMM's streaming layout. */
typedef struct mgc_qweight mgc_qweight;
/* Upload GGUF blocks (host) of an [N][K] weight; wtype 8 or 12 (0 = F32 row-major).
 * K must be a multiple of 128 (256 for Q4_K). */
int mgc_qweight_create(int wtype, const void* w_host, int N, int K, mgc_qweight** out);
void mgc_qweight_destroy(mgc_qweight* w);

/* Quantized linear layer, the MulMat(Q8_0 | Q4_K) dispatch of mg-opencl.cpp:1381-1399
 * (k_quantize_q8 + k_mul_mat_q8_i8 / k_mul_mat_q4k_i8):
 *   y[m*N+n] = act(sum_b dw*dx*idot_b + bias[n]) + resid[m*N+n]
 * x, bias, resid, y are device f32; bias / resid may be NULL; act 0 none, 1 erf-GELU,
 * 2 SiLU.  Uses a per-library scratch for the quantized activation. */
int mgc_qgemm(const mgc_qweight* w, const float* x_dev, int M, const float* bias_dev,
              int act, const float* resid_dev, float* y_dev, void* stream);

/* Upper bound on round_up(M, 128) * K for mgc_qgemm_noalloc: 6 Mi elements, i.e. a fixed
 * 7.5 MiB device array (int8 codes plus two f32 per 32-block) held by every GPU that loads
 * the library, for as long as the process lives. */
#define MGC_NOALLOC_MAX_ELEMS 6291456

/* No counterpart in the reference.  mgc_qgemm for callers that are not allowed to allocate
 * device memory (a host whose pool allocator owns all GPU memory, or code that may not
 * allocate after start-up): same inputs, outputs and results as mgc_qgemm, but the
 * quantized-activation scratch is a fixed array compiled into the library, so the call
 * makes no cudaMalloc / cudaFree.  Returns <0 with a clear message if
 * round_up(M,128) * K > MGC_NOALLOC_MAX_ELEMS, or for an F32 weight.  The first call on
 * each device looks up the array's device address; make that first call before any
 * stream capture.  All calls share the one array and it keeps the previous call's
 * contents (nothing in it needs to start at zero), so calls that can overlap on the GPU --
 * different streams, or different host threads -- race on it: serialise them.  The looked-up
 * address is kept for the life of the process; do not call this after a cudaDeviceReset. */
int mgc_qgemm_noalloc(const mgc_qweight* w, const float* x_dev, int M, const float* bias_dev,
                      int act, const float* resid_dev, float* y_dev, void* stream);

/* F32 linear with the same epilogue (k_mul_mat_t, mg-opencl.cpp:57-98; the MLM head at
 * mg-transformer.cpp:107-108).  w dev [N][K] f32 row-major. */
int mgc_gemm_f32(const float* w_dev, const float* x_dev, int M, int N, int K,
                 const float* bias_dev, int act, const float* resid_dev, float* y_dev,
                 void* stream);

/* LayerNorm + affine over D (k_norm_affine, mg-opencl.cpp:705-727; dispatch :1450-1465).
 * D must be a multiple of 64 and <= 2048. */
int mgc_layernorm_affine(const float* x_dev, const float* gamma_dev, const float* beta_dev,
                         int rows, int D, float eps, float* y_dev, void* stream);

/* fp16-K/V flash attention (k_flash_attention_h, mg-opencl.cpp:859-937; dispatch
 * :1483-1511).  qkv dev [B*S][3*H*Dh] f32 holds the q | k | v projections side by side;
 * out dev [B*S][H*Dh] f32 is the head-merged result (mg-transformer.cpp:84-85).
 * Dh must be 48. */
int mgc_flash_attn(const float* qkv_dev, int B, int S, int H, int Dh, float scale,
                   float* out_dev, void* stream);

/* Token + position embedding (k_get_rows mg-opencl.cpp:667-672 and k_add :947-953). */
int mgc_embed(const float* tok_embd_dev, int vocab, const float* pos_embd_dev, int E,
              const int32_t* tokens_dev, int B, int S, float* out_dev, void* stream);

/* ------------------------------------------------------------------ runtime
 * The CUDA counterpart of mg::OpenCLRuntime (include/mg-opencl.hpp:23-58) specialised to
 * the MaskGIT transformer graph of src/mg-transformer.cpp:32-111. */
typedef struct mgc_runtime mgc_runtime;
/* Load a GGUF (mg-model.cpp:139-201 format), upload and repack every weight.
 * max_rows = largest B*S a forward will see. device = CUDA ordinal.  The runtime owns one
 * CUDA stream and three host threads that copy logits out during mgc_transformer_forward. */
int mgc_runtime_create(const char* gguf_path, int max_rows, int device, mgc_runtime** out);
void mgc_runtime_destroy(mgc_runtime* rt);

/* Column-split tensor parallelism over `world` GPUs, one process (or thread) per rank, all
 * ranks creating their runtime concurrently and then calling every forward with the same
 * arguments (the long-sequence step: batch 4 x 4097 tokens; no counterpart in the reference,
 * which runs on one device).  Rank r holds heads [r*H/G, (r+1)*H/G) of q|k|v, rows
 * [r*E/G, (r+1)*E/G) of attn_o and ffn_down, rows [r*F/G, ...) of ffn_up and a 1/G slice of
 * the MLM head; NCCL all-gathers (loaded with dlopen on first use) join the slices.  Every rank
 * returns the full logits, equal to the single-GPU runtime's.  n_head and n_ffn/128 must be
 * divisible by world.  id: 128 bytes from mgc_tp_unique_id on one rank, shared by the host. */
int mgc_tp_unique_id(uint8_t id_out[128]);
int mgc_runtime_create_tp(const char* gguf_path, int max_rows, int device, int rank, int world,
                          const uint8_t id[128], mgc_runtime** out);
/* n_layer n_head n_embd n_ffn head_dim vocab n_tokens mask_id codebook wtype */
int mgc_runtime_hparams(const mgc_runtime* rt, int32_t out[10]);
const char* mgc_runtime_device_name(const mgc_runtime* rt);

/* The TransformerFwd callback (include/mg-generate.hpp:15): tokens host [B*S] int32 ->
 * logits host [B*S*vocab] f32, row-major s-outer / v-inner; synchronous.  The logits come back
 * in four row chunks, each copied to `logits` by its own host thread as its DMA lands. */
int mgc_transformer_forward(mgc_runtime* rt, const int32_t* tokens_host, int B, int S,
                            float* logits_host);
/* Same forward with device buffers, enqueued on the runtime's stream (replayed from a
 * CUDA graph captured on first use for each (B, S)).  Not synchronised on return. */
int mgc_transformer_forward_dev(mgc_runtime* rt, const int32_t* tokens_dev, int B, int S,
                                float* logits_dev);
/* Forward that also copies the 51 named verification tensors (the MG_DUMP_NAMED hook of
 * mg-opencl.cpp:1631-1641): embd_post_norm, blk.i.attn_post, blk.i.ffn_post, output_norm,
 * output_logits, each [B*S][width] f32, concatenated into dump_host. */
int mgc_transformer_forward_dump(mgc_runtime* rt, const int32_t* tokens_host, int B, int S,
                                 float* logits_host, float* dump_host);
/* Synchronise the runtime's stream. */
int mgc_runtime_sync(mgc_runtime* rt);
/* Raw cudaStream_t of the runtime. */
void* mgc_runtime_stream(mgc_runtime* rt);

/* Decode loop (generate(), src/mg-generate.cpp:53-123, without the VQGAN): B independent
 * images, image i with class_ids[i] and std::mt19937_64(seeds[i]); forwards are batched.
 * The per-position softmax and categorical draw run on the device (the host draws the
 * uniforms in the reference's order; only the sampled codes and their probabilities come
 * back), the confidence / re-mask step on the host.
 * tokens_out host [B][S] = the final sampled sequence (class token first). */
int mgc_generate(mgc_runtime* rt, int B, const int32_t* class_ids, const uint64_t* seeds,
                 int steps, float temperature, int32_t* tokens_out);

/* Number of kernels the runtime's last forward enqueued (all are this library's own). */
int mgc_runtime_kernel_count(const mgc_runtime* rt);

/* Times one op class of the forward as it runs inside the step: captures a CUDA graph of the
 * forward's launches of that class only (op = a name of mgc_profile_report, e.g. "MulMat(q)"),
 * on the runtime's own buffers (their contents are whatever the last forward left), replays it
 * `iters` times between CUDA events and returns the mean milliseconds per replay; *launches
 * (optional) = kernels per replay.  No counterpart in the reference (it is the live, in-graph
 * counterpart of the per-op profile of mg-opencl.hpp:50-53). */
int mgc_runtime_time_op(mgc_runtime* rt, const char* op, int B, int S, int iters, float* ms_per_replay,
                        int* launches);

/* Per-op-type profile (OpenCLRuntime::profile_enable/reset/report, mg-opencl.hpp:50-53).
 * When enabled, forwards run eagerly with CUDA events around each kernel. */
int mgc_profile_enable(mgc_runtime* rt, int on);
int mgc_profile_reset(mgc_runtime* rt);
/* Writes "name count ms\n" lines (descending by ms) into buf (NUL-terminated). */
int mgc_profile_report(mgc_runtime* rt, char* buf, size_t buflen);

/* ---------------------------------------------------------------- VQGAN decoder
 * The CUDA counterpart of build_vqgan_decoder + compute (include/mg-vqgan.hpp:12,
 * src/mg-vqgan.cpp:67-108) behind the reference's VqganFwd callback
 * (include/mg-generate.hpp:17: grid [n_tokens] -> HWC float [R][R][3]).  The GGUF must carry
 * the vqgan.* tensors (F32) and the maskgit.vqgan.* keys (tools/convert_to_gguf.py:203-208).
 * Activations are NHWC f32 on the device; the whole decode is one CUDA graph per image count. */
typedef struct mgc_vqgan mgc_vqgan;
/* Loads the decoder onto `device` with buffers for up to max_images grids per call. */
int mgc_vqgan_create(const char* gguf_path, int max_images, int device, mgc_vqgan** out);
/* n_tokens of one grid, output resolution R, codebook size (any pointer may be null). */
int mgc_vqgan_info(const mgc_vqgan* v, int* n_tokens, int* resolution, int* codebook_size);
/* Host grid [n_images][n_tokens] (ids in [0, codebook_size), else -1 and nothing runs) ->
 * host image [n_images][R][R][3] f32, unclamped (mg-generate.cpp:141-144 clamps when it makes
 * bytes).  Synchronous.  Grid cell p = y * sqrt(n_tokens) + x.  Returns -1 if a kernel gave up
 * a bounded wait (the device error word, read and cleared). */
int mgc_vqgan_decode(mgc_vqgan* v, const int32_t* grid, int n_images, float* image_hwc);
/* The same, returned as the bytes of the reference's mg::Image (mg-generate.cpp:141-144:
 * clamp to [0, 1], * 255 + 0.5, truncated), host rgb [n_images][R][R][3] uint8. */
int mgc_vqgan_decode_rgb8(mgc_vqgan* v, const int32_t* grid, int n_images, uint8_t* rgb);
/* The whole of mg::generate (src/mg-generate.cpp:39-171) for B images: the decode loop of
 * mgc_generate on rt, then each final grid (class token dropped) through the VQGAN decoder in
 * batches of v's max_images, as mgc_vqgan_decode_rgb8.  rgb host [B][R][R][3] uint8;
 * tokens_out (optional) host [B][n_tokens + 1] as mgc_generate. */
int mgc_generate_images(mgc_runtime* rt, mgc_vqgan* v, int B, const int32_t* class_ids, const uint64_t* seeds,
                        int steps, float temperature, uint8_t* rgb, int32_t* tokens_out);
/* The same on device buffers, enqueued on `stream` (null = legacy default stream) without a
 * sync; ids outside the codebook decode as a zero latent. */
int mgc_vqgan_decode_device(mgc_vqgan* v, const int32_t* grid_dev, int n_images, float* image_dev,
                            void* stream);
/* Kernels the last decode launched (all this library's own). */
int mgc_vqgan_launches(const mgc_vqgan* v);
/* Times one kernel class of the decode as it runs inside it: a CUDA graph of that class's
 * launches only for n_images (op: "conv_tc", "conv_simt", "conv_out", "splitk_reduce",
 * "groupnorm", "split", "gather" or "all"), on the decoder's own buffers, replayed `iters`
 * times between CUDA events on its stream; *ms_per_replay = mean ms, *launches (optional) =
 * kernels per replay. */
int mgc_vqgan_time_op(mgc_vqgan* v, const char* op, int n_images, int iters, float* ms_per_replay,
                      int* launches);
void mgc_vqgan_destroy(mgc_vqgan* v);

#ifdef __cplusplus
}
#endif
#endif
