/* mgo.h -- CPU restatement ("oracle") of edge_maskgit's quantized transformer hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library links, loads or calls this
 * code; it is the checker that the CUDA path is compared against.  Only tests/, the
 * smoke() check in __graft_entry__.py and the cpu_baseline / reference legs of bench.py
 * use it.
 *
 * Every function restates one piece of the reference (chenxugz/edge_maskgit) and cites the
 * file:line it follows.  Conventions:
 *   - activations are row-major [rows][K] f32 (the reference's x[m*K + k]);
 *   - weights are the raw GGUF block bytes, rows [N][K/32]x34 B (Q8_0) or
 *     [N][K/256]x144 B (Q4_K), exactly as tools/convert_to_gguf.py writes them;
 *   - all float arithmetic is IEEE single precision, compiled with -ffp-contract=off, and
 *     every place the reference's OpenCL compiler may contract a*b+c is written as an
 *     explicit fmaf() so the CUDA kernels can reproduce it bit for bit.
 */
#ifndef MGO_H
#define MGO_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- fp16 helpers (IEEE binary16, round to nearest even) ---- */
float    mgo_f16_to_f32(uint16_t h);
uint16_t mgo_f32_to_f16(float f);

/* ---- weight packers: tools/convert_to_gguf.py:109-124 (Q8_0) and :68-106 (Q4_K) ---- */
void mgo_pack_q8_0(const float* w, int64_t N, int64_t K, uint8_t* out);
void mgo_pack_q4_k(const float* w, int64_t N, int64_t K, uint8_t* out);
/* dequant formulas: DEQ_Q8 mg-opencl.cpp:386-387, deq_q4k_elem mg-opencl.cpp:252-262 */
void mgo_dequant(int wtype, const uint8_t* w, int64_t N, int64_t K, float* out);

/* ---- activation quantizer: k_quantize_q8, mg-opencl.cpp:424-434 ----
 * qx int8 [M][K], dx f32 [M][K/32]; sumx (optional, may be NULL) int32 [M][K/32] is the
 * per-block sum of qx that k_mul_mat_q4k_i8 forms at mg-opencl.cpp:561-565. */
void mgo_quantize_act(const float* x, int64_t M, int64_t K, int8_t* qx, float* dx, int32_t* sumx);

/* ---- int8-dot GEMM: k_mul_mat_q8_i8 mg-opencl.cpp:440-494 / k_mul_mat_q4k_i8 :504-590 ----
 * wtype 8 = Q8_0, 12 = Q4_K.  y[m*N+n] = act(acc + bias[n]) + resid[m*N+n]; act 0 none,
 * 1 erf-GELU (mg-opencl.cpp:36-40), 2 SiLU.  bias / resid may be NULL.
 * Per block b (ascending):  Q8_0: acc = fmaf(dw*dx, (float)idot, acc)
 *                           Q4_K (mg-opencl.cpp:572, difference first):
 *                                 t = fmaf(scl*dx, (float)idot, -((mnl*dx)*(float)sumx));
 *                                 acc = acc + t
 * idot_out (optional) receives the raw int32 block dots [M][N][K/32]. */
void mgo_qgemm(int wtype, const uint8_t* w, const int8_t* qx, const float* dx,
               const int32_t* sumx, int64_t M, int64_t N, int64_t K,
               const float* bias, int act, const float* resid, float* y, int32_t* idot_out);
/* The same GEMM in the order the CUDA kernel accumulates Q4_K (Q8_0 is identical):
 *   acc = fmaf(scl*dx, (float)idot, acc); acc = fmaf(-mnl, dx*(float)sumx, acc)
 * -- two roundings into acc instead of one.  Used to check the kernel bit for bit; the
 * kernel is checked against mgo_qgemm within a tolerance. */
void mgo_qgemm_fused(int wtype, const uint8_t* w, const int8_t* qx, const float* dx,
                     const int32_t* sumx, int64_t M, int64_t N, int64_t K,
                     const float* bias, int act, const float* resid, float* y, int32_t* idot_out);

/* F32 GEMM with the same fused epilogue (k_mul_mat_t, mg-opencl.cpp:57-98): the MLM head.
 * w [N][K] f32 row-major.  acc = fmaf(w, x, acc) over k ascending. */
void mgo_gemm_f32(const float* w, const float* x, int64_t M, int64_t N, int64_t K,
                  const float* bias, int act, const float* resid, float* y);

/* LayerNorm + affine over D: k_norm_affine mg-opencl.cpp:705-727 (64-lane strided partial
 * sums, shared-memory tree, then (x-mean)*inv*gamma+beta as one fmaf). */
void mgo_layernorm_affine(const float* x, const float* gamma, const float* beta,
                          int64_t rows, int64_t D, float eps, float* y);

/* fp16-K/V flash attention: k_flash_attention_h mg-opencl.cpp:859-937.  qkv is the fused
 * projection output [B*S][3*H*Dh] (q | k | v column blocks); out is [B*S][H*Dh] (heads
 * merged, i.e. after the permute+cont of mg-transformer.cpp:84). */
void mgo_flash_attn(const float* qkv, int64_t B, int64_t S, int64_t H, int64_t Dh,
                    float scale, float* out);

/* token + position embedding: k_get_rows mg-opencl.cpp:667-672 + k_add :947-953 */
void mgo_embed(const float* tok_embd, int64_t vocab, const float* pos_embd, int64_t E,
               const int32_t* tokens, int64_t B, int64_t S, float* out);

/* ---- whole-model oracle (build_transformer, mg-transformer.cpp:32-111) ---- */
typedef struct mgo_model mgo_model;
mgo_model* mgo_model_load(const char* gguf_path);   /* NULL on error, see mgo_last_error */
void       mgo_model_free(mgo_model*);
const char* mgo_last_error(void);
/* hparams: n_layer n_head n_embd n_ffn head_dim vocab n_tokens mask_id codebook wtype */
void       mgo_model_hparams(const mgo_model*, int32_t out[10]);
/* tokens [B][S] -> logits [B*S][vocab].  dump (optional) receives the 51 named tensors
 * in order embd_post_norm, blk.i.attn_post, blk.i.ffn_post (i ascending), output_norm,
 * output_logits, each [B*S][width] f32, concatenated. */
int  mgo_forward(mgo_model*, const int32_t* tokens, int B, int S, float* logits, float* dump);

/* ---- decode loop: generate() mg-generate.cpp:39-123 (sampling part; VQGAN excluded) ----
 * fwd(user, tokens[B*S], logits[B*S*vocab]) is the transformer callback.  Image i uses
 * class_ids[i] and its own std::mt19937_64(seeds[i]).  tokens_out [B][S] receives
 * `result` (the final sampled sequence incl. class token) per image. */
typedef int (*mgo_fwd_fn)(void* user, const int32_t* tokens, int B, int S, float* logits);
int  mgo_generate(const mgo_model*, mgo_fwd_fn fwd, void* user, int B,
                  const int32_t* class_ids, const uint64_t* seeds, int steps,
                  float temperature, int32_t* tokens_out);
/* convenience forward callback bound to the oracle model (user = mgo_model*) */
int  mgo_forward_cb(void* user, const int32_t* tokens, int B, int S, float* logits);

#ifdef __cplusplus
}
#endif
#endif
