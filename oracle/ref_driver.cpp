// ref_driver.cpp -- C entry points over the UNMODIFIED reference mg-core (compiled from
// the reference's own sources where they lie, see oracle/Makefile).  TEST INFRASTRUCTURE:
// used to pin the oracle (mgo.cpp) against the reference itself and as the timed CPU
// baseline.  Nothing in the shipped library uses it.
//
//  mgref_forward : Model::load + build_transformer + mg::compute (the reference's scalar
//                  F32 executor, src/mg-cpu/mg-cpu.cpp), i.e. the reference CPU path.
//                  Its weights must be F32 (mg-cpu cannot read Q8_0/Q4_K), so callers
//                  pass the dequantised twin GGUF.  Named tensors are dumped like
//                  tools/verify-opencl-transformer.cpp:67-85.
//  mgref_vqgan   : Model::load + build_vqgan_decoder (src/mg-vqgan.cpp) + mg::compute on one
//                  token grid; the {W,H,3} image is returned HWC, the order of the VqganFwd
//                  callback (src/mg-generate.cpp:137-140, tools/main.cpp:147-151).
//  mgref_generate: mg::generate (src/mg-generate.cpp) with a caller-supplied transformer
//                  callback and a VQGAN callback that only captures the token grid.
#include "mg-generate.hpp"
#include "mg-model.hpp"
#include "mg-tensor.hpp"
#include "mg-transformer.hpp"
#include "mg-vqgan.hpp"

#include <cstring>
#include <exception>
#include <string>
#include <vector>

static std::string g_ref_err;

extern "C" {

const char* mgref_last_error(void) { return g_ref_err.c_str(); }

int mgref_forward(const char* gguf, const int32_t* tokens, int B, int S, float* logits,
                  float* dump, int n_threads) {
    try {
        mg::Context wctx(64 << 20);
        auto model = mg::Model::load(gguf, wctx);
        mg::Context ctx(3ull << 30);
        mg::Tensor* tok = ctx.tensor2d(mg::Type::I32, S, B);
        std::memcpy(tok->data, tokens, sizeof(int32_t) * B * S);
        mg::Tensor* out = mg::build_transformer(ctx, *model, tok);
        mg::Graph g; g.build_forward(out);
        mg::compute(ctx, g, n_threads);
        std::memcpy(logits, out->data, out->nbytes());
        if (dump) {
            const int L = model->hparams().n_layer;
            std::vector<std::string> order{"embd_post_norm"};
            for (int i = 0; i < L; i++) {
                order.push_back("blk." + std::to_string(i) + ".attn_post");
                order.push_back("blk." + std::to_string(i) + ".ffn_post");
            }
            order.push_back("output_norm"); order.push_back("output_logits");
            size_t off = 0;
            for (auto& nm : order)
                for (mg::Tensor* t : g.nodes)
                    if (t->name == nm) {
                        std::memcpy(reinterpret_cast<char*>(dump) + off, t->data, t->nbytes());
                        off += t->nbytes();
                        break;
                    }
        }
        return 0;
    } catch (const std::exception& e) { g_ref_err = e.what(); return -1; }
}

int mgref_vqgan(const char* gguf, const int32_t* grid, float* hwc) {
    try {
        mg::Context wctx(64 << 20);
        auto model = mg::Model::load(gguf, wctx);
        const int n_tok = model->hparams().n_tokens;
        mg::Context vctx(3ull << 30);
        mg::Tensor* gt = vctx.tensor1d(mg::Type::I32, n_tok);
        std::memcpy(gt->data, grid, sizeof(int32_t) * n_tok);
        mg::Tensor* img = mg::build_vqgan_decoder(vctx, *model, gt);
        mg::Graph g; g.build_forward(img);
        mg::compute(vctx, g, 1);
        const int64_t W = img->ne[0], H = img->ne[1];
        const float* o = static_cast<const float*>(img->data);
        for (int64_t y = 0; y < H; y++)
            for (int64_t x = 0; x < W; x++)
                for (int c = 0; c < 3; c++) hwc[(y * W + x) * 3 + c] = o[x + W * (y + H * c)];
        return 0;
    } catch (const std::exception& e) { g_ref_err = e.what(); return -1; }
}

typedef int (*mgref_fwd_fn)(void* user, const int32_t* tokens, int B, int S, float* logits);

int mgref_generate(const char* gguf, mgref_fwd_fn fwd, void* user, int class_id,
                   unsigned long long seed, int steps, float temperature, int32_t* grid_out) {
    try {
        mg::Context wctx(64 << 20);
        auto model = mg::Model::load(gguf, wctx);
        const int S = model->hparams().n_tokens + 1;
        const int n_tok = model->hparams().n_tokens;
        mg::GenConfig cfg; cfg.class_id = class_id; cfg.steps = steps; cfg.seed = seed;
        cfg.temperature = temperature;
        bool ok = true;
        mg::TransformerFwd tf = [&](const int32_t* t, float* l) {
            if (fwd(user, t, 1, S, l) != 0) ok = false;
        };
        mg::VqganFwd vf = [&](const int32_t* grid, float*) {
            std::memcpy(grid_out, grid, sizeof(int32_t) * n_tok);
        };
        mg::generate(*model, cfg, false, tf, vf, nullptr, nullptr);
        if (!ok) { g_ref_err = "transformer callback failed"; return -1; }
        return 0;
    } catch (const std::exception& e) { g_ref_err = e.what(); return -1; }
}

}  // extern "C"
