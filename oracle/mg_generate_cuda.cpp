// mg_generate_cuda.cpp -- the reference's own decode loop with this repository's CUDA backend,
// wired exactly as INTEGRATION.md's `--backend cuda` branch of tools/main.cpp does it.
// TEST INFRASTRUCTURE: compiled by oracle/Makefile against the UNMODIFIED reference sources
// (Model::load, generate(): src/mg-model.cpp, src/mg-generate.cpp) and libmgcuda.so; the GPU
// tests run it and compare its grid with mgc_generate's.  It shows that the C ABI (through
// include/mgc.hpp) links into, and drives, the reference program unchanged.
//
//   mg_generate_cuda MODEL.gguf CLASS SEED STEPS OUT.bin [IMAGE.bin [RGB.bin]]
//     OUT.bin   = the n_tokens grid (int32)
//     IMAGE.bin = the decoded image, HWC f32 [R][R][3], from the CUDA VQGAN decoder as the
//                 VqganFwd callback (given only for a GGUF that carries the decoder)
//     RGB.bin   = the bytes of the mg::Image that generate() returns
#include "mg-generate.hpp"
#include "mg-model.hpp"
#include "mg-tensor.hpp"
#include "mgc.hpp"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <memory>
#include <vector>

int main(int argc, char** argv) {
    if (argc < 6 || argc > 8) {
        std::fprintf(stderr, "usage: %s MODEL.gguf CLASS SEED STEPS OUT.bin [IMAGE.bin [RGB.bin]]\n", argv[0]);
        return 2;
    }
    try {
        mg::Context wctx(64 << 20);
        auto model = mg::Model::load(argv[1], wctx);
        const int S = model->hparams().n_tokens + 1;
        const int n_tok = model->hparams().n_tokens;
        // the `--backend cuda` branch: a runtime on GPU 0 and its TransformerFwd
        mgc::Runtime rt(argv[1], S, 0);
        mg::TransformerFwd fwd = rt.transformer_fwd(S);
        std::vector<int32_t> grid(n_tok);
        // and, with IMAGE.bin, the VQGAN decoder's VqganFwd
        std::unique_ptr<mgc::Vqgan> vq;
        if (argc >= 7) vq.reset(new mgc::Vqgan(argv[1], 1, 0));
        std::vector<float> image;
        mg::VqganFwd vq_fwd = vq ? vq->vqgan_fwd() : mg::VqganFwd();
        mg::VqganFwd vfwd = [&](const int32_t* g, float* hwc) {
            std::memcpy(grid.data(), g, sizeof(int32_t) * n_tok);
            if (vq_fwd) {
                vq_fwd(g, hwc);
                image.assign(hwc, hwc + (size_t)vq->resolution() * vq->resolution() * 3);
            }
        };
        mg::GenConfig cfg;
        cfg.class_id = std::atoi(argv[2]);
        cfg.seed = std::strtoull(argv[3], nullptr, 10);
        cfg.steps = std::atoi(argv[4]);
        mg::GenStats stats;
        const mg::Image img = mg::generate(*model, cfg, false, fwd, vfwd, &stats, nullptr);
        FILE* f = std::fopen(argv[5], "wb");
        if (!f || std::fwrite(grid.data(), sizeof(int32_t), grid.size(), f) != grid.size()) {
            std::fprintf(stderr, "cannot write %s\n", argv[5]);
            return 1;
        }
        std::fclose(f);
        if (vq) {
            FILE* fi = std::fopen(argv[6], "wb");
            if (!fi || std::fwrite(image.data(), sizeof(float), image.size(), fi) != image.size()) {
                std::fprintf(stderr, "cannot write %s\n", argv[6]);
                return 1;
            }
            std::fclose(fi);
        }
        if (argc == 8) {
            FILE* fr = std::fopen(argv[7], "wb");
            if (!fr || std::fwrite(img.rgb.data(), 1, img.rgb.size(), fr) != img.rgb.size()) {
                std::fprintf(stderr, "cannot write %s\n", argv[7]);
                return 1;
            }
            std::fclose(fr);
        }
        std::printf("transformer_ms %.3f steps %d\n", stats.transformer_ms, stats.steps);
        return 0;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        return 1;
    }
}
