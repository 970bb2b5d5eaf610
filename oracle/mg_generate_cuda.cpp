// mg_generate_cuda.cpp -- the reference's own decode loop with this repository's CUDA backend,
// wired exactly as INTEGRATION.md's `--backend cuda` branch of tools/main.cpp does it.
// TEST INFRASTRUCTURE: compiled by oracle/Makefile against the UNMODIFIED reference sources
// (Model::load, generate(): src/mg-model.cpp, src/mg-generate.cpp) and libmgcuda.so; the GPU
// tests run it and compare its grid with mgc_generate's.  It shows that the C ABI (through
// include/mgc.hpp) links into, and drives, the reference program unchanged.
//
//   mg_generate_cuda MODEL.gguf CLASS SEED STEPS OUT.bin   -> OUT.bin = the n_tokens grid (int32)
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
    if (argc != 6) {
        std::fprintf(stderr, "usage: %s MODEL.gguf CLASS SEED STEPS OUT.bin\n", argv[0]);
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
        mg::VqganFwd vfwd = [&](const int32_t* g, float*) { std::memcpy(grid.data(), g, sizeof(int32_t) * n_tok); };
        mg::GenConfig cfg;
        cfg.class_id = std::atoi(argv[2]);
        cfg.seed = std::strtoull(argv[3], nullptr, 10);
        cfg.steps = std::atoi(argv[4]);
        mg::GenStats stats;
        mg::generate(*model, cfg, false, fwd, vfwd, &stats, nullptr);
        FILE* f = std::fopen(argv[5], "wb");
        if (!f || std::fwrite(grid.data(), sizeof(int32_t), grid.size(), f) != grid.size()) {
            std::fprintf(stderr, "cannot write %s\n", argv[5]);
            return 1;
        }
        std::fclose(f);
        std::printf("transformer_ms %.3f steps %d\n", stats.transformer_ms, stats.steps);
        return 0;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        return 1;
    }
}
