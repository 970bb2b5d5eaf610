// mgc.hpp -- C++ convenience layer over the C ABI of mgc.h for C++ hosts such as the
// reference's tools/main.cpp.  Header-only; errors become std::runtime_error, the
// reference's convention (its TransformerFwd callbacks throw, include/mg-generate.hpp:15 and
// src/mg-generate.cpp:73-76).
#ifndef MGC_HPP
#define MGC_HPP
#include <cstdint>
#include <functional>
#include <stdexcept>
#include <string>

#include "mgc.h"

namespace mgc {

inline void check(int rc, const char* what) {
    if (rc != 0) throw std::runtime_error(std::string("cuda backend: ") + what + ": " + mgc_last_error());
}

// One transformer runtime on one GPU: owns the uploaded weights, the CUDA stream and graphs.
class Runtime {
public:
    // gguf_path: the same GGUF the reference loads (Q8_0 / Q4_K / F32 linears);
    // max_rows: the largest B*S a forward will see (n_tokens + 1 for the decode loop).
    Runtime(const std::string& gguf_path, int max_rows, int device = 0) {
        check(mgc_runtime_create(gguf_path.c_str(), max_rows, device, &rt_), "runtime_create");
    }
    ~Runtime() { mgc_runtime_destroy(rt_); }
    Runtime(const Runtime&) = delete;
    Runtime& operator=(const Runtime&) = delete;

    // tokens [B*S] int32 -> logits [B*S*vocab] f32, host memory, synchronous.
    void forward(const int32_t* tokens, int B, int S, float* logits) {
        check(mgc_transformer_forward(rt_, tokens, B, S, logits), "transformer_forward");
    }
    // A callable with the shape of mg::TransformerFwd (std::function<void(const int32_t*,
    // float*)>) for one image of S tokens; the Runtime must outlive it.
    std::function<void(const int32_t*, float*)> transformer_fwd(int S) {
        return [this, S](const int32_t* tokens, float* logits) { forward(tokens, 1, S, logits); };
    }
    mgc_runtime* handle() { return rt_; }

private:
    mgc_runtime* rt_ = nullptr;
};

// The VQGAN decoder on one GPU (mgc_vqgan_*).
class Vqgan {
public:
    Vqgan(const std::string& gguf_path, int max_images = 1, int device = 0) {
        check(mgc_vqgan_create(gguf_path.c_str(), max_images, device, &v_), "vqgan_create");
        check(mgc_vqgan_info(v_, &n_tokens_, &resolution_, nullptr), "vqgan_info");
    }
    ~Vqgan() { mgc_vqgan_destroy(v_); }
    Vqgan(const Vqgan&) = delete;
    Vqgan& operator=(const Vqgan&) = delete;

    // grid [n][n_tokens] -> image [n][R][R][3] HWC f32, host memory, synchronous.
    void decode(const int32_t* grid, float* image_hwc, int n = 1) {
        check(mgc_vqgan_decode(v_, grid, n, image_hwc), "vqgan_decode");
    }
    // A callable with the shape of mg::VqganFwd (std::function<void(const int32_t*, float*)>,
    // include/mg-generate.hpp:17); the Vqgan must outlive it.
    std::function<void(const int32_t*, float*)> vqgan_fwd() {
        return [this](const int32_t* grid, float* hwc) { decode(grid, hwc, 1); };
    }
    int resolution() const { return resolution_; }
    int n_tokens() const { return n_tokens_; }
    mgc_vqgan* handle() { return v_; }

private:
    mgc_vqgan* v_ = nullptr;
    int n_tokens_ = 0, resolution_ = 0;
};

}  // namespace mgc
#endif
