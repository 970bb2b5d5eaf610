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

}  // namespace mgc
#endif
