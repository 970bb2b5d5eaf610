// noalloc.cu -- mgc_qgemm_noalloc: the quantized linear layer for callers that may not
// allocate device memory.
//
// Some hosts embed this library where cudaMalloc is off limits: a custom allocator owns
// all device memory (an inference server with a fixed memory pool), or the call runs in a
// context whose rules forbid allocation after start-up (real-time or safety-certified
// code, plugin hosts that audit allocations).  mgc_qgemm needs scratch for the quantized
// activation and grows a library buffer with cudaMalloc on demand; this entry point
// instead uses a fixed scratch array compiled into the library, so it never allocates.
#include "../../include/mgc.h"
#include "kernels.h"

#include <cstdio>
#include <mutex>
#include <string>

namespace {

// Fixed scratch for the quantized activation, in the tile layout of kernels.h: per 128 x 128
// tile the int8 codes, then the per-block scales and the Q4_K correction terms (20480 bytes
// per 16384 codes).  MGC_NOALLOC_MAX_ELEMS bounds Mpad*K (Mpad = M rounded up to 128).
// Every GPU that loads the library holds these bytes until the process exits.
constexpr size_t kMaxElems = MGC_NOALLOC_MAX_ELEMS;
constexpr size_t kScratchBytes = kMaxElems / 16384 * mgc::kActTile;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_mu;

// Errors are reported through mgc_last_error(), like every other entry point.
int fail(const std::string& m) { mgc::set_last_error(m.c_str()); return -1; }

}  // namespace

extern "C" int mgc_qgemm_noalloc(const mgc_qweight* wq, const float* x_dev, int M, const float* bias_dev,
                                 int act, const float* resid_dev, float* y_dev, void* stream) {
    if (!wq || !x_dev || !y_dev || M <= 0) return fail("mgc_qgemm_noalloc: bad arguments");
    const mgc::QWeight& w = wq->w;
    if (w.wtype != MGC_Q8_0 && w.wtype != MGC_Q4_K) {
        return fail("mgc_qgemm_noalloc: weight must be Q8_0 or Q4_K");
    }
    if (w.K % 128 != 0 || (w.wtype == MGC_Q4_K && w.K % 256 != 0)) {
        return fail("mgc_qgemm_noalloc: unsupported shape K = " + std::to_string(w.K) +
                    " (K must be a multiple of 128, 256 for Q4_K)");
    }
    const int Mpad = mgc::round_up(M, 128);
    if ((size_t)Mpad * (size_t)w.K > kMaxElems) {
        return fail("mgc_qgemm_noalloc: round_up(M,128) * K = " + std::to_string((size_t)Mpad * w.K) +
                    " exceeds the fixed scratch limit MGC_NOALLOC_MAX_ELEMS = " + std::to_string(kMaxElems));
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        return fail("mgc_qgemm_noalloc: no usable current device");
    }
    void* base;
    {
        // First call on a device: resolve the scratch array's device address (the symbol's
        // host-side name is not a device pointer).  Make this first call before any stream
        // capture.  The address is cached for the life of the process: after a
        // cudaDeviceReset the module is reloaded and the array may move, so the library must
        // not be used across a device reset.
        std::lock_guard<std::mutex> lk(g_mu);
        if (!g_scratch_ptr[dev]) {
            void* p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
            if (e != cudaSuccess || !p) {
                return fail(std::string("mgc_qgemm_noalloc: cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
            }
            g_scratch_ptr[dev] = p;
        }
        base = g_scratch_ptr[dev];
    }
    mgc::ActQ a;
    a.Mpad = Mpad;
    a.q = (int8_t*)base;
    cudaStream_t st = (cudaStream_t)stream;
    // An error left by earlier, unrelated work is reported as such, not as this call's failure.
    const cudaError_t prior = cudaGetLastError();
    if (prior != cudaSuccess) {
        return fail(std::string("mgc_qgemm_noalloc: a CUDA error was pending before this call: ") +
                    cudaGetErrorString(prior));
    }
    mgc::launch_quant_act_tiled(x_dev, M, w.K, a, w.wtype == MGC_Q4_K, st);
    const cudaError_t eq = cudaGetLastError();
    if (eq != cudaSuccess) {
        return fail(std::string("mgc_qgemm_noalloc: quantizer launch failed: ") + cudaGetErrorString(eq));
    }
    const int rc = mgc::launch_qgemm(w, a, M, bias_dev, act, resid_dev, y_dev, st);
    if (rc == -2) {
        return fail("mgc_qgemm_noalloc: unsupported GEMM configuration M = " + std::to_string(M) + ", N = " +
                    std::to_string(w.N) + ", K = " + std::to_string(w.K));
    }
    if (rc != 0) {
        return fail(std::string("mgc_qgemm_noalloc: GEMM launch failed: ") + cudaGetErrorString(cudaGetLastError()));
    }
    return 0;
}
