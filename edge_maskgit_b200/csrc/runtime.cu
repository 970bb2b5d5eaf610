// runtime.cu -- the C ABI of libmgcuda.so: kernel-level entry points, the GGUF-backed
// transformer runtime (the CUDA counterpart of mg::OpenCLRuntime, include/mg-opencl.hpp),
// and the decode loop of src/mg-generate.cpp.
#include "../../include/mgc.h"
#include "gguf.h"
#include "kernels.h"
#include "pack.h"
#include "ptx.cuh"
#include "tp.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <condition_variable>
#include <map>
#include <mutex>
#include <memory>
#include <random>
#include <set>
#include <stdexcept>
#include <string>
#include <thread>
#include <tuple>
#include <unordered_map>
#include <vector>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace mgc {
__device__ int g_dev_error = 0;
int g_launch_count = 0;

__global__ void spin_kernel(long long cycles) {
    const long long t0 = clock64();
    while (clock64() - t0 < cycles) {}
}
void launch_spin(long long cycles, cudaStream_t st) { spin_kernel<<<1, 1, 0, st>>>(cycles); }

// Self-test of the bounded-wait path every pipelined kernel uses: waits on an mbarrier that
// nothing arrives on.  mbar_wait gives up after its cycle limit (~2 s), records `code` in the
// device error word and returns, so the kernel ends and the context stays usable.
__global__ void wait_timeout_selftest_kernel(int code) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x != 0) return;
    abort_flag = 0;
    mbar_init(&bar, 1);
    mbar_fence_init();
    mbar_wait(&bar, 0, (volatile int*)&abort_flag, code);
}

void set_max_shared_carveout(const void* kernel) {
    static std::mutex mu;
    static std::set<std::pair<const void*, int>> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    if (done.insert({kernel, dev}).second)
        cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
}
}

using namespace mgc;

namespace {

thread_local std::string g_err;

struct Err : std::runtime_error { using std::runtime_error::runtime_error; };

#define CK(call)                                                                        \
    do {                                                                                \
        cudaError_t e_ = (call);                                                        \
        if (e_ != cudaSuccess)                                                          \
            throw Err(std::string(#call) + ": " + cudaGetErrorString(e_));              \
    } while (0)

template <class F>
int guard(F&& f) {
    try { f(); return 0; }
    catch (const std::exception& e) { g_err = e.what(); return -1; }
}

template <class T>
T* dalloc(size_t n) {
    void* p = nullptr;
    CK(cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)));
    return (T*)p;
}
template <class T>
T* dupload(const T* h, size_t n) {
    T* d = dalloc<T>(n);
    CK(cudaMemcpy(d, h, n * sizeof(T), cudaMemcpyHostToDevice));
    return d;
}

// Upload an [N][K] weight given as GGUF bytes (Q8_0 / Q4_K blocks, or row-major F32).
QWeight upload_weight(int wtype, const void* host, int N, int K) {
    QWeight w;
    w.wtype = wtype; w.N = N; w.K = K;
    if (wtype == 0) { w.f32 = dupload((const float*)host, (size_t)N * K); return w; }
    if (wtype != 8 && wtype != 12) throw Err("unsupported weight type " + std::to_string(wtype));
    if (K % 128 != 0 || (wtype == 12 && K % 256 != 0)) throw Err("qweight: K must be a multiple of 128 (256 for Q4_K)");
    w.Npad = round_up(N, 128);
    std::vector<int8_t> q; std::vector<float> sc;
    repack(wtype, (const uint8_t*)host, N, K, w.Npad, q, sc);
    w.q = dupload(q.data(), q.size());
    w.s = dupload(sc.data(), sc.size());
    return w;
}
void free_weight(QWeight& w) {
    cudaFree(w.q); cudaFree(w.s); cudaFree(w.f32);
    w = QWeight{};
}

// Quantized-activation tiles for up to Mpad rows and K columns (kernels.h layout).
ActQ alloc_actq(int Mpad, int K) {
    ActQ a;
    a.Mpad = Mpad;
    const size_t bytes = (size_t)(K / 128) * (Mpad / 128) * kActTile;
    a.q = dalloc<int8_t>(bytes);
    CK(cudaMemset(a.q, 0, bytes));
    return a;
}
void free_actq(ActQ& a) { cudaFree(a.q); a = ActQ{}; }

// Library scratch used by the standalone mgc_qgemm entry point (grown on demand, per device).
struct Scratch { ActQ a; int Mpad = 0, K = 0, N = 0; float* attn = nullptr; size_t attn_n = 0; SplitK sk; };

// Split-K scratch for up to 4 splits of an [rows][N] output.
SplitK alloc_splitk(int Mpad, int N) {
    SplitK k;
    k.part_floats = (size_t)4 * Mpad * N;
    k.part = dalloc<float>(k.part_floats);
    k.n_counters = ((N + 31) / 32) * (Mpad / 128);
    k.counters = dalloc<int>(k.n_counters);
    CK(cudaMemset(k.counters, 0, sizeof(int) * k.n_counters));
    return k;
}
void free_splitk(SplitK& k) { cudaFree(k.part); cudaFree(k.counters); k = SplitK{}; }
std::map<int, Scratch> g_scratch;
std::mutex g_scratch_mu;

}  // namespace


void mgc::set_last_error(const char* msg) { g_err = msg; }

extern "C" {

const char* mgc_last_error(void) { return g_err.c_str(); }

int mgc_selftest_wait_timeout(int code, void* stream) {
    return guard([&] {
        if (code <= 0) throw Err("mgc_selftest_wait_timeout: code must be positive");
        wait_timeout_selftest_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(code);
        CK(cudaPeekAtLastError());
        CK(cudaStreamSynchronize((cudaStream_t)stream));
    });
}

int mgc_device_error(void) {
    int v = 0;
    int rc = guard([&] {
        CK(cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(int)));
        const int zero = 0;
        CK(cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(int)));
    });
    return rc != 0 ? rc : v;
}

int mgc_pack_q8_0(const float* w, int64_t N, int64_t K, uint8_t* out) {
    if (!w || !out || N <= 0 || K <= 0 || K % 32) { g_err = "mgc_pack_q8_0: K must be a positive multiple of 32"; return -1; }
    pack_q8_0(w, N, K, out);
    return 0;
}
int mgc_pack_q4_k(const float* w, int64_t N, int64_t K, uint8_t* out) {
    if (!w || !out || N <= 0 || K <= 0 || K % 256) { g_err = "mgc_pack_q4_k: K must be a positive multiple of 256"; return -1; }
    pack_q4_k(w, N, K, out);
    return 0;
}
int mgc_dequant(int wtype, const uint8_t* w, int64_t N, int64_t K, float* out) {
    if (!(wtype == 8 && K % 32 == 0) && !(wtype == 12 && K % 256 == 0)) { g_err = "mgc_dequant: bad type or K"; return -1; }
    dequant(wtype, w, N, K, out);
    return 0;
}

int mgc_quantize_act(const float* x, int M, int K, int8_t* qx, float* dx, int32_t* sumx, void* stream) {
    if (M <= 0 || K <= 0 || K % 32) { g_err = "mgc_quantize_act: K must be a positive multiple of 32"; return -1; }
    return guard([&] {
        launch_quant_act_plain(x, M, K, qx, dx, sumx, (cudaStream_t)stream);
        CK(cudaPeekAtLastError());
    });
}

int mgc_qweight_create(int wtype, const void* w_host, int N, int K, mgc_qweight** out) {
    return guard([&] {
        if (!w_host || !out || N <= 0 || K <= 0) throw Err("mgc_qweight_create: bad arguments");
        auto* q = new mgc_qweight();
        try { q->w = upload_weight(wtype, w_host, N, K); }
        catch (...) { delete q; throw; }
        int dev; CK(cudaGetDevice(&dev));
        CK(cudaSetDevice(dev));
        if (qgemm_prepare() != 0) throw Err("qgemm: cannot set shared-memory limit");
        *out = q;
    });
}
void mgc_qweight_destroy(mgc_qweight* w) {
    if (!w) return;
    free_weight(w->w);
    delete w;
}

int mgc_qgemm(const mgc_qweight* wq, const float* x, int M, const float* bias, int act, const float* resid,
              float* y, void* stream) {
    return guard([&] {
        if (!wq || !x || !y || M <= 0) throw Err("mgc_qgemm: bad arguments");
        const QWeight& w = wq->w;
        cudaStream_t st = (cudaStream_t)stream;
        if (w.wtype == 0) {
            launch_gemm_f32(w.f32, x, M, w.N, w.K, bias, act, resid, y, st);
            CK(cudaPeekAtLastError());
            return;
        }
        int dev; CK(cudaGetDevice(&dev));
        std::lock_guard<std::mutex> lk(g_scratch_mu);
        Scratch& s = g_scratch[dev];
        const int Mpad = round_up(M, 128);
        if (s.Mpad < Mpad || s.K < w.K || s.N < w.N) {
            CK(cudaStreamSynchronize(st));
            free_actq(s.a);
            free_splitk(s.sk);
            s.Mpad = std::max(s.Mpad, Mpad);
            s.K = std::max(s.K, w.K);
            s.N = std::max(s.N, w.N);
            s.a = alloc_actq(s.Mpad, s.K);
            s.sk = alloc_splitk(s.Mpad, s.N);
        }
        launch_quant_act_tiled(x, M, w.K, s.a, w.wtype == 12, st);
        if (launch_qgemm(w, s.a, M, bias, act, resid, y, st, &s.sk) != 0)
            throw Err(std::string("qgemm launch failed: ") + cudaGetErrorString(cudaGetLastError()));
    });
}

int mgc_gemm_f32(const float* w, const float* x, int M, int N, int K, const float* bias, int act,
                 const float* resid, float* y, void* stream) {
    return guard([&] {
        if (M <= 0 || N <= 0 || K <= 0) throw Err("mgc_gemm_f32: bad sizes");
        launch_gemm_f32(w, x, M, N, K, bias, act, resid, y, (cudaStream_t)stream);
        CK(cudaPeekAtLastError());
    });
}

int mgc_layernorm_affine(const float* x, const float* gamma, const float* beta, int rows, int D, float eps,
                         float* y, void* stream) {
    return guard([&] {
        if (rows <= 0 || D % 64 || D > 2048 || D <= 0) throw Err("mgc_layernorm_affine: D must be a multiple of 64, <= 2048");
        launch_ln(x, gamma, beta, rows, D, eps, y, nullptr, false, (cudaStream_t)stream);
        CK(cudaPeekAtLastError());
    });
}

int mgc_flash_attn(const float* qkv, int B, int S, int H, int Dh, float scale, float* out, void* stream) {
    return guard([&] {
        if (B <= 0 || S <= 0 || H <= 0) throw Err("mgc_flash_attn: bad sizes");
        if (Dh != 48) throw Err("mgc_flash_attn: head_dim must be 48");
        int dev; CK(cudaGetDevice(&dev));
        std::lock_guard<std::mutex> lk(g_scratch_mu);
        Scratch& sc = g_scratch[dev];
        const size_t need = attn_scratch_floats(B, S, H);
        if (sc.attn_n < need) {
            CK(cudaStreamSynchronize((cudaStream_t)stream));
            cudaFree(sc.attn);
            sc.attn = dalloc<float>(need);
            sc.attn_n = need;
        }
        if (launch_flash_attn(qkv, B, S, H, Dh, scale, out, sc.attn, sc.attn_n, (cudaStream_t)stream) != 0)
            throw Err(std::string("mgc_flash_attn: launch failed: ") + cudaGetErrorString(cudaGetLastError()));
    });
}

int mgc_embed(const float* tok, int vocab, const float* pos, int E, const int32_t* tokens, int B, int S,
              float* out, void* stream) {
    return guard([&] {
        if (E % 64 || E > 2048 || B <= 0 || S <= 0) throw Err("mgc_embed: E must be a multiple of 64, <= 2048");
        launch_embed(tok, vocab, pos, E, tokens, B, S, out, (cudaStream_t)stream);
        CK(cudaPeekAtLastError());
    });
}

}  // extern "C"

// ============================================================================ runtime
struct LayerW {
    QWeight qkv, o, up, down;
    float *bqkv = nullptr, *bo = nullptr, *bup = nullptr, *bdown = nullptr;
    float *g1 = nullptr, *b1 = nullptr, *g2 = nullptr, *b2 = nullptr;
};

struct ProfRow { double ms = 0; int n = 0; };

// Host side of the logits read-back: chunk c of the pinned staging buffer is copied to the
// caller's buffer by thread c (the calling thread takes chunk 0) as soon as its device-to-host
// copy has landed, so the host copy is split four ways and overlaps the remaining DMA.
struct ReadPool {
    static constexpr int kChunks = 4;
    std::vector<std::thread> th;
    std::mutex mu;
    std::condition_variable cv, done_cv;
    unsigned gen = 0;
    int pending = 0;
    bool stop = false;
    float* dst = nullptr;
    const float* src = nullptr;
    size_t off[kChunks + 1] = {};
    cudaEvent_t ev[kChunks] = {};

    void chunk(int c) {
        if (off[c + 1] == off[c]) return;
        cudaEventSynchronize(ev[c]);
        std::memcpy(dst + off[c], src + off[c], sizeof(float) * (off[c + 1] - off[c]));
    }
    void start(int device) {
        for (int c = 1; c < kChunks; c++)
            th.emplace_back([this, c, device] {
                cudaSetDevice(device);
                unsigned seen = 0;
                for (;;) {
                    {
                        std::unique_lock<std::mutex> lk(mu);
                        cv.wait(lk, [&] { return stop || gen != seen; });
                        if (stop) return;
                        seen = gen;
                    }
                    chunk(c);
                    std::lock_guard<std::mutex> lk(mu);
                    if (--pending == 0) done_cv.notify_one();
                }
            });
    }
    // copy [0, total) floats once the events have fired; off[] must be set by the caller
    void run(float* d, const float* s) {
        cudaEventSynchronize(ev[0]);   // the forward is done: wake the helpers only now
        {
            std::lock_guard<std::mutex> lk(mu);
            dst = d; src = s; pending = kChunks - 1; ++gen;
        }
        cv.notify_all();
        chunk(0);
        std::unique_lock<std::mutex> lk(mu);
        done_cv.wait(lk, [&] { return pending == 0; });
    }
    ~ReadPool() {
        { std::lock_guard<std::mutex> lk(mu); stop = true; }
        cv.notify_all();
        for (auto& t : th) t.join();
    }
};

struct mgc_runtime {
    int device = 0;
    std::string dev_name;
    cudaStream_t st = nullptr;
    // hparams
    int n_layer = 0, n_head = 0, E = 0, F = 0, Dh = 0, V = 0, n_tokens = 0, mask_id = -1, codebook = 0;
    int n_pos = 0, wtype = 0;
    float eps = 1e-12f, choice_temp = 4.5f;
    // weights
    float *tok = nullptr, *pos = nullptr, *g0 = nullptr, *b0 = nullptr;
    std::vector<LayerW> layers;
    QWeight proj;
    float *bproj = nullptr, *gout = nullptr, *bout = nullptr, *obias = nullptr;
    bool any_q4k = false;
    std::vector<float*> f32_allocs;
    // activations
    int max_rows = 0, Mpad = 0;
    float *x = nullptr, *t = nullptr, *qkv = nullptr, *att = nullptr, *ff = nullptr, *logits = nullptr;
    int32_t* tokens = nullptr;
    ActQ aE, aF;
    SplitK sk;                       // split-K partials of the quantized GEMMs
    float* attn_scratch = nullptr;   // key-split partials of the attention
    size_t attn_scratch_n = 0;
    // host staging (pinned)
    int32_t* h_tokens = nullptr;
    int* h_err = nullptr;   // pinned copy of the device error word, read back after each forward
    // decode-loop sampling on the device (mgc_generate): uniforms in, sampled code + probability out
    double* d_r = nullptr; int32_t* d_sid = nullptr; float* d_psid = nullptr;
    double* h_r = nullptr; int32_t* h_sid = nullptr; float* h_psid = nullptr;
    float* h_logits = nullptr;
    // logits read-back in row chunks (ReadPool)
    ReadPool rd;
    // CUDA graphs keyed by (B, S, tokens ptr, logits ptr)
    std::map<std::tuple<int, int, const void*, const void*>, cudaGraphExec_t> graphs;
    // profiling
    bool prof = false;
    bool fuse = true;        // fused epilogue quantizers (MGC_NO_FUSE=1 runs them as separate kernels)
    int last_launches = 0;   // kernels enqueued by the last forward
    std::string only_op;     // non-empty: enqueue_forward enqueues only this op class
    // column-split tensor parallelism (mgc_runtime_create_tp): this rank's share of every layer
    int tp_rank = 0, tp_world = 1;
    ncclComm_t comm = nullptr;
    int Eg = 0, Fg = 0, Hl = 0, Vg = 0;   // local widths: E/G, F/G, heads H/G, vocabulary slice
    float* gbuf = nullptr;                 // [G][rows][Eg] all-gathered column slices
    float* head_w = nullptr;               // [Vg][E] this rank's vocabulary rows (zero padded)
    float* head_b = nullptr;               // [Vg]
    float* lgbuf = nullptr;                // [G][rows][Vg] all-gathered logits slices
    float* lg_loc = nullptr;               // [rows][Vg]
    std::map<std::string, ProfRow> prof_rows;

    float* up_f32(const GgufTensor& t, size_t n) {
        if (t.type != 0) throw Err("expected an F32 tensor");
        float* d = dupload((const float*)t.data, n);
        f32_allocs.push_back(d);
        return d;
    }
};

namespace {

// A run of rows [row0, row0 + nrows) of an [N][K] GGUF tensor (nrows < 0: all rows).
struct RowRange { std::string name; int row0 = 0, nrows = -1; };

QWeight load_linear(const Gguf& g, const std::vector<RowRange>& parts, int K, bool& any_q4k) {
    // several [N_i][K] weights (or row ranges of them) of one type stacked along N (q|k|v):
    // rows are independent and stored back to back, so concatenating their GGUF bytes is the
    // same as one [sum N_i][K] weight.
    std::vector<uint8_t> bytes;
    int N = 0; uint32_t type = 0;
    for (size_t i = 0; i < parts.size(); i++) {
        const GgufTensor& t = g.req(parts[i].name);
        if (t.ne[0] != K) throw Err("tensor '" + parts[i].name + "' has unexpected K");
        if (i == 0) type = t.type;
        else if (t.type != type) throw Err("fused weights of different types");
        const int rows = (int)t.ne[1], r0 = parts[i].row0, nr = parts[i].nrows < 0 ? rows : parts[i].nrows;
        if (r0 < 0 || r0 + nr > rows) throw Err("row range outside tensor '" + parts[i].name + "'");
        const size_t row_bytes = t.bytes / (size_t)rows;
        bytes.insert(bytes.end(), t.data + (size_t)r0 * row_bytes, t.data + (size_t)(r0 + nr) * row_bytes);
        N += nr;
    }
    if (type == 12) any_q4k = true;
    return upload_weight((int)type, bytes.data(), N, K);
}

// One linear layer: quantized path reads the tiled activation `a`, F32 path the f32 `xin`.
void linear(mgc_runtime* rt, const QWeight& w, const float* xin, const ActQ& a, int M, const float* bias,
            int act, const float* resid, float* y) {
    if (w.wtype == 0) { launch_gemm_f32(w.f32, xin, M, w.N, w.K, bias, act, resid, y, rt->st); return; }
    if (launch_qgemm(w, a, M, bias, act, resid, y, rt->st, &rt->sk) != 0)
        throw Err(std::string("qgemm launch failed: ") + cudaGetErrorString(cudaGetLastError()));
}

// One column-split forward on this rank (tensor parallel over rt->tp_world GPUs, every rank
// enqueueing the same sequence): the layer structure of enqueue_forward with each linear
// computing this rank's output columns and NCCL all-gathers where a full row is needed next.
// Every output element is computed as on one GPU (same K order, same quantized inputs), and
// the attention of a head is the same kernel, so the logits equal the single-GPU forward's.
//   q|k|v: this rank's heads (no exchange before attention) -> attention -> all-gather the
//   head-merged slices -> quantizer over the gathered layout -> attn_o (E/G columns, residual
//   slice read in place) -> all-gather -> LayerNorm over the gathered layout (full rows on
//   every rank, + quantizer) -> ffn_up (F/G columns, GELU, quantizes into the full activation
//   tiles at its own column offset) -> all-gather of those int8 tiles in place -> ffn_down ->
//   all-gather -> LayerNorm.  output_proj and its LayerNorm run replicated; the MLM head is
//   split by vocabulary rows and its logits all-gathered.
// Column-split tensor-parallel forward (one stream; the NCCL all-gathers are captured into the
// step graph).  The attention's key split is chosen from the single-GPU launch shape, so every
// head is reduced in the same order as on one GPU.
void enqueue_forward_tp(mgc_runtime* rt, const int32_t* tokens, int B, int S, float* logits) {
    const int R = B * S, E = rt->E, g = rt->tp_rank, Eg = rt->Eg, Fg = rt->Fg, Vg = rt->Vg;
    cudaStream_t st = rt->st;
    const bool qc = rt->any_q4k;
    const long long slice = (long long)R * Eg;   // floats per rank block of gbuf
    auto gather = [&](const void* send, void* recv, size_t bytes) {
        const std::string e = tp_all_gather(send, recv, bytes, rt->comm, st);
        if (!e.empty()) throw Err(e);
    };
    auto q = [&](const QWeight& w, const ActQ& a, const float* bias, int act, const float* resid, int resid_ld,
                 float* y, const ActQ* qo, int qo_n0, const AttnPrepOut* ap) {
        if (w.wtype == 0) throw Err("tensor parallel needs quantized linears");
        if (launch_qgemm(w, a, R, bias, act, resid, y, st, nullptr, qo, qc, ap, resid_ld, qo_n0) != 0)
            throw Err(std::string("qgemm launch failed: ") + cudaGetErrorString(cudaGetLastError()));
    };
    const int launches0 = g_launch_count;
    launch_embed_ln(rt->tok, rt->V, rt->pos, E, tokens, B, S, rt->g0, rt->b0, rt->eps, rt->x, &rt->aE, qc, st);
    const float scale = 1.0f / std::sqrt((float)rt->Dh);
    const long attn_ctas = (long)((S + 127) / 128) * rt->n_head * B;   // the single-GPU launch
    // ffn_up writes chunks [g*Fg/128, (g+1)*Fg/128) of the full activation tiles: one contiguous run
    const size_t f_slice = (size_t)(Fg / 128) * (rt->Mpad / 128) * kActTile;
    for (int l = 0; l < rt->n_layer; l++) {
        const LayerW& L = rt->layers[l];
        const AttnPrepOut ap = attn_prep_out(rt->attn_scratch, B, S, rt->Hl);
        q(L.qkv, rt->aE, L.bqkv, 0, nullptr, 0, nullptr, nullptr, 0, &ap);
        if (launch_flash_attn(nullptr, B, S, rt->Hl, rt->Dh, scale, rt->att, rt->attn_scratch, rt->attn_scratch_n, st,
                              nullptr, false, nullptr, true, attn_ctas) != 0)
            throw Err("flash attention launch failed");
        gather(rt->att, rt->gbuf, sizeof(float) * (size_t)slice);
        if (!launch_quant_blocked(rt->gbuf, Eg, slice, R, E, rt->aE, qc, st)) throw Err("gathered quantizer failed");
        q(L.o, rt->aE, L.bo, 0, rt->x + (size_t)g * Eg, E, rt->t, nullptr, 0, nullptr);
        gather(rt->t, rt->gbuf, sizeof(float) * (size_t)slice);
        if (!launch_ln_blocked(rt->gbuf, Eg, slice, L.g1, L.b1, R, E, rt->eps, rt->x, &rt->aE, qc, st))
            throw Err("gathered LayerNorm failed");
        q(L.up, rt->aE, L.bup, 1, nullptr, 0, nullptr, &rt->aF, g * Fg, nullptr);
        gather(rt->aF.q + (size_t)g * f_slice, rt->aF.q, f_slice);
        q(L.down, rt->aF, L.bdown, 0, rt->x + (size_t)g * Eg, E, rt->t, nullptr, 0, nullptr);
        gather(rt->t, rt->gbuf, sizeof(float) * (size_t)slice);
        if (!launch_ln_blocked(rt->gbuf, Eg, slice, L.g2, L.b2, R, E, rt->eps, rt->x, &rt->aE, qc, st))
            throw Err("gathered LayerNorm failed");
    }
    if (launch_qgemm(rt->proj, rt->aE, R, rt->bproj, 1, nullptr, rt->t, st, nullptr) != 0)
        throw Err(std::string("qgemm launch failed: ") + cudaGetErrorString(cudaGetLastError()));
    launch_ln(rt->t, rt->gout, rt->bout, R, E, rt->eps, rt->x, nullptr, false, st);
    launch_gemm_f32(rt->head_w, rt->x, R, Vg, E, rt->head_b, 0, nullptr, rt->lg_loc, st);
    gather(rt->lg_loc, rt->lgbuf, sizeof(float) * (size_t)R * Vg);
    launch_ungather_cols(rt->lgbuf, R, Vg, rt->V, logits, st);
    CK(cudaPeekAtLastError());
    rt->last_launches = g_launch_count - launches0;
}

// Enqueue one transformer forward (build_transformer, mg-transformer.cpp:32-111) on rt->st.
// dump (device, optional) receives the 51 named tensors back to back.
void enqueue_forward(mgc_runtime* rt, const int32_t* tokens, int B, int S, float* logits, float* dump) {
    if (rt->tp_world > 1) {
        if (dump || rt->prof || !rt->only_op.empty())
            throw Err("tensor-parallel runtime: no dump / per-op profile (use a single-GPU runtime)");
        if (B * S > rt->max_rows) throw Err("forward: B*S exceeds the runtime's max_rows");
        if (S > rt->n_pos) throw Err("forward: S exceeds n_positions");
        enqueue_forward_tp(rt, tokens, B, S, logits);
        return;
    }
    const int R = B * S, E = rt->E, F = rt->F;
    if (R > rt->max_rows) throw Err("forward: B*S exceeds the runtime's max_rows");
    if (S > rt->n_pos) throw Err("forward: S exceeds n_positions");
    cudaStream_t st = rt->st;
    size_t doff = 0;
    auto put = [&](const float* src, int w) {
        if (!dump) return;
        CK(cudaMemcpyAsync(dump + doff, src, sizeof(float) * (size_t)R * w, cudaMemcpyDeviceToDevice, st));
        doff += (size_t)R * w;
    };
    // Profiling: a bounded spin kernel holds the GPU while the host enqueues every op with an
    // event pair, so the events time GPU execution only (no host launch gaps).
    struct Ev { const char* name; cudaEvent_t a, b; };
    std::vector<Ev> evs;
    if (rt->prof) launch_spin(2000000, st);   // ~1 ms at 2 GHz
    auto op = [&](const char* name, auto&& fn) {
        // op-class timing (mgc_runtime_time_op): enqueue only the launches of one op class
        if (!rt->only_op.empty() && rt->only_op != name) return;
        if (!rt->prof) { fn(); return; }
        Ev e{name, nullptr, nullptr};
        CK(cudaEventCreate(&e.a)); CK(cudaEventCreate(&e.b));
        CK(cudaEventRecord(e.a, st));
        fn();
        CK(cudaEventRecord(e.b, st));
        evs.push_back(e);
    };
    const int launches0 = g_launch_count;
    const bool qc = rt->any_q4k;
    const char* mm = rt->wtype == 0 ? "MulMat(f32)" : "MulMat(q)";
    op("GetRows+Norm", [&] { launch_embed_ln(rt->tok, rt->V, rt->pos, E, tokens, B, S, rt->g0, rt->b0, rt->eps,
                                              rt->x, &rt->aE, qc, st); });
    put(rt->x, E);
    const float scale = 1.0f / std::sqrt((float)rt->Dh);
    for (int l = 0; l < rt->n_layer; l++) {
        const LayerW& L = rt->layers[l];
        // the QKV epilogue writes the attention's f16 Q/K/V tiles directly (no f32 qkv round trip)
        const bool fprep = rt->fuse && L.qkv.wtype != 0;
        if (fprep) {
            op(mm, [&] {
                const AttnPrepOut ap = attn_prep_out(rt->attn_scratch, B, S, rt->n_head);
                if (launch_qgemm(L.qkv, rt->aE, R, L.bqkv, 0, nullptr, nullptr, st, &rt->sk, nullptr, false, &ap) != 0)
                    throw Err(std::string("qgemm launch failed: ") + cudaGetErrorString(cudaGetLastError()));
            });
        } else {
            op(mm, [&] { linear(rt, L.qkv, rt->x, rt->aE, R, L.bqkv, 0, nullptr, rt->qkv); });
        }
        bool att_quantized = false;
        op("FlashAttention", [&] {
            const bool fq = rt->fuse && L.o.wtype != 0;
            if (launch_flash_attn(rt->qkv, B, S, rt->n_head, rt->Dh, scale, rt->att, rt->attn_scratch,
                                  rt->attn_scratch_n, st, fq ? &rt->aE : nullptr, qc, &att_quantized, fprep) != 0)
                throw Err("flash attention launch failed");
        });
        if (L.o.wtype != 0 && !att_quantized)
            op("Quantize", [&] { launch_quant_act_tiled(rt->att, R, E, rt->aE, qc, st); });
        op(mm, [&] { linear(rt, L.o, rt->att, rt->aE, R, L.bo, 0, rt->x, rt->t); });
        op("Norm", [&] { launch_ln(rt->t, L.g1, L.b1, R, E, rt->eps, rt->x, &rt->aE, qc, st); });
        put(rt->x, E);
        if (L.up.wtype != 0 && L.down.wtype != 0 && rt->fuse) {
            // ffn_up's epilogue quantizes GELU(x W_up + b) straight into ffn_down's input tiles
            op(mm, [&] {
                if (launch_qgemm(L.up, rt->aE, R, L.bup, 1, nullptr, nullptr, st, &rt->sk, &rt->aF, qc) != 0)
                    throw Err(std::string("qgemm launch failed: ") + cudaGetErrorString(cudaGetLastError()));
            });
        } else {
            op(mm, [&] { linear(rt, L.up, rt->x, rt->aE, R, L.bup, 1, nullptr, rt->ff); });
            if (L.down.wtype != 0) op("Quantize", [&] { launch_quant_act_tiled(rt->ff, R, F, rt->aF, qc, st); });
        }
        op(mm, [&] { linear(rt, L.down, rt->ff, rt->aF, R, L.bdown, 0, rt->x, rt->t); });
        op("Norm", [&] { launch_ln(rt->t, L.g2, L.b2, R, E, rt->eps, rt->x, &rt->aE, qc, st); });
        put(rt->x, E);
    }
    op(mm, [&] { linear(rt, rt->proj, rt->x, rt->aE, R, rt->bproj, 1, nullptr, rt->t); });
    op("Norm", [&] { launch_ln(rt->t, rt->gout, rt->bout, R, E, rt->eps, rt->x, nullptr, false, st); });
    put(rt->x, E);
    op("MulMat(f32)", [&] { launch_gemm_f32(rt->tok, rt->x, R, rt->V, E, rt->obias, 0, nullptr, logits, st); });
    put(logits, rt->V);
    CK(cudaPeekAtLastError());
    rt->last_launches = g_launch_count - launches0;
    if (rt->prof) {
        CK(cudaStreamSynchronize(st));
        for (Ev& e : evs) {
            float ms = 0;
            CK(cudaEventElapsedTime(&ms, e.a, e.b));
            ProfRow& r = rt->prof_rows[e.name]; r.ms += ms; r.n++;
            cudaEventDestroy(e.a); cudaEventDestroy(e.b);
        }
    }
}

// Grow the attention scratch (prep tiles + key-split partials) for B images of S tokens; the
// captured graphs hold the old pointer, so they are dropped.  Never called inside a capture.
void ensure_attn_scratch(mgc_runtime* rt, int B, int S) {
    const size_t need = attn_scratch_floats(B, S, rt->Hl);
    if (rt->attn_scratch_n >= need) return;
    CK(cudaStreamSynchronize(rt->st));
    for (auto& kv : rt->graphs) cudaGraphExecDestroy(kv.second);
    rt->graphs.clear();
    cudaFree(rt->attn_scratch);
    rt->attn_scratch = nullptr;
    rt->attn_scratch = dalloc<float>(need);
    CK(cudaMemset(rt->attn_scratch, 0, need * sizeof(float)));   // padded keys of the prep tiles stay finite
    rt->attn_scratch_n = need;
}

// Forward through a cached CUDA graph (captured on the first call for this key).
void run_forward(mgc_runtime* rt, const int32_t* tokens, int B, int S, float* logits) {
    ensure_attn_scratch(rt, B, S);
    if (rt->prof) { enqueue_forward(rt, tokens, B, S, logits, nullptr); return; }
    auto key = std::make_tuple(B, S, (const void*)tokens, (const void*)logits);
    auto it = rt->graphs.find(key);
    if (it == rt->graphs.end()) {
        cudaGraph_t g;
        CK(cudaStreamBeginCapture(rt->st, cudaStreamCaptureModeThreadLocal));
        try { enqueue_forward(rt, tokens, B, S, logits, nullptr); }
        catch (...) { cudaStreamEndCapture(rt->st, &g); if (g) cudaGraphDestroy(g); throw; }
        CK(cudaStreamEndCapture(rt->st, &g));
        cudaGraphExec_t ex;
        CK(cudaGraphInstantiate(&ex, g, 0));
        cudaGraphDestroy(g);
        it = rt->graphs.emplace(key, ex).first;
    }
    CK(cudaGraphLaunch(it->second, rt->st));
}

// v >= 0: a value of the device error word already read back (asynchronously, in stream order)
void check_dev_error(int v = -1) {
    if (v < 0) CK(cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(int)));
    if (v != 0) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(int));
        throw Err("a kernel gave up waiting (device error code " + std::to_string(v) + ")");
    }
}

void destroy_runtime(mgc_runtime* rt) {
    if (!rt) return;
    cudaSetDevice(rt->device);
    if (rt->st) cudaStreamSynchronize(rt->st);
    for (auto& kv : rt->graphs) cudaGraphExecDestroy(kv.second);
    tp_comm_destroy(rt->comm);
    cudaFree(rt->gbuf); cudaFree(rt->lgbuf); cudaFree(rt->lg_loc);
    for (auto& L : rt->layers) { free_weight(L.qkv); free_weight(L.o); free_weight(L.up); free_weight(L.down); }
    free_weight(rt->proj);
    for (float* p : rt->f32_allocs) cudaFree(p);
    cudaFree(rt->x); cudaFree(rt->t); cudaFree(rt->qkv); cudaFree(rt->att); cudaFree(rt->ff);
    cudaFree(rt->logits); cudaFree(rt->tokens); cudaFree(rt->attn_scratch);
    free_splitk(rt->sk);
    free_actq(rt->aE); free_actq(rt->aF);
    if (rt->h_tokens) cudaFreeHost(rt->h_tokens);
    if (rt->h_err) cudaFreeHost(rt->h_err);
    cudaFree(rt->d_r); cudaFree(rt->d_sid); cudaFree(rt->d_psid);
    if (rt->h_r) cudaFreeHost(rt->h_r);
    if (rt->h_sid) cudaFreeHost(rt->h_sid);
    if (rt->h_psid) cudaFreeHost(rt->h_psid);
    if (rt->h_logits) cudaFreeHost(rt->h_logits);
    for (cudaEvent_t& e : rt->rd.ev)
        if (e) cudaEventDestroy(e);
    if (rt->st) cudaStreamDestroy(rt->st);
    delete rt;
}

}  // namespace

extern "C" {

}  // extern "C"

namespace {

// Shared body of mgc_runtime_create (world == 1) and mgc_runtime_create_tp.
void create_runtime(const char* path, int max_rows, int device, int rank, int world, const ncclUniqueId* id,
                    mgc_runtime** out) {
        if (!path || !out || max_rows <= 0) throw Err("mgc_runtime_create: bad arguments");
        if (world < 1 || rank < 0 || rank >= world) throw Err("mgc_runtime_create_tp: bad rank / world");
        std::unique_ptr<mgc_runtime, void (*)(mgc_runtime*)> rt(new mgc_runtime(), destroy_runtime);
        rt->device = device;
        rt->tp_rank = rank;
        rt->tp_world = world;
        if (const char* e = std::getenv("MGC_NO_FUSE")) rt->fuse = e[0] != '1';
        CK(cudaSetDevice(device));
        cudaDeviceProp prop;
        CK(cudaGetDeviceProperties(&prop, device));
        rt->dev_name = prop.name;
        if (prop.major != 10) throw Err(std::string("libmgcuda needs an sm_100 GPU, found ") + prop.name);
        CK(cudaStreamCreateWithFlags(&rt->st, cudaStreamNonBlocking));
        for (cudaEvent_t& e : rt->rd.ev) CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        rt->rd.start(device);
        if (qgemm_prepare() != 0 || attn_prepare() != 0) throw Err("cannot set kernel shared-memory limits");
        Gguf g;
        g.open(path);
        rt->n_layer = g.geti("maskgit.n_layer", 0); rt->n_head = g.geti("maskgit.n_head", 0);
        rt->E = g.geti("maskgit.n_embd", 0); rt->F = g.geti("maskgit.n_ffn", 0);
        rt->Dh = g.geti("maskgit.head_dim", 0); rt->V = g.geti("maskgit.vocab_size", 0);
        rt->n_tokens = g.geti("maskgit.n_tokens", 0); rt->mask_id = g.geti("maskgit.mask_token_id", -1);
        rt->codebook = g.geti("maskgit.vqgan.codebook_size", 0);
        rt->eps = g.getf("maskgit.layernorm_eps", 1e-12f);
        rt->choice_temp = g.getf("maskgit.sampling.choice_temperature", 4.5f);
        const int E = rt->E, F = rt->F;
        if (E <= 0 || F <= 0 || rt->n_head * rt->Dh != E || E % 128 || F % 128)
            throw Err("unsupported hyper-parameters (n_embd / n_ffn must be multiples of 128)");
        const GgufTensor& tok = g.req("token_embd.weight");
        const GgufTensor& pos = g.req("pos_embd.weight");
        if (tok.ne[0] != E || tok.ne[1] != rt->V || pos.ne[0] != E) throw Err("embedding shapes do not match hparams");
        rt->n_pos = (int)pos.ne[1];
        rt->tok = rt->up_f32(tok, (size_t)E * rt->V);
        rt->pos = rt->up_f32(pos, (size_t)E * rt->n_pos);
        rt->g0 = rt->up_f32(g.req("token_embd_norm.weight"), E);
        rt->b0 = rt->up_f32(g.req("token_embd_norm.bias"), E);
        // column split over `world` ranks: whole heads of q|k|v, E/G rows of attn_o and
        // ffn_down, F/G rows of ffn_up (each rank computes those output columns in full)
        const int G = world;
        if (G > 1 && (rt->n_head % G || F % (128 * G) || (E / G) % 32 || (E / G) % 8))
            throw Err("tensor parallel: n_head and n_ffn/128 must divide by the world size");
        rt->Eg = E / G; rt->Fg = F / G; rt->Hl = rt->n_head / G;
        const int Eg = rt->Eg, Fg = rt->Fg;
        auto bias_slice = [&](const GgufTensor& t, int n, int r0, int nr) {
            if (t.type != 0 || (int)t.ne[0] != n) throw Err("unexpected bias tensor");
            float* d = dupload((const float*)t.data + r0, (size_t)nr);
            rt->f32_allocs.push_back(d);
            return d;
        };
        bool q4 = false;
        for (int l = 0; l < rt->n_layer; l++) {
            const std::string p = "blk." + std::to_string(l) + ".";
            LayerW L;
            L.qkv = load_linear(g, {{p + "attn_q.weight", rank * Eg, Eg}, {p + "attn_k.weight", rank * Eg, Eg},
                                    {p + "attn_v.weight", rank * Eg, Eg}}, E, q4);
            L.o = load_linear(g, {{p + "attn_o.weight", rank * Eg, Eg}}, E, q4);
            L.up = load_linear(g, {{p + "ffn_up.weight", rank * Fg, Fg}}, E, q4);
            L.down = load_linear(g, {{p + "ffn_down.weight", rank * Eg, Eg}}, F, q4);
            std::vector<float> bqkv;
            for (const char* nm : {"attn_q.bias", "attn_k.bias", "attn_v.bias"}) {
                const GgufTensor& t = g.req(p + nm);
                bqkv.insert(bqkv.end(), (const float*)t.data + rank * Eg, (const float*)t.data + (rank + 1) * Eg);
            }
            L.bqkv = dupload(bqkv.data(), bqkv.size());
            rt->f32_allocs.push_back(L.bqkv);
            L.bo = bias_slice(g.req(p + "attn_o.bias"), E, rank * Eg, Eg);
            L.bup = bias_slice(g.req(p + "ffn_up.bias"), F, rank * Fg, Fg);
            L.bdown = bias_slice(g.req(p + "ffn_down.bias"), E, rank * Eg, Eg);
            L.g1 = rt->up_f32(g.req(p + "attn_norm.weight"), E);
            L.b1 = rt->up_f32(g.req(p + "attn_norm.bias"), E);
            L.g2 = rt->up_f32(g.req(p + "ffn_norm.weight"), E);
            L.b2 = rt->up_f32(g.req(p + "ffn_norm.bias"), E);
            rt->layers.push_back(L);
        }
        rt->proj = load_linear(g, {{"output_proj.weight"}}, E, q4);
        rt->bproj = rt->up_f32(g.req("output_proj.bias"), E);
        rt->gout = rt->up_f32(g.req("output_norm.weight"), E);
        rt->bout = rt->up_f32(g.req("output_norm.bias"), E);
        rt->obias = rt->up_f32(g.req("output.bias"), rt->V);
        rt->any_q4k = q4;
        rt->wtype = rt->n_layer > 0 ? rt->layers[0].qkv.wtype : rt->proj.wtype;
        // activations
        rt->max_rows = max_rows;
        rt->Mpad = round_up(max_rows, 128);
        const size_t R = (size_t)rt->Mpad;
        rt->x = dalloc<float>(R * E); rt->t = dalloc<float>(R * E); rt->qkv = dalloc<float>(R * 3 * E);
        rt->att = dalloc<float>(R * E); rt->ff = dalloc<float>(R * F); rt->logits = dalloc<float>(R * rt->V);
        rt->tokens = dalloc<int32_t>(R);
        rt->aE = alloc_actq(rt->Mpad, E);
        rt->aF = alloc_actq(rt->Mpad, F);
        rt->sk = alloc_splitk(rt->Mpad, std::max(3 * E, F));
        rt->attn_scratch_n = attn_scratch_floats(1, rt->Mpad, rt->Hl);
        rt->attn_scratch = dalloc<float>(rt->attn_scratch_n);
        CK(cudaMemset(rt->attn_scratch, 0, rt->attn_scratch_n * sizeof(float)));
        CK(cudaMallocHost(&rt->h_tokens, sizeof(int32_t) * R));
        CK(cudaMallocHost(&rt->h_err, sizeof(int)));
        rt->d_r = dalloc<double>(R); rt->d_sid = dalloc<int32_t>(R); rt->d_psid = dalloc<float>(R);
        CK(cudaMallocHost(&rt->h_r, sizeof(double) * R));
        CK(cudaMallocHost(&rt->h_sid, sizeof(int32_t) * R));
        CK(cudaMallocHost(&rt->h_psid, sizeof(float) * R));
        CK(cudaMallocHost(&rt->h_logits, sizeof(float) * R * rt->V));
        if (G > 1) {
            // the MLM head (token_embd as F32 weight) split by vocabulary rows, padded to Vg
            const int V = rt->V, Vg = (V + G - 1) / G, v0 = std::min(V, rank * Vg), nv = std::min(V, v0 + Vg) - v0;
            rt->Vg = Vg;
            std::vector<float> hw((size_t)Vg * E, 0.0f), hb(Vg, 0.0f);
            std::memcpy(hw.data(), (const float*)tok.data + (size_t)v0 * E, sizeof(float) * (size_t)nv * E);
            std::memcpy(hb.data(), (const float*)g.req("output.bias").data + v0, sizeof(float) * nv);
            rt->head_w = dupload(hw.data(), hw.size());
            rt->head_b = dupload(hb.data(), hb.size());
            rt->f32_allocs.push_back(rt->head_w);
            rt->f32_allocs.push_back(rt->head_b);
            rt->gbuf = dalloc<float>(R * E);
            rt->lgbuf = dalloc<float>((size_t)G * R * Vg);
            rt->lg_loc = dalloc<float>(R * Vg);
            const std::string e = tp_comm_init(&rt->comm, G, *id, rank);
            if (!e.empty()) throw Err(e);
        }
        CK(cudaDeviceSynchronize());
        // one eager forward: sets every kernel's attributes outside any later stream capture
        CK(cudaMemsetAsync(rt->tokens, 0, sizeof(int32_t) * R, rt->st));
        enqueue_forward(rt.get(), rt->tokens, 1, std::min(max_rows, rt->n_pos), rt->logits, nullptr);
        CK(cudaStreamSynchronize(rt->st));
        check_dev_error();
        *out = rt.release();
}

}  // namespace

extern "C" {

int mgc_runtime_create(const char* path, int max_rows, int device, mgc_runtime** out) {
    return guard([&] { create_runtime(path, max_rows, device, 0, 1, nullptr, out); });
}

int mgc_tp_unique_id(uint8_t out[128]) {
    return guard([&] {
        static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id size");
        if (!out) throw Err("mgc_tp_unique_id: bad arguments");
        ncclUniqueId id;
        const std::string e = tp_unique_id(&id);
        if (!e.empty()) throw Err(e);
        std::memcpy(out, &id, sizeof(id));
    });
}

int mgc_runtime_create_tp(const char* path, int max_rows, int device, int rank, int world, const uint8_t id[128],
                          mgc_runtime** out) {
    return guard([&] {
        if (!id) throw Err("mgc_runtime_create_tp: bad arguments");
        ncclUniqueId uid;
        std::memcpy(&uid, id, sizeof(uid));
        create_runtime(path, max_rows, device, rank, world, &uid, out);
    });
}

void mgc_runtime_destroy(mgc_runtime* rt) { destroy_runtime(rt); }

int mgc_runtime_hparams(const mgc_runtime* rt, int32_t o[10]) {
    if (!rt) return -1;
    const int32_t v[10] = {rt->n_layer, rt->n_head, rt->E, rt->F, rt->Dh, rt->V, rt->n_tokens, rt->mask_id,
                           rt->codebook, rt->wtype};
    std::memcpy(o, v, sizeof(v));
    return 0;
}
const char* mgc_runtime_device_name(const mgc_runtime* rt) { return rt ? rt->dev_name.c_str() : ""; }
void* mgc_runtime_stream(mgc_runtime* rt) { return rt ? (void*)rt->st : nullptr; }

int mgc_runtime_sync(mgc_runtime* rt) {
    return guard([&] {
        CK(cudaSetDevice(rt->device));
        CK(cudaStreamSynchronize(rt->st));
        check_dev_error();
    });
}

int mgc_transformer_forward_dev(mgc_runtime* rt, const int32_t* tokens_dev, int B, int S, float* logits_dev) {
    return guard([&] {
        if (!rt || B <= 0 || S <= 0) throw Err("mgc_transformer_forward_dev: bad arguments");
        CK(cudaSetDevice(rt->device));
        run_forward(rt, tokens_dev, B, S, logits_dev);
    });
}

int mgc_transformer_forward(mgc_runtime* rt, const int32_t* tokens, int B, int S, float* logits) {
    return guard([&] {
        if (!rt || !tokens || !logits || B <= 0 || S <= 0) throw Err("mgc_transformer_forward: bad arguments");
        const size_t R = (size_t)B * S, nl = R * rt->V;
        if ((int)R > rt->max_rows) throw Err("forward: B*S exceeds the runtime's max_rows");
        CK(cudaSetDevice(rt->device));
        std::memcpy(rt->h_tokens, tokens, sizeof(int32_t) * R);
        CK(cudaMemcpyAsync(rt->tokens, rt->h_tokens, sizeof(int32_t) * R, cudaMemcpyHostToDevice, rt->st));
        run_forward(rt, rt->tokens, B, S, rt->logits);
        constexpr int NCH = ReadPool::kChunks;
        size_t* off = rt->rd.off;
        for (int c = 0; c <= NCH; c++) off[c] = (R * c / NCH) * rt->V;   // whole rows per chunk
        CK(cudaMemcpyFromSymbolAsync(rt->h_err, g_dev_error, sizeof(int), 0, cudaMemcpyDeviceToHost, rt->st));
        for (int c = 0; c < NCH; c++) {
            if (off[c + 1] == off[c]) continue;
            CK(cudaMemcpyAsync(rt->h_logits + off[c], rt->logits + off[c], sizeof(float) * (off[c + 1] - off[c]),
                               cudaMemcpyDeviceToHost, rt->st));
            CK(cudaEventRecord(rt->rd.ev[c], rt->st));
        }
        rt->rd.run(logits, rt->h_logits);
        check_dev_error(*rt->h_err);
    });
}

int mgc_transformer_forward_dump(mgc_runtime* rt, const int32_t* tokens, int B, int S, float* logits,
                                 float* dump_host) {
    return guard([&] {
        if (!rt || !tokens || !logits || !dump_host) throw Err("mgc_transformer_forward_dump: bad arguments");
        const size_t R = (size_t)B * S;
        if ((int)R > rt->max_rows) throw Err("forward: B*S exceeds the runtime's max_rows");
        const size_t ndump = R * ((size_t)rt->E * (2 * rt->n_layer + 2) + rt->V);
        CK(cudaSetDevice(rt->device));
        ensure_attn_scratch(rt, B, S);
        float* d_dump = dalloc<float>(ndump);
        try {
            CK(cudaMemcpyAsync(rt->tokens, tokens, sizeof(int32_t) * R, cudaMemcpyHostToDevice, rt->st));
            enqueue_forward(rt, rt->tokens, B, S, rt->logits, d_dump);
            CK(cudaMemcpyAsync(logits, rt->logits, sizeof(float) * R * rt->V, cudaMemcpyDeviceToHost, rt->st));
            CK(cudaMemcpyAsync(dump_host, d_dump, sizeof(float) * ndump, cudaMemcpyDeviceToHost, rt->st));
            CK(cudaStreamSynchronize(rt->st));
            check_dev_error();
        } catch (...) { cudaFree(d_dump); throw; }
        cudaFree(d_dump);
    });
}

// generate() sampling (mg-generate.cpp:24-35 helpers, :53-123 loop) for B independent
// images; the same libstdc++ mt19937_64 / uniform_real_distribution<double> streams.
int mgc_generate(mgc_runtime* rt, int B, const int32_t* class_ids, const uint64_t* seeds, int steps,
                 float temperature, int32_t* tokens_out) {
    return guard([&] {
        if (!rt || B <= 0 || !class_ids || !seeds || !tokens_out || steps <= 0) throw Err("mgc_generate: bad arguments");
        const int CB = rt->codebook, MASK = rt->mask_id, S = rt->n_tokens + 1;
        const size_t vocab = (size_t)rt->V;
        if (B * S > rt->max_rows) throw Err("mgc_generate: B*S exceeds max_rows");
        if (CB <= 0 || CB > rt->V) throw Err("mgc_generate: bad codebook size");
        const float ct = temperature < 0 ? rt->choice_temp : temperature;
        std::vector<std::mt19937_64> rng;
        for (int i = 0; i < B; i++) rng.emplace_back(seeds[i]);
        std::vector<int32_t> tokens((size_t)B * S, MASK), sampled(S), result((size_t)B * S);
        for (int i = 0; i < B; i++) tokens[(size_t)i * S] = class_ids[i] + CB;
        std::vector<float> selp(S), conf(S);
        const size_t R = (size_t)B * S;
        CK(cudaSetDevice(rt->device));
        ensure_attn_scratch(rt, B, S);
        for (int step = 0; step < steps; step++) {
            // forward on the device; the logits stay there (no read-back)
            std::memcpy(rt->h_tokens, tokens.data(), sizeof(int32_t) * R);
            CK(cudaMemcpyAsync(rt->tokens, rt->h_tokens, sizeof(int32_t) * R, cudaMemcpyHostToDevice, rt->st));
            run_forward(rt, rt->tokens, B, S, rt->logits);
            // the categorical uniforms of every position, in generate()'s draw order (one per
            // position, before the step's gumbel draws), drawn while the forward runs
            for (int i = 0; i < B; i++) {
                std::uniform_real_distribution<double> u(0.0, 1.0);
                for (int s = 0; s < S; s++) rt->h_r[(size_t)i * S + s] = u(rng[i]);
            }
            CK(cudaMemcpyAsync(rt->d_r, rt->h_r, sizeof(double) * R, cudaMemcpyHostToDevice, rt->st));
            launch_sample_codes(rt->logits, (int)R, (int)vocab, CB, rt->d_r, rt->d_sid, rt->d_psid, rt->st);
            CK(cudaMemcpyAsync(rt->h_sid, rt->d_sid, sizeof(int32_t) * R, cudaMemcpyDeviceToHost, rt->st));
            CK(cudaMemcpyAsync(rt->h_psid, rt->d_psid, sizeof(float) * R, cudaMemcpyDeviceToHost, rt->st));
            CK(cudaMemcpyFromSymbolAsync(rt->h_err, g_dev_error, sizeof(int), 0, cudaMemcpyDeviceToHost, rt->st));
            CK(cudaStreamSynchronize(rt->st));
            check_dev_error(*rt->h_err);
            for (int i = 0; i < B; i++) {
                std::mt19937_64& r = rng[i];
                int32_t* tk = tokens.data() + (size_t)i * S;
                for (int s = 0; s < S; s++) {
                    const bool unknown = tk[s] == MASK;
                    sampled[s] = unknown ? rt->h_sid[(size_t)i * S + s] : tk[s];
                    selp[s] = unknown ? rt->h_psid[(size_t)i * S + s] : INFINITY;   // known tokens: max confidence
                }
                std::copy(sampled.begin(), sampled.end(), result.begin() + (size_t)i * S);
                const float ratio = (float)(step + 1) / steps;
                const float mask_ratio = std::cos((float)M_PI / 2.f * ratio);
                int n_unknown = 0;
                for (int s = 0; s < S; s++) n_unknown += tk[s] == MASK;
                int mask_len = (int)std::floor(rt->n_tokens * mask_ratio);
                mask_len = std::max(1, std::min(mask_len, n_unknown - 1));
                const float temp = ct * (1.f - ratio);
                for (int s = 0; s < S; s++) {
                    std::uniform_real_distribution<double> u(1e-12, 1.0);
                    const float gm = (float)(-std::log(-std::log(u(r))));
                    conf[s] = std::log(selp[s]) + temp * gm;
                }
                std::vector<float> sorted(conf);
                std::nth_element(sorted.begin(), sorted.begin() + mask_len, sorted.end());
                const float cutoff = sorted[mask_len];
                for (int s = 0; s < S; s++) tk[s] = conf[s] < cutoff ? MASK : sampled[s];
            }
        }
        std::memcpy(tokens_out, result.data(), sizeof(int32_t) * B * S);
    });
}

int mgc_runtime_kernel_count(const mgc_runtime* rt) { return rt ? rt->last_launches : -1; }

int mgc_runtime_time_op(mgc_runtime* rt, const char* op, int B, int S, int iters, float* ms_per_replay,
                        int* launches) {
    return guard([&] {
        if (!rt || !op || !op[0] || B <= 0 || S <= 0 || iters <= 0 || !ms_per_replay)
            throw Err("mgc_runtime_time_op: bad arguments");
        if (B * S > rt->max_rows) throw Err("mgc_runtime_time_op: B*S exceeds max_rows");
        CK(cudaSetDevice(rt->device));
        ensure_attn_scratch(rt, B, S);
        CK(cudaStreamSynchronize(rt->st));
        cudaGraph_t g = nullptr;
        cudaGraphExec_t ex = nullptr;
        cudaEvent_t e0 = nullptr, e1 = nullptr;
        rt->only_op = op;
        const bool prof = rt->prof;
        rt->prof = false;
        auto restore = [&] {
            rt->only_op.clear();
            rt->prof = prof;
            if (ex) cudaGraphExecDestroy(ex);
            if (e0) cudaEventDestroy(e0);
            if (e1) cudaEventDestroy(e1);
        };
        try {
            CK(cudaStreamBeginCapture(rt->st, cudaStreamCaptureModeThreadLocal));
            try { enqueue_forward(rt, rt->tokens, B, S, rt->logits, nullptr); }
            catch (...) { cudaStreamEndCapture(rt->st, &g); if (g) cudaGraphDestroy(g); throw; }
            CK(cudaStreamEndCapture(rt->st, &g));
            CK(cudaGraphInstantiate(&ex, g, 0));
            cudaGraphDestroy(g);
            if (launches) *launches = rt->last_launches;
            CK(cudaEventCreate(&e0));
            CK(cudaEventCreate(&e1));
            for (int i = 0; i < 2; i++) CK(cudaGraphLaunch(ex, rt->st));   // warm-up
            CK(cudaEventRecord(e0, rt->st));
            for (int i = 0; i < iters; i++) CK(cudaGraphLaunch(ex, rt->st));
            CK(cudaEventRecord(e1, rt->st));
            CK(cudaEventSynchronize(e1));
            float ms = 0;
            CK(cudaEventElapsedTime(&ms, e0, e1));
            *ms_per_replay = ms / iters;
            check_dev_error();
        } catch (...) { restore(); throw; }
        restore();
    });
}

int mgc_profile_enable(mgc_runtime* rt, int on) { if (!rt) return -1; rt->prof = on != 0; return 0; }
int mgc_profile_reset(mgc_runtime* rt) { if (!rt) return -1; rt->prof_rows.clear(); return 0; }
int mgc_profile_report(mgc_runtime* rt, char* buf, size_t len) {
    if (!rt || !buf || len == 0) return -1;
    std::vector<std::pair<std::string, ProfRow>> rows(rt->prof_rows.begin(), rt->prof_rows.end());
    std::sort(rows.begin(), rows.end(), [](auto& a, auto& b) { return a.second.ms > b.second.ms; });
    std::string s;
    for (auto& r : rows) {
        char line[128];
        std::snprintf(line, sizeof line, "%s %d %.4f\n", r.first.c_str(), r.second.n, r.second.ms);
        s += line;
    }
    std::snprintf(buf, len, "%s", s.c_str());
    return 0;
}

}  // extern "C"
