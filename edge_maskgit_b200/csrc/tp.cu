// tp.cu -- the pieces of column-split tensor parallelism that are not GEMM / attention kernels:
// NCCL, loaded on first use (single-GPU users of the library never need it), and the copy that
// turns all-gathered vocabulary slices of the logits into row-major logits.
//
// NCCL is opened with dlopen("libnccl.so.2"): in a process that already loaded NCCL (PyTorch
// does) the loader returns that copy, otherwise the system library.  Only the five entry points
// below are used; their C signatures are NCCL's public API (nccl.h).
#include "kernels.h"
#include "ptx.cuh"
#include "tp.h"

#include <dlfcn.h>
#include <mutex>
#include <string>

namespace mgc {

namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    const char* (*get_error_string)(ncclResult_t) = nullptr;
    std::string error;
};

NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) { api.error = std::string("cannot load libnccl.so.2: ") + dlerror(); return; }
        api.get_unique_id = (decltype(api.get_unique_id))dlsym(h, "ncclGetUniqueId");
        api.comm_init_rank = (decltype(api.comm_init_rank))dlsym(h, "ncclCommInitRank");
        api.all_gather = (decltype(api.all_gather))dlsym(h, "ncclAllGather");
        api.comm_destroy = (decltype(api.comm_destroy))dlsym(h, "ncclCommDestroy");
        api.get_error_string = (decltype(api.get_error_string))dlsym(h, "ncclGetErrorString");
        if (!api.get_unique_id || !api.comm_init_rank || !api.all_gather || !api.comm_destroy || !api.get_error_string)
            api.error = "libnccl.so.2 lacks an expected entry point";
    });
    return api;
}

std::string nccl_msg(const char* what, ncclResult_t r) {
    NcclApi& a = nccl();
    return std::string(what) + ": " + (a.get_error_string ? a.get_error_string(r) : "nccl error");
}

}  // namespace

std::string tp_unique_id(ncclUniqueId* id) {
    NcclApi& a = nccl();
    if (!a.error.empty()) return a.error;
    const ncclResult_t r = a.get_unique_id(id);
    return r == ncclSuccess ? std::string() : nccl_msg("ncclGetUniqueId", r);
}

std::string tp_comm_init(ncclComm_t* comm, int world, const ncclUniqueId& id, int rank) {
    NcclApi& a = nccl();
    if (!a.error.empty()) return a.error;
    const ncclResult_t r = a.comm_init_rank(comm, world, id, rank);
    return r == ncclSuccess ? std::string() : nccl_msg("ncclCommInitRank", r);
}

std::string tp_all_gather(const void* send, void* recv, size_t bytes, ncclComm_t comm, cudaStream_t st) {
    NcclApi& a = nccl();
    const ncclResult_t r = a.all_gather(send, recv, bytes, ncclChar, comm, st);
    return r == ncclSuccess ? std::string() : nccl_msg("ncclAllGather", r);
}

void tp_comm_destroy(ncclComm_t comm) {
    if (comm && nccl().comm_destroy) nccl().comm_destroy(comm);
}

// [G][R][Vg] vocabulary slices -> [R][V] row-major logits (columns >= V dropped)
__global__ void ungather_cols_kernel(const float* __restrict__ src, int R, int Vg, int V, float* __restrict__ dst) {
    griddep_wait();   // inputs come from the preceding kernel (no-op without PDL)
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)R * V) return;
    const int r = (int)(i / V), v = (int)(i % V), g = v / Vg;
    dst[i] = src[((long long)g * R + r) * Vg + (v - g * Vg)];
}

void launch_ungather_cols(const float* src, int R, int Vg, int V, float* dst, cudaStream_t st) {
    ++g_launch_count;
    const long long n = (long long)R * V;
    launch_k(ungather_cols_kernel, (unsigned)((n + 255) / 256), 256, 0, st, src, R, Vg, V, dst);
}

}  // namespace mgc
