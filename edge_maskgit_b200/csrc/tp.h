// tp.h -- column-split tensor parallelism helpers (tp.cu): NCCL loaded on first use, and the
// logits un-gather.  Functions return an empty string on success, else the error message.
#pragma once
#include <string>

#include <cuda_runtime.h>
#include <nccl.h>

namespace mgc {

std::string tp_unique_id(ncclUniqueId* id);
std::string tp_comm_init(ncclComm_t* comm, int world, const ncclUniqueId& id, int rank);
std::string tp_all_gather(const void* send, void* recv, size_t bytes, ncclComm_t comm, cudaStream_t st);
void tp_comm_destroy(ncclComm_t comm);
void launch_ungather_cols(const float* src, int R, int Vg, int V, float* dst, cudaStream_t st);

}  // namespace mgc
