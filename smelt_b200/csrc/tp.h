// Tensor-parallel communicator for the GPT-2 XL configuration: NCCL all-reduce of
// the row-split projection partial sums over NVLink. NCCL is loaded at run time
// (dlopen of libnccl.so.2) so the library has no link-time NCCL dependency and
// shares whichever NCCL the process already loaded.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

namespace gpt2q {
struct TpComm;
TpComm* tp_create(int tp_size, int tp_rank, const void* nccl_unique_id, int device);
// red = all-reduce-sum(red) over the ranks, then x += red (n floats).
int tp_allreduce_add(TpComm* c, float* red, float* x, size_t n, cudaStream_t st);
const char* tp_last_error(const TpComm* c);
void tp_destroy(TpComm* c);
}  // namespace gpt2q
