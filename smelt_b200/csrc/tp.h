// Tensor-parallel communicator for the GPT-2 XL configuration. The row-split projections
// (attn c_proj, mlp c_proj) leave one partial sum per rank; the ranks combine them without a
// library collective: every rank's partial stays in its own memory, mapped into the peers'
// address space (CUDA IPC over NVLink), and one kernel per residual update
//   1. tells every peer that this rank's partial is complete (a release store of an epoch
//      into the peer's flag word, one per thread block),
//   2. waits (bounded) for the peers' epochs,
//   3. sums the partials in rank order straight from peer memory, adds the residual stream
//      (every rank gets bit-identical rows) and
//   4. applies the LayerNorm that follows, writing the next linear's input.
// NCCL (loaded at run time with dlopen) bootstraps the handle exchange; where the GPUs cannot
// map each other's memory the partials are summed by an NCCL all-reduce instead.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>

namespace gpt2q {
struct TpComm;
// part_elems: floats of one partial buffer ([Mmax][d]).
TpComm* tp_create(int tp_size, int tp_rank, const void* nccl_unique_id, int device, size_t part_elems);
// Where this rank's projection writes its partial for residual update `parity` (0: attention
// projection, 1: MLP projection; the two alternate, so a buffer is rewritten only after every
// peer has finished reading it).
float* tp_partial(TpComm* c, int parity);
// x[m] += sum over ranks of partial[m] (rank order), m < M; then, when g != nullptr,
// h = LayerNorm(x) (eps) with the fp16 hi/lo split in hhi / hlo.
int tp_reduce_ln(TpComm* c, int parity, float* x, int M, int d, const float* g, const float* b, float eps, float* h,
                 __half* hhi, __half* hlo, cudaStream_t st);
// Reads and clears the device error word (0 = fine, > 0 a bounded wait for a peer gave up).
int tp_take_error(TpComm* c, cudaStream_t st);
// Device address of the communicator's error word (null without a communicator).
const int* tp_err_word(const TpComm* c);
bool tp_peer_mapped(const TpComm* c);
const char* tp_last_error(const TpComm* c);
void tp_destroy(TpComm* c);
}  // namespace gpt2q
