// NCCL all-reduce for tensor-parallel handles (see tp.h).
#include <dlfcn.h>
#include <nccl.h>

#include <string>

#include "tp.h"

namespace gpt2q {

struct TpComm {
    void* lib = nullptr;
    ncclComm_t comm = nullptr;
    std::string err;
    ncclResult_t (*init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*destroy)(ncclComm_t) = nullptr;
    const char* (*err_str)(ncclResult_t) = nullptr;
};

__global__ void k_add_inplace(float* __restrict__ x, const float* __restrict__ y, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        x[i] = x[i] + y[i];
}

TpComm* tp_create(int tp_size, int tp_rank, const void* id, int device) {
    TpComm* c = new TpComm();
    c->lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!c->lib) {
        c->err = std::string("dlopen libnccl.so.2: ") + dlerror();
        return c;
    }
    c->init_rank = (decltype(c->init_rank))dlsym(c->lib, "ncclCommInitRank");
    c->all_reduce = (decltype(c->all_reduce))dlsym(c->lib, "ncclAllReduce");
    c->destroy = (decltype(c->destroy))dlsym(c->lib, "ncclCommDestroy");
    c->err_str = (decltype(c->err_str))dlsym(c->lib, "ncclGetErrorString");
    if (!c->init_rank || !c->all_reduce || !c->destroy || !c->err_str) {
        c->err = "NCCL symbols missing";
        return c;
    }
    cudaSetDevice(device);
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    ncclResult_t r = c->init_rank(&c->comm, tp_size, uid, tp_rank);
    if (r != ncclSuccess) c->err = std::string("ncclCommInitRank: ") + c->err_str(r);
    return c;
}

int tp_allreduce_add(TpComm* c, float* red, float* x, size_t n, cudaStream_t st) {
    ncclResult_t r = c->all_reduce(red, red, n, ncclFloat32, ncclSum, c->comm, st);
    if (r != ncclSuccess) {
        c->err = std::string("ncclAllReduce: ") + c->err_str(r);
        return -1;
    }
    int blocks = (int)((n + 255) / 256);
    if (blocks > 148 * 4) blocks = 148 * 4;
    k_add_inplace<<<blocks, 256, 0, st>>>(x, red, n);
    if (cudaGetLastError() != cudaSuccess) {
        c->err = "add kernel launch failed";
        return -1;
    }
    return 0;
}

const char* tp_last_error(const TpComm* c) { return c ? c->err.c_str() : "no communicator"; }

void tp_destroy(TpComm* c) {
    if (!c) return;
    if (c->comm && c->destroy) c->destroy(c->comm);
    delete c;
}

}  // namespace gpt2q
