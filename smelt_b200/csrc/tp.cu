// Tensor-parallel residual updates over peer memory (see tp.h).
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <string>

#include "common.cuh"
#include "tp.h"

namespace gpt2q {

namespace {

constexpr int TP_MAX = 8;     // ranks
constexpr int TP_MAXB = 128;  // thread blocks of the reduce kernel (one flag word each per rank)
constexpr int TP_THREADS = 256;
constexpr int TP_V4 = 2;      // float4 per thread and row: d <= 2048, d % 4 == 0
constexpr uint32_t TP_SPIN = 1u << 24;  // bounded wait, ~1 s with the back-off below

struct TpArgs {
    const float* part[TP_MAX];  // rank q's partial buffer of this parity (peer pointer, or ours)
    uint32_t* flags[TP_MAX];    // rank q's flag array [TP_MAX][TP_MAXB]
    uint32_t* my_flags;         // ours
    uint32_t* ep;               // [TP_MAXB] epoch of each block of this rank
    int* err;
    int n, me;
    float* x;
    int M, d;
    const float *g, *b;
    float eps;
    float* h;
    __half *hhi, *hlo;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// 16 bytes of peer (or own) memory, fetched again rather than from a cached copy: the buffer
// is rewritten every other residual update.
__device__ __forceinline__ float4 ld_cv4(const float* p) { return __ldcv(reinterpret_cast<const float4*>(p)); }

__device__ __forceinline__ float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();  // red is reused by consecutive calls
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < TP_THREADS / 32; ++w) s += red[w];
    return s;
}

// Block b: rendezvous of block b on every rank, then rows b, b + G, ...: x += sum_q part_q
// (rank order), then the LayerNorm of the row (gpt2.rs:178-185) when g is set.
__global__ void __launch_bounds__(TP_THREADS) k_tp_reduce_ln(TpArgs a) {
    __shared__ uint32_t e_s;
    __shared__ float red[TP_THREADS / 32];
    const int blk = blockIdx.x, tid = threadIdx.x;
    if (tid == 0) {
        const uint32_t e = a.ep[blk] + 1;
        a.ep[blk] = e;
        e_s = e;
        // this rank's partial was written by the preceding kernel, complete before this one
        // started: announce it to every rank
        for (int q = 0; q < a.n; ++q) st_release_sys(a.flags[q] + a.me * TP_MAXB + blk, e);
    }
    __syncthreads();
    const uint32_t e = e_s;
    if (tid < a.n) {
        const uint32_t* f = a.my_flags + tid * TP_MAXB + blk;
        uint32_t i = 0;
        while ((int)(ld_acquire_sys(f) - e) < 0) {
            if (++i == TP_SPIN) {
                atomicExch(a.err, 1);
                break;
            }
            __nanosleep(64);
        }
    }
    __syncthreads();
    for (int m = blk; m < a.M; m += gridDim.x) {
        // every rank's slice of the row in flight at once, then the sum in rank order
        float4 pv[TP_MAX][TP_V4];
#pragma unroll
        for (int q = 0; q < TP_MAX; ++q)
#pragma unroll
            for (int k = 0; k < TP_V4; ++k) {
                const int i = (tid + k * TP_THREADS) * 4;
                pv[q][k] = (q < a.n && i < a.d) ? ld_cv4(a.part[q] + (size_t)m * a.d + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        float v[TP_V4][4];
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < TP_V4; ++k) {
            const int i = (tid + k * TP_THREADS) * 4;
            if (i < a.d) {
                float4 r = pv[0][k];
#pragma unroll
                for (int q = 1; q < TP_MAX; ++q) {
                    if (q < a.n) {
                        r.x += pv[q][k].x;
                        r.y += pv[q][k].y;
                        r.z += pv[q][k].z;
                        r.w += pv[q][k].w;
                    }
                }
                float4* xp = reinterpret_cast<float4*>(a.x + (size_t)m * a.d + i);
                const float4 x0 = *xp;
                const float4 y = make_float4(x0.x + r.x, x0.y + r.y, x0.z + r.z, x0.w + r.w);
                *xp = y;
                v[k][0] = y.x;
                v[k][1] = y.y;
                v[k][2] = y.z;
                v[k][3] = y.w;
                s += (y.x + y.y) + (y.z + y.w);
            } else {
                v[k][0] = v[k][1] = v[k][2] = v[k][3] = 0.f;
            }
        }
        if (!a.g) continue;  // uniform across the block
        const float mean = block_sum(s, red) / (float)a.d;
        float q2 = 0.f;
#pragma unroll
        for (int k = 0; k < TP_V4; ++k) {
            const int i = (tid + k * TP_THREADS) * 4;
            if (i < a.d) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float t = v[k][e] - mean;
                    q2 += t * t;
                }
            }
        }
        const float rstd = __frcp_rn(sqrtf(block_sum(q2, red) / (float)a.d + a.eps));
#pragma unroll
        for (int k = 0; k < TP_V4; ++k) {
            const int i = (tid + k * TP_THREADS) * 4;
            if (i < a.d) {
                const size_t o = (size_t)m * a.d + i;
                const float4 g4 = *reinterpret_cast<const float4*>(a.g + i);
                const float4 b4 = *reinterpret_cast<const float4*>(a.b + i);
                const float y[4] = {(v[k][0] - mean) * rstd * g4.x + b4.x, (v[k][1] - mean) * rstd * g4.y + b4.y,
                                    (v[k][2] - mean) * rstd * g4.z + b4.z, (v[k][3] - mean) * rstd * g4.w + b4.w};
                *reinterpret_cast<float4*>(a.h + o) = make_float4(y[0], y[1], y[2], y[3]);
                __half2 h01, h23, l01, l23;
                split_hl2(y[0], y[1], h01, l01);
                split_hl2(y[2], y[3], h23, l23);
                *reinterpret_cast<__half2*>(a.hhi + o) = h01;
                *reinterpret_cast<__half2*>(a.hhi + o + 2) = h23;
                *reinterpret_cast<__half2*>(a.hlo + o) = l01;
                *reinterpret_cast<__half2*>(a.hlo + o + 2) = l23;
            }
        }
    }
}

}  // namespace

struct TpComm {
    void* lib = nullptr;
    ncclComm_t comm = nullptr;
    std::string err;
    ncclResult_t (*init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*destroy)(ncclComm_t) = nullptr;
    const char* (*err_str)(ncclResult_t) = nullptr;
    int n = 1, me = 0;
    size_t part_elems = 0;
    float* part[2] = {nullptr, nullptr};   // ours
    uint32_t* flags = nullptr;             // ours [TP_MAX][TP_MAXB]
    uint32_t* ep = nullptr;                // [TP_MAXB]
    int* d_err = nullptr;
    bool peer = false;                     // partials read from peer memory
    float* peer_part[2][TP_MAX] = {};      // mapped (ours at [me])
    uint32_t* peer_flags[TP_MAX] = {};
};

namespace {

bool fail(TpComm* c, const std::string& what) {
    c->err = what;
    return false;
}

// Exchanges CUDA IPC handles of the partial buffers and the flag array through an NCCL
// all-gather and maps the peers' buffers. False (with peer = false) where the GPUs cannot map
// each other's memory.
bool map_peers(TpComm* c, cudaStream_t st) {
    constexpr int H = (int)sizeof(cudaIpcMemHandle_t);
    cudaIpcMemHandle_t mine[3];
    if (cudaIpcGetMemHandle(&mine[0], c->part[0]) != cudaSuccess ||
        cudaIpcGetMemHandle(&mine[1], c->part[1]) != cudaSuccess ||
        cudaIpcGetMemHandle(&mine[2], c->flags) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    char *dsend = nullptr, *drecv = nullptr;
    if (cudaMalloc(&dsend, 3 * H) != cudaSuccess || cudaMalloc(&drecv, (size_t)3 * H * c->n) != cudaSuccess) {
        cudaFree(dsend);
        return false;
    }
    std::string all((size_t)3 * H * c->n, '\0');
    bool ok = cudaMemcpy(dsend, mine, 3 * H, cudaMemcpyHostToDevice) == cudaSuccess &&
              c->all_gather(dsend, drecv, 3 * H, ncclChar, c->comm, st) == ncclSuccess &&
              cudaStreamSynchronize(st) == cudaSuccess &&
              cudaMemcpy(&all[0], drecv, all.size(), cudaMemcpyDeviceToHost) == cudaSuccess;
    cudaFree(dsend);
    cudaFree(drecv);
    if (!ok) return false;
    for (int q = 0; q < c->n; ++q) {
        if (q == c->me) {
            c->peer_part[0][q] = c->part[0];
            c->peer_part[1][q] = c->part[1];
            c->peer_flags[q] = c->flags;
            continue;
        }
        cudaIpcMemHandle_t hq[3];
        memcpy(hq, &all[(size_t)3 * H * q], 3 * H);
        void* p[3] = {nullptr, nullptr, nullptr};
        for (int k = 0; k < 3; ++k) {
            if (cudaIpcOpenMemHandle(&p[k], hq[k], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                cudaGetLastError();
                return false;
            }
        }
        c->peer_part[0][q] = static_cast<float*>(p[0]);
        c->peer_part[1][q] = static_cast<float*>(p[1]);
        c->peer_flags[q] = static_cast<uint32_t*>(p[2]);
    }
    return true;
}

}  // namespace

TpComm* tp_create(int tp_size, int tp_rank, const void* id, int device, size_t part_elems) {
    TpComm* c = new TpComm();
    c->n = tp_size;
    c->me = tp_rank;
    c->part_elems = part_elems;
    if (tp_size > TP_MAX) {
        fail(c, "at most 8 tensor-parallel ranks");
        return c;
    }
    c->lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!c->lib) {
        fail(c, std::string("dlopen libnccl.so.2: ") + dlerror());
        return c;
    }
    c->init_rank = (decltype(c->init_rank))dlsym(c->lib, "ncclCommInitRank");
    c->all_reduce = (decltype(c->all_reduce))dlsym(c->lib, "ncclAllReduce");
    c->all_gather = (decltype(c->all_gather))dlsym(c->lib, "ncclAllGather");
    c->destroy = (decltype(c->destroy))dlsym(c->lib, "ncclCommDestroy");
    c->err_str = (decltype(c->err_str))dlsym(c->lib, "ncclGetErrorString");
    if (!c->init_rank || !c->all_reduce || !c->all_gather || !c->destroy || !c->err_str) {
        fail(c, "NCCL symbols missing");
        return c;
    }
    cudaSetDevice(device);
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    ncclResult_t r = c->init_rank(&c->comm, tp_size, uid, tp_rank);
    if (r != ncclSuccess) {
        fail(c, std::string("ncclCommInitRank: ") + c->err_str(r));
        return c;
    }
    const size_t fbytes = (size_t)TP_MAX * TP_MAXB * 4;
    if (cudaMalloc(&c->part[0], part_elems * 4) != cudaSuccess || cudaMalloc(&c->part[1], part_elems * 4) != cudaSuccess ||
        cudaMalloc(&c->flags, fbytes) != cudaSuccess || cudaMalloc(&c->ep, TP_MAXB * 4) != cudaSuccess ||
        cudaMalloc(&c->d_err, 4) != cudaSuccess || cudaMemset(c->flags, 0, fbytes) != cudaSuccess ||
        cudaMemset(c->ep, 0, TP_MAXB * 4) != cudaSuccess || cudaMemset(c->d_err, 0, 4) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess) {
        fail(c, "tensor-parallel buffers: out of device memory");
        return c;
    }
    cudaStream_t st;
    if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) {
        fail(c, "stream creation failed");
        return c;
    }
    c->peer = map_peers(c, st);
    // every rank must take the same path: agree through one more all-gather
    int* dflag = nullptr;
    int* dall = nullptr;
    int mine = c->peer ? 1 : 0;
    bool ok = cudaMalloc(&dflag, 4) == cudaSuccess && cudaMalloc(&dall, 4 * TP_MAX) == cudaSuccess &&
              cudaMemcpy(dflag, &mine, 4, cudaMemcpyHostToDevice) == cudaSuccess &&
              c->all_gather(dflag, dall, 1, ncclInt32, c->comm, st) == ncclSuccess &&
              cudaStreamSynchronize(st) == cudaSuccess;
    int all[TP_MAX] = {0};
    if (ok) ok = cudaMemcpy(all, dall, 4 * tp_size, cudaMemcpyDeviceToHost) == cudaSuccess;
    cudaFree(dflag);
    cudaFree(dall);
    cudaStreamDestroy(st);
    if (!ok) {
        fail(c, "tensor-parallel bootstrap all-gather failed");
        return c;
    }
    for (int q = 0; q < tp_size; ++q) c->peer = c->peer && all[q] == 1;
    return c;
}

float* tp_partial(TpComm* c, int parity) { return c->part[parity & 1]; }

bool tp_peer_mapped(const TpComm* c) { return c && c->peer; }

int tp_reduce_ln(TpComm* c, int parity, float* x, int M, int d, const float* g, const float* b, float eps, float* h,
                 __half* hhi, __half* hlo, cudaStream_t st) {
    if (M <= 0) return 0;
    if (d > TP_THREADS * TP_V4 * 4 || d % 4 != 0 || (size_t)M * d > c->part_elems) {
        c->err = "tensor-parallel reduce: row too wide, not a multiple of 4, or too many rows";
        return -1;
    }
    TpArgs a{};
    parity &= 1;
    if (c->peer) {
        for (int q = 0; q < c->n; ++q) {
            a.part[q] = c->peer_part[parity][q];
            a.flags[q] = c->peer_flags[q];
        }
        a.n = c->n;
        a.me = c->me;
    } else {
        // no peer mapping: NCCL sums the partials in place, the kernel adds the one buffer
        ncclResult_t r = c->all_reduce(c->part[parity], c->part[parity], (size_t)M * d, ncclFloat32, ncclSum, c->comm, st);
        if (r != ncclSuccess) {
            c->err = std::string("ncclAllReduce: ") + c->err_str(r);
            return -1;
        }
        a.part[0] = c->part[parity];
        a.flags[0] = c->flags;
        a.n = 1;
        a.me = 0;
    }
    a.my_flags = c->flags;
    a.ep = c->ep;
    a.err = c->d_err;
    a.x = x;
    a.M = M;
    a.d = d;
    a.g = g;
    a.b = b;
    a.eps = eps;
    a.h = h;
    a.hhi = hhi;
    a.hlo = hlo;
    const int grid = M < TP_MAXB ? M : TP_MAXB;
    k_tp_reduce_ln<<<grid, TP_THREADS, 0, st>>>(a);
    if (cudaGetLastError() != cudaSuccess) {
        c->err = "tensor-parallel reduce launch failed";
        return -1;
    }
    return 0;
}

int tp_take_error(TpComm* c, cudaStream_t st) {
    if (!c || !c->d_err) return 0;
    int h = 0;
    if (cudaMemcpyAsync(&h, c->d_err, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess) return -1;
    if (cudaStreamSynchronize(st) != cudaSuccess) return -1;
    if (h != 0) cudaMemsetAsync(c->d_err, 0, 4, st);
    return h;
}

const int* tp_err_word(const TpComm* c) { return c ? c->d_err : nullptr; }

const char* tp_last_error(const TpComm* c) { return c ? c->err.c_str() : "no communicator"; }

void tp_destroy(TpComm* c) {
    if (!c) return;
    for (int q = 0; q < c->n && q < TP_MAX; ++q) {
        if (q == c->me) continue;
        for (int k = 0; k < 2; ++k)
            if (c->peer_part[k][q]) cudaIpcCloseMemHandle(c->peer_part[k][q]);
        if (c->peer_flags[q]) cudaIpcCloseMemHandle(c->peer_flags[q]);
    }
    cudaFree(c->part[0]);
    cudaFree(c->part[1]);
    cudaFree(c->flags);
    cudaFree(c->ep);
    cudaFree(c->d_err);
    if (c->comm && c->destroy) c->destroy(c->comm);
    delete c;
}

}  // namespace gpt2q
