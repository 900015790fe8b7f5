// gpt2q_argmax_noalloc: greedy argmax over device logits that allocates nothing.
//
// Some callers of this library cannot allocate device memory at the moment they need a
// greedy pick: code that must not stall the device (cudaMalloc / cudaFree can synchronise
// the whole device, which breaks latency budgets of a running decode loop), and hosts whose
// device memory is owned by another framework's pool, where a stray cudaMalloc can fail
// even though memory is nominally free. For them this entry point runs the same two argmax kernels as the
// decode path, but their per-row scratch slot lives in a fixed array compiled into the
// library instead of a buffer allocated by a handle.
//
// Limits and caveats:
//  - at most GPT2Q_NOALLOC_MAX_ROWS rows per call (8 KiB of scratch, held by every GPU
//    that loads the library until the process exits); larger calls fail with GPT2Q_EARG;
//  - a call looks up the array's device address, except while `stream` reports an active
//    capture, when it uses the address an earlier call found: the first call on a device does
//    this set-up and should come before any stream capture;
//  - every call shares the one array: calls whose kernels overlap on the GPU (different
//    streams without ordering between them) race and give wrong tokens. Serialise them.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "gpt2q.h"
#include "kernels.h"

namespace gpt2q {
void set_global_error(const std::string& msg);  // runtime.cu
}

namespace {

// One (total-order key, index) slot per row, consumed and cleared by the finaliser.
static __device__ __align__(256) unsigned long long g_noalloc_best[GPT2Q_NOALLOC_MAX_ROWS];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned long long* g_dev_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device, looked up on every call (so a
// module reloaded after a device reset gets its new address) except while the stream reports
// an active capture, when the address an earlier call found is used.
int scratch_for_current_device(cudaStream_t st, unsigned long long** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        gpt2q::set_global_error("gpt2q_argmax_noalloc: no usable current CUDA device");
        return GPT2Q_ECUDA;
    }
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cs) != cudaSuccess) cs = cudaStreamCaptureStatusNone;
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_dev_ptr[dev] || cs == cudaStreamCaptureStatusNone) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_best);
        if (e != cudaSuccess || !p) {
            gpt2q::set_global_error(std::string("gpt2q_argmax_noalloc: cudaGetSymbolAddress failed: ") +
                                    cudaGetErrorString(e));
            return GPT2Q_ECUDA;
        }
        g_dev_ptr[dev] = static_cast<unsigned long long*>(p);
    }
    *out = g_dev_ptr[dev];
    return GPT2Q_OK;
}

}  // namespace

extern "C" int gpt2q_argmax_noalloc(const float* d_logits, int vocab, int ld, int n_rows, uint32_t* d_next,
                                    void* stream) {
    if (!d_logits || !d_next || vocab <= 0 || ld < vocab || n_rows <= 0) {
        gpt2q::set_global_error("gpt2q_argmax_noalloc: null pointer or bad vocab / ld / n_rows");
        return GPT2Q_EARG;
    }
    if (n_rows > GPT2Q_NOALLOC_MAX_ROWS) {
        gpt2q::set_global_error("gpt2q_argmax_noalloc: n_rows " + std::to_string(n_rows) + " exceeds the maximum " +
                                std::to_string(GPT2Q_NOALLOC_MAX_ROWS));
        return GPT2Q_EARG;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    unsigned long long* best = nullptr;
    int rc = scratch_for_current_device(st, &best);
    if (rc != GPT2Q_OK) return rc;
    // the previous call may have stopped before its finaliser cleared the slots
    cudaError_t e = cudaMemsetAsync(best, 0, (size_t)n_rows * sizeof(unsigned long long), st);
    if (e == cudaSuccess)
        e = gpt2q::launch_argmax(d_logits, vocab, ld, n_rows, best, d_next, nullptr, nullptr, 0, nullptr, nullptr, st);
    if (e != cudaSuccess) {
        gpt2q::set_global_error(std::string("gpt2q_argmax_noalloc: ") + cudaGetErrorString(e));
        return GPT2Q_ECUDA;
    }
    return GPT2Q_OK;
}
