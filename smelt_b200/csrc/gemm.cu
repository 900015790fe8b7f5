// Tensor-core linear: placeholder until the tcgen05 kernel lands; usable() is false
// so every linear runs on the CUDA-core path.
#include "gemm.h"

namespace gpt2q {

bool GemmPlan::usable(const QW& w, int M) const {
    (void)w;
    return enabled && M >= min_m;
}

int gemm_init(GemmPlan& p, int device) {
    (void)device;
    p.enabled = false;
    return 0;
}

void gemm_destroy(GemmPlan& p) { p.enabled = false; }

cudaError_t launch_linear_tc(const GemmPlan& p, const QW& w, const float* X, int ldx, int M, const Epi& e,
                             cudaStream_t st) {
    (void)p; (void)w; (void)X; (void)ldx; (void)M; (void)e; (void)st;
    return cudaErrorNotSupported;
}

}  // namespace gpt2q
