// Tensor-core (tcgen05 / TMEM) dequant-fused linear for large M (prefill and
// large-batch decode). See gemm.cu.
#pragma once
#include <cuda_runtime.h>

#include "common.cuh"

namespace gpt2q {

struct GemmPlan {
    bool enabled = false;
    int min_m = 1 << 30;  // use the tensor-core path when M >= min_m
    bool usable(const QW& w, int M) const;
};

int gemm_init(GemmPlan& p, int device);
void gemm_destroy(GemmPlan& p);
cudaError_t launch_linear_tc(const GemmPlan& p, const QW& w, const float* X, int ldx, int M, const Epi& e,
                             cudaStream_t st);

}  // namespace gpt2q
