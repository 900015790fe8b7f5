// Backward kernels of the GPT-2 trunk (the reference's plasticity path, cu/backward.cu and
// gpu_backward.rs), batched over positions. All fp32; weights stay in their uploaded atom and
// are dequantised exactly ((float)q * f16(scale)) in registers.
#pragma once
#include <cuda_runtime.h>

#include "common.cuh"

namespace gpt2q {

// Epilogues of the input-gradient GEMM reduction.
enum BwdEpi : int {
    BWD_STORE = 0,     // out[t][c] = sum
    BWD_ADD = 1,       // out[t][c] += sum
    BWD_GELU_BWD = 2,  // out[t][c] = sum * gelu'(xpre[t][c])
};

// Scratch launch_bwd_linear needs for T rows of a W [rows][cols]: split partials (floats) and
// per-tile tickets (unsigned, zeroed once; every launch leaves them at zero).
size_t bwd_linear_part_floats(int T, int rows, int cols);
size_t bwd_linear_counters(int T, int cols);

// dX[t][c] = epi(sum_r dY[t][r] * W[r][c]) for t < T, c < W.cols, r < W.rows (transposed
// product of k_lin_input_grad, cu/backward.cu:18-27, over T positions at once). Row splits
// are summed in fixed order by the last CTA of each tile.
cudaError_t launch_bwd_linear(const QW& w, const float* dY, int ldy, int T, float* part, unsigned* counters, int epi,
                              float* out, int ldo, const float* xpre, int ldx, cudaStream_t st);

// LayerNorm backward per row (k_ln_backward, cu/backward.cu:38-115): out[t] = (epi) dx of row
// t given the saved pre-LN row x[t] and dY[t]. dg/db (may be null) accumulate dY*xhat and dY
// and are only allowed for T == 1.
cudaError_t launch_bwd_ln(const float* dY, int ldy, const float* x, int ldx, const float* g, float eps, int n, int T,
                          int epi, float* out, int ldo, float* dg, float* db, cudaStream_t st);

// out[i] = gelu(x[i]) (tanh form; optional fp16 hi/lo copies for a tensor-core consumer) and
// the GELU backward dx[i] = dy[i] * gelu'(x[i]) (k_gelu_bwd, cu/backward.cu:117-139).
cudaError_t launch_gelu_fwd(const float* x, float* out, __half* ohi, __half* olo, size_t n, cudaStream_t st);
cudaError_t launch_gelu_bwd(const float* x, const float* dy, float* dx, size_t n, cudaStream_t st);

// Causal training-form attention forward for T positions (head dim hd, n_head heads) over
// row-major q/k/v with row strides ldq/ldk/ldv, head h at column h*hd; out [T][ldo] and,
// when ohi is not null, its fp16 hi/lo split (same stride).
cudaError_t launch_attn_fwd_train(const float* q, int ldq, const float* k, int ldk, const float* v, int ldv, int T,
                                  int n_head, int hd, float* out, int ldo, __half* ohi, __half* olo, cudaStream_t st);

// Its backward (k_attn_bwd_train, cu/backward.cu:141-225): dq overwritten; dk/dv overwritten
// (accumulate == 0) or accumulated into (accumulate != 0). `stats` holds 3 * n_head * T floats.
cudaError_t launch_attn_bwd_train(const float* q, int ldq, const float* k, int ldk, const float* v, int ldv,
                                  const float* dy, int lddy, int T, int n_head, int hd, float* dq, int lddq, float* dk,
                                  int lddk, float* dv, int lddv, int accumulate, float* stats, cudaStream_t st);

}  // namespace gpt2q
