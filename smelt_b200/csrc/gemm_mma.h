// Batched-decode linear on the warp-level tensor cores (mma.sync over the exact fp16 values of the
// int8 / int4 weights, group scales applied in fp32) for 1..MMA_MAX_M tokens. See gemm_mma.cu.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <string>

#include "common.cuh"

namespace gpt2q {

constexpr int MMA_MAX_M = 64;             // tokens per launch (8 fragments of 8)
constexpr int MMA_MAX_WARPS = 16;         // warps per CTA, each a group range of the CTA's K range
constexpr int MMA_MAX_SPLITS = 8;         // K splits over the CTAs of a cluster
constexpr int MMA_MAX_TILES = 1024;       // matrices of more 16-row tiles (the tied head) use the tcgen05 GEMM
constexpr int MMA_MAX_SMEM = 225 * 1024;  // staged activations + warp and cluster partials per CTA

// Per-process set-up on the current device (call when a handle is created, outside any capture).
void mma_init();
bool mma_usable(const QW& w, int M);
// mma_usable, and a work layout whose staged activations fit in shared memory exists (with room
// for a folded LayerNorm's statistics when `ln`).
bool mma_fits(const QW& w, int M, bool ln = false);
// A LayerNorm folded into the linear that consumes it: with X = g * x (the gain applied by the
// residual linear that produced x, Epi::ln_g), W LN(x) + bias = rstd (W X - mean W g) + W b + bias
// per token, the mean and rstd combined from the (mean, M2) of 16-element tiles that the
// producer wrote (Epi::stats), and c1 = W g, c2b = W b + bias precomputed per output row.
struct LnFold {
    const float2* stats;  // [token][stats_ld]: tiles 0..n_tiles-1 of a token contiguous
    int stats_ld, n_tiles;
    float eps;
    const float* c1;   // [rows]
    const float* c2b;  // [rows]
};

// X = x_hi + x_lo, fp16 [M][ldx] written by the previous kernel; ldx % 8 == 0. err: device word
// set when the bounded wait for the staged activations gives up. With `ln`, X = g * x and the
// epilogue completes the LayerNorm (see LnFold).
cudaError_t launch_linear_mma(const QW& w, const __half* xhi, const __half* xlo, int ldx, int M, int* err,
                              const Epi& e, cudaStream_t st, const LnFold* ln = nullptr);
// The tied lm head on the warp-level tensor cores for 1..MMA_MAX_M tokens (k_head_mma): one CTA
// per SM stages x = x_hi + x_lo (fp16 [M][ldx], ldx % 8 == 0) once and its warps run whole 16-row
// tiles of W over the full K; out[m][n] for n < w.rows (row stride ldo >= w.rows). `usable` when
// the atom is int8 / int4 and the staged rows fit in shared memory.
bool head_mma_usable(const QW& w, int M, int ldx);
cudaError_t launch_head_mma(const QW& w, const __half* xhi, const __half* xlo, int ldx, int M, float* out, int ldo,
                            int* err, cudaStream_t st);
// Largest number of 16-row tiles per CTA among the launches since the last mma_init (one count
// for the process).
int mma_tiles_per_cta_max();
// Phase stamps of the launch selected by GPT2Q_MMA_TRACE ("" when none), as JSON.
std::string mma_trace_json();

}  // namespace gpt2q
