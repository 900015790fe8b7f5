// Tensor-core (tcgen05 / TMEM / TMA) dequant-fused linear for large M (prefill and
// batched decode). See gemm.cu.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

#include <string>

#include "common.cuh"

namespace gpt2q {

struct GemmState;

// Activation operand of the tensor-core linear: x = hi + lo, fp16 [Mmax][ld] buffers
// written by the producing kernel (LayerNorm, attention, GELU epilogue).
struct XSplit {
    const __half* hi;
    const __half* lo;
    int ld;
};

struct GemmPlan {
    bool enabled = false;
    int min_m = 1 << 30;         // the tensor-core path serves M >= min_m
    int presplit_min_m = 1 << 30;  // ... and reads the fp16 hi/lo weight copies for M >= this
    int Mmax = 0, Kmax = 0;
    int* err = nullptr;   // device error word (bounded-wait timeouts)
    // One-shot test switch, next to err: while it is non-zero, the rank-1 CTA of a split-K
    // cluster skips sending its partials, so the peers' bounded waits run out; the launch
    // that does so clears it. Armed at creation by GPT2Q_TEST_SPLITK_STALL=1 (tests only).
    int* fault = nullptr;
    // Split-K partials of the wide tiles (more than 64 tokens), exchanged through L2; one
    // buffer serves every launch on the stream because a launch writes it only after its
    // dependent-launch wait, when the launch before has finished reading it.
    float* part = nullptr;
    size_t part_floats = 0;
    // Products of the wide (more than 64 tokens) tiles: 3 = W_hi X_hi + W_lo X_hi + W_hi X_lo
    // (about 22 bits on both operands), 2 = the exact dequantised weights times fp16
    // activations, 1 = fp16-rounded weights times fp16 activations. Logits max-abs against the
    // oracle on the GPT-2 small / medium / XL workload shapes: 3.2e-5, 2.0e-3, 3.2e-3. All
    // three hold 2e-2, but 1 and 2 flip greedy tokens whose top-2 logits are closer than
    // that (one of 200 sequences of a d = 384 decode batch at 2 products), so the default
    // is 3. GPT2Q_TC_PRODUCTS selects 1 or 2 when the handle is created.
    int products = 3;
    size_t presplit_bytes = 0;
    GemmState* state = nullptr;
    bool usable(const QW& w, int M) const;
};

int gemm_init(GemmPlan& p, int device, int Mmax, int Kmax);
void gemm_destroy(GemmPlan& p);
// Prepare a weight for the tensor-core path: TMA descriptors, the power-of-two prescale
// derived from an upper bound of max |dequantised weight| and, when `presplit`, the
// exact fp16 hi/lo copy used by the compute-bound prefill regime.
int gemm_register_weight(GemmPlan& p, const QW& w, float max_abs_w, bool presplit, cudaStream_t st);
cudaError_t launch_linear_tc(const GemmPlan& p, const QW& w, const XSplit& x, int M, const Epi& e,
                             cudaStream_t st);
// The tied lm head over 1..64 tokens on kind::i8 (int8 weights registered with this plan, K a
// multiple of 64): pieces / xscale as written by launch_head_pieces with MP = 32 (M <= 32) or 64.
bool head_i8_usable(const GemmPlan& p, const QW& w, int M);
cudaError_t launch_head_i8(const GemmPlan& p, const QW& w, const uint8_t* pieces, const float* xscale, int M,
                           float* out, int ldo, cudaStream_t st);
// Phase stamps of the launch selected by GPT2Q_TC_TRACE ("" when none), as JSON.
std::string gemm_trace_json(const GemmPlan& p);
// Reads and clears the device error word (0 = no error). Synchronises `st`.
int gemm_take_error(GemmPlan& p, cudaStream_t st);

}  // namespace gpt2q
