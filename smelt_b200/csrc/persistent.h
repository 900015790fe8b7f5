// Persistent single-sequence decode: the whole GPT-2 step (embed, every layer, ln_f, tied
// head, greedy argmax) in ONE launch of 12 thread-block clusters x 8 CTAs, for as many
// consecutive steps as asked. Replaces, for batch 1, the per-kernel decode whose launch and
// ramp latencies (about 50 launches per token) dominate a 21 us weight-streaming floor.
//
// Layout of the work (GPT-2 with head dim 64, one cluster per attention head, CS = 8 CTAs):
//   * Every CTA streams a private, pre-packed copy of exactly the weight bytes it uses, in
//     the order it uses them, through a ring of shared-memory slots filled by 1-D bulk copies
//     (cp.async.bulk, no multicast). The stream runs ahead of the computation across layer and
//     step boundaries, so HBM stays busy while the dependency chain advances.
//   * Per layer, cluster h owns attention head h: q/k/v rows of the head (8 per CTA), causal
//     attention split over positions (partials combined through distributed shared memory),
//     and the head's slice of attn c_proj (split-K by head). It also owns 256 c_fc rows
//     (32 per CTA) and the matching 32-column slice of mlp c_proj (split-K).
//   * The two split-K sums per layer cross clusters through "LL" words: {fp32 value, 32-bit
//     epoch} written with one 8-byte store and polled until the epoch matches, so the data
//     and its arrival flag travel together. Every CTA keeps its own copy of the residual
//     stream x; all copies are bit-identical because every sum runs in a fixed order.
//   * Cluster-internal synchronisation uses mbarriers with remote arrives (bounded waits);
//     the weight-producer warp never joins them.
// Every wait is bounded. On timeout a CTA records an error, raises a global abort flag and
// all CTAs run to the end without waiting, so the kernel always exits.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "common.cuh"

namespace gpt2q {

struct MkLayer {  // fp32 per-layer vectors
    const float *ln1_g, *ln1_b, *ln2_g, *ln2_b, *b_qkv, *b_proj, *b_fc, *b_mproj;
};

struct MkParams {
    const uint8_t* stream;  // per-CTA weight streams, cta_bytes apart
    size_t cta_bytes;
    int seg_bytes;          // one ring slot (= one stream segment)
    int d, n_layer, n_head, vocab, n_ctx, head_rows;  // head_rows: lm-head rows per CTA (last CTA fewer)
    float ln_eps, attn_scale;
    const MkLayer* layers;
    const float *lnf_g, *lnf_b;
    QW wte, wpe;
    float* kv;  // KV arena [slot][layer][K|V][head][n_ctx][64]
    size_t kv_slot, kv_layer, kv_sel, kv_head;  // strides in floats
    const int* slot;      // sequence slot (device)
    int* pos;             // position of the first step; advanced by `steps`
    uint32_t* tok;        // token of the first step; replaced by the last prediction
    uint32_t* next;       // last prediction
    uint32_t* genlog;     // [n_ctx]: token predicted from each position
    float* logits;        // [vocab]: logits of the last step
    unsigned long long *p1, *p2, *best;  // LL exchange words
    uint32_t* epoch;      // LL epoch counter, advanced by `steps`
    int* err;
    int* abort_flag;
    int steps;
    unsigned long long* trace;  // optional [grid][MK_TRACE] globaltimer stamps of the first step
    // optional post-ln_f adapter h += B (A h): device descriptor {a [r][d], b [d][r], r} read at
    // every step's head (layout of AdapterDesc, kernels.h); null or r == 0 means none
    const void* adapter;
};

constexpr int MK_TRACE = 48;  // trace slots per CTA: stamps (globaltimer) except the counters below
constexpr bool mk_trace_counter(int k) { return k == 24 || k == 27 || k == 28 || (k >= 32 && k < 40); }

struct MkPlan {
    bool enabled = false;
    std::string why;      // reason when disabled
    int clusters = 0;     // = n_head
    int seg_bytes = 0;
    size_t cta_bytes = 0;
    int head_rows = 0;
    size_t smem = 0;
    uint8_t* stream = nullptr;
    MkLayer* layers = nullptr;
    unsigned long long *p1 = nullptr, *p2 = nullptr, *best = nullptr;
    uint32_t* epoch = nullptr;
    int* err = nullptr;  // [0] error word, [1] abort flag
    unsigned long long* trace = nullptr;  // allocated when GPT2Q_MK_TRACE is set at create
};

constexpr int MK_CS = 8;  // CTAs per cluster

// Weight tensors the persistent decode needs (all core.i8.b32.f16scale).
struct MkWeights {
    QW wte, wpe;
    std::vector<QW> attn, proj, fc, mproj;
    std::vector<MkLayer> layers;  // host copy of the per-layer vector pointers
};

// Checks eligibility, packs the per-CTA weight streams and allocates the exchange buffers.
// On any unmet requirement the plan stays disabled (plan.why says why) and returns
// cudaSuccess; a CUDA failure is returned as such.
cudaError_t mk_setup(MkPlan& plan, const MkWeights& w, int d, int n_layer, int n_head, int vocab, int n_ctx,
                     int device, cudaStream_t st);
void mk_destroy(MkPlan& plan);
cudaError_t launch_decode_persistent(const MkPlan& plan, const MkParams& p, cudaStream_t st);
// Reads and clears the error word and abort flag: 0 = fine, >0 = a bounded wait gave up.
int mk_take_error(const MkPlan& plan, cudaStream_t st);

}  // namespace gpt2q
