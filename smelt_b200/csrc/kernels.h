// Host-side launchers of the gpt2q CUDA kernels (definitions in kernels.cu).
#pragma once
#include <string>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace gpt2q {

// KV arena geometry: [slot][layer][K|V][head][n_ctx][hd] fp32.
struct KVGeom {
    float* base;
    size_t slot_stride, layer_stride, sel_stride, head_stride;
    int hd;
    int n_slots;  // slots in the arena (n_ctx = head_stride / hd)
};

// Prefill attention work item: 64 query rows of one sequence.
struct AttnTile {
    int row0;  // first activation row of the sequence
    int q0;    // first query position of the tile
    int T;     // sequence length
    int slot;  // KV slot
};

cudaError_t launch_embed(const QW& wte, const QW& wpe, const uint32_t* tok, const int* pos, float* x,
                         int d, int M, cudaStream_t st);
// y = LayerNorm(x rows) and, when yhi != null, its fp16 hi/lo split (row stride ldy).
cudaError_t launch_layernorm(const float* x, int ldx, const int* rows, float* y, int ldy, __half* yhi, __half* ylo,
                             const float* g, const float* b, int d, float eps, int M, cudaStream_t st);
// out = epilogue(X[M][K] . W^T) on CUDA cores (fp32 FMA, weights dequantised in registers).
cudaError_t launch_linear_simt(const QW& w, const float* X, int ldx, int M, const Epi& e,
                               cudaStream_t st);
// Post-ln_f plastic adapter of the reference's GPU path (cu/gpt2.cu:196-215): the published
// generation (A [r][d], B [d][r], r; r = 0 means none) lives in device memory, so a captured
// step reads whichever generation is current when it runs.
struct AdapterDesc {
    const float* a;
    const float* b;
    int r;
};
// rows of h (ld floats apart): h += B (A h), and the fp16 hi/lo copy rewritten.
cudaError_t launch_adapter(const AdapterDesc* desc, float* h, __half* hhi, __half* hlo, int ld, int d, int rows,
                           int max_r, cudaStream_t st);
// terms[i] = (l[i][target[i]] - max_i) - ln(sum_j exp(l[i][j] - max_i)) in f64, rows i < rows
// of logits l [rows][ld] (one block per row, fixed-order reductions).
cudaError_t launch_nll_rows(const float* logits, int vocab, int ld, int rows, const int* targets, double* terms,
                            cudaStream_t st);
// err: device error word set when a bounded wait for the staged K/V rows gives up.
cudaError_t launch_attn_decode(const float* q, int ldq, const KVGeom& g, size_t layer_off, const int* slot,
                               const int* pos, float* out, __half* ohi, __half* olo, int ldo, int n_head, int B,
                               float scale, int* err, cudaStream_t st);
cudaError_t launch_attn_prefill(const float* q, int ldq, const KVGeom& g, size_t layer_off,
                                const AttnTile* tiles, int n_tiles, float* out, __half* ohi, __half* olo, int ldo,
                                int n_head, float scale, cudaStream_t st);
// Causal prefill attention on the tensor cores (attn_tc.cu): tiles of 128 queries, head dim 64,
// scale 1/8. Bounded waits record a timeout in `err`.
// Phase stamps of the traced tensor-core attention launch (GPT2Q_ATTN_TRACE), JSON; "" if none.
std::string attn_tc_trace_json();
cudaError_t launch_attn_prefill_tc(const float* q, int ldq, const KVGeom& g, size_t layer_off, const AttnTile* tiles,
                                   int n_tiles, float* out, __half* ohi, __half* olo, int ldo, int n_head, int* err,
                                   cudaStream_t st);
// Greedy argmax per row (total order, ties -> last index). `best` holds one zeroed u64 per
// row; the finaliser consumes and re-zeroes it, writes next[], and optionally logs the
// token at genlog[b][gpos[b]], feeds it back (tok_adv) and advances pos_adv.
cudaError_t launch_argmax(const float* logits, int V, int ld, int B, unsigned long long* best, uint32_t* next,
                          uint32_t* genlog, const int* gpos, int n_ctx, uint32_t* tok_adv, int* pos_adv,
                          cudaStream_t st);
// Programmatic dependent launch on/off (GPT2Q_NO_PDL=1 disables it).
bool pdl_enabled();
cudaError_t launch_dequant(const QW& w, float* out, cudaStream_t st);
// ln_f rows 0..M-1 of h ([M][ldh], K wide) as the int8 pieces and 2^-S scales of the kind::i8 lm
// head (gemm.h launch_head_i8), for MP = 32 or 64 token slots.
cudaError_t launch_head_pieces(const float* h, int ldh, int M, int K, int MP, int8_t* pieces, float* xscale,
                               cudaStream_t st);
// c1[n] = sum_k W[n][k] g[k], c2b[n] = sum_k W[n][k] b[k] + bias[n] (bias may be null): the
// constants of a LayerNorm folded into the linear W that follows it (computed in double).
cudaError_t launch_ln_fold(const QW& w, const float* g, const float* b, const float* bias, float* c1, float* c2b,
                           cudaStream_t st);
// Upload-time layout conversion from the SMT payload (raw, on device).
cudaError_t launch_repack_q8(const uint8_t* raw, int rows, int cols, uint8_t* q, __half* s, int sstride,
                             cudaStream_t st);
cudaError_t launch_repack_q4(const uint8_t* raw, int rows, int cols, uint8_t* q, __half* s, int sstride,
                             cudaStream_t st);
// Bounded host-lag helper for profiling (see kernels.cu).
cudaError_t launch_sleep(unsigned long long ns, cudaStream_t st);
cudaError_t launch_f16_to_f32(const __half* src, float* dst, size_t n, cudaStream_t st);

}  // namespace gpt2q
