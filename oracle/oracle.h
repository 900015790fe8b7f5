/* CPU oracle for the quantized GPT-2 forward.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker that the CUDA path is
 * compared against; it is never linked into, loaded by, or called from the
 * product library (smelt_b200/, include/gpt2q.h). Only tests/, the smoke entry
 * and the CPU-baseline leg of bench.py may load it.
 *
 * It restates, in C++17 compiled with -ffp-contract=off (Rust never contracts
 * a*b+c unless mul_add is written, so neither may we), the reference's CPU
 * executor and numeric atoms of LukasParke/smelt:
 *   experiments/model-lab/src/atoms.rs:10-164     f16 codec, q8_encode, gemv_q8/gemv_f16
 *   experiments/model-lab/src/gpt2.rs:121-396     vec_f32, matmul, layernorm, vec_row,
 *                                                 step, empty_kv, nll_per_token,
 *                                                 generate_greedy, argmax
 *   experiments/model-lab/src/bin/pack.rs:47-84   Conv1D transpose + atom policy
 *   experiments/perf-lab/src/bin/atoms.rs:9-209   int4 atom math, perf-lab RNG, metrics
 *   experiments/model-lab/src/gpu_backward.rs:835-856  xorshift64* Rng
 *   experiments/model-lab/src/bin/bwparity.rs:215-305  independent f64 forward
 *
 * Parity pin: the perf-lab atom experiment (int4 q4_sym_b32_f16scale, bf16,
 * mxfp4, two-level int4 over five seeded distributions) is re-run by
 * orc_perf_atoms() and compared with the reference's committed output
 * docs/experiments/results/atoms.log:4-23. That pins the f16 codec, the int4
 * quantizer and the perf-lab RNG. The forward itself has no golden logits in
 * the reference for synthetic weights; it is pinned by restatement plus the
 * independent f64 forward and an HF-transformers float64 cross-check in tests.
 */
#ifndef SMELT_ORACLE_H
#define SMELT_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- numeric atoms (atoms.rs) ---- */
uint16_t orc_f32_to_f16(float x);
float orc_f16_to_f32(uint16_t h);
/* q8: 34 B per 32 values; q4: 18 B per 32 values. n % 32 == 0. */
void orc_q8_encode(const float* x, size_t n, uint8_t* out);
void orc_q4_encode(const float* x, size_t n, uint8_t* out);
/* y[r-r0] += dot(W_row_r, x) for r in [r0, r_end) (atoms.rs:89-164). */
void orc_gemv_q8(const uint8_t* w, const float* x, float* y, size_t rows, size_t cols,
                 size_t r0, size_t r_end);
void orc_gemv_q4(const uint8_t* w, const float* x, float* y, size_t rows, size_t cols,
                 size_t r0, size_t r_end);
void orc_gemv_f16(const uint8_t* w, const float* x, float* y, size_t rows, size_t cols,
                  size_t r0, size_t r_end);
void orc_gemv_f32(const uint8_t* w, const float* x, float* y, size_t rows, size_t cols,
                  size_t r0, size_t r_end);

/* ---- converter policy (pack.rs:47-84) ----
 * policy: "auto" (Q8 for 2-D numel>=4096 else F16), "core.f16", "core.i8.b32.f16scale",
 * "q4auto" (int4 for 2-D numel>=4096 else F16), "f32" (every tensor core.f32).
 * hf_shape is the HF safetensors shape; Conv1D weights are transposed to [out,in].
 * out_bytes must hold orc_pack_size(...) bytes. atom_out receives the atom name. */
size_t orc_pack_size(const char* name, int ndim, const int64_t* hf_shape, const char* policy);
int orc_pack_tensor(const char* name, int ndim, const int64_t* hf_shape, const float* data,
                    const char* policy, int64_t* shape_out, char* atom_out, size_t atom_cap,
                    uint8_t* out_bytes);

/* ---- RNG (gpu_backward.rs:835-856 xorshift64*, perf-lab Box-Muller) ---- */
uint64_t orc_rng_new(uint64_t seed);
/* Fills n normals N(0, std) drawn with uniform=(next>>11)/2^53 and the perf-lab
 * Box-Muller formula; state is advanced in place. */
void orc_rng_normal_f32(uint64_t* state, float* out, size_t n, double stdv);
void orc_rng_below(uint64_t* state, uint32_t* out, size_t n, uint64_t bound);

/* ---- perf-lab atom experiment (perf-lab/src/bin/atoms.rs:177-209) ----
 * Writes 20 (rms_rel_err, cos_sim) pairs in the order of atoms.log:4-23. */
void orc_perf_atoms(double* out40, size_t n_per_dist);

/* ---- engine (gpt2.rs) ---- */
typedef struct orc_engine orc_engine;
orc_engine* orc_engine_new(int n_embd, int n_layer, int n_head, int n_ctx, int vocab,
                           float ln_eps, int threads);
int orc_engine_add(orc_engine* e, const char* name, const char* atom, int ndim,
                   const int64_t* shape, const uint8_t* data, uint64_t len);
void orc_engine_free(orc_engine* e);
/* kv layout: [n_layer][2][n_ctx * n_embd] f32, caller-owned, zero-initialised. */
size_t orc_kv_floats(const orc_engine* e);
int orc_engine_step(const orc_engine* e, uint32_t tok, int pos, float* kv, float* logits);
/* T consecutive steps of one sequence at positions pos0..pos0+T-1 (kv rows 0..pos0-1 written by
 * earlier steps), computed over all positions at once with bit-identical results; writes the K/V
 * rows and the vocab logits of the last position. */
int orc_engine_prefill(const orc_engine* e, const uint32_t* ids, int T, int pos0, float* kv,
                       float* logits_last);
int orc_vec_f32(const orc_engine* e, const char* name, float* out, uint64_t n);
int orc_vec_row(const orc_engine* e, const char* name, uint32_t row, float* out, uint64_t n);
/* Returns number of generated tokens written to out (<= steps). */
int orc_generate_greedy(const orc_engine* e, const uint32_t* prompt, int n_prompt, int steps,
                        uint32_t* out);
double orc_nll_per_token(const orc_engine* e, const uint32_t* ids, int n);
/* Post-ln_f adapter h += B (A h) applied by every later step (gpu.rs:188-194,
 * cu/gpt2.cu:196-215); A [r][d], B [d][r]; r = 0 clears. */
int orc_set_adapter(orc_engine* e, const float* a, const float* b, int r);
uint32_t orc_argmax(const float* v, size_t n);
/* Independent float64 forward over T positions (bwparity.rs:215-305) on the
 * dequantised weights; logits_out is [T][vocab] f64. */
int orc_forward_f64(const orc_engine* e, const uint32_t* ids, int T, double* logits_out);

#ifdef __cplusplus
}
#endif
#endif
