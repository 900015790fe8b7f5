/* gpt2q — B200 (sm_100a) GPT-2 forward over group-quantized weights.
 *
 * C-ABI boundary of the smelt_b200 library (libgpt2q.so). It replaces the CUDA
 * executor of LukasParke/smelt's model-lab (experiments/model-lab/src/gpu.rs,
 * kernels in src/cu/gpt2.cu) and keeps the shape of its Rust API so a thin FFI
 * crate restores `Gpu::new / step / clear_kv`. Citations below are paths inside
 * that project.
 *
 * Conventions
 *  - Every call returns an int status: GPT2Q_OK (0) or a negative GPT2Q_E* code.
 *    Nothing aborts or panics; gpt2q_last_error() gives the message.
 *  - One handle per GPU. A handle is not thread-safe; distinct handles may be
 *    driven from distinct threads.
 *  - Host buffers are caller-owned; gpt2q_create copies every tensor, so the
 *    caller keeps ownership (gpu.rs:114-127 copies too).
 *  - Weight payloads use the SMT TENSORS layout (model-lab/src/bin/pack.rs:68-94):
 *      "core.i8.b32.f16scale"  [rows][cols/32] blocks of 34 B: f16 scale LE + 32 x int8
 *      "core.i4.b32.f16scale"  [rows][cols/32] blocks of 18 B: f16 scale LE + 16 B, byte j =
 *                              elem j (low nibble) | elem j+16 (high nibble), two's complement
 *      "core.f16"              IEEE half, little endian
 *      "core.f32"              IEEE float (fp32 weights)
 *    2-D weights are [out, in] (pack.rs transposes HF Conv1D at convert time).
 *  - Tensor names follow the HF GPT-2 names used by the pack: wte.weight,
 *    wpe.weight, ln_f.{weight,bias}, h.{L}.ln_1/ln_2.{weight,bias},
 *    h.{L}.attn.c_attn/c_proj.{weight,bias}, h.{L}.mlp.c_fc/c_proj.{weight,bias}.
 *  - Greedy argmax follows gpt2.rs:390-396: IEEE total order, ties -> LAST index.
 */
#ifndef GPT2Q_H
#define GPT2Q_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GPT2Q_OK 0
#define GPT2Q_EARG -1      /* bad argument / shape / name */
#define GPT2Q_EOOM -2      /* device allocation failed */
#define GPT2Q_ECUDA -3     /* CUDA runtime error */
#define GPT2Q_ENCCL -4     /* NCCL error (tensor-parallel handles) */
#define GPT2Q_ETIMEOUT -5  /* a bounded device-side wait gave up */
#define GPT2Q_EUNSUP -6    /* unsupported configuration */

typedef struct gpt2q_handle gpt2q_handle;

/* Model architecture (gpt2.rs:11-19 Meta) plus capacity of this handle. */
typedef struct gpt2q_config {
    int32_t n_embd;
    int32_t n_layer;
    int32_t n_head;
    int32_t n_ctx;
    int32_t vocab;
    float ln_eps;
    int32_t max_seqs;   /* KV-cache slots (sequences resident at once); >= 1 */
    int32_t max_tokens; /* tokens per prefill chunk (activation workspace); 0 = default */
} gpt2q_config;

/* One tensor record of the SMT TENSORS section (format.rs:17-28 TensorRecord). */
typedef struct gpt2q_tensor_desc {
    const char* name;
    const char* atom;
    int32_t ndim;
    int64_t shape[2];
    const void* data; /* host pointer to the payload */
    uint64_t len;     /* payload bytes */
} gpt2q_tensor_desc;

/* Replaces Gpu::new(&Engine) (gpu.rs:75-157): uploads every tensor (quantized
 * ones stay quantized in HBM), allocates the KV arena for cfg->max_seqs
 * sequences of n_ctx positions and the activation workspace. */
int gpt2q_create(const gpt2q_config* cfg, const gpt2q_tensor_desc* tensors, int n_tensors,
                 int device, gpt2q_handle** out);

/* Tensor-parallel handle (no counterpart in the reference, which is single-GPU,
 * gpu.rs:76): rank `tp_rank` of `tp_size` keeps its column slice of c_attn
 * (whole heads) and c_fc and its row slice of attn/mlp c_proj; the two c_proj
 * partial sums per layer are added by the library's own kernel from peer memory
 * when the GPUs can map each other's memory (gpt2q_info "tp_peer_mapped"), else
 * by an NCCL all-reduce. nccl_id points to the 128-byte ncclUniqueId made by
 * rank 0 and shared by the caller. */
int gpt2q_create_tp(const gpt2q_config* cfg, const gpt2q_tensor_desc* tensors, int n_tensors,
                    int device, int tp_size, int tp_rank, const void* nccl_id,
                    gpt2q_handle** out);

/* Frees everything; replaces the Drop of Gpu. Safe on NULL. */
void gpt2q_destroy(gpt2q_handle* h);

/* Last error message of this handle (or of the last failed create when h is NULL). */
const char* gpt2q_last_error(const gpt2q_handle* h);

/* Replaces Gpu::clear_kv (gpu.rs:203-209). slots == NULL clears every slot. */
int gpt2q_reset_kv(gpt2q_handle* h, const int32_t* slots, int n_slots);

/* Exactly Gpu::step (gpu.rs:212-379): batch 1, KV slot 0, token `tok` at
 * position `pos`; writes vocab fp32 logits to host `logits`. */
int gpt2q_step(gpt2q_handle* h, uint32_t tok, int32_t pos, float* logits);

/* Batched decode: one token per sequence. Sequence i feeds tok[i] at pos[i]
 * into KV slot slots[i] (slots == NULL: slot i), attends over positions
 * 0..pos[i] of that slot. Optional outputs (host, may be NULL): logits
 * [n_seq][vocab], next_tok [n_seq] (greedy argmax). Engine::step batched over
 * sequences (gpt2.rs:227-332). */
int gpt2q_decode(gpt2q_handle* h, const uint32_t* tok, const int32_t* pos, const int32_t* slots,
                 int n_seq, float* logits, uint32_t* next_tok);

/* Prefill whole prompts starting at position 0. Sequence i owns tokens
 * [seq_offsets[i], seq_offsets[i+1]) and KV slot slots[i] (NULL: slot i).
 * Optional host outputs: logits_last [n_seq][vocab] at each prompt's last
 * position, next_tok [n_seq]. Equivalent to feeding every prompt token through
 * Engine::step (gpt2.rs:373-381) but computed as one batched pass. */
int gpt2q_prefill(gpt2q_handle* h, const uint32_t* tokens, const int32_t* seq_offsets,
                  const int32_t* slots, int n_seq, float* logits_last, uint32_t* next_tok);

/* Continues the sequences of the previous gpt2q_prefill/gpt2q_decode call for
 * `steps` more greedy decode steps entirely on the device: each step feeds the
 * previous step's argmax token at position+1. Optional host output
 * out_tokens [steps][n_seq]. Fails with GPT2Q_EARG when a position would reach n_ctx. */
int gpt2q_decode_steps(gpt2q_handle* h, int steps, uint32_t* out_tokens);

/* generate_greedy (gpt2.rs:367-388) for a batch of prompts: prefill, then
 * steps-1 device-side decode steps; out [n_seq][steps]. Prompts are clipped the
 * same way (positions > n_ctx-1 stop generation; missing tokens are written as
 * UINT32_MAX). */
int gpt2q_generate_greedy(gpt2q_handle* h, const uint32_t* tokens, const int32_t* seq_offsets,
                          int n_seq, int steps, uint32_t* out);

/* Publish a plastic adapter applied to the post-ln_f hidden state of every later step and
 * prefill: h += B (A h), A [r][d] and B [d][r] fp32 row-major, 1 <= r <= 256
 * (Gpu::set_adapter gpu.rs:188-194, k_adapter_apply cu/gpt2.cu:196-215). The copy is made
 * on the handle's stream: work enqueued before the call sees the previous generation, work
 * after it the new one (RCU-style). Host buffers may be reused when the call returns. */
int gpt2q_set_adapter(gpt2q_handle* h, const float* A, const float* B, int r);
/* Remove the adapter (Gpu::clear_adapter, gpu.rs:195). */
int gpt2q_clear_adapter(gpt2q_handle* h);

/* Teacher-forced negative log-likelihood per token of ids[0..n-1]
 * (nll_per_token, gpt2.rs:347-364): the mean over positions p = 0..n-2 of
 * -(logit[ids[p+1]] - max) + ln(sum exp(logit - max)), with the log-sum-exp in f64.
 * One prefill over the sequence in cache slot `slot` (its KV cache is overwritten),
 * the head on every position, and the per-position terms on the device: logits
 * never leave the GPU; only the n-1 f64 terms are read back and summed in order.
 * 2 <= n <= min(n_ctx, max_tokens). */
int gpt2q_nll(gpt2q_handle* h, const uint32_t* ids, int n, int slot, double* out_nll);

/* Dequantize a weight tensor exactly as Engine::vec_f32 (gpt2.rs:121-142)
 * into host `out` (n floats). Computed on the device from the uploaded bytes. */
int gpt2q_dequant(gpt2q_handle* h, const char* name, float* out, uint64_t n);

/* Number of kernel launches issued so far (Gpu::launches, gpu.rs:70). A CUDA
 * graph replay counts the kernels it contains. */
uint64_t gpt2q_launches(const gpt2q_handle* h);

/* Launch on this CUDA stream (a cudaStream_t) instead of the handle's own. */
int gpt2q_set_stream(gpt2q_handle* h, void* stream);

/* Wait for all work of the handle. */
int gpt2q_sync(gpt2q_handle* h);

/* Per-launch timing (CUDA events around every kernel; disables CUDA graphs
 * while on). gpt2q_profile_read writes a JSON object
 * {"kernel": {"launches": n, "ms": t, "bytes": algorithmic bytes}, ...}. */
int gpt2q_profile(gpt2q_handle* h, int enable);
int gpt2q_profile_read(gpt2q_handle* h, char* json, size_t cap);

/* Runs one decode step of the current sequences; the first launch of every kernel
 * type (the argmax excepted) is replayed `reps` times back to back in a CUDA graph with
 * the step's own arguments and timed with CUDA events. Writes JSON
 * {"kernel": {"us": per-launch time, "bytes": algorithmic bytes per launch,
 *  "per_step": launches per decode step}, ...}. The replays repeat residual
 * additions, so decode results after this call are not meaningful until the next
 * prefill. */
int gpt2q_profile_kernels(gpt2q_handle* h, int reps, char* json, size_t cap);

/* Which execution paths this handle uses, as JSON:
 * {"persistent_decode": bool, "persistent_why": reason when false,
 *  "persistent_ctas": CTAs of the persistent launch, "tensor_core": bool}.
 * The persistent decode serves every single-sequence decode step (gpt2q_step,
 * gpt2q_decode with n_seq = 1, gpt2q_decode_steps with one sequence); the
 * environment variable GPT2Q_NO_PERSISTENT at create time turns it off.
 * No counterpart in the reference (gpu.rs has one kernel sequence). */
int gpt2q_info(gpt2q_handle* h, char* json, size_t cap);

/* Greedy argmax (IEEE total order, ties -> last index) of n_rows rows of device fp32
 * logits (row stride ld >= vocab floats) into device d_next[n_rows], on `stream` (a
 * cudaStream_t; NULL = legacy default stream). Allocates nothing: its per-row scratch is
 * a fixed array inside the library, for callers that cannot allocate device memory at
 * that point (a decode loop that must not synchronise the device, or code under another
 * framework's memory pool). No counterpart in the reference. Limit: n_rows <=
 * GPT2Q_NOALLOC_MAX_ROWS, else GPT2Q_EARG. A call looks up the scratch array's device
 * address (cudaGetSymbolAddress) unless `stream` reports an active capture, when it uses
 * the address an earlier call found; the first call on a device therefore does the set-up and
 * should come before any stream capture. All calls share the scratch, so calls that overlap on
 * the GPU race; serialise them. Errors are reported by gpt2q_last_error(NULL). */
#define GPT2Q_NOALLOC_MAX_ROWS 1024
int gpt2q_argmax_noalloc(const float* d_logits, int vocab, int ld, int n_rows, uint32_t* d_next, void* stream);

/* Workload utilities for seeded synthetic weights/tokens (no counterpart in the
 * reference's GPU API): xorshift64* Rng of model-lab/src/gpu_backward.rs:835-856
 * (Rng::new(seed) = seed ^ 0x9E3779B97F4A7C15) with the Box-Muller normal of
 * perf-lab/src/bin/atoms.rs:78-83. `state` is advanced in place. */
uint64_t gpt2q_rng_new(uint64_t seed);
/* Converter group quantisers (host, multithreaded): n % 32 == 0 values -> SMT payload.
 * q8: atoms.rs:65-78 (34 B per group); q4: perf-lab atoms.rs:89-99 math, 18 B per group. */
int gpt2q_quantize_q8(const float* x, size_t n, uint8_t* out);
int gpt2q_quantize_q4(const float* x, size_t n, uint8_t* out);
void gpt2q_rng_normal_f32(uint64_t* state, float* out, size_t n, double stdv);
void gpt2q_rng_below(uint64_t* state, uint32_t* out, size_t n, uint64_t bound);

/* SMT container loading (Engine::load, gpt2.rs:43-89, over PackReader, format.rs:94-175).
 * The file is memory-mapped; with verify != 0 the merkle content_id (format.rs:121-145: blake3
 * over the sorted BLAKE3 digests of every section) and every tensor digest (first 16 bytes of
 * blake3 of its payload, gpt2.rs:91-110) are checked on all host threads, and a mismatch fails
 * with GPT2Q_EARG and a message naming the section or tensor. META.arch supplies n_embd,
 * n_layer, n_head, n_ctx, vocab_size and ln_eps; the TENSORS records become the tensor list of
 * gpt2q_create. Errors are reported by gpt2q_last_error(NULL). */
int gpt2q_create_from_smt(const char* path, int device, int max_seqs, int max_tokens, int verify,
                          gpt2q_handle** out);

/* Parses (and with verify != 0 verifies) an SMT container without touching a GPU; writes JSON
 * {"content_id": hex, "verified": bool, "arch": {...}, "tensors": [{name, atom, len, shape}]}. */
int gpt2q_smt_inspect(const char* path, int verify, char* json, size_t cap);

/* BLAKE3 (32-byte output, unkeyed) of len bytes, the hash the SMT digests use; host threads
 * hash the subtrees of large inputs. */
int gpt2q_blake3(const void* data, uint64_t len, uint8_t* out32);

/* ---- Backward of the trunk (the reference's plasticity path: cu/backward.cu, gpu_backward.rs) ----
 *
 * Input gradient of the whole trunk for one sequence (trunk_input_grad, gpu_backward.rs:651-790,
 * over the activations of bwparity.rs forward_stash:448-580): the forward over ids[0..n-1]
 * (positions 0..n-1) keeps every activation the backward needs on the device, then
 * dlogits [n][vocab] (host) is propagated through the tied head, ln_f and every layer, all
 * positions at once. Writes dx [n][n_embd] (host): the gradient with respect to the embedding
 * output wte[ids[p]] + wpe[p] at each position. lnf_out (host, may be NULL) receives the ln_f
 * output [n][n_embd], which the tied head's weight gradient needs (dlogits[p][v] * lnf_out[p]).
 * The plastic adapter is not part of the trunk. 1 <= n <= n_ctx; single-GPU handles only. */
int gpt2q_trunk_input_grad(gpt2q_handle* h, const uint32_t* ids, int n, const float* dlogits, float* dx,
                           float* lnf_out);

/* Per-op backward kernels with the BwdOps signatures (gpu_backward.rs:69-93): host buffers,
 * uploaded and downloaded per call on `device`, like GpuBackward's methods (gpu_backward.rs:
 * 307-377). Errors are reported by gpt2q_last_error(NULL).
 * lin_input_grad: dx[i] = sum_r w[r*cols+i] * dy[r] (k_lin_input_grad); cols % 4 == 0. */
int gpt2q_bwd_lin_input_grad(int device, const float* w, const float* dy, int rows, int cols, float* dx);
/* LayerNorm backward of one n-vector (k_ln_backward); dg and db accumulate. */
int gpt2q_bwd_ln_backward(int device, const float* dy, const float* x, const float* g, const float* b, float eps,
                          int n, float* dx, float* dg, float* db);
/* dx[i] = dy[i] * gelu'(x_pre[i]) for the tanh GELU (k_gelu_bwd). */
int gpt2q_bwd_gelu(int device, const float* x_pre, const float* dy, int n, float* dx);
/* Causal training-form attention backward (k_attn_bwd_train): q/k/v/dy [t][stride], head h
 * at column h*hd, stride/hd heads; dq overwritten, dk and dv accumulate. t <= 1024, hd <= 128. */
int gpt2q_bwd_attn_train(int device, const float* q, const float* k, const float* v, const float* dy, int t, int hd,
                         int stride, float* dq, float* dk, float* dv);

#ifdef __cplusplus
}
#endif
#endif /* GPT2Q_H */
