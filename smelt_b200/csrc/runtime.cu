// gpt2q host runtime: the C-ABI of include/gpt2q.h.
//
// Replaces the CUDA executor of LukasParke/smelt (experiments/model-lab/src/gpu.rs):
//  - weights are uploaded once, quantized atoms stay quantized in HBM and are
//    repacked into a 16-byte aligned layout (int8/nibbles + f16 scale rows);
//  - the KV cache is one arena [slot][layer][K|V][head][n_ctx][hd] fp32, i.e. a
//    contiguous cache per sequence (the reference keeps one [n_ctx][d] buffer per
//    layer for a single sequence, gpu.rs:128-134);
//  - a decode step is a fixed kernel sequence captured once per batch size in a
//    CUDA graph; greedy argmax runs on the device and feeds the next step, so a
//    multi-step decode never returns to the host between tokens;
//  - a single sequence on an eligible int8 model decodes through one persistent
//    launch (persistent.h) that runs any number of steps.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "gpt2q.h"
#include "gemm.h"
#include "gemm_mma.h"
#include "backward.h"
#include "kernels.h"
#include "persistent.h"
#include "tp.h"

using namespace gpt2q;

namespace gpt2q {
void set_global_error(const std::string& msg);
}

namespace {

std::string g_create_error;

struct DevBuf {
    void* p = nullptr;
    size_t bytes = 0;
};

struct Linear {
    QW w{};
    float* bias = nullptr;
    int rows = 0, cols = 0;
    std::string name;
    size_t weight_bytes = 0;  // q + scale bytes read by one full pass over W
    float max_abs_w = 0.f;    // upper bound of |dequantised weight| (tensor-core prescale)
    // the LayerNorm before this linear folded into its epilogue: W g and W b + bias per row
    float* ln_c1 = nullptr;
    float* ln_c2b = nullptr;
};

struct LayerW {
    float *ln1_g = nullptr, *ln1_b = nullptr, *ln2_g = nullptr, *ln2_b = nullptr;
    Linear attn, proj, fc, mproj;
};

struct ProfAgg {
    uint64_t launches = 0;
    double ms = 0.0;
    double bytes = 0.0;
};

struct ProfRec {
    std::string name;
    cudaEvent_t a, b;
    double bytes;
};

float half_bits_to_float(uint16_t h) {
    __half_raw r;
    r.x = h;
    return __half2float(__half(r));
}

int atom_id(const std::string& a) {
    if (a == "core.i8.b32.f16scale") return ATOM_Q8;
    if (a == "core.i4.b32.f16scale") return ATOM_Q4;
    if (a == "core.f16") return ATOM_F16;
    if (a == "core.f32") return ATOM_F32;
    return -1;
}

size_t payload_bytes(int atom, size_t numel) {
    switch (atom) {
        case ATOM_Q8: return numel / 32 * 34;
        case ATOM_Q4: return numel / 32 * 18;
        case ATOM_F16: return numel * 2;
        default: return numel * 4;
    }
}

}  // namespace

struct gpt2q_handle {
    gpt2q_config cfg{};
    int device = 0;
    int hd = 64;
    int H_local = 0;   // heads held by this handle
    int d_local = 0;   // H_local * hd
    int fc_local = 0;  // c_fc rows held by this handle
    int tp_size = 1, tp_rank = 0;
    cudaStream_t own_stream = nullptr, stream = nullptr;
    bool use_graphs = true;
    std::string err;
    std::vector<DevBuf> allocs;

    Linear wte, wpe;
    float *lnf_g = nullptr, *lnf_b = nullptr;
    std::vector<LayerW> layers;
    std::map<std::string, const Linear*> lin_by_name;
    std::map<std::string, std::pair<float*, size_t>> vec_by_name;

    KVGeom kv{};
    int Mmax = 0;
    float *x = nullptr, *h = nullptr, *qb = nullptr, *att = nullptr, *f = nullptr, *logits = nullptr;
    // fp16 hi/lo copies of the linear inputs (h: LayerNorm out, att: attention out, f: GELU out)
    __half *h_hi = nullptr, *h_lo = nullptr, *att_hi = nullptr, *att_lo = nullptr, *f_hi = nullptr, *f_lo = nullptr;
    unsigned long long* best = nullptr;  // argmax slots, one per sequence
    // plastic adapter (allocated on first use): two generations of A/B buffers, alternating,
    // and the device descriptor a step reads
    static constexpr int AD_MAX_R = 256;
    bool adapter_on = false;
    int ad_gen = 0;
    float* ad_a[2] = {nullptr, nullptr};
    float* ad_b[2] = {nullptr, nullptr};
    AdapterDesc* d_adapter = nullptr;
    // teacher-forced NLL (allocated on first use): head logits of up to NLL_ROWS positions,
    // the target ids and the per-position f64 terms
    float* nll_logits = nullptr;
    int* nll_tgt = nullptr;
    double* nll_terms = nullptr;
    int* kerr = nullptr;  // device error word of the CUDA-core kernels' bounded waits
    // trunk backward workspace (grown on demand, freed by destroy)
    float* bwd_ws = nullptr;
    size_t bwd_ws_floats = 0;
    // prefill scratch
    uint32_t* p_tok = nullptr;
    int *p_pos = nullptr, *p_slot = nullptr, *p_lastrow = nullptr, *p_lastpos = nullptr;
    AttnTile* p_tiles = nullptr;
    int max_tiles = 0;
    // decode state
    uint32_t *d_tok = nullptr, *d_next = nullptr, *d_genlog = nullptr;
    int *d_pos = nullptr, *d_slot = nullptr;
    int cur_n = 0;
    std::vector<int> hpos, hslot;  // host mirror of the decode state
    // host staging (pinned)
    int* h_stage = nullptr;
    size_t h_stage_ints = 0;
    int* h_err = nullptr;  // pinned: the device error words, read with the step's outputs

    std::map<int, std::pair<cudaGraphExec_t, uint64_t>> dec_graphs;  // 2 B + adapter -> (graph, kernels)
    bool capturing = false;
    uint64_t capture_kernels = 0;
    uint64_t launches = 0;

    // kernel-timing pass (gpt2q_profile_kernels): name -> (us per launch, bytes per launch)
    int ktime_reps = 0;
    std::map<std::string, std::pair<double, double>> ktime_res;
    std::map<std::string, int> ktime_count;

    bool prof = false;
    std::vector<ProfRec> prof_pending;
    std::vector<cudaEvent_t> ev_pool;
    std::map<std::string, ProfAgg> prof_agg;

    GemmPlan gemm;  // tensor-core path for large M
    // warp-level tensor-core path (mma.sync) for mma_min_m <= M <= MMA_MAX_M tokens, and the
    // scratch of its K split over CTAs; GPT2Q_MMA_DISABLE=1 / GPT2Q_MMA_MIN_M at creation
    bool mma_on = true;
    int mma_min_m = 1;  // measured 2.7-4.4x faster than the CUDA-core GEMV at 2-12 tokens
    // LayerNorms inside a layer folded into the warp-level linear that consumes them, from the
    // per-tile statistics the residual linear before them writes ([MMA_MAX_M][n_embd / 16]);
    // GPT2Q_LN_FUSE=0 at creation keeps the LayerNorm launches
    bool ln_fuse = true;
    float2* ln_stats = nullptr;
    // the tied head on kind::i8 (int8 head weights) where the tcgen05 head does not run (fewer
    // than its minimum of 16 rows): pieces of the ln_f output [d/32][3][64][32] and their scales
    // [64][d/32]. GPT2Q_HEAD_I8 at creation: 0 = never, 2 = for every 1..64 rows (tests)
    int head_i8 = 1;
    // the tied head on the warp-level tensor cores (k_head_mma), ahead of the i8 head: 0 = never,
    // 1 = where the tcgen05 head does not run (fewer than 16 rows), 2 = for every 1..64 rows
    // (tests). GPT2Q_HEAD_MMA at creation; off under GPT2Q_MMA_DISABLE=1 and GPT2Q_HEAD_I8=2
    int head_mma = 1;
    int8_t* head_pieces = nullptr;
    float* head_xscale = nullptr;
    MkPlan mk;      // persistent single-sequence decode
    TpComm* tp = nullptr;

    int fail(int code, const std::string& m) {
        err = m;
        return code;
    }
    template <class T>
    T* dalloc(size_t bytes) {
        void* p = nullptr;
        if (bytes == 0) bytes = 16;
        if (cudaMalloc(&p, bytes) != cudaSuccess) return nullptr;
        allocs.push_back({p, bytes});
        return reinterpret_cast<T*>(p);
    }
};

#define CK(call)                                                                        \
    do {                                                                                \
        cudaError_t e_ = (call);                                                        \
        if (e_ != cudaSuccess)                                                          \
            return H->fail(GPT2Q_ECUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
    } while (0)

namespace {

// ------------------------------------------------------------------ launch bookkeeping
int launched(gpt2q_handle* H, const char* name, double bytes, cudaError_t e, cudaEvent_t a, cudaEvent_t b) {
    if (e != cudaSuccess) return H->fail(GPT2Q_ECUDA, std::string(name) + ": " + cudaGetErrorString(e));
    if (H->capturing) {
        H->capture_kernels++;
    } else {
        H->launches++;
    }
    if (a) {
        cudaEventRecord(b, H->stream);
        H->prof_pending.push_back({name, a, b, bytes});
    }
    return GPT2Q_OK;
}

cudaEvent_t pooled_event(gpt2q_handle* H) {
    if (H->ev_pool.empty()) {
        cudaEvent_t e = nullptr;
        cudaEventCreate(&e);
        return e;
    }
    cudaEvent_t e = H->ev_pool.back();
    H->ev_pool.pop_back();
    return e;
}

// Steady-state time of one kernel launch: `reps` back-to-back launches with the very same
// arguments captured in one CUDA graph, timed with CUDA events on the handle's stream.
// Only kernels that may run repeatedly without leaving the buffers out of bounds are
// timed this way (not the argmax finaliser, which advances positions).
template <class F>
int time_kernel(gpt2q_handle* H, const char* name, double bytes, F&& f) {
    cudaError_t e = f();
    if (e != cudaSuccess) return H->fail(GPT2Q_ECUDA, std::string(name) + ": " + cudaGetErrorString(e));
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ex = nullptr;
    CK(cudaStreamBeginCapture(H->stream, cudaStreamCaptureModeThreadLocal));
    for (int r = 0; r < H->ktime_reps; ++r) f();
    CK(cudaStreamEndCapture(H->stream, &g));
    e = cudaGraphInstantiate(&ex, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return H->fail(GPT2Q_ECUDA, std::string("kernel timing graph: ") + cudaGetErrorString(e));
    cudaEvent_t a = pooled_event(H), b = pooled_event(H);
    e = cudaGraphLaunch(ex, H->stream);
    if (e == cudaSuccess) e = cudaEventRecord(a, H->stream);
    if (e == cudaSuccess) e = cudaGraphLaunch(ex, H->stream);
    if (e == cudaSuccess) e = cudaEventRecord(b, H->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(H->stream);
    float ms = 0.f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, a, b);
    H->ev_pool.push_back(a);
    H->ev_pool.push_back(b);
    cudaGraphExecDestroy(ex);
    if (e != cudaSuccess) return H->fail(GPT2Q_ECUDA, std::string("kernel timing: ") + cudaGetErrorString(e));
    H->ktime_res[name] = {ms * 1000.0 / H->ktime_reps, bytes};
    H->launches += 1 + 2 * (uint64_t)H->ktime_reps;
    return GPT2Q_OK;
}

template <class F>
int run_kernel(gpt2q_handle* H, const char* name, double bytes, F&& f) {
    if (H->ktime_reps > 0 && !H->capturing) {
        H->ktime_count[name]++;
        if (!H->ktime_res.count(name) && std::strcmp(name, "argmax") != 0) return time_kernel(H, name, bytes, f);
    }
    cudaEvent_t a = nullptr, b = nullptr;
    if (H->prof && !H->capturing) {
        a = pooled_event(H);
        b = pooled_event(H);
        cudaEventRecord(a, H->stream);
    }
    return launched(H, name, bytes, f(), a, b);
}

#define RUN(name, bytes, expr)                                              \
    do {                                                                    \
        int rc_ = run_kernel(H, name, (double)(bytes), [&]() { return (expr); }); \
        if (rc_ != GPT2Q_OK) return rc_;                                    \
    } while (0)

// ------------------------------------------------------------------ upload
struct Src {
    const gpt2q_tensor_desc* d = nullptr;
};

int upload_vec(gpt2q_handle* H, const gpt2q_tensor_desc* t, size_t n, size_t off, size_t cnt, float** out) {
    int a = atom_id(t->atom);
    if (t->ndim != 1 || (size_t)t->shape[0] != n)
        return H->fail(GPT2Q_EARG, std::string("tensor ") + t->name + ": expected 1-D of length " + std::to_string(n));
    if (a != ATOM_F16 && a != ATOM_F32)
        return H->fail(GPT2Q_EARG, std::string("tensor ") + t->name + ": 1-D tensors must be core.f16 or core.f32");
    if (t->len != payload_bytes(a, n)) return H->fail(GPT2Q_EARG, std::string("tensor ") + t->name + ": bad length");
    float* d = H->dalloc<float>(cnt * 4);
    if (!d) return H->fail(GPT2Q_EOOM, "cudaMalloc vector");
    if (a == ATOM_F32) {
        CK(cudaMemcpyAsync(d, reinterpret_cast<const float*>(t->data) + off, cnt * 4, cudaMemcpyHostToDevice,
                           H->stream));
        CK(cudaStreamSynchronize(H->stream));
    } else {
        __half* tmp = nullptr;
        CK(cudaMalloc(&tmp, cnt * 2));
        CK(cudaMemcpyAsync(tmp, reinterpret_cast<const uint16_t*>(t->data) + off, cnt * 2, cudaMemcpyHostToDevice,
                           H->stream));
        CK(launch_f16_to_f32(tmp, d, cnt, H->stream));
        CK(cudaStreamSynchronize(H->stream));
        CK(cudaFree(tmp));
    }
    *out = d;
    H->vec_by_name[t->name] = {d, cnt};
    return GPT2Q_OK;
}

// Upload a 2-D weight [rows][cols]; keep the row ranges `rsel` and columns [c0, c1).
int upload_linear(gpt2q_handle* H, const gpt2q_tensor_desc* t, int rows, int cols,
                  const std::vector<std::pair<int, int>>& rsel, int c0, int c1, Linear* L) {
    int a = atom_id(t->atom);
    if (a < 0) return H->fail(GPT2Q_EARG, std::string("tensor ") + t->name + ": unknown atom " + t->atom);
    if (t->ndim != 2 || t->shape[0] != rows || t->shape[1] != cols)
        return H->fail(GPT2Q_EARG, std::string("tensor ") + t->name + ": expected shape [" + std::to_string(rows) +
                                       ", " + std::to_string(cols) + "]");
    if (cols % 32 != 0) return H->fail(GPT2Q_EUNSUP, std::string("tensor ") + t->name + ": cols must be a multiple of 32");
    if (t->len != payload_bytes(a, (size_t)rows * cols))
        return H->fail(GPT2Q_EARG, std::string("tensor ") + t->name + ": payload length does not match shape/atom");
    const size_t row_bytes = payload_bytes(a, (size_t)cols);
    int out_rows = 0;
    for (auto& r : rsel) out_rows += r.second;
    const int out_cols = c1 - c0;
    const size_t out_row_bytes = payload_bytes(a, (size_t)out_cols);
    const size_t col_off = payload_bytes(a, (size_t)c0);
    const bool whole = (rsel.size() == 1 && rsel[0].first == 0 && rsel[0].second == rows && c0 == 0 && c1 == cols);
    std::vector<uint8_t> sliced;
    const uint8_t* src = reinterpret_cast<const uint8_t*>(t->data);
    if (!whole) {
        sliced.resize((size_t)out_rows * out_row_bytes);
        size_t o = 0;
        for (auto& r : rsel)
            for (int i = 0; i < r.second; ++i, ++o)
                std::memcpy(sliced.data() + o * out_row_bytes, src + (size_t)(r.first + i) * row_bytes + col_off,
                            out_row_bytes);
        src = sliced.data();
    }
    const size_t raw_bytes = (size_t)out_rows * out_row_bytes;
    if (a == ATOM_Q8 || a == ATOM_Q4) {
        const size_t blk = (a == ATOM_Q8) ? 34 : 18;
        const float qmax = (a == ATOM_Q8) ? 127.f : 8.f;
        float smax = 0.f;
        for (size_t o = 0; o + blk <= raw_bytes; o += blk) {
            const uint16_t hb = (uint16_t)(src[o] | (src[o + 1] << 8));
            const float sv = std::fabs(half_bits_to_float(hb));
            if (sv > smax && std::isfinite(sv)) smax = sv;
        }
        L->max_abs_w = smax * qmax;
    }
    L->rows = out_rows;
    L->cols = out_cols;
    L->name = t->name;
    QW& w = L->w;
    w.rows = out_rows;
    w.cols = out_cols;
    w.atom = a;
    w.sstride = 0;
    w.s = nullptr;
    if (a == ATOM_F16 || a == ATOM_F32) {
        uint8_t* q = H->dalloc<uint8_t>(raw_bytes);
        if (!q) return H->fail(GPT2Q_EOOM, "cudaMalloc weight");
        CK(cudaMemcpyAsync(q, src, raw_bytes, cudaMemcpyHostToDevice, H->stream));
        CK(cudaStreamSynchronize(H->stream));
        w.q = q;
        w.qstride = (a == ATOM_F16 ? 2 : 4) * (size_t)out_cols;
        L->weight_bytes = raw_bytes;
    } else {
        const int nblk = out_cols / 32;
        w.sstride = (nblk + 7) / 8 * 8;
        w.qstride = (a == ATOM_Q8) ? (size_t)out_cols : (size_t)out_cols / 2;
        uint8_t* q = H->dalloc<uint8_t>(w.qstride * out_rows);
        __half* s = H->dalloc<__half>((size_t)w.sstride * out_rows * 2);
        if (!q || !s) return H->fail(GPT2Q_EOOM, "cudaMalloc weight");
        CK(cudaMemsetAsync(s, 0, (size_t)w.sstride * out_rows * 2, H->stream));
        uint8_t* raw = nullptr;
        CK(cudaMalloc(&raw, raw_bytes));
        CK(cudaMemcpyAsync(raw, src, raw_bytes, cudaMemcpyHostToDevice, H->stream));
        if (a == ATOM_Q8)
            CK(launch_repack_q8(raw, out_rows, out_cols, q, s, w.sstride, H->stream));
        else
            CK(launch_repack_q4(raw, out_rows, out_cols, q, s, w.sstride, H->stream));
        CK(cudaStreamSynchronize(H->stream));
        CK(cudaFree(raw));
        w.q = q;
        w.s = s;
        L->weight_bytes = w.qstride * out_rows + (size_t)nblk * 2 * out_rows;
    }
    H->lin_by_name[t->name] = L;
    return GPT2Q_OK;
}

// ------------------------------------------------------------------ forward pieces
Epi epi_store(float* out, int ldo, const float* bias) {
    Epi e{};
    e.kind = EPI_STORE;
    e.out = out;
    e.ldo = ldo;
    e.bias = bias;
    return e;
}

double linear_bytes(const Linear& L, int M, int extra_out_rw) {
    return (double)L.weight_bytes + (double)M * L.cols * 4 + (double)M * L.rows * 4 * extra_out_rw;
}

// Linear input: fp32 rows for the CUDA-core kernel and their fp16 hi/lo split for the
// tensor-core kernel (both written by the producer).
struct In {
    const float* f;
    const __half* hi;
    const __half* lo;
    int ld;
};

// The linear runs on the warp-level tensor-core kernel (with room for an applied LayerNorm).
bool takes_mma(const gpt2q_handle* H, const Linear& L, const In& X, int M, bool ln) {
    return X.hi && H->mma_on && M >= H->mma_min_m && M <= MMA_MAX_M && X.ld % 8 == 0 && mma_fits(L.w, M, ln);
}

// The linear reads the fp32 copy of its activations only on the CUDA-core path; their producer
// (LayerNorm, attention, the c_fc GELU epilogue) skips that copy otherwise.
bool reads_f32(const gpt2q_handle* H, const Linear& L, const In& X, int M) {
    return !(X.hi && (takes_mma(H, L, X, M, false) || H->gemm.usable(L.w, M)));
}

// With `ln` the warp-level kernel completes the LayerNorm folded into it (the caller checked
// ln_fusable).
int linear(gpt2q_handle* H, const char* name, const Linear& L, const In& X, int M, const Epi& e,
           const LnFold* ln = nullptr) {
    const int extra = (e.kind == EPI_RESID) ? 2 : 1;
    const double bytes = linear_bytes(L, M, extra);
    if (ln) {
        RUN(name, bytes, launch_linear_mma(L.w, X.hi, X.lo, X.ld, M, H->kerr, e, H->stream, ln));
    } else if (takes_mma(H, L, X, M, false)) {
        RUN(name, bytes, launch_linear_mma(L.w, X.hi, X.lo, X.ld, M, H->kerr, e, H->stream));
    } else if (X.hi && H->gemm.usable(L.w, M)) {
        const XSplit xs{X.hi, X.lo, X.ld};
        RUN(name, bytes, launch_linear_tc(H->gemm, L.w, xs, M, e, H->stream));
    } else {
        RUN(name, bytes, launch_linear_simt(L.w, X.f, X.ld, M, e, H->stream));
    }
    return GPT2Q_OK;
}

// Residual update of a row-split projection under tensor parallelism: this rank's partial
// (+bias on rank 0) into its exchange buffer `parity`, then one kernel sums the ranks'
// partials from peer memory into x and applies the LayerNorm (g, b) that follows, when given.
int tp_residual(gpt2q_handle* H, const char* name, const Linear& L, const In& X, int M, int parity, const float* g,
                const float* b) {
    const int d = H->cfg.n_embd;
    Epi e = epi_store(tp_partial(H->tp, parity), d, H->tp_rank == 0 ? L.bias : nullptr);
    int rc = linear(H, name, L, X, M, e);
    if (rc) return rc;
    // timed like every other kernel in profiling mode (the time includes the wait for the peers)
    cudaEvent_t a = nullptr, ev_b = nullptr;
    if (H->prof && !H->capturing) {
        a = pooled_event(H);
        ev_b = pooled_event(H);
        cudaEventRecord(a, H->stream);
    }
    rc = tp_reduce_ln(H->tp, parity, H->x, M, d, g, b, H->cfg.ln_eps, H->h, H->h_hi, H->h_lo, H->stream);
    if (rc) return H->fail(GPT2Q_ENCCL, tp_last_error(H->tp));
    const double bytes = (double)M * d * 4 * (H->tp_size + 3);  // partials of every rank, x in/out, LN out
    return launched(H, "tp_reduce_ln", bytes, cudaSuccess, a, ev_b);
}

Epi epi_qkv(gpt2q_handle* H, int layer, const int* slot, const int* pos, const float* bias) {
    Epi e{};
    e.kind = EPI_QKV;
    e.bias = bias;
    e.out = H->qb;
    e.ldo = H->d_local;
    e.kv = H->kv.base;
    e.slot = slot;
    e.pos = pos;
    e.d_local = H->d_local;
    e.hd = H->hd;
    e.slot_stride = H->kv.slot_stride;
    e.layer_off = (size_t)layer * H->kv.layer_stride;
    e.sel_stride = H->kv.sel_stride;
    e.head_stride = H->kv.head_stride;
    return e;
}

// A LayerNorm between the residual linear `prod` and the linear `cons` that consumes it is
// folded into `cons` when both take the warp-level kernel: prod writes the per-tile statistics
// of its new residual rows and g * x as cons's activations; cons's epilogue completes the
// LayerNorm with its precomputed W g and W b + bias.
bool ln_fusable(const gpt2q_handle* H, const Linear& prod, const In& pin, const Linear& cons, const In& cin, int M) {
    const int d = H->cfg.n_embd;
    return H->ln_fuse && H->tp_size == 1 && cons.ln_c1 && d % 16 == 0 && d / 16 <= 128 &&
           takes_mma(H, prod, pin, M, false) && takes_mma(H, cons, cin, M, true);
}

// One transformer block over M activation rows (gpt2.rs:238-322). attn_fn runs the
// attention of this layer (decode or prefill form).
template <class AttnFn>
int block(gpt2q_handle* H, int layer, int M, const int* slot, const int* pos, AttnFn&& attn_fn) {
    const int d = H->cfg.n_embd;
    const float eps = H->cfg.ln_eps;
    LayerW& Lw = H->layers[layer];
    const In hin{H->h, H->h_hi, H->h_lo, d};
    const In ain{H->att, H->att_hi, H->att_lo, H->d_local};
    const In fin{H->f, H->f_hi, H->f_lo, H->fc_local};
    // LN1 (after the previous layer's mlp c_proj) and LN2 (after attn c_proj) folded into qkv and
    // c_fc where the kernels allow it
    const bool fuse1 = layer > 0 && ln_fusable(H, H->layers[layer - 1].mproj, fin, Lw.attn, hin, M);
    const bool fuse2 = ln_fusable(H, Lw.proj, ain, Lw.fc, hin, M);
    const LayerW* next = layer + 1 < H->cfg.n_layer ? &H->layers[layer + 1] : nullptr;
    const bool fuse1_next = next && ln_fusable(H, Lw.mproj, fin, next->attn, hin, M);
    const LnFold ln1{H->ln_stats, d / 16, d / 16, eps, Lw.attn.ln_c1, Lw.attn.ln_c2b};
    const LnFold ln2{H->ln_stats, d / 16, d / 16, eps, Lw.fc.ln_c1, Lw.fc.ln_c2b};
    // under tensor parallelism every LayerNorm after the first is applied by the residual
    // reduction before it
    const bool tp = H->tp_size > 1;
    if (!(tp && layer > 0) && !fuse1)
        RUN("layernorm", (double)M * d * 8,
            launch_layernorm(H->x, d, nullptr, reads_f32(H, Lw.attn, hin, M) ? H->h : nullptr, d, H->h_hi, H->h_lo,
                             Lw.ln1_g, Lw.ln1_b, d, eps, M, H->stream));
    int rc = linear(H, "linear_qkv", Lw.attn, hin, M, epi_qkv(H, layer, slot, pos, Lw.attn.bias), fuse1 ? &ln1 : nullptr);
    if (rc) return rc;
    rc = attn_fn(layer);
    if (rc) return rc;
    if (tp) {
        rc = tp_residual(H, "linear_attn_proj", Lw.proj, ain, M, 0, Lw.ln2_g, Lw.ln2_b);
    } else {
        Epi e = epi_store(H->x, d, Lw.proj.bias);
        e.kind = EPI_RESID;
        if (fuse2) {
            e.stats = H->ln_stats;
            e.stats_ld = d / 16;
            e.ln_g = Lw.ln2_g;
            e.out_hi = H->h_hi;
            e.out_lo = H->h_lo;
        }
        rc = linear(H, "linear_attn_proj", Lw.proj, ain, M, e);
    }
    if (rc) return rc;
    if (!tp && !fuse2)
        RUN("layernorm", (double)M * d * 8,
            launch_layernorm(H->x, d, nullptr, reads_f32(H, Lw.fc, hin, M) ? H->h : nullptr, d, H->h_hi, H->h_lo,
                             Lw.ln2_g, Lw.ln2_b, d, eps, M, H->stream));
    {
        Epi e = epi_store(reads_f32(H, Lw.mproj, fin, M) ? H->f : nullptr, H->fc_local, Lw.fc.bias);
        e.kind = EPI_GELU;
        e.out_hi = H->f_hi;
        e.out_lo = H->f_lo;
        rc = linear(H, "linear_fc_gelu", Lw.fc, hin, M, e, fuse2 ? &ln2 : nullptr);
        if (rc) return rc;
    }
    if (tp) {
        // the next layer's first LayerNorm; after the last layer the final one runs on its own
        // (prefill normalises only the last row of each sequence)
        const bool last = layer + 1 == H->cfg.n_layer;
        const LayerW* nx = last ? nullptr : &H->layers[layer + 1];
        rc = tp_residual(H, "linear_mlp_proj", Lw.mproj, fin, M, 1, nx ? nx->ln1_g : nullptr, nx ? nx->ln1_b : nullptr);
    } else {
        Epi e = epi_store(H->x, d, Lw.mproj.bias);
        e.kind = EPI_RESID;
        if (fuse1_next) {
            e.stats = H->ln_stats;
            e.stats_ld = d / 16;
            e.ln_g = next->ln1_g;
            e.out_hi = H->h_hi;
            e.out_lo = H->h_lo;
        }
        rc = linear(H, "linear_mlp_proj", Lw.mproj, fin, M, e);
    }
    return rc;
}

// The tied head over rows 0..M-1 of h into out (row stride vocab). Below the tcgen05 head's 16
// rows it runs on the warp-level tensor cores (k_head_mma; 8 rows: 22 us), else on kind::i8 over
// exact int8 pieces of h (int8 head weights), instead of the CUDA-core GEMV: measured at 2 and 8
// rows, 124 and 223 us -> 35 us per head. From 16 rows the f16 hi/lo tile is faster (28.5 us at
// 32 rows against 36 us for either): each of the i8 path's 24 groups per tile needs its own TMEM
// drain and scaling in the epilogue.
int head(gpt2q_handle* H, int M, float* out) {
    const int d = H->cfg.n_embd, V = H->cfg.vocab;
    const bool mma = H->head_mma == 2 || (H->head_mma == 1 && !H->gemm.usable(H->wte.w, M));
    if (mma && H->mma_on && H->head_i8 != 2 && H->h_hi && head_mma_usable(H->wte.w, M, d)) {
        RUN("linear_head", linear_bytes(H->wte, M, 1),
            launch_head_mma(H->wte.w, H->h_hi, H->h_lo, d, M, out, V, H->kerr, H->stream));
        return GPT2Q_OK;
    }
    const bool want = H->head_i8 == 2 || (H->head_i8 == 1 && !H->gemm.usable(H->wte.w, M));
    if (want && H->head_pieces && head_i8_usable(H->gemm, H->wte.w, M)) {
        const int MP = M <= 32 ? 32 : 64;
        RUN("head_pieces", (double)M * d * 4 + (double)MP * d * 3,
            launch_head_pieces(H->h, d, M, d, MP, H->head_pieces, H->head_xscale, H->stream));
        RUN("linear_head", (double)H->wte.weight_bytes + (double)M * V * 4,
            launch_head_i8(H->gemm, H->wte.w, reinterpret_cast<const uint8_t*>(H->head_pieces), H->head_xscale, M,
                           out, V, H->stream));
        return GPT2Q_OK;
    }
    return linear(H, "linear_head", H->wte, In{H->h, H->h_hi, H->h_lo, d}, M, epi_store(out, V, nullptr));
}

// The published adapter, applied to `rows` rows of h after ln_f (gpu.rs:364-367).
int apply_adapter(gpt2q_handle* H, int rows) {
    if (!H->adapter_on) return GPT2Q_OK;
    const int d = H->cfg.n_embd;
    RUN("adapter", (double)rows * d * 8,
        launch_adapter(H->d_adapter, H->h, H->h_hi, H->h_lo, d, d, rows, gpt2q_handle::AD_MAX_R, H->stream));
    return GPT2Q_OK;
}

// Decode step for B sequences reading d_tok/d_pos/d_slot; argmax advances the state.
int enqueue_decode(gpt2q_handle* H, int B) {
    const int d = H->cfg.n_embd;
    const float scale = 1.0f / std::sqrt((float)H->hd);
    RUN("embed", (double)B * d * 6, launch_embed(H->wte.w, H->wpe.w, H->d_tok, H->d_pos, H->x, d, B, H->stream));
    double kv_bytes = 0;
    for (int b = 0; b < B && b < (int)H->hpos.size(); ++b) kv_bytes += 2.0 * (H->hpos[b] + 1) * H->d_local * 4;
    for (int l = 0; l < H->cfg.n_layer; ++l) {
        int rc = block(H, l, B, H->d_slot, H->d_pos, [&](int layer) {
            const In ain{H->att, H->att_hi, H->att_lo, H->d_local};
            float* att32 = reads_f32(H, H->layers[layer].proj, ain, B) ? H->att : nullptr;
            RUN("attn_decode", kv_bytes + (double)B * H->d_local * 8,
                launch_attn_decode(H->qb, H->d_local, H->kv, (size_t)layer * H->kv.layer_stride, H->d_slot,
                                   H->d_pos, att32, H->att_hi, H->att_lo, H->d_local, H->H_local, B, scale,
                                   H->kerr, H->stream));
            return GPT2Q_OK;
        });
        if (rc) return rc;
    }
    RUN("layernorm", (double)B * d * 8,
        launch_layernorm(H->x, d, nullptr, H->h, d, H->h_hi, H->h_lo, H->lnf_g, H->lnf_b, d, H->cfg.ln_eps, B,
                         H->stream));
    int rc = apply_adapter(H, B);
    if (rc) return rc;
    rc = head(H, B, H->logits);
    if (rc) return rc;
    RUN("argmax", (double)B * H->cfg.vocab * 4,
        launch_argmax(H->logits, H->cfg.vocab, H->cfg.vocab, B, H->best, H->d_next, H->d_genlog, H->d_pos,
                      H->cfg.n_ctx, H->d_tok, H->d_pos, H->stream));
    H->launches += H->capturing ? 0 : 1;  // argmax is two kernels
    if (H->capturing) H->capture_kernels++;
    return GPT2Q_OK;
}

int flush_profile(gpt2q_handle* H) {
    if (H->prof_pending.empty()) return GPT2Q_OK;
    CK(cudaStreamSynchronize(H->stream));
    for (auto& r : H->prof_pending) {
        float ms = 0.f;
        cudaEventElapsedTime(&ms, r.a, r.b);
        auto& g = H->prof_agg[r.name];
        g.launches++;
        g.ms += ms;
        g.bytes += r.bytes;
        H->ev_pool.push_back(r.a);
        H->ev_pool.push_back(r.b);
    }
    H->prof_pending.clear();
    return GPT2Q_OK;
}

// `steps` greedy steps of the single current sequence in one persistent launch.
int run_persistent(gpt2q_handle* H, int steps) {
    const gpt2q_config& c = H->cfg;
    MkParams p{};
    p.stream = H->mk.stream;
    p.cta_bytes = H->mk.cta_bytes;
    p.seg_bytes = H->mk.seg_bytes;
    p.d = c.n_embd;
    p.n_layer = c.n_layer;
    p.n_head = c.n_head;
    p.vocab = c.vocab;
    p.n_ctx = c.n_ctx;
    p.head_rows = H->mk.head_rows;
    p.ln_eps = c.ln_eps;
    p.attn_scale = 1.0f / std::sqrt((float)H->hd);
    p.layers = H->mk.layers;
    p.lnf_g = H->lnf_g;
    p.lnf_b = H->lnf_b;
    p.wte = H->wte.w;
    p.wpe = H->wpe.w;
    p.kv = H->kv.base;
    p.kv_slot = H->kv.slot_stride;
    p.kv_layer = H->kv.layer_stride;
    p.kv_sel = H->kv.sel_stride;
    p.kv_head = H->kv.head_stride;
    p.slot = H->d_slot;
    p.pos = H->d_pos;
    p.tok = H->d_tok;
    p.next = H->d_next;
    p.genlog = H->d_genlog;
    p.logits = H->logits;
    p.p1 = H->mk.p1;
    p.p2 = H->mk.p2;
    p.best = H->mk.best;
    p.epoch = H->mk.epoch;
    p.err = H->mk.err;
    p.abort_flag = H->mk.err + 1;
    p.steps = steps;
    p.trace = H->mk.trace;
    p.adapter = H->adapter_on ? H->d_adapter : nullptr;
    int rc = run_kernel(H, "decode_persistent", (double)H->mk.cta_bytes * 8 * H->mk.clusters * steps,
                        [&]() { return launch_decode_persistent(H->mk, p, H->stream); });
    if (rc) return rc;
    H->hpos[0] += steps;
    return GPT2Q_OK;
}

bool use_persistent(const gpt2q_handle* H, int B) {
    // the persistent kernel computes ln_f and the adapter stage itself
    return B == 1 && H->mk.enabled && !H->capturing && H->ktime_reps == 0;
}


// Run one decode step for the current state (graph replay when possible).
int run_decode_step(gpt2q_handle* H, int B) {
    if (use_persistent(H, B)) return run_persistent(H, 1);
    const bool graph_ok = H->use_graphs && !H->prof && H->stream != nullptr;
    if (graph_ok) {
        const int key = 2 * B + (H->adapter_on ? 1 : 0);  // the adapter stage is captured only when on
        auto it = H->dec_graphs.find(key);
        if (it == H->dec_graphs.end()) {
            cudaGraph_t g = nullptr;
            CK(cudaStreamBeginCapture(H->stream, cudaStreamCaptureModeThreadLocal));
            H->capturing = true;
            H->capture_kernels = 0;
            int rc = enqueue_decode(H, B);
            H->capturing = false;
            cudaError_t ce = cudaStreamEndCapture(H->stream, &g);
            if (rc) {
                if (g) cudaGraphDestroy(g);
                return rc;
            }
            if (ce != cudaSuccess) return H->fail(GPT2Q_ECUDA, std::string("graph capture: ") + cudaGetErrorString(ce));
            cudaGraphExec_t ex = nullptr;
            ce = cudaGraphInstantiate(&ex, g, 0);
            cudaGraphDestroy(g);
            if (ce != cudaSuccess) return H->fail(GPT2Q_ECUDA, std::string("graph instantiate: ") + cudaGetErrorString(ce));
            it = H->dec_graphs.emplace(key, std::make_pair(ex, H->capture_kernels)).first;
        }
        CK(cudaGraphLaunch(it->second.first, H->stream));
        H->launches += it->second.second;
    } else {
        if (H->prof) CK(launch_sleep(20000000ull, H->stream));  // host runs ahead of the GPU
        int rc = enqueue_decode(H, B);
        if (rc) return rc;
        if (H->prof) {
            rc = flush_profile(H);
            if (rc) return rc;
        }
    }
    for (int b = 0; b < B; ++b) H->hpos[b] += 1;
    return GPT2Q_OK;
}

int check_tokens(gpt2q_handle* H, const uint32_t* tok, size_t n) {
    for (size_t i = 0; i < n; ++i)
        if (tok[i] >= (uint32_t)H->cfg.vocab)
            return H->fail(GPT2Q_EARG, "token id " + std::to_string(tok[i]) + " >= vocab");
    return GPT2Q_OK;
}

int ensure_stage(gpt2q_handle* H, size_t ints) {
    if (H->h_stage_ints >= ints) return GPT2Q_OK;
    if (H->h_stage) cudaFreeHost(H->h_stage);
    H->h_stage = nullptr;
    H->h_stage_ints = 0;
    CK(cudaMallocHost(&H->h_stage, ints * 4));
    H->h_stage_ints = ints;
    return GPT2Q_OK;
}

// Prefill of one chunk of sequences [s0, s1) whose tokens fit the workspace.
// layers_only: stop after the last transformer block (x holds the residual stream of every
// prompt row), for callers that need more than the last position's logits.
int prefill_chunk(gpt2q_handle* H, const uint32_t* tokens, const int32_t* offs, const int32_t* slots, int s0,
                  int s1, bool layers_only = false) {
    const int d = H->cfg.n_embd;
    const int base = offs[s0];
    const int M = offs[s1] - base;
    const int ns = s1 - s0;
    // host staging: tok[M] pos[M] slot[M] lastrow[ns] lastpos[ns] tiles[4*nt]
    // attention tiles: 128 queries on the tensor cores, 64 on the CUDA cores
    const bool attn_tc = H->gemm.enabled && H->hd == 64 && !std::getenv("GPT2Q_ATTN_CORES");
    const int qt = attn_tc ? 128 : 64;
    int nt = 0;
    for (int s = s0; s < s1; ++s) nt += (offs[s + 1] - offs[s] + qt - 1) / qt;
    if (nt > H->max_tiles) return H->fail(GPT2Q_EARG, "too many attention tiles in one prefill chunk");
    int rc = ensure_stage(H, (size_t)3 * M + 2 * ns + 4 * (size_t)nt);
    if (rc) return rc;
    int* st_tok = H->h_stage;
    int* st_pos = st_tok + M;
    int* st_slot = st_pos + M;
    int* st_lrow = st_slot + M;
    int* st_lpos = st_lrow + ns;
    AttnTile* st_tiles = reinterpret_cast<AttnTile*>(st_lpos + ns);
    int ti = 0;
    for (int s = s0; s < s1; ++s) {
        const int T = offs[s + 1] - offs[s];
        const int r0 = offs[s] - base;
        const int slot = slots ? slots[s] : s;
        for (int t = 0; t < T; ++t) {
            st_tok[r0 + t] = (int)tokens[offs[s] + t];
            st_pos[r0 + t] = t;
            st_slot[r0 + t] = slot;
        }
        st_lrow[s - s0] = r0 + T - 1;
        st_lpos[s - s0] = T - 1;
        for (int q0 = 0; q0 < T; q0 += qt) st_tiles[ti++] = AttnTile{r0, q0, T, slot};
    }
    CK(cudaMemcpyAsync(H->p_tok, st_tok, (size_t)M * 4, cudaMemcpyHostToDevice, H->stream));
    CK(cudaMemcpyAsync(H->p_pos, st_pos, (size_t)M * 4, cudaMemcpyHostToDevice, H->stream));
    CK(cudaMemcpyAsync(H->p_slot, st_slot, (size_t)M * 4, cudaMemcpyHostToDevice, H->stream));
    CK(cudaMemcpyAsync(H->p_lastrow, st_lrow, (size_t)ns * 4, cudaMemcpyHostToDevice, H->stream));
    CK(cudaMemcpyAsync(H->p_lastpos, st_lpos, (size_t)ns * 4, cudaMemcpyHostToDevice, H->stream));
    CK(cudaMemcpyAsync(H->p_tiles, st_tiles, (size_t)nt * sizeof(AttnTile), cudaMemcpyHostToDevice, H->stream));

    const float scale = 1.0f / std::sqrt((float)H->hd);
    if (H->prof) CK(launch_sleep(20000000ull, H->stream));
    double kv_bytes = 0;
    for (int s = s0; s < s1; ++s) {
        const double T = offs[s + 1] - offs[s];
        kv_bytes += 2.0 * T * H->d_local * 4;
    }
    RUN("embed", (double)M * d * 6, launch_embed(H->wte.w, H->wpe.w, H->p_tok, H->p_pos, H->x, d, M, H->stream));
    for (int l = 0; l < H->cfg.n_layer; ++l) {
        rc = block(H, l, M, H->p_slot, H->p_pos, [&](int layer) {
            const In ain{H->att, H->att_hi, H->att_lo, H->d_local};
            float* att32 = reads_f32(H, H->layers[layer].proj, ain, M) ? H->att : nullptr;
            if (attn_tc)
                RUN("attn_prefill_tc", kv_bytes + (double)M * H->d_local * 8,
                    launch_attn_prefill_tc(H->qb, H->d_local, H->kv, (size_t)layer * H->kv.layer_stride, H->p_tiles,
                                           nt, att32, H->att_hi, H->att_lo, H->d_local, H->H_local, H->gemm.err,
                                           H->stream));
            else
                RUN("attn_prefill", kv_bytes + (double)M * H->d_local * 8,
                    launch_attn_prefill(H->qb, H->d_local, H->kv, (size_t)layer * H->kv.layer_stride, H->p_tiles, nt,
                                        att32, H->att_hi, H->att_lo, H->d_local, H->H_local, scale, H->stream));
            return GPT2Q_OK;
        });
        if (rc) return rc;
    }
    if (layers_only) return GPT2Q_OK;
    // ln_f + tied head for the last position of each sequence only.
    RUN("layernorm", (double)ns * d * 8,
        launch_layernorm(H->x, d, H->p_lastrow, H->h, d, H->h_hi, H->h_lo, H->lnf_g, H->lnf_b, d, H->cfg.ln_eps, ns,
                         H->stream));
    rc = apply_adapter(H, ns);
    if (rc) return rc;
    float* lg = H->logits + (size_t)s0 * H->cfg.vocab;
    rc = head(H, ns, lg);
    if (rc) return rc;
    RUN("argmax", (double)ns * H->cfg.vocab * 4,
        launch_argmax(lg, H->cfg.vocab, H->cfg.vocab, ns, H->best + s0, H->d_next + s0,
                      H->d_genlog + (size_t)s0 * H->cfg.n_ctx, H->p_lastpos, H->cfg.n_ctx, H->d_tok + s0, nullptr,
                      H->stream));
    H->launches += 1;  // argmax is two kernels
    // the staging buffer is reused by the next chunk
    CK(cudaStreamSynchronize(H->stream));
    if (H->prof) return flush_profile(H);
    return GPT2Q_OK;
}

int do_prefill(gpt2q_handle* H, const uint32_t* tokens, const int32_t* offs, const int32_t* slots, int n_seq) {
    if (n_seq <= 0 || n_seq > H->cfg.max_seqs) return H->fail(GPT2Q_EARG, "n_seq out of range [1, max_seqs]");
    if (!tokens || !offs) return H->fail(GPT2Q_EARG, "null tokens/seq_offsets");
    if (offs[0] != 0) return H->fail(GPT2Q_EARG, "seq_offsets[0] must be 0");
    std::vector<char> used(H->cfg.max_seqs, 0);
    for (int s = 0; s < n_seq; ++s) {
        const int T = offs[s + 1] - offs[s];
        if (T <= 0 || T > H->cfg.n_ctx) return H->fail(GPT2Q_EARG, "prompt length out of range [1, n_ctx]");
        const int slot = slots ? slots[s] : s;
        if (slot < 0 || slot >= H->cfg.max_seqs || used[slot]) return H->fail(GPT2Q_EARG, "bad or repeated slot");
        used[slot] = 1;
    }
    int rc = check_tokens(H, tokens, (size_t)offs[n_seq]);
    if (rc) return rc;
    int s0 = 0;
    while (s0 < n_seq) {
        int s1 = s0;
        while (s1 < n_seq && offs[s1 + 1] - offs[s0] <= H->Mmax) s1++;
        if (s1 == s0) return H->fail(GPT2Q_EARG, "prompt longer than max_tokens");
        rc = prefill_chunk(H, tokens, offs, slots, s0, s1);
        if (rc) return rc;
        s0 = s1;
    }
    // decode state: next token at position T for every sequence
    H->cur_n = n_seq;
    H->hpos.assign(n_seq, 0);
    H->hslot.assign(n_seq, 0);
    const int M = H->cfg.max_seqs;
    rc = ensure_stage(H, (size_t)2 * M);
    if (rc) return rc;
    for (int s = 0; s < n_seq; ++s) {
        H->hpos[s] = offs[s + 1] - offs[s];
        H->hslot[s] = slots ? slots[s] : s;
        H->h_stage[s] = H->hpos[s];
        H->h_stage[M + s] = H->hslot[s];
    }
    // pos | slot are adjacent on the device: one copy
    CK(cudaMemcpyAsync(H->d_pos, H->h_stage, (size_t)2 * M * 4, cudaMemcpyHostToDevice, H->stream));
    CK(cudaStreamSynchronize(H->stream));
    return GPT2Q_OK;
}

int do_decode(gpt2q_handle* H, const uint32_t* tok, const int32_t* pos, const int32_t* slots, int n_seq) {
    if (n_seq <= 0 || n_seq > H->cfg.max_seqs) return H->fail(GPT2Q_EARG, "n_seq out of range [1, max_seqs]");
    if (!tok || !pos) return H->fail(GPT2Q_EARG, "null tok/pos");
    int rc = check_tokens(H, tok, (size_t)n_seq);
    if (rc) return rc;
    const int M = H->cfg.max_seqs;
    rc = ensure_stage(H, (size_t)3 * M);
    if (rc) return rc;
    std::vector<char> used(H->cfg.max_seqs, 0);
    H->hpos.assign(n_seq, 0);
    H->hslot.assign(n_seq, 0);
    for (int i = 0; i < n_seq; ++i) {
        const int slot = slots ? slots[i] : i;
        if (pos[i] < 0 || pos[i] >= H->cfg.n_ctx) return H->fail(GPT2Q_EARG, "pos out of range [0, n_ctx)");
        if (slot < 0 || slot >= H->cfg.max_seqs || used[slot]) return H->fail(GPT2Q_EARG, "bad or repeated slot");
        used[slot] = 1;
        H->h_stage[i] = (int)tok[i];
        H->h_stage[M + i] = pos[i];
        H->h_stage[2 * M + i] = slot;
        H->hpos[i] = pos[i];
        H->hslot[i] = slot;
    }
    // one copy of the tok | pos | slot block (entries past n_seq are not read by this step)
    CK(cudaMemcpyAsync(H->d_tok, H->h_stage, (size_t)3 * M * 4, cudaMemcpyHostToDevice, H->stream));
    H->cur_n = n_seq;
    return run_decode_step(H, n_seq);
}

int check_device_error(gpt2q_handle* H) {
    int e = gemm_take_error(H->gemm, H->stream);
    if (e == 0) e = mk_take_error(H->mk, H->stream);
    if (e == 0 && H->tp) e = tp_take_error(H->tp, H->stream);
    if (e == 0 && H->kerr) {
        int h = 0;
        if (cudaMemcpyAsync(&h, H->kerr, 4, cudaMemcpyDeviceToHost, H->stream) != cudaSuccess ||
            cudaStreamSynchronize(H->stream) != cudaSuccess)
            e = -1;
        else if (h != 0) {
            cudaMemsetAsync(H->kerr, 0, 4, H->stream);
            e = h;
        }
    }
    if (e > 0) return H->fail(GPT2Q_ETIMEOUT, "a bounded device-side wait timed out (error word " + std::to_string(e) + ")");
    if (e < 0) return H->fail(GPT2Q_ECUDA, "reading the device error word failed");
    return GPT2Q_OK;
}

// The outputs and every device error word in one round trip: the words are copied to pinned
// memory behind the outputs and inspected after a single synchronisation; only a non-zero word
// takes the slow path that clears it and reports the error.
int read_outputs(gpt2q_handle* H, int n, const float* dlogits, float* logits, uint32_t* next) {
    if (logits)
        CK(cudaMemcpyAsync(logits, dlogits, (size_t)n * H->cfg.vocab * 4, cudaMemcpyDeviceToHost, H->stream));
    if (!H->h_err) {
        if (next) CK(cudaMemcpyAsync(next, H->d_next, (size_t)n * 4, cudaMemcpyDeviceToHost, H->stream));
        CK(cudaStreamSynchronize(H->stream));
        return check_device_error(H);
    }
    // the next tokens land in pinned memory (a direct copy to pageable memory is staged by the
    // driver) and are copied out after the synchronisation
    int* h_next = H->h_err + 16;
    if (next) CK(cudaMemcpyAsync(h_next, H->d_next, (size_t)n * 4, cudaMemcpyDeviceToHost, H->stream));
    int nw = 0;
    auto word = [&](const int* d, int count) -> cudaError_t {
        if (!d) return cudaSuccess;
        const cudaError_t e = cudaMemcpyAsync(H->h_err + nw, d, (size_t)count * 4, cudaMemcpyDeviceToHost, H->stream);
        nw += count;
        return e;
    };
    CK(word(H->gemm.enabled ? H->gemm.err : nullptr, 1));
    CK(word(H->mk.err, 2));
    CK(word(tp_err_word(H->tp), 1));
    CK(word(H->kerr, 1));
    CK(cudaStreamSynchronize(H->stream));
    if (next) std::memcpy(next, h_next, (size_t)n * 4);
    for (int i = 0; i < nw; ++i)
        if (H->h_err[i] != 0) return check_device_error(H);
    return GPT2Q_OK;
}

const gpt2q_tensor_desc* find(const std::map<std::string, const gpt2q_tensor_desc*>& m, const std::string& n) {
    auto it = m.find(n);
    return it == m.end() ? nullptr : it->second;
}

// Column range [c0,c1) of a row-split projection for rank r (multiples of 32 along K).
std::pair<int, int> k_split(int K, int parts_total, int r0, int r1, int unit) {
    (void)parts_total;
    return {r0 * unit, std::min(K, r1 * unit)};
}

int create_common(const gpt2q_config* cfg, const gpt2q_tensor_desc* tensors, int n_tensors, int device,
                  int tp_size, int tp_rank, const void* nccl_id, gpt2q_handle** out) {
    if (!cfg || !tensors || !out) {
        g_create_error = "null argument";
        return GPT2Q_EARG;
    }
    *out = nullptr;
    std::unique_ptr<gpt2q_handle> H(new gpt2q_handle());
    H->cfg = *cfg;
    H->device = device;
    H->tp_size = tp_size;
    H->tp_rank = tp_rank;
    auto bail = [&](int code) {
        g_create_error = H->err;
        gpt2q_destroy(H.release());
        return code;
    };
    const gpt2q_config& c = H->cfg;
    if (c.n_embd <= 0 || c.n_layer <= 0 || c.n_head <= 0 || c.n_ctx <= 0 || c.vocab <= 0 || c.max_seqs <= 0 ||
        c.n_embd % c.n_head != 0) {
        H->err = "invalid config";
        return bail(GPT2Q_EARG);
    }
    H->hd = c.n_embd / c.n_head;
    if (H->hd != 64) {
        H->err = "head dim must be 64 (all GPT-2 sizes)";
        return bail(GPT2Q_EUNSUP);
    }
    if (tp_size < 1 || tp_rank < 0 || tp_rank >= tp_size || tp_size > c.n_head) {
        H->err = "invalid tensor-parallel rank/size";
        return bail(GPT2Q_EARG);
    }
    if (cudaSetDevice(device) != cudaSuccess) {
        H->err = "cudaSetDevice failed";
        return bail(GPT2Q_ECUDA);
    }
    if (cudaStreamCreateWithFlags(&H->own_stream, cudaStreamNonBlocking) != cudaSuccess) {
        H->err = "cudaStreamCreate failed";
        return bail(GPT2Q_ECUDA);
    }
    H->stream = H->own_stream;
    if (const char* e = std::getenv("GPT2Q_NO_GRAPH")) H->use_graphs = (e[0] == '0');

    std::map<std::string, const gpt2q_tensor_desc*> by;
    for (int i = 0; i < n_tensors; ++i) {
        if (!tensors[i].name || !tensors[i].atom || !tensors[i].data) {
            H->err = "tensor descriptor with null field";
            return bail(GPT2Q_EARG);
        }
        by[tensors[i].name] = &tensors[i];
    }
    auto need = [&](const std::string& n) -> const gpt2q_tensor_desc* {
        const gpt2q_tensor_desc* t = find(by, n);
        if (!t) H->err = "missing tensor '" + n + "'";
        return t;
    };
    const int d = c.n_embd, hd = H->hd;
    // heads of this rank: contiguous, first (n_head % tp) ranks get one extra
    const int hbase = c.n_head / tp_size, hrem = c.n_head % tp_size;
    const int h0 = tp_rank * hbase + std::min(tp_rank, hrem);
    const int hn = hbase + (tp_rank < hrem ? 1 : 0);
    H->H_local = hn;
    H->d_local = hn * hd;

    const gpt2q_tensor_desc* t;
    int rc;
    if (!(t = need("wte.weight"))) return bail(GPT2Q_EARG);
    if ((rc = upload_linear(H.get(), t, c.vocab, d, {{0, c.vocab}}, 0, d, &H->wte))) return bail(rc);
    if (!(t = need("wpe.weight"))) return bail(GPT2Q_EARG);
    if ((rc = upload_linear(H.get(), t, c.n_ctx, d, {{0, c.n_ctx}}, 0, d, &H->wpe))) return bail(rc);
    if (!(t = need("ln_f.weight")) || (rc = upload_vec(H.get(), t, d, 0, d, &H->lnf_g))) return bail(t ? rc : GPT2Q_EARG);
    if (!(t = need("ln_f.bias")) || (rc = upload_vec(H.get(), t, d, 0, d, &H->lnf_b))) return bail(t ? rc : GPT2Q_EARG);
    H->layers.resize(c.n_layer);
    int fc_rows = -1;
    for (int l = 0; l < c.n_layer; ++l) {
        LayerW& L = H->layers[l];
        const std::string p = "h." + std::to_string(l) + ".";
        auto vec = [&](const std::string& n, size_t len, size_t off, size_t cnt, float** dst) -> int {
            const gpt2q_tensor_desc* tt = need(p + n);
            if (!tt) return GPT2Q_EARG;
            return upload_vec(H.get(), tt, len, off, cnt, dst);
        };
        if ((rc = vec("ln_1.weight", d, 0, d, &L.ln1_g)) || (rc = vec("ln_1.bias", d, 0, d, &L.ln1_b)) ||
            (rc = vec("ln_2.weight", d, 0, d, &L.ln2_g)) || (rc = vec("ln_2.bias", d, 0, d, &L.ln2_b)))
            return bail(rc);
        // c_attn: rows [q | k | v], each d wide; keep this rank's heads of each block.
        if (!(t = need(p + "attn.c_attn.weight"))) return bail(GPT2Q_EARG);
        std::vector<std::pair<int, int>> qkv_rows = {{h0 * hd, hn * hd}, {d + h0 * hd, hn * hd}, {2 * d + h0 * hd, hn * hd}};
        if ((rc = upload_linear(H.get(), t, 3 * d, d, qkv_rows, 0, d, &L.attn))) return bail(rc);
        {
            const gpt2q_tensor_desc* tb = need(p + "attn.c_attn.bias");
            if (!tb) return bail(GPT2Q_EARG);
            // three slices of the bias, concatenated
            float* dst = H->dalloc<float>((size_t)3 * hn * hd * 4);
            if (!dst) return bail(GPT2Q_EOOM);
            for (int k = 0; k < 3; ++k) {
                float* part = nullptr;
                if ((rc = upload_vec(H.get(), tb, 3 * d, (size_t)k * d + h0 * hd, (size_t)hn * hd, &part))) return bail(rc);
                if (cudaMemcpyAsync(dst + (size_t)k * hn * hd, part, (size_t)hn * hd * 4, cudaMemcpyDeviceToDevice,
                                    H->stream) != cudaSuccess)
                    return bail(GPT2Q_ECUDA);
            }
            L.attn.bias = dst;
            H->vec_by_name[p + "attn.c_attn.bias"] = {dst, (size_t)3 * hn * hd};
        }
        // attn c_proj: [d, d], keep this rank's K columns (its heads' outputs).
        if (!(t = need(p + "attn.c_proj.weight"))) return bail(GPT2Q_EARG);
        if ((rc = upload_linear(H.get(), t, d, d, {{0, d}}, h0 * hd, (h0 + hn) * hd, &L.proj))) return bail(rc);
        if ((rc = vec("attn.c_proj.bias", d, 0, d, &L.proj.bias))) return bail(rc);
        // mlp c_fc [inter, d]: row split in multiples of 32.
        if (!(t = need(p + "mlp.c_fc.weight"))) return bail(GPT2Q_EARG);
        if (t->ndim != 2) {
            H->err = "mlp.c_fc.weight must be 2-D";
            return bail(GPT2Q_EARG);
        }
        const int inter = (int)t->shape[0];
        if (fc_rows >= 0 && inter != fc_rows) {
            H->err = "c_fc rows differ between layers";
            return bail(GPT2Q_EARG);
        }
        fc_rows = inter;
        if (inter % (32 * tp_size) != 0 && tp_size > 1) {
            H->err = "c_fc rows must split into multiples of 32";
            return bail(GPT2Q_EUNSUP);
        }
        const int fper = inter / tp_size;
        const int f0 = tp_rank * fper;
        if ((rc = upload_linear(H.get(), t, inter, d, {{f0, fper}}, 0, d, &L.fc))) return bail(rc);
        if ((rc = vec("mlp.c_fc.bias", inter, f0, fper, &L.fc.bias))) return bail(rc);
        if (!(t = need(p + "mlp.c_proj.weight"))) return bail(GPT2Q_EARG);
        if ((rc = upload_linear(H.get(), t, d, inter, {{0, d}}, f0, f0 + fper, &L.mproj))) return bail(rc);
        if ((rc = vec("mlp.c_proj.bias", d, 0, d, &L.mproj.bias))) return bail(rc);
        H->fc_local = fper;
    }
    (void)k_split;

    // KV arena [slot][layer][K|V][head][n_ctx][hd]
    H->kv.hd = hd;
    H->kv.n_slots = c.max_seqs;
    H->kv.head_stride = (size_t)c.n_ctx * hd;
    H->kv.sel_stride = (size_t)hn * H->kv.head_stride;
    H->kv.layer_stride = 2 * H->kv.sel_stride;
    H->kv.slot_stride = (size_t)c.n_layer * H->kv.layer_stride;
    H->kv.base = H->dalloc<float>(H->kv.slot_stride * c.max_seqs * 4);
    if (!H->kv.base) {
        H->err = "cudaMalloc KV arena (" + std::to_string(H->kv.slot_stride * c.max_seqs * 4) + " bytes)";
        return bail(GPT2Q_EOOM);
    }
    if (cudaMemsetAsync(H->kv.base, 0, H->kv.slot_stride * c.max_seqs * 4, H->stream) != cudaSuccess)
        return bail(GPT2Q_ECUDA);

    const int max_tokens = c.max_tokens > 0 ? c.max_tokens : 8192;
    H->Mmax = std::max(c.max_seqs, max_tokens);
    const size_t M = (size_t)H->Mmax;
    H->max_tiles = (int)(M / 64 + c.max_seqs + 1);
    H->x = H->dalloc<float>(M * d * 4);
    H->h = H->dalloc<float>(M * d * 4);
    H->qb = H->dalloc<float>(M * H->d_local * 4);
    H->att = H->dalloc<float>(M * H->d_local * 4);
    H->f = H->dalloc<float>(M * H->fc_local * 4);
    H->logits = H->dalloc<float>((size_t)c.max_seqs * c.vocab * 4);
    H->h_hi = H->dalloc<__half>(M * d * 2);
    H->h_lo = H->dalloc<__half>(M * d * 2);
    H->att_hi = H->dalloc<__half>(M * H->d_local * 2);
    H->att_lo = H->dalloc<__half>(M * H->d_local * 2);
    H->f_hi = H->dalloc<__half>(M * H->fc_local * 2);
    H->f_lo = H->dalloc<__half>(M * H->fc_local * 2);
    H->best = H->dalloc<unsigned long long>((size_t)c.max_seqs * 8);
    H->kerr = H->dalloc<int>(4);
    if (const char* e = std::getenv("GPT2Q_MMA_DISABLE")) H->mma_on = e[0] != '1';
    if (const char* e = std::getenv("GPT2Q_MMA_MIN_M")) H->mma_min_m = std::max(1, std::atoi(e));
    if (H->mma_on) mma_init();
    if (const char* e = std::getenv("GPT2Q_LN_FUSE")) H->ln_fuse = e[0] != '0';
    if (const char* e = std::getenv("GPT2Q_HEAD_I8")) H->head_i8 = std::atoi(e);
    if (const char* e = std::getenv("GPT2Q_HEAD_MMA")) H->head_mma = std::max(0, std::min(2, std::atoi(e)));
    if (d % 32 == 0) {
        const size_t pb = (size_t)(d / 32) * 3 * 64 * 32, sb = (size_t)64 * (d / 32) * 4;
        H->head_pieces = H->dalloc<int8_t>(pb);
        H->head_xscale = H->dalloc<float>(sb);
        if (!H->head_pieces || !H->head_xscale || cudaMemset(H->head_pieces, 0, pb) != cudaSuccess ||
            cudaMemset(H->head_xscale, 0, sb) != cudaSuccess)
            return bail(GPT2Q_EOOM);
    }
    H->ln_stats = H->dalloc<float2>((size_t)((d + 15) / 16) * MMA_MAX_M * 8);

    H->p_tok = H->dalloc<uint32_t>(M * 4);
    H->p_pos = H->dalloc<int>(M * 4);
    H->p_slot = H->dalloc<int>(M * 4);
    H->p_lastrow = H->dalloc<int>((size_t)c.max_seqs * 4);
    H->p_lastpos = H->dalloc<int>((size_t)c.max_seqs * 4);
    H->p_tiles = H->dalloc<AttnTile>((size_t)H->max_tiles * sizeof(AttnTile));
    // tok | pos | slot in one block (max_seqs each), so a step's inputs are one host copy
    int* dstate = H->dalloc<int>((size_t)3 * c.max_seqs * 4);
    H->d_tok = reinterpret_cast<uint32_t*>(dstate);
    H->d_pos = dstate ? dstate + c.max_seqs : nullptr;
    H->d_slot = dstate ? dstate + 2 * c.max_seqs : nullptr;
    H->d_next = H->dalloc<uint32_t>((size_t)c.max_seqs * 4);
    // pinned: 16 error-word slots, then the next tokens of up to max_seqs sequences
    if (cudaMallocHost(&H->h_err, (16 + (size_t)c.max_seqs) * sizeof(int)) != cudaSuccess) H->h_err = nullptr;
    H->d_genlog = H->dalloc<uint32_t>((size_t)c.max_seqs * c.n_ctx * 4);
    if (!H->x || !H->h || !H->qb || !H->att || !H->f || !H->logits || !H->p_tok || !H->p_pos || !H->p_slot ||
        !H->p_lastrow || !H->p_lastpos || !H->p_tiles || !H->d_tok || !H->d_next || !H->d_pos || !H->d_slot ||
        !H->d_genlog || !H->h_hi || !H->h_lo || !H->att_hi || !H->att_lo ||
        !H->f_hi || !H->f_lo || !H->best || !H->kerr) {
        H->err = "cudaMalloc workspace";
        return bail(GPT2Q_EOOM);
    }
    if (cudaMemsetAsync(H->d_genlog, 0xff, (size_t)c.max_seqs * c.n_ctx * 4, H->stream) != cudaSuccess ||
        cudaMemsetAsync(H->best, 0, (size_t)c.max_seqs * 8, H->stream) != cudaSuccess ||
        cudaMemsetAsync(H->kerr, 0, 4, H->stream) != cudaSuccess)
        return bail(GPT2Q_ECUDA);
    {
        const int Kmax = std::max(std::max(d, H->fc_local), H->d_local);
        if (gemm_init(H->gemm, device, H->Mmax, Kmax) != 0) {
            H->err = "tensor-core linear init failed";
            return bail(GPT2Q_ECUDA);
        }
        for (auto& kv : H->lin_by_name) {
            const Linear* L = kv.second;
            // layer weights also get the fp16 hi/lo copy for compute-bound prefill; the tied
            // head only ever multiplies the last position of each prompt
            const bool presplit = kv.first.rfind("h.", 0) == 0;
            if (gemm_register_weight(H->gemm, L->w, L->max_abs_w, presplit, H->stream) != 0) {
                H->err = "tensor map for " + kv.first + " failed";
                return bail(GPT2Q_ECUDA);
            }
        }
    }
    if (tp_size == 1 && H->mma_on && H->ln_fuse) {
        // the constants of LN1 / LN2 folded into qkv / c_fc on the warp-level decode path
        for (auto& L : H->layers) {
            const std::pair<Linear*, std::pair<const float*, const float*>> pairs[2] = {
                {&L.attn, {L.ln1_g, L.ln1_b}}, {&L.fc, {L.ln2_g, L.ln2_b}}};
            for (const auto& pr : pairs) {
                Linear* lin = pr.first;
                const float* g = pr.second.first;
                const float* b = pr.second.second;
                if ((lin->w.atom != ATOM_Q8 && lin->w.atom != ATOM_Q4) || !g || !b) continue;
                lin->ln_c1 = H->dalloc<float>((size_t)lin->rows * 4);
                lin->ln_c2b = H->dalloc<float>((size_t)lin->rows * 4);
                if (!lin->ln_c1 || !lin->ln_c2b) return bail(GPT2Q_EOOM);
                if (launch_ln_fold(lin->w, g, b, lin->bias, lin->ln_c1, lin->ln_c2b, H->stream) != cudaSuccess)
                    return bail(GPT2Q_ECUDA);
            }
        }
    }
    if (tp_size == 1) {
        MkWeights mw;
        mw.wte = H->wte.w;
        mw.wpe = H->wpe.w;
        bool have_all = H->lnf_g && H->lnf_b;
        for (auto& L : H->layers) {
            mw.attn.push_back(L.attn.w);
            mw.proj.push_back(L.proj.w);
            mw.fc.push_back(L.fc.w);
            mw.mproj.push_back(L.mproj.w);
            mw.layers.push_back(MkLayer{L.ln1_g, L.ln1_b, L.ln2_g, L.ln2_b, L.attn.bias, L.proj.bias, L.fc.bias,
                                        L.mproj.bias});
            have_all = have_all && L.ln1_g && L.ln1_b && L.ln2_g && L.ln2_b && L.attn.bias && L.proj.bias &&
                       L.fc.bias && L.mproj.bias;
        }
        if (have_all) {
            const cudaError_t me = mk_setup(H->mk, mw, d, c.n_layer, c.n_head, c.vocab, c.n_ctx, device, H->stream);
            if (me != cudaSuccess) {
                H->err = std::string("persistent decode setup: ") + cudaGetErrorString(me);
                return bail(GPT2Q_ECUDA);
            }
        } else {
            H->mk.why = "a LayerNorm or bias vector is missing";
        }
    }
    if (tp_size > 1) {
        H->tp = tp_create(tp_size, tp_rank, nccl_id, device, M * d);
        if (!H->tp || tp_last_error(H->tp)[0]) {
            H->err = std::string("NCCL init: ") + (H->tp ? tp_last_error(H->tp) : "failed");
            return bail(GPT2Q_ENCCL);
        }
    }
    if (cudaStreamSynchronize(H->stream) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        H->err = "device sync after upload failed";
        return bail(GPT2Q_ECUDA);
    }
    *out = H.release();
    return GPT2Q_OK;
}


// ------------------------------------------------------------------ trunk input gradient
// Forward over one sequence with the activations the backward needs (the stash of the
// reference's bwparity.rs forward_stash:448-580: per layer the residual entering the layer,
// the residual after the attention branch, q|k|v with bias and the pre-GELU c_fc output; the
// input of ln_f and its output), then trunk_input_grad (gpu_backward.rs:651-790) with every op
// batched over the T positions. Weights are read in their uploaded atoms; the dequantised
// values are exactly Engine::vec_f32's, the f32 weights the reference's backward uses.
int trunk_grad(gpt2q_handle* H, const uint32_t* ids, int T, const float* dlogits, float* dx_out, float* lnf_out) {
    // The stash feeds a backward that amplifies activation rounding (fp16 activations in the
    // forward gave 6 % relative error in dx at 128 positions): the wide tiles compute all
    // three products here, whatever GPT2Q_TC_PRODUCTS selected for inference.
    struct Products {
        GemmPlan& g;
        int saved;
        ~Products() { g.products = saved; }
    } keep{H->gemm, H->gemm.products};
    H->gemm.products = 3;
    const int d = H->cfg.n_embd, L = H->cfg.n_layer, V = H->cfg.vocab, NH = H->cfg.n_head, hd = H->hd;
    const int F = H->fc_local, d3 = 3 * d;
    const float eps = H->cfg.ln_eps;
    auto up64 = [](size_t n) { return (n + 63) / 64 * 64; };
    size_t part_n = bwd_linear_part_floats(T, V, d);
    for (const LayerW& lw : H->layers) {
        part_n = std::max(part_n, bwd_linear_part_floats(T, lw.attn.rows, lw.attn.cols));
        part_n = std::max(part_n, bwd_linear_part_floats(T, lw.proj.rows, lw.proj.cols));
        part_n = std::max(part_n, bwd_linear_part_floats(T, lw.fc.rows, lw.fc.cols));
        part_n = std::max(part_n, bwd_linear_part_floats(T, lw.mproj.rows, lw.mproj.cols));
    }
    const size_t Td = up64((size_t)T * d), TF = up64((size_t)T * F), T3 = up64((size_t)T * d3);
    const size_t n_ctr = up64(bwd_linear_counters(T, std::max(F, d3)));
    const size_t need = (size_t)(L + 1) * Td + (size_t)L * (Td + T3 + TF)  // stash
                        + Td                                               // ln_f output
                        + 2 * Td + TF                                      // h, att, gelu(fc)
                        + 2 * Td + TF                                      // their fp16 hi/lo splits
                        + up64((size_t)T * V)                              // dlogits
                        + 3 * Td + TF + T3                                 // G, DH, DATT, DFC, DQKV
                        + up64(part_n) + up64((size_t)3 * NH * T) + up64((size_t)2 * T) + n_ctr;
    if (H->bwd_ws_floats < need) {
        if (H->bwd_ws) {
            CK(cudaStreamSynchronize(H->stream));
            cudaFree(H->bwd_ws);
            H->bwd_ws = nullptr;
            H->bwd_ws_floats = 0;
        }
        if (cudaMalloc(&H->bwd_ws, need * 4) != cudaSuccess) {
            H->bwd_ws = nullptr;
            return H->fail(GPT2Q_EOOM, "trunk backward workspace (" + std::to_string(need * 4) + " bytes)");
        }
        H->bwd_ws_floats = need;
        // the split-reduction tickets sit at the end; every launch leaves them at zero
        CK(cudaMemsetAsync(H->bwd_ws + need - n_ctr, 0, n_ctr * 4, H->stream));
    }
    float* w = H->bwd_ws;
    auto take = [&](size_t n) {
        float* p = w;
        w += n;
        return p;
    };
    float* xs = take((size_t)(L + 1) * Td);  // x_in of layer l at l*Td; x_L is ln_f's input
    float* xmid = take((size_t)L * Td);
    float* qkv = take((size_t)L * T3);
    float* fcpre = take((size_t)L * TF);
    float* lnf = take(Td);
    float* hb = take(Td);
    float* att = take(Td);
    float* fb = take(TF);
    __half* hb_hi = reinterpret_cast<__half*>(take(Td / 2));
    __half* hb_lo = reinterpret_cast<__half*>(take(Td / 2));
    __half* att_hi = reinterpret_cast<__half*>(take(Td / 2));
    __half* att_lo = reinterpret_cast<__half*>(take(Td / 2));
    __half* fb_hi = reinterpret_cast<__half*>(take(TF / 2));
    __half* fb_lo = reinterpret_cast<__half*>(take(TF / 2));
    float* DL = take(up64((size_t)T * V));
    float* G = take(Td);
    float* DH = take(Td);
    float* DATT = take(Td);
    float* DFC = take(TF);
    float* DQKV = take(T3);
    float* part = take(up64(part_n));
    float* stats = take(up64((size_t)3 * NH * T));
    int* d_ids = reinterpret_cast<int*>(take(up64((size_t)2 * T)));
    int* d_pos = d_ids + T;
    unsigned* ctr = reinterpret_cast<unsigned*>(H->bwd_ws + H->bwd_ws_floats - n_ctr);

    std::vector<int> hi(2 * (size_t)T);
    for (int p = 0; p < T; ++p) {
        hi[p] = (int)ids[p];
        hi[T + p] = p;
    }
    CK(cudaMemcpyAsync(d_ids, hi.data(), hi.size() * 4, cudaMemcpyHostToDevice, H->stream));
    CK(cudaMemcpyAsync(DL, dlogits, (size_t)T * V * 4, cudaMemcpyHostToDevice, H->stream));

    // ---- forward with the stash ----
    RUN("embed", (double)T * d * 8,
        launch_embed(H->wte.w, H->wpe.w, reinterpret_cast<const uint32_t*>(d_ids), d_pos, xs, d, T, H->stream));
    for (int l = 0; l < L; ++l) {
        const LayerW& lw = H->layers[l];
        float* xin = xs + (size_t)l * Td;
        float* xm = xmid + (size_t)l * Td;
        float* qk = qkv + (size_t)l * T3;
        float* fp = fcpre + (size_t)l * TF;
        float* xo = xs + (size_t)(l + 1) * Td;
        // the linears take the tensor-core path for T >= 16 (fp16 hi/lo split inputs), as prefill does
        RUN("layernorm", (double)T * d * 8,
            launch_layernorm(xin, d, nullptr, hb, d, hb_hi, hb_lo, lw.ln1_g, lw.ln1_b, d, eps, T, H->stream));
        int rc = linear(H, "linear_qkv", lw.attn, In{hb, hb_hi, hb_lo, d}, T, epi_store(qk, d3, lw.attn.bias));
        if (rc) return rc;
        RUN("attn_train", (double)T * d3 * 4,
            launch_attn_fwd_train(qk, d3, qk + d, d3, qk + 2 * d, d3, T, NH, hd, att, d, att_hi, att_lo, H->stream));
        CK(cudaMemcpyAsync(xm, xin, (size_t)T * d * 4, cudaMemcpyDeviceToDevice, H->stream));
        Epi er = epi_store(xm, d, lw.proj.bias);
        er.kind = EPI_RESID;
        rc = linear(H, "linear_proj", lw.proj, In{att, att_hi, att_lo, d}, T, er);
        if (rc) return rc;
        RUN("layernorm", (double)T * d * 8,
            launch_layernorm(xm, d, nullptr, hb, d, hb_hi, hb_lo, lw.ln2_g, lw.ln2_b, d, eps, T, H->stream));
        rc = linear(H, "linear_fc", lw.fc, In{hb, hb_hi, hb_lo, d}, T, epi_store(fp, F, lw.fc.bias));
        if (rc) return rc;
        RUN("gelu", (double)T * F * 8, launch_gelu_fwd(fp, fb, fb_hi, fb_lo, (size_t)T * F, H->stream));
        CK(cudaMemcpyAsync(xo, xm, (size_t)T * d * 4, cudaMemcpyDeviceToDevice, H->stream));
        Epi em = epi_store(xo, d, lw.mproj.bias);
        em.kind = EPI_RESID;
        rc = linear(H, "linear_mproj", lw.mproj, In{fb, fb_hi, fb_lo, F}, T, em);
        if (rc) return rc;
    }
    const float* xL = xs + (size_t)L * Td;
    RUN("layernorm", (double)T * d * 8,
        launch_layernorm(xL, d, nullptr, lnf, d, nullptr, nullptr, H->lnf_g, H->lnf_b, d, eps, T, H->stream));

    // ---- backward: head, ln_f, then the layers in reverse ----
    // algorithmic bytes: the weights once, dY, the output (and the GELU input or the added-to output)
    auto bwd_lin = [&](const char* name, const Linear& Lw, const float* dY, int ldy, int epi, float* out, int ldo,
                       const float* xpre, int ldx) {
        const double bytes = (double)Lw.weight_bytes + (double)T * (Lw.rows + (epi == BWD_STORE ? 1 : 2) * Lw.cols) * 4;
        return run_kernel(H, name, bytes, [&]() {
            return launch_bwd_linear(Lw.w, dY, ldy, T, part, ctr, epi, out, ldo, xpre, ldx, H->stream);
        });
    };
    int rc = bwd_lin("bwd_linear_head", H->wte, DL, V, BWD_STORE, DH, d, nullptr, 0);
    if (rc) return rc;
    RUN("bwd_ln", (double)T * d * 16,
        launch_bwd_ln(DH, d, xL, d, H->lnf_g, eps, d, T, BWD_STORE, G, d, nullptr, nullptr, H->stream));
    for (int l = L - 1; l >= 0; --l) {
        const LayerW& lw = H->layers[l];
        const float* xin = xs + (size_t)l * Td;
        const float* xm = xmid + (size_t)l * Td;
        const float* qk = qkv + (size_t)l * T3;
        const float* fp = fcpre + (size_t)l * TF;
        // MLP branch: d_fc = gelu'(fc_pre) * (W_mproj^T g), dh2 = W_fc^T d_fc, g += LN2^T(dh2)
        rc = bwd_lin("bwd_linear_mproj", lw.mproj, G, d, BWD_GELU_BWD, DFC, F, fp, F);
        if (rc) return rc;
        rc = bwd_lin("bwd_linear_fc", lw.fc, DFC, F, BWD_STORE, DH, d, nullptr, 0);
        if (rc) return rc;
        RUN("bwd_ln", (double)T * d * 16,
            launch_bwd_ln(DH, d, xm, d, lw.ln2_g, eps, d, T, BWD_ADD, G, d, nullptr, nullptr, H->stream));
        // attention branch on g = d(x_mid): c_proj^T, attention backward, c_attn^T, LN1^T
        rc = bwd_lin("bwd_linear_proj", lw.proj, G, d, BWD_STORE, DATT, d, nullptr, 0);
        if (rc) return rc;
        RUN("bwd_attn", (double)T * d3 * 8,
            launch_attn_bwd_train(qk, d3, qk + d, d3, qk + 2 * d, d3, DATT, d, T, NH, hd, DQKV, d3, DQKV + d, d3,
                                  DQKV + 2 * d, d3, 0, stats, H->stream));
        H->launches++;  // query-row and key-row kernels
        rc = bwd_lin("bwd_linear_qkv", lw.attn, DQKV, d3, BWD_STORE, DH, d, nullptr, 0);
        if (rc) return rc;
        RUN("bwd_ln", (double)T * d * 16,
            launch_bwd_ln(DH, d, xin, d, lw.ln1_g, eps, d, T, BWD_ADD, G, d, nullptr, nullptr, H->stream));
    }
    CK(cudaMemcpyAsync(dx_out, G, (size_t)T * d * 4, cudaMemcpyDeviceToHost, H->stream));
    if (lnf_out) CK(cudaMemcpyAsync(lnf_out, lnf, (size_t)T * d * 4, cudaMemcpyDeviceToHost, H->stream));
    CK(cudaStreamSynchronize(H->stream));
    return check_device_error(H);
}
}  // namespace

// Message for gpt2q_last_error(NULL), used by calls that have no handle.
void gpt2q::set_global_error(const std::string& msg) { g_create_error = msg; }

// =================================================================== C-ABI
extern "C" {

int gpt2q_create(const gpt2q_config* cfg, const gpt2q_tensor_desc* tensors, int n_tensors, int device,
                 gpt2q_handle** out) {
    return create_common(cfg, tensors, n_tensors, device, 1, 0, nullptr, out);
}

int gpt2q_create_tp(const gpt2q_config* cfg, const gpt2q_tensor_desc* tensors, int n_tensors, int device,
                    int tp_size, int tp_rank, const void* nccl_id, gpt2q_handle** out) {
    if (tp_size > 1 && !nccl_id) {
        g_create_error = "nccl_id required for tp_size > 1";
        return GPT2Q_EARG;
    }
    return create_common(cfg, tensors, n_tensors, device, tp_size, tp_rank, nccl_id, out);
}

void gpt2q_destroy(gpt2q_handle* H) {
    if (!H) return;
    cudaSetDevice(H->device);
    if (H->stream) cudaStreamSynchronize(H->stream);
    for (auto& g : H->dec_graphs) cudaGraphExecDestroy(g.second.first);
    H->dec_graphs.clear();
    for (auto& r : H->prof_pending) {
        cudaEventDestroy(r.a);
        cudaEventDestroy(r.b);
    }
    for (auto e : H->ev_pool) cudaEventDestroy(e);
    if (H->tp) tp_destroy(H->tp);
    gemm_destroy(H->gemm);
    mk_destroy(H->mk);
    for (auto& a : H->allocs) cudaFree(a.p);
    if (H->bwd_ws) cudaFree(H->bwd_ws);
    if (H->h_stage) cudaFreeHost(H->h_stage);
    if (H->h_err) cudaFreeHost(H->h_err);
    if (H->own_stream) cudaStreamDestroy(H->own_stream);
    delete H;
}

const char* gpt2q_last_error(const gpt2q_handle* H) { return H ? H->err.c_str() : g_create_error.c_str(); }

int gpt2q_reset_kv(gpt2q_handle* H, const int32_t* slots, int n_slots) {
    if (!H) return GPT2Q_EARG;
    CK(cudaSetDevice(H->device));
    if (!slots) {
        CK(cudaMemsetAsync(H->kv.base, 0, H->kv.slot_stride * H->cfg.max_seqs * 4, H->stream));
    } else {
        for (int i = 0; i < n_slots; ++i) {
            if (slots[i] < 0 || slots[i] >= H->cfg.max_seqs) return H->fail(GPT2Q_EARG, "slot out of range");
            CK(cudaMemsetAsync(H->kv.base + (size_t)slots[i] * H->kv.slot_stride, 0, H->kv.slot_stride * 4, H->stream));
        }
    }
    CK(cudaStreamSynchronize(H->stream));
    return GPT2Q_OK;
}

int gpt2q_step(gpt2q_handle* H, uint32_t tok, int32_t pos, float* logits) {
    if (!H) return GPT2Q_EARG;
    CK(cudaSetDevice(H->device));
    const int32_t slot = 0;
    int rc = do_decode(H, &tok, &pos, &slot, 1);
    if (rc) return rc;
    return read_outputs(H, 1, H->logits, logits, nullptr);
}

int gpt2q_decode(gpt2q_handle* H, const uint32_t* tok, const int32_t* pos, const int32_t* slots, int n_seq,
                 float* logits, uint32_t* next_tok) {
    if (!H) return GPT2Q_EARG;
    CK(cudaSetDevice(H->device));
    int rc = do_decode(H, tok, pos, slots, n_seq);
    if (rc) return rc;
    return read_outputs(H, n_seq, H->logits, logits, next_tok);
}

int gpt2q_prefill(gpt2q_handle* H, const uint32_t* tokens, const int32_t* seq_offsets, const int32_t* slots,
                  int n_seq, float* logits_last, uint32_t* next_tok) {
    if (!H) return GPT2Q_EARG;
    CK(cudaSetDevice(H->device));
    int rc = do_prefill(H, tokens, seq_offsets, slots, n_seq);
    if (rc) return rc;
    return read_outputs(H, n_seq, H->logits, logits_last, next_tok);
}

int gpt2q_decode_steps(gpt2q_handle* H, int steps, uint32_t* out_tokens) {
    if (!H) return GPT2Q_EARG;
    if (steps < 0) return H->fail(GPT2Q_EARG, "steps < 0");
    if (H->cur_n <= 0) return H->fail(GPT2Q_EARG, "no sequences to continue (call prefill or decode first)");
    CK(cudaSetDevice(H->device));
    const int B = H->cur_n;
    std::vector<int> start = H->hpos;
    for (int b = 0; b < B; ++b)
        if (H->hpos[b] + steps > H->cfg.n_ctx)
            return H->fail(GPT2Q_EARG, "decode_steps would run past n_ctx");
    if (steps > 0 && use_persistent(H, B)) {
        int rc = run_persistent(H, steps);
        if (rc) return rc;
    } else {
        for (int s = 0; s < steps; ++s) {
            int rc = run_decode_step(H, B);
            if (rc) return rc;
        }
    }
    if (out_tokens && steps > 0) {
        // genlog[b][p] holds the token predicted from position p
        std::vector<uint32_t> row(H->cfg.n_ctx);
        CK(cudaStreamSynchronize(H->stream));
        for (int b = 0; b < B; ++b) {
            CK(cudaMemcpyAsync(row.data() + start[b], H->d_genlog + (size_t)b * H->cfg.n_ctx + start[b],
                               (size_t)steps * 4, cudaMemcpyDeviceToHost, H->stream));
            CK(cudaStreamSynchronize(H->stream));
            for (int s = 0; s < steps; ++s) out_tokens[(size_t)s * B + b] = row[start[b] + s];
        }
    }
    CK(cudaStreamSynchronize(H->stream));
    return check_device_error(H);
}

int gpt2q_generate_greedy(gpt2q_handle* H, const uint32_t* tokens, const int32_t* seq_offsets, int n_seq, int steps,
                          uint32_t* out) {
    if (!H) return GPT2Q_EARG;
    if (steps <= 0 || !out) return H->fail(GPT2Q_EARG, "steps must be >= 1 and out non-null");
    CK(cudaSetDevice(H->device));
    std::vector<uint32_t> first(n_seq > 0 ? n_seq : 1);
    int rc = gpt2q_prefill(H, tokens, seq_offsets, nullptr, n_seq, nullptr, first.data());
    if (rc) return rc;
    for (size_t i = 0; i < (size_t)n_seq * steps; ++i) out[i] = UINT32_MAX;
    for (int s = 0; s < n_seq; ++s) out[(size_t)s * steps] = first[s];
    // sequence s may generate tokens predicted from positions T_s-1 .. n_ctx-1
    std::vector<int> room(n_seq);
    int common = steps - 1;
    for (int s = 0; s < n_seq; ++s) {
        const int T = seq_offsets[s + 1] - seq_offsets[s];
        room[s] = std::min(steps - 1, H->cfg.n_ctx - T);
        common = std::min(common, room[s]);
    }
    if (common > 0) {
        std::vector<uint32_t> buf((size_t)common * n_seq);
        rc = gpt2q_decode_steps(H, common, buf.data());
        if (rc) return rc;
        for (int k = 0; k < common; ++k)
            for (int s = 0; s < n_seq; ++s) out[(size_t)s * steps + 1 + k] = buf[(size_t)k * n_seq + s];
    }
    // sequences with more room continue alone (the others stopped at n_ctx, gpt2.rs:374)
    for (int k = common; k < steps - 1; ++k) {
        std::vector<uint32_t> tk;
        std::vector<int32_t> ps, sl;
        std::vector<int> who;
        for (int s = 0; s < n_seq; ++s) {
            if (k < room[s]) {
                const int T = seq_offsets[s + 1] - seq_offsets[s];
                tk.push_back(out[(size_t)s * steps + k]);
                ps.push_back(T + k);
                sl.push_back(s);
                who.push_back(s);
            }
        }
        if (who.empty()) break;
        std::vector<uint32_t> nx(who.size());
        rc = gpt2q_decode(H, tk.data(), ps.data(), sl.data(), (int)who.size(), nullptr, nx.data());
        if (rc) return rc;
        for (size_t i = 0; i < who.size(); ++i) out[(size_t)who[i] * steps + 1 + k] = nx[i];
    }
    return GPT2Q_OK;
}

int gpt2q_set_adapter(gpt2q_handle* H, const float* A, const float* B, int r) {
    if (!H) return GPT2Q_EARG;
    if (!A || !B || r < 1 || r > gpt2q_handle::AD_MAX_R)
        return H->fail(GPT2Q_EARG, "adapter: A and B required, 1 <= r <= 256");
    CK(cudaSetDevice(H->device));
    const int d = H->cfg.n_embd;
    if (!H->d_adapter) {
        for (int k = 0; k < 2; ++k) {
            H->ad_a[k] = H->dalloc<float>((size_t)gpt2q_handle::AD_MAX_R * d * 4);
            H->ad_b[k] = H->dalloc<float>((size_t)gpt2q_handle::AD_MAX_R * d * 4);
        }
        H->d_adapter = H->dalloc<AdapterDesc>(sizeof(AdapterDesc));
        if (!H->ad_a[0] || !H->ad_a[1] || !H->ad_b[0] || !H->ad_b[1] || !H->d_adapter)
            return H->fail(GPT2Q_EOOM, "adapter buffers");
    }
    // RCU publish on the handle's stream: the other generation's buffers are free once every
    // step enqueued before the previous publish has run, which stream order guarantees
    const int g = H->ad_gen ^ 1;
    CK(cudaMemcpyAsync(H->ad_a[g], A, (size_t)r * d * 4, cudaMemcpyHostToDevice, H->stream));
    CK(cudaMemcpyAsync(H->ad_b[g], B, (size_t)r * d * 4, cudaMemcpyHostToDevice, H->stream));
    const AdapterDesc desc{H->ad_a[g], H->ad_b[g], r};
    CK(cudaMemcpyAsync(H->d_adapter, &desc, sizeof(desc), cudaMemcpyHostToDevice, H->stream));
    CK(cudaStreamSynchronize(H->stream));  // the host descriptor goes out of scope
    H->ad_gen = g;
    H->adapter_on = true;
    return GPT2Q_OK;
}

int gpt2q_clear_adapter(gpt2q_handle* H) {
    if (!H) return GPT2Q_EARG;
    if (!H->d_adapter) return GPT2Q_OK;
    CK(cudaSetDevice(H->device));
    const AdapterDesc desc{nullptr, nullptr, 0};
    CK(cudaMemcpyAsync(H->d_adapter, &desc, sizeof(desc), cudaMemcpyHostToDevice, H->stream));
    CK(cudaStreamSynchronize(H->stream));
    H->adapter_on = false;
    return GPT2Q_OK;
}

int gpt2q_nll(gpt2q_handle* H, const uint32_t* ids, int n, int slot, double* out) {
    if (!H) return GPT2Q_EARG;
    if (!ids || !out) return H->fail(GPT2Q_EARG, "null ids/out");
    if (n < 2 || n > H->cfg.n_ctx || n > H->Mmax) return H->fail(GPT2Q_EARG, "n out of range [2, min(n_ctx, max_tokens)]");
    if (slot < 0 || slot >= H->cfg.max_seqs) return H->fail(GPT2Q_EARG, "slot out of range");
    CK(cudaSetDevice(H->device));
    int rc = check_tokens(H, ids, (size_t)n);
    if (rc) return rc;
    constexpr int NLL_ROWS = 256;
    const int d = H->cfg.n_embd, V = H->cfg.vocab, R = n - 1;
    if (!H->nll_logits) {
        H->nll_logits = H->dalloc<float>((size_t)NLL_ROWS * V * 4);
        H->nll_tgt = H->dalloc<int>((size_t)H->cfg.n_ctx * 4);
        H->nll_terms = H->dalloc<double>((size_t)H->cfg.n_ctx * 8);
        if (!H->nll_logits || !H->nll_tgt || !H->nll_terms) return H->fail(GPT2Q_EOOM, "NLL buffers");
    }
    const int32_t offs[2] = {0, n};
    const int32_t slots[1] = {slot};
    rc = prefill_chunk(H, ids, offs, slots, 0, 1, true);
    if (rc) return rc;
    // positions 0..n-2 predict ids[1..n-1]: ln_f over their rows, the head in chunks, the terms
    std::vector<int> tgt(R);
    for (int p = 0; p < R; ++p) tgt[p] = (int)ids[p + 1];
    CK(cudaMemcpyAsync(H->nll_tgt, tgt.data(), (size_t)R * 4, cudaMemcpyHostToDevice, H->stream));
    RUN("layernorm", (double)R * d * 8,
        launch_layernorm(H->x, d, nullptr, H->h, d, H->h_hi, H->h_lo, H->lnf_g, H->lnf_b, d, H->cfg.ln_eps, R,
                         H->stream));
    rc = apply_adapter(H, R);
    if (rc) return rc;
    for (int r0 = 0; r0 < R; r0 += NLL_ROWS) {
        const int rows = std::min(NLL_ROWS, R - r0);
        const size_t o = (size_t)r0 * d;
        rc = linear(H, "linear_head", H->wte, In{H->h + o, H->h_hi + o, H->h_lo + o, d}, rows,
                    epi_store(H->nll_logits, V, nullptr));
        if (rc) return rc;
        RUN("nll", (double)rows * V * 4,
            launch_nll_rows(H->nll_logits, V, V, rows, H->nll_tgt + r0, H->nll_terms + r0, H->stream));
    }
    std::vector<double> terms(R);
    CK(cudaMemcpyAsync(terms.data(), H->nll_terms, (size_t)R * 8, cudaMemcpyDeviceToHost, H->stream));
    CK(cudaStreamSynchronize(H->stream));
    rc = check_device_error(H);
    if (rc) return rc;
    // the reference's accumulation: total -= term in position order, then the mean
    double total = 0.0;
    for (int p = 0; p < R; ++p) total -= terms[p];
    *out = total / (double)R;
    // the slot's cache now holds this sequence; its decode state is not advanced
    return GPT2Q_OK;
}

int gpt2q_trunk_input_grad(gpt2q_handle* H, const uint32_t* ids, int n, const float* dlogits, float* dx,
                           float* lnf_out) {
    if (!H) return GPT2Q_EARG;
    if (!ids || !dlogits || !dx) return H->fail(GPT2Q_EARG, "null ids/dlogits/dx");
    if (n < 1 || n > H->cfg.n_ctx) return H->fail(GPT2Q_EARG, "n out of range [1, n_ctx]");
    if (H->tp_size > 1) return H->fail(GPT2Q_EUNSUP, "trunk backward needs a single-GPU handle");
    if (H->hd > 128) return H->fail(GPT2Q_EUNSUP, "trunk backward needs head dim <= 128");
    CK(cudaSetDevice(H->device));
    const int rc = check_tokens(H, ids, (size_t)n);
    if (rc) return rc;
    return trunk_grad(H, ids, n, dlogits, dx, lnf_out);
}

int gpt2q_dequant(gpt2q_handle* H, const char* name, float* out, uint64_t n) {
    if (!H || !name || !out) return GPT2Q_EARG;
    CK(cudaSetDevice(H->device));
    auto it = H->lin_by_name.find(name);
    if (it != H->lin_by_name.end()) {
        const QW& w = it->second->w;
        if ((uint64_t)w.rows * w.cols != n) return H->fail(GPT2Q_EARG, "dequant: n does not match tensor size");
        float* tmp = nullptr;
        CK(cudaMalloc(&tmp, n * 4));
        cudaError_t e = launch_dequant(w, tmp, H->stream);
        if (e == cudaSuccess) e = cudaMemcpyAsync(out, tmp, n * 4, cudaMemcpyDeviceToHost, H->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(H->stream);
        cudaFree(tmp);
        if (e != cudaSuccess) return H->fail(GPT2Q_ECUDA, std::string("dequant: ") + cudaGetErrorString(e));
        return GPT2Q_OK;
    }
    auto iv = H->vec_by_name.find(name);
    if (iv != H->vec_by_name.end()) {
        if (iv->second.second != n) return H->fail(GPT2Q_EARG, "dequant: n does not match tensor size");
        CK(cudaMemcpyAsync(out, iv->second.first, n * 4, cudaMemcpyDeviceToHost, H->stream));
        CK(cudaStreamSynchronize(H->stream));
        return GPT2Q_OK;
    }
    return H->fail(GPT2Q_EARG, std::string("dequant: unknown tensor ") + name);
}

uint64_t gpt2q_launches(const gpt2q_handle* H) { return H ? H->launches : 0; }

int gpt2q_set_stream(gpt2q_handle* H, void* stream) {
    if (!H) return GPT2Q_EARG;
    CK(cudaStreamSynchronize(H->stream));
    H->stream = stream ? reinterpret_cast<cudaStream_t>(stream) : H->own_stream;
    // graphs were instantiated for launch on any stream; they stay valid
    return GPT2Q_OK;
}

int gpt2q_sync(gpt2q_handle* H) {
    if (!H) return GPT2Q_EARG;
    CK(cudaSetDevice(H->device));
    CK(cudaStreamSynchronize(H->stream));
    return GPT2Q_OK;
}

int gpt2q_profile(gpt2q_handle* H, int enable) {
    if (!H) return GPT2Q_EARG;
    int rc = flush_profile(H);
    if (rc) return rc;
    H->prof = enable != 0;
    if (H->prof) {
        H->prof_agg.clear();
        while (H->ev_pool.size() < 2048) {
            cudaEvent_t e = nullptr;
            CK(cudaEventCreate(&e));
            H->ev_pool.push_back(e);
        }
    }
    return GPT2Q_OK;
}

int gpt2q_profile_kernels(gpt2q_handle* H, int reps, char* json, size_t cap) {
    if (!H || !json || cap == 0 || reps <= 0) return GPT2Q_EARG;
    if (H->cur_n <= 0) return H->fail(GPT2Q_EARG, "profile_kernels: no sequences (call prefill or decode first)");
    CK(cudaSetDevice(H->device));
    for (int b = 0; b < H->cur_n; ++b)
        if (H->hpos[b] + 1 > H->cfg.n_ctx) return H->fail(GPT2Q_EARG, "profile_kernels: positions at n_ctx");
    H->ktime_reps = reps;
    H->ktime_res.clear();
    H->ktime_count.clear();
    int rc = enqueue_decode(H, H->cur_n);
    H->ktime_reps = 0;
    if (rc) return rc;
    CK(cudaStreamSynchronize(H->stream));
    for (int b = 0; b < H->cur_n; ++b) H->hpos[b] += 1;
    std::string s = "{";
    bool first = true;
    for (auto& kv : H->ktime_count) {
        auto it = H->ktime_res.find(kv.first);
        if (it == H->ktime_res.end()) continue;
        char buf[256];
        std::snprintf(buf, sizeof buf, "%s\"%s\": {\"us\": %.4f, \"bytes\": %.0f, \"per_step\": %d}",
                      first ? "" : ", ", kv.first.c_str(), it->second.first, it->second.second, kv.second);
        s += buf;
        first = false;
    }
    s += "}";
    if (s.size() + 1 > cap) return H->fail(GPT2Q_EARG, "profile_kernels: buffer too small");
    std::memcpy(json, s.c_str(), s.size() + 1);
    return check_device_error(H);
}

int gpt2q_info(gpt2q_handle* H, char* json, size_t cap) {
    if (!H || !json || cap == 0) return GPT2Q_EARG;
    std::string why;
    for (char ch : H->mk.why) why += (ch == '"' || ch == '\\') ? '\'' : ch;
    const std::string head = std::string("{\"persistent_decode\": ") + (H->mk.enabled ? "true" : "false") +
                          ", \"persistent_why\": \"" + why + "\", \"persistent_ctas\": " +
                          std::to_string(H->mk.enabled ? MK_CS * H->mk.clusters : 0) +
                          ", \"tensor_core\": " + (H->gemm.enabled ? "true" : "false") +
                          ", \"tc_products\": " + std::to_string(H->gemm.products) +
                          ", \"mma_tiles_per_cta_max\": " + std::to_string(mma_tiles_per_cta_max()) +
                          ", \"tp_size\": " + std::to_string(H->tp_size) +
                          ", \"tp_peer_mapped\": " + (tp_peer_mapped(H->tp) ? "true" : "false");
    std::string tr;
    if (H->mk.trace) {
        // phase stamps (ns since the first stamp of CTA 0) of the last persistent launch
        const int G = MK_CS * H->mk.clusters;
        std::vector<unsigned long long> t((size_t)G * MK_TRACE);
        CK(cudaMemcpy(t.data(), H->mk.trace, t.size() * 8, cudaMemcpyDeviceToHost));
        tr = ", \"persistent_trace\": [";
        for (int g = 0; g < G; ++g) {
            tr += g ? ", [" : "[";
            for (int k = 0; k < MK_TRACE; ++k) {
                const unsigned long long raw = t[(size_t)g * MK_TRACE + k];
                const bool counter = mk_trace_counter(k);
                const long long v = counter ? (long long)raw : raw ? (long long)(raw - t[0]) : -1;
                tr += (k ? ", " : "") + std::to_string(v);
            }
            tr += "]";
        }
        tr += "]";
    }
    const std::string gt = gemm_trace_json(H->gemm);
    if (!gt.empty()) tr += ", \"tc_trace\": " + gt;
    const std::string mt = mma_trace_json();
    if (!mt.empty()) tr += ", \"mma_trace\": " + mt;
    const std::string at = attn_tc_trace_json();
    if (!at.empty()) tr += ", \"attn_trace\": " + at;
    const std::string s = head + tr + "}";
    if (s.size() + 1 > cap) return H->fail(GPT2Q_EARG, "info: buffer too small");
    std::memcpy(json, s.c_str(), s.size() + 1);
    return GPT2Q_OK;
}

int gpt2q_profile_read(gpt2q_handle* H, char* json, size_t cap) {
    if (!H || !json || cap == 0) return GPT2Q_EARG;
    int rc = flush_profile(H);
    if (rc) return rc;
    std::string s = "{";
    bool first = true;
    for (auto& kv : H->prof_agg) {
        char buf[256];
        std::snprintf(buf, sizeof buf, "%s\"%s\": {\"launches\": %llu, \"ms\": %.6f, \"bytes\": %.0f}", first ? "" : ", ",
                      kv.first.c_str(), (unsigned long long)kv.second.launches, kv.second.ms, kv.second.bytes);
        s += buf;
        first = false;
    }
    s += "}";
    if (s.size() + 1 > cap) return H->fail(GPT2Q_EARG, "profile_read: buffer too small");
    std::memcpy(json, s.c_str(), s.size() + 1);
    return GPT2Q_OK;
}

}  // extern "C"
