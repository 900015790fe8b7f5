// Persistent single-sequence decode kernel and its weight-stream packer (see persistent.h).
//
// Reference semantics per step (experiments/model-lab/src/gpt2.rs:227-331, gpu.rs:212-376):
// x = wte[tok] + wpe[pos]; per layer x += c_proj(attn(LN1(x))) + b, x += mproj(gelu(c_fc(LN2(x)))) + b;
// logits = wte . LN_f(x); next = argmax with ties to the last index (gpt2.rs:390-396).
#include "persistent.h"

#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "kernels.h"
#include "tcgen05.cuh"

namespace gpt2q {
namespace {

constexpr int NWC = 8;         // warps
constexpr int NCT = NWC * 32;  // threads
constexpr int THREADS = NCT;
constexpr int NSLOT = 6;       // ring slots (bulk copies in flight per CTA)
constexpr int HD = 64;         // head dim
constexpr int APS = HD + 2;    // attention partial: m, l, o[64]
constexpr uint32_t SPIN = 1u << 22;
constexpr int BEST_STRIDE = 32;  // argmax words 256 bytes apart: pollers spread over L2 slices

// Per-layer vector block in shared memory (floats): LN1 g|b, LN2 g|b (d each), then this
// CTA's slices of the q/k/v bias (3 x 8), attn c_proj bias (d/8), c_fc bias (32) and
// mlp c_proj bias (d/8).
struct VecLayout {
    int ln1g, ln1b, ln2g, ln2b, bqkv, bproj, bfc, bmproj, total;
    __host__ __device__ explicit VecLayout(int d) {
        const int dsl = d / MK_CS;
        ln1g = 0;
        ln1b = d;
        ln2g = 2 * d;
        ln2b = 3 * d;
        bqkv = 4 * d;
        bproj = bqkv + 24;
        bfc = bproj + dsl;
        bmproj = bfc + 32;
        total = bmproj + dsl;
    }
};

// ------------------------------------------------------------------ primitives
__device__ __forceinline__ bool aborted(const MkParams& p) { return *(volatile const int*)p.abort_flag != 0; }

__device__ __noinline__ void raise_error(const MkParams& p, int code) {
    atomicCAS(p.err, 0, code);
    atomicExch(p.abort_flag, 1);
}

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const unsigned long long t = __shfl_xor_sync(0xffffffffu, v, o);
        v = t > v ? t : v;
    }
    return v;
}

// Wait for a ring slot's bulk copy; gives up on abort or after SPIN polls.
__device__ __forceinline__ bool ring_wait(uint64_t* bar, uint32_t parity, const MkParams& p) {
    for (uint32_t i = 0; i < SPIN; ++i) {
        if (tc::mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 255u && aborted(p)) return false;
    }
    raise_error(p, 1);
    return false;
}

// Wait for our own bulk copies before exit: bounded, ignores the abort flag.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity, const MkParams& p) {
    for (uint32_t i = 0; i < SPIN; ++i)
        if (tc::mbar_try_wait(bar, parity)) return;
    raise_error(p, 4);
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     tc::smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(tc::smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(tc::smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }


__device__ __forceinline__ void ll_store(unsigned long long* a, float v, uint32_t e) {
    const unsigned long long w = ((unsigned long long)e << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(a), "l"(w) : "memory");
}

__device__ __forceinline__ void ll_store_raw(unsigned long long* a, unsigned long long w) {
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(a), "l"(w) : "memory");
}

__device__ __forceinline__ unsigned long long ll_load(const unsigned long long* a) {
    unsigned long long w;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(a) : "memory");
    return w;
}

// Sum of the n <= 16 LL words a[0], a[stride], ... (fixed index order) once all carry epoch e.
// Every poll round issues all its loads before testing any of them. `rounds` (optional)
// receives the number of poll rounds.
__device__ __forceinline__ float ll_sum(const unsigned long long* a, size_t stride, int n, uint32_t e,
                                        const MkParams& p, uint32_t* rounds = nullptr) {
    float v[16];
    unsigned long long w[16];
    uint32_t pending = n >= 32 ? 0xFFFFFFFFu : ((1u << n) - 1u);
    uint32_t it = 0;
    for (; pending && it < SPIN; ++it) {
#pragma unroll
        for (int i = 0; i < 16; ++i)
            if (pending & (1u << i)) w[i] = ll_load(a + (size_t)i * stride);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            if ((pending & (1u << i)) && (uint32_t)(w[i] >> 32) == e) {
                v[i] = __uint_as_float((uint32_t)w[i]);
                pending &= ~(1u << i);
            }
        }
        if (pending) {
            __nanosleep(32);
            if ((it & 63u) == 63u && aborted(p)) break;
        }
    }
    if (pending && !aborted(p)) raise_error(p, 3);
    if (rounds) *rounds = it;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i)
        if (i < n) s += (pending & (1u << i)) ? 0.f : v[i];
    return s;
}

// R int8 rows (row stride K bytes, scale stride K/32 halves) against one fp32 vector in
// shared memory; warp-wide. The R accumulation chains are independent and share every
// activation load; every lane returns all R sums. KC > 0 fixes K at compile time (full unroll).
template <int R, int KC>
__device__ __forceinline__ void dot_q8_rows(const uint8_t* q, const __half* s, const float* x, int Kr, int lane,
                                            float (&out)[R]) {
    const int K = KC > 0 ? KC : Kr;
    const int gs = K >> 5;
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.f;
    auto body = [&](int c) {
        const float4 xv = *reinterpret_cast<const float4*>(x + c);
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const uint32_t w = *reinterpret_cast<const uint32_t*>(q + (size_t)r * K + c);
            float f[4];
            i8x4_to_f32(w, f);
            float t = f[0] * xv.x;
            t = fmaf(f[1], xv.y, t);
            t = fmaf(f[2], xv.z, t);
            t = fmaf(f[3], xv.w, t);
            acc[r] = fmaf(t, __half2float(s[r * gs + (c >> 5)]), acc[r]);
        }
    };
    if constexpr (KC > 0) {
#pragma unroll
        for (int i = 0; i < KC / 128; ++i) body(lane * 4 + 128 * i);
    } else {
#pragma unroll 2
        for (int c = lane * 4; c < K; c += 128) body(c);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1)
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
#pragma unroll
    for (int r = 0; r < R; ++r) out[r] = acc[r];
}

// ---- int8 tensor-core dot products (mma.sync m16n8k32, s8 x s8 -> s32) ----
// An fp32 vector x is written exactly enough as four int8 "pieces" per 32-wide group g:
// x = 2^-S_g (p0 + p1 2^-7 + p2 2^-14 + p3 2^-21) + r with |r| <= 2^(E_g - 28), E_g the
// exponent of max |x| over the group (|p0| <= 64, |p1..p3| <= 64). The pieces are the columns
// 0..3 of the mma's B operand, so one instruction gives the exact integer dot products of 16
// weight rows with all four pieces; the int32 results are combined in fp32 and scaled by the
// weight group's f16 scale and 2^-S_g.
__device__ __forceinline__ void mma_s8_16x8x32(int (&c)[4], const uint4& a, uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

// Warp-wide: the four pieces of x[32*ks + lane] into pc[p][32*ks + lane] (pc rows d bytes
// apart); returns 2^-S for the group.
__device__ __forceinline__ float split_pieces(const float* x, int ks, int lane, int8_t* pc, int d) {
    const float v0 = x[32 * ks + lane];
    // max |x| of the group by its bit pattern (non-negative floats order as unsigned integers);
    // S = 5 - floor(log2 max) so that |x| 2^S < 64, capped at 126 (tiny or zero groups)
    const uint32_t mb = __reduce_max_sync(0xffffffffu, __float_as_uint(v0) & 0x7FFFFFFFu);
    const int S = min(126, 132 - (int)(mb >> 23));
    float v = v0 * __uint_as_float((uint32_t)(127 + S) << 23);  // exact power-of-two scaling
    const float p0 = rintf(v);
    v = (v - p0) * 128.f;
    const float p1 = rintf(v);
    v = (v - p1) * 128.f;
    const float p2 = rintf(v);
    v = (v - p2) * 128.f;
    const float p3 = rintf(v);
    int8_t* o = pc + 32 * ks + lane;
    o[0] = (int8_t)(int)p0;
    o[d] = (int8_t)(int)p1;
    o[2 * d] = (int8_t)(int)p2;
    o[3 * d] = (int8_t)(int)p3;
    return __uint_as_float((uint32_t)(127 - S) << 23);  // 2^-S, S in [-122, 126]
}

// B fragments of x for this warp's groups ks = warp + 8 i (i < 4, ks < gsn): pieces go through
// pc ([4][d] bytes; each warp writes and reads only its own groups), f[i] = 2^-S of group ks.
__device__ __forceinline__ void vec_fragments(const float* x, int d, int8_t* pc, int warp, int lane, float (&f)[4],
                                              uint32_t (&b0)[4], uint32_t (&b1)[4]) {
    const int gsn = d >> 5;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int ks = warp + NWC * i;
        f[i] = ks < gsn ? split_pieces(x, ks, lane, pc, d) : 0.f;
    }
    __syncwarp();
    const int n = lane >> 2, t4 = 4 * (lane & 3);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int ks = warp + NWC * i;
        const bool ok = ks < gsn && n < 4;
        b0[i] = ok ? *reinterpret_cast<const uint32_t*>(pc + n * d + 32 * ks + t4) : 0u;
        b1[i] = ok ? *reinterpret_cast<const uint32_t*>(pc + n * d + 32 * ks + 16 + t4) : 0u;
    }
}

// Weights of the result columns lane (g, t) holds: pieces 2t and 2t+1 (columns 4..7 are zero).
__device__ __forceinline__ float piece_w_lo(int lane) {
    return (lane & 3) == 0 ? 1.f : ((lane & 3) == 1 ? 0x1p-14f : 0.f);
}
__device__ __forceinline__ float piece_w_hi(int lane) {
    return (lane & 3) == 0 ? 0x1p-7f : ((lane & 3) == 1 ? 0x1p-21f : 0.f);
}

// 32 weight rows of a fragment-ordered segment (block 2 ks + mt of 512 bytes: lane's 16 bytes
// are its A registers; scales Ss [32][gsn]) against x's fragments: this warp's k-groups summed
// in group order; per-warp row sums to red32[warp][32] (the caller syncs and adds the warps).
__device__ __forceinline__ void rows32_mma(const uint8_t* S, const __half* Ss, int gsn, const float (&f)[4],
                                           const uint32_t (&b0)[4], const uint32_t (&b1)[4], int warp, int lane,
                                           float* red32) {
    const float wlo = piece_w_lo(lane), whi = piece_w_hi(lane);
    const int gr = lane >> 2;
    float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int ks = warp + NWC * i;
        if (ks < gsn) {
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
                const uint4 a = *reinterpret_cast<const uint4*>(S + ((size_t)(2 * ks + mt) * 32 + lane) * 16);
                int c[4];
                mma_s8_16x8x32(c, a, b0[i], b1[i]);
                const float sa = __half2float(Ss[(mt * 16 + gr) * gsn + ks]) * f[i];
                const float sb = __half2float(Ss[(mt * 16 + gr + 8) * gsn + ks]) * f[i];
                const float va = fmaf((float)c[1], whi, (float)c[0] * wlo);
                const float vb = fmaf((float)c[3], whi, (float)c[2] * wlo);
                acc[mt][0] = fmaf(va, sa, acc[mt][0]);
                acc[mt][1] = fmaf(vb, sb, acc[mt][1]);
            }
        }
    }
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            acc[mt][u] += __shfl_xor_sync(0xffffffffu, acc[mt][u], 1);
            acc[mt][u] += __shfl_xor_sync(0xffffffffu, acc[mt][u], 2);
        }
    if ((lane & 3) == 0) {
        red32[warp * 32 + gr] = acc[0][0];
        red32[warp * 32 + gr + 8] = acc[0][1];
        red32[warp * 32 + 16 + gr] = acc[1][0];
        red32[warp * 32 + 24 + gr] = acc[1][1];
    }
}

__device__ __forceinline__ void softmax_update(float s, float v0, float v1, float& m, float& l, float& o0,
                                               float& o1) {
    const float mn = fmaxf(m, s);
    const float cf = expf(m - mn), pf = expf(s - mn);
    l = l * cf + pf;
    o0 = o0 * cf + pf * v0;
    o1 = o1 * cf + pf * v1;
    m = mn;
}

// Bulk copies of layer l's vectors (this CTA's slices) into vb, completing on `bar`; one thread.
__device__ __forceinline__ void fetch_layer_vectors(const MkParams& p, const MkLayer& lw, int h, int rank, float* vb,
                                                    uint64_t* bar) {
    const int d = p.d, dsl = d / MK_CS;
    const VecLayout V(d);
    const uint32_t dv = (uint32_t)d * 4;
    tc::mbar_arrive_expect_tx(bar, 4 * dv + 3 * 32 + 2 * (uint32_t)dsl * 4 + 128);
    bulk_g2s(vb + V.ln1g, lw.ln1_g, dv, bar);
    bulk_g2s(vb + V.ln1b, lw.ln1_b, dv, bar);
    bulk_g2s(vb + V.ln2g, lw.ln2_g, dv, bar);
    bulk_g2s(vb + V.ln2b, lw.ln2_b, dv, bar);
    for (int sel = 0; sel < 3; ++sel) bulk_g2s(vb + V.bqkv + sel * 8, lw.b_qkv + sel * d + h * HD + rank * 8, 32, bar);
    bulk_g2s(vb + V.bproj, lw.b_proj + rank * dsl, (uint32_t)dsl * 4, bar);
    bulk_g2s(vb + V.bfc, lw.b_fc + (h * MK_CS + rank) * 32, 128, bar);
    bulk_g2s(vb + V.bmproj, lw.b_mproj + rank * dsl, (uint32_t)dsl * 4, bar);
}

// Warm L2 with this CTA's block of cached K/V rows (positions < pos) of layer l.
__device__ __forceinline__ void prefetch_kv(const MkParams& p, int slot, int l, int h, int rank, int pos) {
    const int T = pos + 1;
    const int per = (T + MK_CS - 1) / MK_CS;
    const int t0 = rank * per, t1 = min(pos, t0 + per);
    if (t1 <= t0) return;
    const float* k = p.kv + (size_t)slot * p.kv_slot + (size_t)l * p.kv_layer + (size_t)h * p.kv_head + (size_t)t0 * HD;
    prefetch_l2(k, (uint32_t)((t1 - t0) * HD * 4));
    prefetch_l2(k + p.kv_sel, (uint32_t)((t1 - t0) * HD * 4));
}

// One 1-D bulk copy from this CTA's shared memory into CTA `peer` of the cluster, completing
// (tx bytes) on the peer's mbarrier. Source, destination and size are 16-byte multiples.
__device__ __forceinline__ void send_to(uint32_t peer, const void* src_local, const void* dst_same_offset,
                                        uint32_t bytes, const uint64_t* bar_same_offset) {
    const uint32_t dst = tc::map_cluster(tc::smem_u32(dst_same_offset), peer);
    const uint32_t bar = tc::map_cluster(tc::smem_u32(bar_same_offset), peer);
    asm volatile(
        "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "r"(tc::smem_u32(src_local)), "r"(bytes), "r"(bar)
        : "memory");
}

// Wait for the phase with the given parity of a local mbarrier fed by bulk copies. Bounded;
// deliberately not abort-aware, so no copy into this CTA is left in flight at exit.
__device__ __forceinline__ void wait_rx(uint64_t* bar, uint32_t parity, const MkParams& p) {
    for (uint32_t i = 0; i < SPIN; ++i)
        if (tc::mbar_try_wait(bar, parity)) return;
    raise_error(p, 5);
}

// y = LN(x) * g + b over d features with the population variance (gpt2.rs:178-185), g and b
// in shared memory; mean and E[x^2] come from one block reduction (var = E[x^2] - mean^2).
// x is read from `x`; with `xcopy` it is also stored there. Each thread holds columns
// tid + 256 k, k < 4.
__device__ __forceinline__ void layernorm(const float* x, float* xcopy, float* y, const float* g, const float* b,
                                          int d, float eps, float* red) {
    float xv[4];
    float s = 0.f, q = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int c = threadIdx.x + k * NCT;
        xv[k] = 0.f;
        if (c < d) {
            xv[k] = x[c];
            if (xcopy) xcopy[c] = xv[k];
            s += xv[k];
            q = fmaf(xv[k], xv[k], q);
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        s += __shfl_xor_sync(0xffffffffu, s, o);
        q += __shfl_xor_sync(0xffffffffu, q, o);
    }
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        red[2 * warp] = s;
        red[2 * warp + 1] = q;
    }
    __syncthreads();
    float ts = 0.f, tq = 0.f;
#pragma unroll
    for (int w = 0; w < NWC; ++w) {
        ts += red[2 * w];
        tq += red[2 * w + 1];
    }
    const float mean = ts / (float)d;
    const float var = fmaxf(tq / (float)d - mean * mean, 0.f);
    const float rstd = __frcp_rn(sqrtf(var + eps));
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int c = threadIdx.x + k * NCT;
        if (c < d) y[c] = (xv[k] - mean) * rstd * g[c] + b[c];
    }
    __syncthreads();
}

// ------------------------------------------------------------------ the kernel
// Intra-cluster exchanges (each once per layer, each with its own receive mbarrier):
//   QKV  24 q/k/v values of every CTA      -> qkv_in[8][24]
//   ATT  attention partial (m, l, o[64])   -> ap_in[8][APP]
//   X1   x' slice of every rank             -> x1_in[d]
//   MP   mlp c_proj partial of my rows      -> mp_in[8][d/8]
//   X2   x'' slice of every rank            -> x2_in[d]
// A sender stages its data in its own shared memory, fences it for the async proxy and sends
// one bulk copy per peer. Every receive buffer is rewritten only after its reader has used
// it: each next write depends, through the layer's data flow, on that reader's progress.
constexpr int APP = 68;  // attention partial padded to a 16-byte multiple
constexpr int KV_STAGE = 32;  // cached positions per CTA staged in shared memory (else read from L2)
enum { RX_QKV = 0, RX_ATT, RX_X1, RX_MP, RX_X2, RX_N };

// D > 0: the model width known at compile time (GPT-2 small: 768); D = 0: any eligible width.
template <int D>
__global__ void __launch_bounds__(THREADS, 1) k_decode_persistent(const __grid_constant__ MkParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int d = D > 0 ? D : p.d;
    const int L = p.n_layer, H = p.n_head;
    const int seg = p.seg_bytes;
    const int g = blockIdx.x;
    const int h = g / MK_CS;                    // cluster = attention head
    const int rank = (int)tc::cluster_rank();   // CTA within the cluster
    const int G = gridDim.x;
    const int dsl = d / MK_CS;                  // residual columns owned per rank
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const VecLayout VL(d);

    uint8_t* ring = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)NSLOT * seg);  // [NSLOT]
    uint64_t* rx = full + NSLOT;                                               // [RX_N]
    float* xs = reinterpret_cast<float*>(smem + (size_t)NSLOT * seg + 128);   // [d] residual stream
    float* ln = xs + d;                    // [d]
    float* lnf = ln + d;                   // [2d]: ln_f g | b
    float* vbuf = lnf + 2 * d;             // [2][VL.total]: per-layer vectors, double buffered
    float* qkv_in = vbuf + 2 * VL.total;   // [8][24]
    float* ap_in = qkv_in + MK_CS * 24;    // [8][APP]
    float* x1_in = ap_in + MK_CS * APP;    // [d]
    float* mp_in = x1_in + d;              // [8][dsl]
    float* x2_in = mp_in + d;              // [d]
    float* qkv_out = x2_in + d;            // [24] (+8 pad)
    float* ap_out = qkv_out + 32;          // [APP]
    float* x_out = ap_out + APP;           // [dsl]: x' then x'' slice
    float* mpart = x_out + dsl;            // [d]
    float* wred = mpart + d;               // [8][APS]: per-warp attention partials
    float* atth = wred + NWC * APS;        // [64]
    float* fs = atth + HD;                 // [32]
    float* red = fs + 32;                  // [16]
    float* kst = red + 16;                 // [2][KV_STAGE][64]: this CTA's cached K | V rows
    uint64_t* kvbar = reinterpret_cast<uint64_t*>(kst + 2 * KV_STAGE * HD);
    uint64_t* vbar = kvbar + 1;  // [2]: per-layer vectors, one per buffer
    unsigned long long* bw = reinterpret_cast<unsigned long long*>(vbar + 2);  // [8]
    MkLayer* lws = reinterpret_cast<MkLayer*>(bw + 8);                         // [n_layer]
    const uint32_t rx_bytes[RX_N] = {(uint32_t)(MK_CS * 24 * 4), (uint32_t)(MK_CS * APP * 4), (uint32_t)(d * 4),
                                     (uint32_t)(d * 4), (uint32_t)(d * 4)};

    const int row0_head = g * p.head_rows;
    const int rows_head = max(0, min(p.vocab, row0_head + p.head_rows) - row0_head);
    const int nseg_head = (rows_head + 31) / 32;
    const int nseg = 3 * L + nseg_head;
    const int total = p.steps * nseg;
    const int n_layers_total = p.steps * L;
    const uint8_t* stream = p.stream + (size_t)g * p.cta_bytes;

    // ring: segment i lives in slot i % NSLOT; a slot is refilled as soon as it is released
    int iss = 0, iss_seg = 0;  // next segment to issue, and its index within a step (thread 0)
    auto issue_next = [&]() {
        const int s = iss % NSLOT;
        tc::mbar_arrive_expect_tx(&full[s], (uint32_t)seg);
        bulk_g2s(ring + (size_t)s * seg, stream + (size_t)iss_seg * seg, (uint32_t)seg, &full[s]);
        ++iss;
        iss_seg = (iss_seg + 1 == nseg) ? 0 : iss_seg + 1;
    };
    int rc = 0;  // ring segments consumed
    auto seg_wait = [&]() -> const uint8_t* {
        const int s = rc % NSLOT;
        ring_wait(&full[s], (uint32_t)((rc / NSLOT) & 1), p);
        return ring + (size_t)s * seg;
    };
    auto seg_release = [&]() {  // call after a __syncthreads that follows the last read
        if (tid == 0 && iss < total) issue_next();
        ++rc;
    };
    // staged data (written by this CTA's threads before a __syncthreads) -> every CTA of the cluster
    auto send_all = [&](const float* src, const float* dst, uint32_t bytes, int which) {
        if (warp == 0 && lane < MK_CS) send_to((uint32_t)lane, src, dst, bytes, &rx[which]);
    };
    int gl = 0;  // layers started in this launch: receive phase parity and vector buffer
    auto rx_wait = [&](int which) { wait_rx(&rx[which], (uint32_t)(gl & 1), p); };
    auto rx_rearm = [&](int which) {  // after the last read of this layer's data (past a __syncthreads)
        if (tid == 0 && gl + 1 < n_layers_total) tc::mbar_arrive_expect_tx(&rx[which], rx_bytes[which]);
    };

    const uint32_t epoch0 = *reinterpret_cast<volatile uint32_t*>(p.epoch);
    const int pos0 = *reinterpret_cast<volatile int*>(p.pos);
    const int slot = *p.slot;
    uint32_t tok = *reinterpret_cast<volatile uint32_t*>(p.tok);

    if (tid == 0) {
        for (int i = 0; i < NSLOT; ++i) tc::mbar_init(&full[i], 1);
        for (int i = 0; i < RX_N; ++i) tc::mbar_init(&rx[i], 1);
        tc::mbar_init(kvbar, 1);
        tc::mbar_init(&vbar[0], 1);
        tc::mbar_init(&vbar[1], 1);
        tc::fence_mbar_init();
        for (int i = 0; i < RX_N; ++i)
            if (n_layers_total > 0) tc::mbar_arrive_expect_tx(&rx[i], rx_bytes[i]);
        while (iss < NSLOT && iss < total) issue_next();
    }
    for (int c = tid; c < d / 4; c += NCT) {
        cp_async16(lnf + 4 * c, p.lnf_g + 4 * c);
        cp_async16(lnf + d + 4 * c, p.lnf_b + 4 * c);
    }
    for (int l = tid; l < L; l += NCT) lws[l] = p.layers[l];
    __syncthreads();
    if (tid == 32) fetch_layer_vectors(p, lws[0], h, rank, vbuf, &vbar[0]);
    cp_async_wait_all();  // ln_f vectors
    tc::cluster_sync();  // every CTA's receive barriers are armed before the first send

    // optional phase stamps: step 0, layer 1 in detail, layer ends, head
    unsigned long long* trace = p.trace ? p.trace + (size_t)g * MK_TRACE : nullptr;
    int tstep = -1, tlayer = -1;
#define MK_TR(k)                                                          \
    do {                                                                  \
        if (trace && tstep == 0 && tid == 0) trace[(k)] = globaltimer(); \
    } while (0)
#define MK_TRL(k)                  \
    do {                           \
        if (tlayer == 1) MK_TR(k); \
    } while (0)

    bool x_remote = false;  // the residual of the next LayerNorm is in x2_in (else in xs)
    int kv_uses = 0;        // completed phases of kvbar
    for (int step = 0; step < p.steps; ++step) {
        const uint32_t e = epoch0 + (uint32_t)step + 1u;
        const int pos = pos0 + step;
        tstep = step;
        MK_TR(0);
        // ---- embed: x = deq(wte[tok]) + deq(wpe[pos]) (every CTA keeps its own copy) ----
        {
            const int8_t* qt = reinterpret_cast<const int8_t*>(p.wte.q) + (size_t)tok * p.wte.qstride;
            const __half* st = p.wte.s + (size_t)tok * p.wte.sstride;
            const int8_t* qp = reinterpret_cast<const int8_t*>(p.wpe.q) + (size_t)pos * p.wpe.qstride;
            const __half* sp = p.wpe.s + (size_t)pos * p.wpe.sstride;
            for (int c = tid; c < d; c += NCT)
                xs[c] = (float)__ldg(qt + c) * __half2float(__ldg(st + (c >> 5))) +
                        (float)__ldg(qp + c) * __half2float(__ldg(sp + (c >> 5)));
            if (tid == 0 && pos + 1 < p.n_ctx && step + 1 < p.steps) {  // next step's position row
                prefetch_l2(qp + p.wpe.qstride, (uint32_t)p.wpe.qstride);
                prefetch_l2(sp + p.wpe.sstride, (uint32_t)(p.wpe.sstride * 2));
            }
            x_remote = false;
        }
        MK_TR(1);
        for (int l = 0; l < L; ++l, ++gl) {
            tlayer = l;
            float* vb = vbuf + (gl & 1) * VL.total;
            wait_rx(&vbar[gl & 1], (uint32_t)((gl >> 1) & 1), p);  // this layer's vectors
            __syncthreads();  // x (local) is complete
            MK_TRL(29);
            float* kcache = p.kv + (size_t)slot * p.kv_slot + (size_t)l * p.kv_layer + (size_t)h * p.kv_head;
            float* vcache = kcache + p.kv_sel;
            // this CTA's block of attention positions; the cached ones (< pos) are staged by TMA
            const int T = pos + 1;
            const int per = (T + MK_CS - 1) / MK_CS;
            const int t0 = rank * per, t1 = min(T, t0 + per), t1c = min(pos, t1);
            const bool staged = per <= KV_STAGE && t1c > t0;
            const unsigned long long tA = (trace && tlayer == 1 && tstep == 0 && tid == 0) ? globaltimer() : 0;
            if (tid == 0) {
                if (staged) {
                    const uint32_t bytes = (uint32_t)((t1c - t0) * HD * 4);
                    tc::mbar_arrive_expect_tx(kvbar, 2 * bytes);
                    bulk_g2s(kst, kcache + (size_t)t0 * HD, bytes, kvbar);
                    bulk_g2s(kst + KV_STAGE * HD, vcache + (size_t)t0 * HD, bytes, kvbar);
                } else if (t1c > t0) {
                    prefetch_kv(p, slot, l, h, rank, pos);
                }
            }
            if (tA) trace[33] = globaltimer() - tA;
            {
                // next layer's vectors (the other buffer is free)
                const int nl = (l + 1 < L) ? l + 1 : 0;
                if (tid == 32 && (l + 1 < L || step + 1 < p.steps))
                    fetch_layer_vectors(p, lws[nl], h, rank, vbuf + ((gl + 1) & 1) * VL.total, &vbar[(gl + 1) & 1]);
            }
            MK_TRL(30);
            // ---- LN1 (residual from the previous layer's exchange, or the embedding) ----
            // (x2_in of the previous layer: its phase parity is that of layer gl - 1)
            if (x_remote) wait_rx(&rx[RX_X2], (uint32_t)((gl - 1) & 1), p);
            layernorm(x_remote ? x2_in : xs, x_remote ? xs : nullptr, ln, vb + VL.ln1g, vb + VL.ln1b, d, p.ln_eps,
                      red);
            if (x_remote && tid == 0 && gl < n_layers_total) tc::mbar_arrive_expect_tx(&rx[RX_X2], rx_bytes[RX_X2]);
            MK_TRL(2);
            const uint8_t* A = seg_wait();
            MK_TRL(3);
            // ---- q/k/v rows of head h (8 of each per CTA), sent to every CTA of the cluster ----
            {
                // warp w: segment rows 3w..3w+2 = (sel, dim) pairs of this CTA's 24 q/k/v rows
                const __half* As = reinterpret_cast<const __half*>(A + (size_t)24 * d);
                float out[3];
                dot_q8_rows<3, D>(A + (size_t)(3 * warp) * d, As + (size_t)(3 * warp) * (d / 32), ln, d, lane, out);
                if (lane < 3) {
                    float v = out[0];
                    if (lane == 1) v = out[1];
                    if (lane == 2) v = out[2];
                    const int r = 3 * warp + lane;                    // segment row = sel * 8 + dim % 8
                    const int sel = r >> 3, i = rank * 8 + (r & 7);  // q|k|v, dim within the head
                    v += vb[VL.bqkv + r];
                    qkv_out[r] = v;
                    if (sel > 0) (sel == 1 ? kcache : vcache)[(size_t)pos * HD + i] = v;
                }
                tc::fence_proxy_async_smem();
                __syncthreads();
                send_all(qkv_out, qkv_in + rank * 24, 24 * 4, RX_QKV);
            }
            MK_TRL(4);
            // ---- causal attention over this CTA's contiguous block of positions ----
            rx_wait(RX_QKV);
            MK_TRL(5);
            {
                // dim i of q/k/v of the step: qkv_in[(i / 8) * 24 + sel * 8 + i % 8]
                const int i0 = 2 * lane;
                const float* qrow = qkv_in + (i0 >> 3) * 24 + (i0 & 7);
                const float q0 = qrow[0], q1 = qrow[1];
                const float2 knew = make_float2(qrow[8], qrow[9]), vnew = make_float2(qrow[16], qrow[17]);
                if (staged) {
                    wait_rx(kvbar, (uint32_t)(kv_uses & 1), p);
                    ++kv_uses;
                }
                const float* kb_ = staged ? kst - (size_t)t0 * HD : kcache;  // row t at kb_ + t * 64
                const float* vb_ = staged ? kst + KV_STAGE * HD - (size_t)t0 * HD : vcache;
                float m = -INFINITY, lsum = 0.f, o0 = 0.f, o1 = 0.f;
                for (int ta = t0 + warp; ta < t1; ta += 2 * NWC) {
                    const int tb2 = ta + NWC;
                    float2 ka, va, kb = make_float2(0.f, 0.f), vb2 = make_float2(0.f, 0.f);
                    if (ta == pos) {
                        ka = knew;
                        va = vnew;
                    } else if (staged) {
                        ka = reinterpret_cast<const float2*>(kb_ + (size_t)ta * HD)[lane];
                        va = reinterpret_cast<const float2*>(vb_ + (size_t)ta * HD)[lane];
                    } else {
                        ka = __ldcg(reinterpret_cast<const float2*>(kcache + (size_t)ta * HD) + lane);
                        va = __ldcg(reinterpret_cast<const float2*>(vcache + (size_t)ta * HD) + lane);
                    }
                    const bool hb = tb2 < t1;
                    if (hb) {
                        if (tb2 == pos) {
                            kb = knew;
                            vb2 = vnew;
                        } else if (staged) {
                            kb = reinterpret_cast<const float2*>(kb_ + (size_t)tb2 * HD)[lane];
                            vb2 = reinterpret_cast<const float2*>(vb_ + (size_t)tb2 * HD)[lane];
                        } else {
                            kb = __ldcg(reinterpret_cast<const float2*>(kcache + (size_t)tb2 * HD) + lane);
                            vb2 = __ldcg(reinterpret_cast<const float2*>(vcache + (size_t)tb2 * HD) + lane);
                        }
                    }
                    const float sa = warp_sum(q0 * ka.x + q1 * ka.y) * p.attn_scale;
                    const float sb = warp_sum(q0 * kb.x + q1 * kb.y) * p.attn_scale;
                    softmax_update(sa, va.x, va.y, m, lsum, o0, o1);
                    if (hb) softmax_update(sb, vb2.x, vb2.y, m, lsum, o0, o1);
                }
                float* wr = wred + warp * APS;
                if (lane == 0) {
                    wr[0] = m;
                    wr[1] = lsum;
                }
                wr[2 + 2 * lane] = o0;
                wr[3 + 2 * lane] = o1;
                __syncthreads();
                rx_rearm(RX_QKV);
                if (tid < HD) {
                    float M = -INFINITY;
#pragma unroll
                    for (int w = 0; w < NWC; ++w) M = fmaxf(M, wred[w * APS]);
                    float Ls = 0.f, O = 0.f;
                    if (M != -INFINITY) {
#pragma unroll
                        for (int w = 0; w < NWC; ++w) {
                            const float f = expf(wred[w * APS] - M);
                            Ls += wred[w * APS + 1] * f;
                            O += wred[w * APS + 2 + tid] * f;
                        }
                    }
                    ap_out[2 + tid] = O;
                    if (tid == 0) {
                        ap_out[0] = M;
                        ap_out[1] = Ls;
                    }
                }
                tc::fence_proxy_async_smem();
                __syncthreads();
                send_all(ap_out, ap_in + rank * APP, APP * 4, RX_ATT);
            }
            MK_TRL(6);
            rx_wait(RX_ATT);
            if (tid < HD) {
                float M = -INFINITY;
#pragma unroll
                for (int r = 0; r < MK_CS; ++r) M = fmaxf(M, ap_in[r * APP]);
                float Ls = 0.f, O = 0.f;
#pragma unroll
                for (int r = 0; r < MK_CS; ++r) {
                    const float f = expf(ap_in[r * APP] - M);
                    Ls += ap_in[r * APP + 1] * f;
                    O += ap_in[r * APP + 2 + tid] * f;
                }
                atth[tid] = O / Ls;
            }
            __syncthreads();
            rx_rearm(RX_ATT);
            MK_TRL(7);
            // ---- attn c_proj, split-K by head: rows rank*dsl.. of W[:, h*64 : h*64+64] ----
            // 8 lanes per row (8 int8 each), 4 rows per warp pass
            unsigned long long* p1 = p.p1 + (size_t)l * H * d;
            {
                const uint8_t* Pq = A + (size_t)24 * d + (size_t)24 * (d / 32) * 2;
                const __half* Ps = reinterpret_cast<const __half*>(Pq + (size_t)dsl * HD);
                const int sub = lane & 7;
                const float4 x0 = *reinterpret_cast<const float4*>(atth + sub * 8);
                const float4 x1 = *reinterpret_cast<const float4*>(atth + sub * 8 + 4);
                constexpr int NP = 4;  // passes in flight
                for (int rb = warp * 4; rb < dsl; rb += NWC * 4 * NP) {
                    float a[NP];
                    uint2 w[NP];
#pragma unroll
                    for (int k = 0; k < NP; ++k) {
                        const int row = rb + k * NWC * 4 + (lane >> 3);
                        w[k] = row < dsl ? *reinterpret_cast<const uint2*>(Pq + (size_t)row * HD + sub * 8)
                                         : make_uint2(0u, 0u);
                    }
#pragma unroll
                    for (int k = 0; k < NP; ++k) {
                        const int row = rb + k * NWC * 4 + (lane >> 3);
                        float f[8];
                        i8x4_to_f32(w[k].x, f);
                        i8x4_to_f32(w[k].y, f + 4);
                        float t0a = f[0] * x0.x, t1a = f[4] * x1.x;
                        t0a = fmaf(f[1], x0.y, t0a);
                        t1a = fmaf(f[5], x1.y, t1a);
                        t0a = fmaf(f[2], x0.z, t0a);
                        t1a = fmaf(f[6], x1.z, t1a);
                        t0a = fmaf(f[3], x0.w, t0a);
                        t1a = fmaf(f[7], x1.w, t1a);
                        a[k] = row < dsl ? (t0a + t1a) * __half2float(Ps[row * 2 + (sub >> 2)]) : 0.f;
                    }
#pragma unroll
                    for (int k = 0; k < NP; ++k) {
                        a[k] += __shfl_xor_sync(0xffffffffu, a[k], 4);
                        a[k] += __shfl_xor_sync(0xffffffffu, a[k], 2);
                        a[k] += __shfl_xor_sync(0xffffffffu, a[k], 1);
                        const int row = rb + k * NWC * 4 + (lane >> 3);
                        if (sub == 0 && row < dsl) ll_store(p1 + (size_t)h * d + rank * dsl + row, a[k], e);
                    }
                }
            }
            __syncthreads();
            seg_release();
            MK_TRL(8);
            // ---- exchange 1: x' = x + sum over heads of the c_proj partials + bias ----
            if (tid < dsl) {
                const int col = rank * dsl + tid;
                uint32_t rounds = 0;
                const float sum = ll_sum(p1 + col, (size_t)d, H, e, p, &rounds);
                if (tlayer == 1) MK_TR(26);
                if (trace && tstep == 0 && tlayer == 1 && tid == 0) trace[27] = rounds;
                x_out[tid] = xs[col] + (sum + vb[VL.bproj + tid]);
            }
            tc::fence_proxy_async_smem();
            __syncthreads();
            send_all(x_out, x1_in + rank * dsl, (uint32_t)dsl * 4, RX_X1);
            MK_TRL(9);
            // ---- LN2 over x' + c_fc rows (32 per CTA) + GELU ----
            rx_wait(RX_X1);
            MK_TRL(10);
            layernorm(x1_in, xs, ln, vb + VL.ln2g, vb + VL.ln2b, d, p.ln_eps, red);
            rx_rearm(RX_X1);
            MK_TRL(11);
            const uint8_t* B = seg_wait();
            MK_TRL(12);
            {
                const __half* Bs = reinterpret_cast<const __half*>(B + (size_t)32 * d);
                float out[4];
                dot_q8_rows<4, D>(B + (size_t)(4 * warp) * d, Bs + (size_t)(4 * warp) * (d / 32), ln, d, lane, out);
                if (lane < 4) {
                    float v = out[0];
#pragma unroll
                    for (int u = 1; u < 4; ++u)
                        if (lane == u) v = out[u];
                    fs[4 * warp + lane] = gelu_tanh(v + vb[VL.bfc + 4 * warp + lane]);
                }
            }
            __syncthreads();
            seg_release();
            MK_TRL(13);
            // ---- mlp c_proj partial over this CTA's 32 c_fc outputs ----
            // 4 lanes per row (8 int8 each), 8 rows per warp pass
            const uint8_t* Cg = seg_wait();
            MK_TRL(14);
            {
                const __half* Cs = reinterpret_cast<const __half*>(Cg + (size_t)32 * d);
                const int sub = lane & 3;
                const float4 x0 = *reinterpret_cast<const float4*>(fs + sub * 8);
                const float4 x1 = *reinterpret_cast<const float4*>(fs + sub * 8 + 4);
                constexpr int NP = 4;  // passes in flight
#pragma unroll 1
                for (int rb = warp * 8; rb < d; rb += NWC * 8 * NP) {
                    uint2 w[NP];
#pragma unroll
                    for (int k = 0; k < NP; ++k) {
                        const int row = rb + k * NWC * 8 + (lane >> 2);
                        w[k] = row < d ? *reinterpret_cast<const uint2*>(Cg + (size_t)row * 32 + sub * 8)
                                       : make_uint2(0u, 0u);
                    }
#pragma unroll
                    for (int k = 0; k < NP; ++k) {
                        float f[8];
                        i8x4_to_f32(w[k].x, f);
                        i8x4_to_f32(w[k].y, f + 4);
                        float t0a = f[0] * x0.x, t1a = f[4] * x1.x;
                        t0a = fmaf(f[1], x0.y, t0a);
                        t1a = fmaf(f[5], x1.y, t1a);
                        t0a = fmaf(f[2], x0.z, t0a);
                        t1a = fmaf(f[6], x1.z, t1a);
                        t0a = fmaf(f[3], x0.w, t0a);
                        t1a = fmaf(f[7], x1.w, t1a);
                        float a = t0a + t1a;
                        a += __shfl_xor_sync(0xffffffffu, a, 2);
                        a += __shfl_xor_sync(0xffffffffu, a, 1);
                        const int row = rb + k * NWC * 8 + (lane >> 2);
                        if (sub == 0 && row < d) mpart[row] = a * __half2float(Cs[row]);
                    }
                }
            }
            MK_TRL(18);
            tc::fence_proxy_async_smem();
            MK_TRL(25);
            __syncthreads();
            MK_TRL(31);
            seg_release();
            // slice j of the partial goes to rank j
            if (warp == 0 && lane < MK_CS)
                send_to((uint32_t)lane, mpart + lane * dsl, mp_in + rank * dsl, (uint32_t)dsl * 4, &rx[RX_MP]);
            MK_TRL(15);
            // ---- cluster sum of the partials of my rows (fixed rank order) -> LL words ----
            unsigned long long* p2 = p.p2 + (size_t)l * H * d;
            rx_wait(RX_MP);
            if (tid < dsl) {
                const int row = rank * dsl + tid;
                float v = 0.f;
#pragma unroll
                for (int r = 0; r < MK_CS; ++r) v += mp_in[r * dsl + tid];
                if (tlayer == 1) MK_TR(16);
                ll_store(p2 + (size_t)h * d + row, v, e);
                // ---- exchange 2: x'' = x' + sum over clusters + bias ----
                uint32_t rounds = 0;
                const float sum = ll_sum(p2 + row, (size_t)d, H, e, p, &rounds);
                if (trace && tstep == 0 && tlayer == 1 && tid == 0) trace[28] = rounds;
                x_out[tid] = xs[row] + (sum + vb[VL.bmproj + tid]);
            }
            tc::fence_proxy_async_smem();
            __syncthreads();
            rx_rearm(RX_MP);
            send_all(x_out, x2_in + rank * dsl, (uint32_t)dsl * 4, RX_X2);
            x_remote = true;
            MK_TRL(17);
            if (l == 0) MK_TR(19);
            if (l == L / 2) MK_TR(20);
        }
        MK_TR(21);
        // ---- ln_f, tied lm head over this CTA's vocabulary rows, argmax ----
        wait_rx(&rx[RX_X2], (uint32_t)((gl - 1) & 1), p);
        layernorm(x2_in, xs, ln, lnf, lnf + d, d, p.ln_eps, red);
        if (tid == 0 && gl < n_layers_total) tc::mbar_arrive_expect_tx(&rx[RX_X2], rx_bytes[RX_X2]);
        x_remote = false;
        const bool want_logits = p.logits != nullptr && step == p.steps - 1;
        unsigned long long best = 0ull;
        unsigned long long t_wait = 0, t_rel = 0, t_dot0 = 0, t_last = trace ? globaltimer() : 0;
        if (p.adapter) {
            // post-ln_f plastic adapter (cu/gpt2.cu:196-215), every CTA on its own copy of the
            // row: ah[j] = sum_i A[j][i] h[i], then h[i] += sum_j B[i][j] ah[j], both sequential
            // fused multiply-adds in the order of k_adapter_apply (wred is free here)
            const AdapterDesc ad = *reinterpret_cast<const AdapterDesc*>(p.adapter);
            if (ad.r > 0) {
                float* ah = wred;
                for (int j = tid; j < ad.r; j += NCT) {
                    const float* ar = ad.a + (size_t)j * d;
                    float s = 0.f;
#pragma unroll 16
                    for (int i = 0; i < d; ++i) s = fmaf(__ldg(ar + i), ln[i], s);
                    ah[j] = s;
                }
                __syncthreads();
                for (int i = tid; i < d; i += NCT) {
                    const float* br = ad.b + (size_t)i * ad.r;
                    float s = 0.f;
#pragma unroll 8
                    for (int j = 0; j < ad.r; ++j) s = fmaf(__ldg(br + j), ah[j], s);
                    ln[i] = ln[i] + s;
                }
                __syncthreads();
            }
        }
        // fragments of the ln_f output (B operands) for this warp's groups, kept in registers for
        // the whole head; mpart is free once the last layer's x'' arrived
        const int gsn = d >> 5;
        float fk[4];
        uint32_t hb0[4], hb1[4];
        vec_fragments(ln, d, reinterpret_cast<int8_t*>(mpart), warp, lane, fk, hb0, hb1);
        // per-warp row sums, double-buffered (2 x [8 warps][32 rows] in wred): one barrier per
        // segment, after which the segment is released while warp 0 reduces its rows
        for (int k = 0; k < nseg_head; ++k) {
            const uint8_t* S = seg_wait();
            if (trace && tid == 0) {
                const unsigned long long now = globaltimer();
                t_wait += now - t_last;
                t_last = now;
                if (k == 0) t_dot0 = now;
            }
            float* hred = wred + (k & 1) * (NWC * 32);
            rows32_mma(S, reinterpret_cast<const __half*>(S + (size_t)32 * d), gsn, fk, hb0, hb1, warp, lane, hred);
            __syncthreads();
            const unsigned long long tR = (trace && tid == 0) ? globaltimer() : 0;
            seg_release();
            if (trace && tid == 0) {
                t_last = globaltimer();
                t_rel += t_last - tR;
                if (k == 0) trace[35] = tR - t_dot0;
            }
            if (tid < 32 && k * 32 + tid < rows_head) {  // rows past the end are zero padding
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < NWC; ++w) v += hred[w * 32 + tid];
                const int row = row0_head + k * 32 + tid;
                const unsigned long long key = argmax_pack(v, row);
                best = key > best ? key : best;
                if (want_logits) p.logits[row] = v;
            }
        }
        best = warp_max_u64(best);
        MK_TR(22);
        if (trace && tstep == 0 && tid == 0) {
            trace[24] = t_wait;
            trace[32] = t_rel;
        }
        if (lane == 0) bw[warp] = best;
        __syncthreads();
        const uint32_t ep16 = (e % 65535u) + 1u;
        if (tid == 0) {
            unsigned long long b = 0ull;
            for (int w = 0; w < NWC; ++w) b = bw[w] > b ? bw[w] : b;
            // (key, index, epoch16): unsigned max of the words orders by key then index
            const unsigned long long word = (b & 0xFFFFFFFF00000000ull) | ((b & 0xFFFFull) << 16) | ep16;
            ll_store_raw(p.best + (size_t)g * BEST_STRIDE, word);
        }
        // ---- exchange 3: every CTA takes the global argmax ----
        unsigned long long mine = 0ull;
        if (tid < G) {
            bool ok = false;
            for (uint32_t it = 0; it < SPIN; ++it) {
                const unsigned long long w = ll_load(p.best + (size_t)tid * BEST_STRIDE);
                if ((uint32_t)(w & 0xFFFFull) == ep16) {
                    mine = w;
                    ok = true;
                    break;
                }
                __nanosleep(32);
                if ((it & 63u) == 63u && aborted(p)) break;
            }
            if (!ok && !aborted(p)) raise_error(p, 3);
        }
        mine = warp_max_u64(mine);
        __syncthreads();
        if (lane == 0) bw[warp] = mine;
        __syncthreads();
        unsigned long long top = 0ull;
#pragma unroll
        for (int w = 0; w < NWC; ++w) top = bw[w] > top ? bw[w] : top;
        const uint32_t next = (uint32_t)((top >> 16) & 0xFFFFull);
        MK_TR(23);
        if (g == 0 && tid == 0) {
            p.genlog[pos] = next;
            if (step == p.steps - 1) {
                *p.next = next;
                *p.tok = next;
                *p.pos = pos + 1;
            }
        }
        tok = next;
        // once per step: this step's K/V rows (plain stores) are released to the cluster, and
        // ordered before the bulk copies that stage them in later steps
        tc::cluster_sync();
        if (tid == 0) asm volatile("fence.proxy.async.global;" ::: "memory");
    }
    if (g == 0 && tid == 0) *p.epoch = epoch0 + (uint32_t)p.steps;
#undef MK_TRL
#undef MK_TR
    // every bulk copy issued has been consumed unless the launch aborted; wait for stragglers
    if (tid == 0)
        for (int i = max(0, total - NSLOT); i < total; ++i) drain_wait(&full[i % NSLOT], (uint32_t)((i / NSLOT) & 1), p);
    tc::cluster_sync();  // no CTA leaves while a peer may still touch its shared memory
}

// ------------------------------------------------------------------ stream packing
struct GatherOp {
    const uint8_t* src;
    uint8_t* dst;
    size_t src_stride;
    int rows, bytes;
};

__global__ void k_gather_rows(const GatherOp* __restrict__ ops) {
    const GatherOp o = ops[blockIdx.x];
    const size_t total = (size_t)o.rows * o.bytes;
    for (size_t i = threadIdx.x; i < total; i += blockDim.x) {
        const size_t r = i / o.bytes, c = i % o.bytes;
        o.dst[i] = o.src[r * o.src_stride + c];
    }
}

// A block of R = 16 MT rows x K int8 columns in mma fragment order: 32-bit word w holds rows
// (mt * 16 + g, + 8 for odd registers) and columns 32 ks + 4 t (+ 16 for registers 2, 3) of source
// rows 0 .. n - 1 (zero past n), with block = w / 128 = ks * MT + mt, lane = (w % 128) / 4 =
// 4 g + t and register w % 4: a lane's four A registers are 16 contiguous bytes.
struct FragPackOp {
    const uint8_t* src;
    size_t src_stride;
    uint8_t* dst;
    int n, MT, K;
};

__global__ void k_pack_frag(const FragPackOp* __restrict__ ops) {
    const FragPackOp o = ops[blockIdx.x];
    const int words = 16 * o.MT * o.K / 4;
    for (int w = threadIdx.x; w < words; w += blockDim.x) {
        const int blk = w >> 7, lanew = (w >> 2) & 31, reg = w & 3;
        const int ks = blk / o.MT, mt = blk - ks * o.MT, gq = lanew >> 2, t = lanew & 3;
        const int row = mt * 16 + gq + ((reg & 1) ? 8 : 0);
        const int col = 32 * ks + ((reg & 2) ? 16 : 0) + 4 * t;
        uint32_t v = 0u;
        if (row < o.n) v = *reinterpret_cast<const uint32_t*>(o.src + (size_t)row * o.src_stride + col);
        reinterpret_cast<uint32_t*>(o.dst)[w] = v;
    }
}

size_t smem_bytes(int d, int seg, int n_layer) {
    const VecLayout V(d);
    const int dsl = d / MK_CS;
    const size_t floats = (size_t)4 * d + 2 * V.total + MK_CS * 24 + MK_CS * APP + 3 * d + 32 + APP + dsl + d +
                          NWC * APS + HD + 32 + 16 + 2 * KV_STAGE * HD;
    return (size_t)NSLOT * seg + 128 + floats * 4 + 3 * 8 + 8 * 8 + sizeof(MkLayer) * n_layer;
}

}  // namespace

cudaError_t mk_setup(MkPlan& plan, const MkWeights& w, int d, int L, int H, int V, int n_ctx, int device,
                     cudaStream_t st) {
    (void)n_ctx;
    plan = MkPlan{};
    auto no = [&](const std::string& why) {
        plan.why = why;
        return cudaSuccess;
    };
    if (std::getenv("GPT2Q_NO_PERSISTENT")) return no("disabled by GPT2Q_NO_PERSISTENT");
    if (H <= 0 || d != HD * H) return no("head dim is not 64");
    if (d % 128 != 0) return no("n_embd is not a multiple of 128");
    if (d / MK_CS > NCT || d > 4 * NCT) return no("n_embd too large");
    if (H > 16) return no("more than 16 heads");
    if (V > 65536 || V <= 0) return no("vocab above 65536");
    if ((int)w.attn.size() != L || (int)w.layers.size() != L) return no("layer count mismatch");
    auto q8 = [](const QW& q, int rows, int cols) { return q.atom == ATOM_Q8 && q.rows == rows && q.cols == cols; };
    if (!q8(w.wte, V, d) || w.wpe.atom != ATOM_Q8 || w.wpe.cols != d) return no("embeddings are not int8");
    for (int l = 0; l < L; ++l)
        if (!q8(w.attn[l], 3 * d, d) || !q8(w.proj[l], d, d) || !q8(w.fc[l], 4 * d, d) || !q8(w.mproj[l], d, 4 * d))
            return no("a layer weight is not int8 or not the full (unsliced) shape");
    const int seg = 34 * d;
    const size_t smem = smem_bytes(d, seg, L);
    int dev_smem = 0;
    cudaError_t e = cudaDeviceGetAttribute(&dev_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    if (e != cudaSuccess) return e;
    if (smem > (size_t)dev_smem) return no("shared memory");
    e = cudaFuncSetAttribute(k_decode_persistent<768>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_decode_persistent<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const int G = MK_CS * H;
    {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(G);
        cfg.blockDim = dim3(THREADS);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = MK_CS;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int ncl = 0;
        e = cudaOccupancyMaxActiveClusters(&ncl, d == 768 ? k_decode_persistent<768> : k_decode_persistent<0>, &cfg);
        if (e != cudaSuccess) return e;
        if (ncl < H) return no("only " + std::to_string(ncl) + " clusters of 8 can be co-resident");
    }
    const int RH = (V + G - 1) / G;
    const int nseg_head_max = (RH + 31) / 32;
    const size_t cta_bytes = (size_t)(3 * L + nseg_head_max) * seg;

    // ---- gather plan: every CTA's segments, in consumption order ----
    uint8_t* stream = nullptr;
    e = cudaMalloc(&stream, cta_bytes * G);
    if (e != cudaSuccess) return e;
    e = cudaMemsetAsync(stream, 0, cta_bytes * G, st);
    std::vector<GatherOp> ops;
    std::vector<FragPackOp> hops;  // lm head segments, in mma fragment order
    auto add = [&](const void* src, size_t stride, uint8_t* dst, int rows, int bytes) {
        if (rows > 0 && bytes > 0) ops.push_back({reinterpret_cast<const uint8_t*>(src), dst, stride, rows, bytes});
    };
    const int gs = d / 32;  // scale groups per row of a d-wide weight
    for (int g = 0; g < G; ++g) {
        const int h = g / MK_CS, j = g % MK_CS;
        uint8_t* base = stream + (size_t)g * cta_bytes;
        for (int l = 0; l < L; ++l) {
            const QW &Wa = w.attn[l], &Wp = w.proj[l], &Wf = w.fc[l], &Wm = w.mproj[l];
            uint8_t* A = base + (size_t)(3 * l) * seg;
            for (int sel = 0; sel < 3; ++sel) {
                const int r0 = sel * d + h * HD + j * 8;
                add(Wa.q + (size_t)r0 * Wa.qstride, Wa.qstride, A + (size_t)sel * 8 * d, 8, d);
                add(reinterpret_cast<const uint8_t*>(Wa.s) + (size_t)r0 * Wa.sstride * 2, (size_t)Wa.sstride * 2,
                    A + (size_t)24 * d + (size_t)sel * 8 * gs * 2, 8, gs * 2);
            }
            const int dsl = d / MK_CS;
            uint8_t* P = A + (size_t)24 * d + (size_t)24 * gs * 2;
            add(Wp.q + (size_t)(j * dsl) * Wp.qstride + h * HD, Wp.qstride, P, dsl, HD);
            add(reinterpret_cast<const uint8_t*>(Wp.s) + (size_t)(j * dsl) * Wp.sstride * 2 + (size_t)h * 2 * 2,
                (size_t)Wp.sstride * 2, P + (size_t)dsl * HD, dsl, 4);
            uint8_t* B = base + (size_t)(3 * l + 1) * seg;
            const int f0 = (h * MK_CS + j) * 32;
            add(Wf.q + (size_t)f0 * Wf.qstride, Wf.qstride, B, 32, d);
            add(reinterpret_cast<const uint8_t*>(Wf.s) + (size_t)f0 * Wf.sstride * 2, (size_t)Wf.sstride * 2,
                B + (size_t)32 * d, 32, gs * 2);
            uint8_t* Cg = base + (size_t)(3 * l + 2) * seg;
            add(Wm.q + f0, Wm.qstride, Cg, d, 32);
            add(reinterpret_cast<const uint8_t*>(Wm.s) + (size_t)(f0 / 32) * 2, (size_t)Wm.sstride * 2,
                Cg + (size_t)32 * d, d, 2);
        }
        const int row0 = g * RH;
        const int rows = std::max(0, std::min(V, row0 + RH) - row0);
        for (int k = 0; k * 32 < rows; ++k) {
            uint8_t* S = base + (size_t)(3 * L + k) * seg;
            const int r0 = row0 + k * 32, n = std::min(32, rows - k * 32);
            hops.push_back({w.wte.q + (size_t)r0 * w.wte.qstride, w.wte.qstride, S, n, 2, d});
            add(reinterpret_cast<const uint8_t*>(w.wte.s) + (size_t)r0 * w.wte.sstride * 2,
                (size_t)w.wte.sstride * 2, S + (size_t)32 * d, n, gs * 2);
        }
    }
    GatherOp* dops = nullptr;
    if (e == cudaSuccess) e = cudaMalloc(&dops, ops.size() * sizeof(GatherOp));
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(dops, ops.data(), ops.size() * sizeof(GatherOp), cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) {
        k_gather_rows<<<(unsigned)ops.size(), 256, 0, st>>>(dops);
        e = cudaGetLastError();
    }
    FragPackOp* dh = nullptr;
    if (e == cudaSuccess && !hops.empty()) e = cudaMalloc(&dh, hops.size() * sizeof(FragPackOp));
    if (e == cudaSuccess && dh)
        e = cudaMemcpyAsync(dh, hops.data(), hops.size() * sizeof(FragPackOp), cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess && dh) {
        k_pack_frag<<<(unsigned)hops.size(), 256, 0, st>>>(dh);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (dops) cudaFree(dops);
    if (dh) cudaFree(dh);
    plan.stream = stream;
    if (e != cudaSuccess) {
        mk_destroy(plan);
        return e;
    }
    // ---- per-layer vectors, exchange words, error words ----
    auto alloc = [&](void** ptr, size_t bytes) {
        if (e == cudaSuccess) e = cudaMalloc(ptr, bytes);
        if (e == cudaSuccess) e = cudaMemsetAsync(*ptr, 0, bytes, st);
    };
    alloc(reinterpret_cast<void**>(&plan.layers), sizeof(MkLayer) * L);
    alloc(reinterpret_cast<void**>(&plan.p1), (size_t)L * H * d * 8);
    alloc(reinterpret_cast<void**>(&plan.p2), (size_t)L * H * d * 8);
    alloc(reinterpret_cast<void**>(&plan.best), (size_t)G * BEST_STRIDE * 8);
    alloc(reinterpret_cast<void**>(&plan.epoch), 16);
    alloc(reinterpret_cast<void**>(&plan.err), 16);
    if (std::getenv("GPT2Q_MK_TRACE")) alloc(reinterpret_cast<void**>(&plan.trace), (size_t)G * MK_TRACE * 8);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(plan.layers, w.layers.data(), sizeof(MkLayer) * L, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        mk_destroy(plan);
        return e;
    }
    plan.clusters = H;
    plan.seg_bytes = seg;
    plan.cta_bytes = cta_bytes;
    plan.head_rows = RH;
    plan.smem = smem;
    plan.enabled = true;
    return cudaSuccess;
}

void mk_destroy(MkPlan& plan) {
    void* ptrs[] = {plan.stream, plan.layers, plan.p1, plan.p2, plan.best, plan.epoch, plan.err, plan.trace};
    for (void* q : ptrs)
        if (q) cudaFree(q);
    plan = MkPlan{};
}

cudaError_t launch_decode_persistent(const MkPlan& plan, const MkParams& p, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(MK_CS * plan.clusters);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = plan.smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = MK_CS;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    if (p.d == 768) return cudaLaunchKernelEx(&cfg, k_decode_persistent<768>, p);
    return cudaLaunchKernelEx(&cfg, k_decode_persistent<0>, p);
}

int mk_take_error(const MkPlan& plan, cudaStream_t st) {
    if (!plan.err) return 0;
    int h[2] = {0, 0};
    if (cudaMemcpyAsync(h, plan.err, 8, cudaMemcpyDeviceToHost, st) != cudaSuccess) return -1;
    if (cudaStreamSynchronize(st) != cudaSuccess) return -1;
    if (h[0] || h[1]) {
        if (cudaMemsetAsync(plan.err, 0, 8, st) != cudaSuccess) return -1;
        if (cudaStreamSynchronize(st) != cudaSuccess) return -1;
        return h[0] ? h[0] : 5;
    }
    return 0;
}

}  // namespace gpt2q
