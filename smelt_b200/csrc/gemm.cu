// Tensor-core dequant-fused linear for sm_100a (tcgen05 + TMEM + TMA).
//
//   out[m][n] = epilogue( sum_k X[m][k] * deq(W)[n][k] )
//
// Precision: each 16-wide k-step issues three MMAs, A_hi*B_hi + A_hi*B_lo + A_lo*B_hi,
// where x = x_hi + x_lo and w' = w * 2^P = w_hi + w_lo are fp16 pairs. w' = q * f16(scale)
// * 2^P is exact in fp32 and the pair is exact for it (the power-of-two prescale keeps
// w_lo a normal fp16), x keeps ~22 bits, and the dropped lo*lo term is ~2^-22 relative:
// fp32-class results from the fp16 tensor pipe with fp32 TMEM accumulation.
//
// The MMA is "swap-AB": weight rows are the MMA M dimension (128 TMEM lanes) and tokens
// are N (BN columns), so a decode batch of 32 still fills M, and the epilogue's stores
// along n are coalesced.
//
// Two weight sources (template PRESPLIT):
//  - decode (false): int8 / int4 tiles stream from HBM and are dequantised in the CTA.
//      warp 0     TMA producer of raw weight tiles [128 rows x 64 k] (64- or 32-byte swizzle)
//      warps 1-4  one weight row each: q -> w' -> (hi, lo), written into 128-byte-swizzled
//                 K-major operand tiles; afterwards the epilogue
//  - prefill (true): one-time exact fp16 hi/lo copies of the weight are TMA-loaded
//      directly (compute-bound regime; no per-CTA conversion).
//   warp 5   one thread issues tcgen05.mma kind::f16 into the fp32 TMEM accumulator
//   warp 6   TMA producer of the activation tiles X_hi / X_lo
//
// Split-K (few row tiles, small batch): the splits of one output tile form a thread-block
// cluster; each CTA parks its partial tile in shared memory and CTA r reduces columns
// r, r+S, ... by reading all S partials over distributed shared memory in fixed order
// (deterministic, no global round trip).
//
// Programmatic dependent launch: weight loads and their conversion start before the
// previous kernel has finished; activations are only touched after griddepcontrol.wait.
// All mbarrier waits are bounded (tcgen05.cuh); a timeout sets the error word.
#include <atomic>
#include <cuda.h>
#include <cuda_fp16.h>

#include <cmath>
#include <cstdio>
#include <string>
#include <cstdlib>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "gemm.h"
#include "kernels.h"
#include "tcgen05.cuh"

namespace gpt2q {

namespace {

constexpr int BM = 128, BK = 64, THREADS = 224;
constexpr int MAX_SPLITS = 16;      // decode tiles (pushed exchange): non-portable clusters up to 16
constexpr int MAX_SPLITS_PULL = 8;  // wider tiles (pulled exchange): portable cluster size

// Token columns per reducing CTA in the split-K exchange (a multiple of 4).
__host__ __device__ constexpr int push_cw(int bn, int splits) { return ((bn + splits - 1) / splits + 3) & ~3; }

template <int BN, bool PRESPLIT, bool DEEP>
struct Cfg {
    // DEEP (decode tiles, small grids): one CTA per SM that, launched early under
    // programmatic dependent launch, streams and dequantises as much of its split-K slice as
    // shared memory holds while it waits for its activations, so mostly MMAs remain once X
    // arrives. Otherwise two CTAs share an SM (BN <= 64) and the rings are short.
    static constexpr int OS = DEEP ? (BN == 32 ? 5 : 4) : 2;  // weight operand (fp16 hi/lo) stages
    // activation (X hi/lo) stages, a ring of their own: a CTA requests several X k-blocks at
    // once when its inputs become ready, instead of one L2 round trip per k-block
    static constexpr int XS = DEEP ? 4 : 2;
    static constexpr int RAW_STAGES = DEEP ? 3 : (BN == 128 ? 4 : 2);  // raw int8/int4 tiles in flight
    // BN <= 64: X_hi and X_lo tiles are adjacent, so one MMA with N = 2 BN multiplies a weight
    // half by both; A_hi and A_lo each accumulate into their own TMEM block of 2 BN columns.
    static constexpr bool DUAL = BN <= 64;
    static constexpr int TMEM_COLS = DUAL ? 4 * BN : BN;
    // Decode tiles exchange split-K partials by pushing them (16-byte remote stores into the
    // peers' shared memory); rank r receives the block of CW token columns it reduces into an
    // area of [splits][128][CW] fp32 (splits * CW <= BN + 32) over the free operand rings.
    static constexpr bool PUSH = BN <= 64;
    static constexpr int XCH_FLOATS = 128 * (BN + 32);
    static constexpr int A_BYTES = BM * 128;                          // one of hi/lo
    static constexpr int B_BYTES = BN * 128;                          // one of hi/lo
    static constexpr int RAW_BYTES = PRESPLIT ? 0 : BM * 64;          // int8 tile (int4 uses half)
    static constexpr int OFF_A = 0;
    static constexpr int OFF_B = OFF_A + OS * 2 * A_BYTES;
    static constexpr int OFF_RAW = OFF_B + XS * 2 * B_BYTES;
    // decode: the CTA's group scales, one padded row per weight row (conflict-free)
    static constexpr int SC_KB = 8;                  // k-blocks of scales staged at a time
    static constexpr int SC_STRIDE = 2 * SC_KB + 1;  // floats per row
    static constexpr int OFF_SC = OFF_RAW + RAW_STAGES * RAW_BYTES;
    static constexpr int SC_BYTES = PRESPLIT ? 0 : BM * SC_STRIDE * 4;
    static constexpr int OFF_BAR = OFF_SC + SC_BYTES;
    static constexpr int N_BAR = 2 * RAW_STAGES + 2 * OS + 2 * XS + 2;
    static constexpr int SMEM = OFF_BAR + N_BAR * 8 + 16 + 1024;  // + tmem slot, flag, alignment slack
    static_assert(SMEM <= 232448, "shared memory per CTA");
    // shallow decode tiles that fit twice in an SM's shared memory share it
    static constexpr int MIN_BLOCKS = (!DEEP && BN <= 64 && SMEM <= 232448 / 2 - 1024) ? 2 : 1;
    static_assert(!PUSH || XCH_FLOATS * 4 <= OFF_RAW, "exchange area must fit in the operand rings");
};

struct TcParams {
    QW w;
    int M, nkb_total, kb_per_split, splits;
    float post;  // 2^-P
    float pre;   // 2^P
    Epi epi;
    int* err;
    int* fault;                 // one-shot split-K stall switch (GemmPlan::fault)
    float4* part;               // split-K partials of the wide tiles (GemmPlan::part)
    int products;               // wide tiles: 1 = W_hi X_hi, 2 = + W_lo X_hi, 3 = + W_hi X_lo
    unsigned long long* trace;  // optional [grid][TC_TRACE] globaltimer stamps (one traced launch)
};

constexpr int TC_TRACE = 16;

__device__ __forceinline__ void tc_stamp(const TcParams& p, int k) {
    if (p.trace) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        const size_t cta = blockIdx.x + (size_t)gridDim.x * (blockIdx.y + (size_t)gridDim.y * blockIdx.z);
        p.trace[cta * TC_TRACE + k] = t;
    }
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, const uint4& v) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}

// ---- exact fp16 dequantisation (two values per instruction) ----
// int8 pair -> half2 exactly: bytes biased by +128 go into the mantissa of 1024 (0x64xx),
// then 1152 is subtracted. int4 nibbles are biased by +8 and 1032 is subtracted.
__device__ __forceinline__ __half2 bytes_to_h2(uint32_t biased, uint32_t sel) {
    const uint32_t v = __byte_perm(biased, 0x64646464u, sel);
    return *reinterpret_cast<const __half2*>(&v);
}

// q (exact fp16 integers) times the prescaled group scale s2 = f16(scale) * 2^P:
// hi = f16(q*s), lo = fma(q, s, -hi) — the residual of the 18-bit product has at most 8
// significant bits, so the fp16 FMA returns it exactly and hi + lo == q*s.
__device__ __forceinline__ void qs_hi_lo(__half2 q, __half2 s2, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __hmul2(q, s2);
    const __half2 l = __hfma2(q, s2, __hneg2(h));
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

// 16 int8 weights (one uint4) of row r, k-chunk c (elements 16c..16c+15), into the
// swizzled hi/lo A tiles (output chunks 2c, 2c+1).
__device__ __forceinline__ void put16_q8(uint32_t a_hi, uint32_t a_lo, int r, int c, const uint4& v, __half2 s2) {
    const __half2 off = __float2half2_rn(1152.0f);
    const uint32_t w[4] = {v.x ^ 0x80808080u, v.y ^ 0x80808080u, v.z ^ 0x80808080u, v.w ^ 0x80808080u};
    uint4 hi[2], lo[2];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half2 q01 = __hsub2(bytes_to_h2(w[i], 0x5140u), off);
        const __half2 q23 = __hsub2(bytes_to_h2(w[i], 0x5342u), off);
        uint32_t* ph = &hi[i >> 1].x + (i & 1) * 2;
        uint32_t* pl = &lo[i >> 1].x + (i & 1) * 2;
        qs_hi_lo(q01, s2, ph[0], pl[0]);
        qs_hi_lo(q23, s2, ph[1], pl[1]);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const uint32_t o = (uint32_t)r * 128u + (uint32_t)(((2 * c + j) ^ (r & 7)) * 16);
        st_shared_v4(a_hi + o, hi[j]);
        st_shared_v4(a_lo + o, lo[j]);
    }
}

// One 32-group of int4 weights (16 packed bytes: byte j = elem j | elem j+16 << 4) of row r,
// k-group c (elements 32c..32c+31) -> output chunks 4c..4c+3.
__device__ __forceinline__ void put32_q4(uint32_t a_hi, uint32_t a_lo, int r, int c, const uint4& v, __half2 s2) {
    const __half2 off = __float2half2_rn(1032.0f);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint4 hi[4], lo[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {  // word i: bytes 4i..4i+3 -> elements 4i.. (low) and 16+4i.. (high)
        const uint32_t ul = (w[i] & 0x0F0F0F0Fu) ^ 0x08080808u;
        const uint32_t uh = ((w[i] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
        uint32_t* phl = &hi[i >> 1].x + (i & 1) * 2;
        uint32_t* pll = &lo[i >> 1].x + (i & 1) * 2;
        uint32_t* phh = &hi[2 + (i >> 1)].x + (i & 1) * 2;
        uint32_t* plh = &lo[2 + (i >> 1)].x + (i & 1) * 2;
        qs_hi_lo(__hsub2(bytes_to_h2(ul, 0x5140u), off), s2, phl[0], pll[0]);
        qs_hi_lo(__hsub2(bytes_to_h2(ul, 0x5342u), off), s2, phl[1], pll[1]);
        qs_hi_lo(__hsub2(bytes_to_h2(uh, 0x5140u), off), s2, phh[0], plh[0]);
        qs_hi_lo(__hsub2(bytes_to_h2(uh, 0x5342u), off), s2, phh[1], plh[1]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t o = (uint32_t)r * 128u + (uint32_t)(((4 * c + j) ^ (r & 7)) * 16);
        st_shared_v4(a_hi + o, hi[j]);
        st_shared_v4(a_lo + o, lo[j]);
    }
}

// Epilogue of output row nn for NJ tokens m_j = mbase + j * mstep (written where m_j < mend).
// Every lane of the warp calls it (the KV-cache token offsets travel by shuffle). All global
// loads of the chunk are issued before its first store, per-row terms are computed once, and
// the operation order per element is that of epi_apply.
template <int NJ>
__device__ __forceinline__ void epi_chunk(const Epi& e, int nn, bool row_ok, const float (&acc)[NJ], int mbase,
                                          int mstep, int mend, float post, const float* resid_pre = nullptr,
                                          const float* bias_pre = nullptr) {
    const int lane = threadIdx.x & 31;
    const bool has_b = e.bias != nullptr;
    const float b = bias_pre ? *bias_pre : ((has_b && row_ok) ? __ldg(e.bias + nn) : 0.f);
    bool ok[NJ];
#pragma unroll
    for (int j = 0; j < NJ; ++j) ok[j] = row_ok && (mbase + j * mstep < mend);
    switch (e.kind) {
        case EPI_STORE: {
#pragma unroll
            for (int j = 0; j < NJ; ++j) {
                float v = acc[j] * post;
                if (has_b) v += b;
                if (ok[j]) e.out[(size_t)(mbase + j * mstep) * e.ldo + nn] = v;
            }
            break;
        }
        case EPI_RESID: {
            float r[NJ];
#pragma unroll
            for (int j = 0; j < NJ; ++j)
                r[j] = resid_pre ? resid_pre[j] : (ok[j] ? e.out[(size_t)(mbase + j * mstep) * e.ldo + nn] : 0.f);
#pragma unroll
            for (int j = 0; j < NJ; ++j)
                if (ok[j]) e.out[(size_t)(mbase + j * mstep) * e.ldo + nn] = r[j] + (acc[j] * post + b);
            break;
        }
        case EPI_GELU: {
#pragma unroll
            for (int j = 0; j < NJ; ++j) {
                float v = acc[j] * post;
                if (has_b) v += b;
                const float gv = gelu_tanh(v);
                const size_t o = (size_t)(mbase + j * mstep) * e.ldo + nn;
                if (ok[j]) {
                    if (e.out) e.out[o] = gv;  // null: the consumer reads only the hi/lo pair
                    if (e.out_hi) {
                        const __half h = __float2half_rn(gv);
                        e.out_hi[o] = h;
                        e.out_lo[o] = __float2half_rn(gv - __half2float(h));
                    }
                }
            }
            break;
        }
        default: {  // EPI_QKV
            // lane l holds the KV-cache offset of token mbase + l * mstep (shuffled in uniform flow)
            const int ml = mbase + lane * mstep;
            long long mine = 0;
            if (lane < NJ && ml < mend)
                mine = (long long)e.slot[ml] * (long long)e.slot_stride + (long long)e.pos[ml] * e.hd;
            const bool isq = nn < e.d_local;
            float* col = e.kv;
            if (!isq && row_ok) {
                const int sel = nn >= 2 * e.d_local ? 1 : 0;  // 0 = K, 1 = V
                const int c = nn - (sel + 1) * e.d_local;
                const int head = c / e.hd, i = c - head * e.hd;
                col = e.kv + e.layer_off + (size_t)sel * e.sel_stride + (size_t)head * e.head_stride + i;
            }
#pragma unroll
            for (int j = 0; j < NJ; ++j) {
                const long long off = __shfl_sync(0xffffffffu, mine, j);
                float v = acc[j] * post;
                if (has_b) v += b;
                if (ok[j]) {
                    if (isq)
                        e.out[(size_t)(mbase + j * mstep) * e.ldo + nn] = v;
                    else
                        col[off] = v;
                }
            }
            break;
        }
    }
}

template <int ATOM, int BN, bool PRESPLIT, bool DEEP>
__global__ void __launch_bounds__(THREADS, (Cfg<BN, PRESPLIT, DEEP>::MIN_BLOCKS))
    k_linear_tc(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_wlo,
                const __grid_constant__ CUtensorMap tm_xhi, const __grid_constant__ CUtensorMap tm_xlo,
                TcParams p) {
    using C = Cfg<BN, PRESPLIT, DEEP>;
    extern __shared__ __align__(1024) uint8_t smem_raw_[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw_) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* raw_full = bars;
    uint64_t* raw_empty = bars + C::RAW_STAGES;
    uint64_t* op_full = bars + 2 * C::RAW_STAGES;
    uint64_t* op_empty = op_full + C::OS;
    uint64_t* x_full = op_empty + C::OS;
    uint64_t* x_empty = x_full + C::XS;
    uint64_t* acc_full = x_empty + C::XS;
    uint64_t* recv_full = acc_full + 1;  // split-K peers' partials have landed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_BAR + C::N_BAR * 8);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // weight-row tiles vary fastest: CTAs running together share activation tiles in L2
    const int n0 = blockIdx.x * BM, m0 = blockIdx.y * BN;
    const int split = blockIdx.z;
    const int kb0 = split * p.kb_per_split;
    const int nkb = min(p.kb_per_split, p.nkb_total - kb0);
    constexpr int RAW_TX = (ATOM == ATOM_Q8) ? BM * 64 : BM * 32;

    if (threadIdx.x == 0) tc_stamp(p, 0);
    if (threadIdx.x == 0) {
        for (int i = 0; i < C::RAW_STAGES; ++i) {
            tc::mbar_init(&raw_full[i], 1);
            tc::mbar_init(&raw_empty[i], 128);
        }
        for (int i = 0; i < C::OS; ++i) {
            // prefill: the weight producer (+tx); decode: the 128 converter threads
            tc::mbar_init(&op_full[i], PRESPLIT ? 1 : 128);
            tc::mbar_init(&op_empty[i], 1);
        }
        for (int i = 0; i < C::XS; ++i) {
            tc::mbar_init(&x_full[i], 1);
            tc::mbar_init(&x_empty[i], 1);
        }
        tc::mbar_init(acc_full, 1);
        tc::mbar_init(recv_full, 1);
        if (C::PUSH && p.splits > 1) {
            // this CTA reduces token columns [rank CW, rank CW + w) of the tile (w <= CW: the last
            // block may be narrower): every other split stores 128 rows x w fp32 into it
            const int rank = (int)tc::cluster_rank();
            const int CW = push_cw(BN, p.splits);
            const int w = min(BN, (rank + 1) * CW) - rank * CW;
            if (w > 0) tc::mbar_arrive_expect_tx(recv_full, (uint32_t)((p.splits - 1) * 128 * w * 4));
        }
        tc::fence_mbar_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(tmem_slot, C::TMEM_COLS);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // dependents may start only once this CTA holds its TMEM columns: a dependent CTA that
    // took them first would wait for this grid while this grid waits for its columns
    tc::pdl_trigger();
    const bool push = C::PUSH && p.splits > 1;
    // split-K exchange over three cluster-barrier phases: 0 = barriers initialised, 1 = every
    // CTA's MMAs are done (its operand rings may be written), 2 = all stores into every CTA
    // have landed (none may exit before)
    if (push) tc::cluster_arrive_relaxed();
    if (threadIdx.x == 0) tc_stamp(p, 1);

    if (warp == 0) {
        // ---------------- weight tile producer (no dependency on earlier kernels) ----------------
        if (lane == 0) {
            tc::prefetch_tmap(&tm_w);
            int issued = 0;
            for (int i = 0; i < nkb; ++i) {
                if (PRESPLIT) {
                    const int s = i % C::OS, use = i / C::OS;
                    if (!tc::mbar_wait_spin(&op_empty[s], (use & 1) ^ 1, p.err)) break;
                    const bool wlo = C::DUAL || p.products >= 2;
                    tc::mbar_arrive_expect_tx(&op_full[s], (wlo ? 2 : 1) * C::A_BYTES);
                    uint8_t* a = smem + C::OFF_A + s * 2 * C::A_BYTES;
                    tc::tma_load_2d(a, &tm_w, (kb0 + i) * BK, n0, &op_full[s]);
                    if (wlo) tc::tma_load_2d(a + C::A_BYTES, &tm_wlo, (kb0 + i) * BK, n0, &op_full[s]);
                } else {
                    const int s = i % C::RAW_STAGES, use = i / C::RAW_STAGES;
                    if (!tc::mbar_wait_spin(&raw_empty[s], (use & 1) ^ 1, p.err)) break;
                    tc::mbar_arrive_expect_tx(&raw_full[s], RAW_TX);
                    const int kx = (kb0 + i) * (ATOM == ATOM_Q8 ? 64 : 32);
                    tc::tma_load_2d(smem + C::OFF_RAW + s * C::RAW_BYTES, &tm_w, kx, n0, &raw_full[s]);
                }
                if (i == 0) tc_stamp(p, 2);
                issued = i + 1;
            }
            tc_stamp(p, 3);
            // drain: every issued copy has landed before the CTA can exit
            if (PRESPLIT) {
                for (int i = (issued > C::OS ? issued - C::OS : 0); i < issued; ++i)
                    tc::mbar_wait(&op_full[i % C::OS], (i / C::OS) & 1, p.err);
            } else {
                for (int i = (issued > C::RAW_STAGES ? issued - C::RAW_STAGES : 0); i < issued; ++i)
                    tc::mbar_wait(&raw_full[i % C::RAW_STAGES], (i / C::RAW_STAGES) & 1, p.err);
            }
        }
    } else if (warp == 6) {
        // ---------------- activation tile producer ----------------
        if (lane == 0) {
            tc::prefetch_tmap(&tm_xhi);
            tc::prefetch_tmap(&tm_xlo);
            tc::pdl_wait();  // X was written by the previous kernel
            tc_stamp(p, 8);
            int issued = 0;
            for (int i = 0; i < nkb; ++i) {
                const int s = i % C::XS, use = i / C::XS;
                if (!tc::mbar_wait_spin(&x_empty[s], (use & 1) ^ 1, p.err)) break;
                const bool xlo = C::DUAL || p.products >= 3;
                tc::mbar_arrive_expect_tx(&x_full[s], (xlo ? 2 : 1) * C::B_BYTES);
                const int kx = (kb0 + i) * BK;
                uint8_t* b = smem + C::OFF_B + s * 2 * C::B_BYTES;
                tc::tma_load_2d(b, &tm_xhi, kx, m0, &x_full[s]);
                if (xlo) tc::tma_load_2d(b + C::B_BYTES, &tm_xlo, kx, m0, &x_full[s]);
                if (i == 0) tc_stamp(p, 9);
                issued = i + 1;
            }
            for (int i = (issued > C::XS ? issued - C::XS : 0); i < issued; ++i)
                tc::mbar_wait(&x_full[i % C::XS], (i / C::XS) & 1, p.err);
        }
    } else if (warp == 5) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_f16_f32(BM, C::DUAL ? 2 * BN : BN);
            for (int i = 0; i < nkb; ++i) {
                const int s = i % C::OS, use = i / C::OS;
                const int xs = i % C::XS, xuse = i / C::XS;
                // single-thread polls: a suspended try_wait may resume well after the phase
                // completes, leaving the tensor pipe idle
                if (!tc::mbar_wait_spin(&op_full[s], use & 1, p.err)) break;
                if (!tc::mbar_wait_spin(&x_full[xs], xuse & 1, p.err)) break;
                if (i == 0) tc_stamp(p, 6);
                tc::tc_fence_after();
                const uint32_t a_hi = tc::smem_u32(smem + C::OFF_A + s * 2 * C::A_BYTES);
                const uint32_t a_lo = a_hi + C::A_BYTES;
                const uint32_t b_hi = tc::smem_u32(smem + C::OFF_B + xs * 2 * C::B_BYTES);
                const uint32_t b_lo = b_hi + C::B_BYTES;
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk) {
                    const uint32_t ko = kk * 32;
                    const uint64_t dah = tc::desc_sw128(a_hi + ko), dal = tc::desc_sw128(a_lo + ko);
                    const uint64_t dbh = tc::desc_sw128(b_hi + ko);
                    const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
                    if constexpr (C::DUAL) {
                        // [X_hi; X_lo] is one 2 BN-row operand: A_hi -> columns 0..2BN, A_lo -> 2BN..4BN
                        tc::mma_f16(tmem, dah, dbh, idesc, acc);
                        tc::mma_f16(tmem + 2 * BN, dal, dbh, idesc, acc);
                    } else {
                        const uint64_t dbl = tc::desc_sw128(b_lo + ko);
                        tc::mma_f16(tmem, dah, dbh, idesc, acc);
                        if (p.products >= 3) tc::mma_f16(tmem, dah, dbl, idesc, 1u);
                        if (p.products >= 2) tc::mma_f16(tmem, dal, dbh, idesc, 1u);
                    }
                }
                tc::mma_commit(&op_empty[s]);
                tc::mma_commit(&x_empty[xs]);
            }
            tc::mma_commit(acc_full);
            tc_stamp(p, 7);
            tc::mbar_wait(acc_full, 0, p.err);  // every MMA has completed before teardown
        }
    } else {
        // ---------------- converters (warps 1-4), then epilogue ----------------
        const int t = threadIdx.x - 32;  // weight row within the tile, 0..127
        if (!PRESPLIT) {
            const int n = n0 + t;
            const bool row_ok = n < p.w.rows;
            const __half* srow = p.w.s + (size_t)(row_ok ? n : 0) * p.w.sstride;
            float* sc = reinterpret_cast<float*>(smem + C::OFF_SC) + t * C::SC_STRIDE;
            bool ok = true;
            for (int i = 0; i < nkb && ok; ++i) {
                if (i % C::SC_KB == 0) {
                    // this row's scales for k-blocks i..i+SC_KB-1, prescaled by 2^P; one burst of
                    // independent loads instead of a dependent global load per k-block
                    const int gbase = (kb0 + i) * 2;
#pragma unroll
                    for (int j = 0; j < 2 * C::SC_KB; ++j) {
                        const int gi = gbase + j;
                        sc[j] = (row_ok && gi < p.w.sstride) ? __half2float(srow[gi]) * p.pre : 0.f;
                    }
                }
                const int rs = i % C::RAW_STAGES, ruse = i / C::RAW_STAGES;
                const int os = i % C::OS, ouse = i / C::OS;
                ok = tc::mbar_wait(&raw_full[rs], ruse & 1, p.err) &&
                     tc::mbar_wait(&op_empty[os], (ouse & 1) ^ 1, p.err);
                if (!ok) break;
                if (i == 0 && t == 0) tc_stamp(p, 4);
                const int jj = 2 * (i % C::SC_KB);
                const __half2 s0 = __float2half2_rn(sc[jj]);
                const __half2 s1 = __float2half2_rn(sc[jj + 1]);
                const uint32_t raw = tc::smem_u32(smem + C::OFF_RAW + rs * C::RAW_BYTES);
                const uint32_t a_hi = tc::smem_u32(smem + C::OFF_A + os * 2 * C::A_BYTES);
                const uint32_t a_lo = a_hi + C::A_BYTES;
                if (ATOM == ATOM_Q8) {
                    // row t: 4 chunks of 16 int8, 64-byte swizzle: chunk c at c ^ ((t >> 1) & 3)
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const uint4 v = ld_shared_v4(raw + t * 64 + ((c ^ ((t >> 1) & 3)) * 16));
                        put16_q8(a_hi, a_lo, t, c, v, (c < 2) ? s0 : s1);
                    }
                } else {
                    // row t: 2 chunks of 16 packed bytes (one 32-group each), 32-byte swizzle
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        const uint4 v = ld_shared_v4(raw + t * 32 + ((c ^ ((t >> 2) & 1)) * 16));
                        put32_q4(a_hi, a_lo, t, c, v, (c == 0) ? s0 : s1);
                    }
                }
                tc::fence_proxy_async_smem();
                tc::mbar_arrive(&raw_empty[rs]);
                tc::mbar_arrive(&op_full[os]);
            }
        }
        if (threadIdx.x == 32) tc_stamp(p, 5);
        // ---- epilogue part 1: TMEM -> (outputs | pushed partial | L2 partial) ----
        // the bias is a weight: its load flies while the MMAs finish
        const int n_epi = n0 + (warp & 3) * 32 + lane;
        const float bias_v = (p.epi.bias && n_epi < p.w.rows) ? __ldg(p.epi.bias + n_epi) : 0.f;
        const bool acc_ok = tc::mbar_wait(acc_full, 0, p.err);
        if (threadIdx.x == 32) tc_stamp(p, 10);
        tc::tc_fence_after();
        if (push) {
            // this CTA's MMAs, and their shared-memory reads, are complete: its operand rings
            // may now receive the peers' partials (phase 1)
            tc::cluster_wait();  // phase 0
            tc::cluster_arrive_relaxed();
        }
        tc::pdl_wait();  // outputs / residual inputs belong to earlier kernels
        if (threadIdx.x == 32) tc_stamp(p, 11);
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;  // TMEM lane owned by this thread
        const int nn = n0 + row;
        const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16);
        float4* gpart = p.part + ((size_t)(blockIdx.x + gridDim.x * blockIdx.y) * p.splits + split) * (BN / 4) * 128;
        const int mend = min(p.M, m0 + BN);
        // push exchange: rank r reduces token columns [r CW, r CW + CW) of the tile
        const int rank = push ? (int)tc::cluster_rank() : 0;
        // test switch (GemmPlan::fault): rank 1 withholds its partials once
        const bool stall = push && rank == 1 && *reinterpret_cast<volatile const int*>(p.fault) != 0;
        const int CW = push_cw(BN, p.splits);
        float* recv = reinterpret_cast<float*>(smem);  // [splits][128][CW]: slot s from split s
        const int own_w = max(0, min(BN, (rank + 1) * CW) - rank * CW);
        // residual rows of this CTA's token columns, loaded while the partials travel
        constexpr int RPRE = 8;
        const bool resid = p.epi.kind == EPI_RESID;
        float rpre[RPRE];
        if (push && resid && own_w <= RPRE) {
#pragma unroll
            for (int j = 0; j < RPRE; ++j) {
                const int m = m0 + rank * CW + j;
                rpre[j] = (j < own_w && nn < p.w.rows && m < mend) ? p.epi.out[(size_t)m * p.epi.ldo + nn] : 0.f;
            }
        }
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
            float v[32];
            if constexpr (C::DUAL) {  // (A_hi X_hi + A_hi X_lo) + (A_lo X_hi + A_lo X_lo)
                float t[32];
                tc::tmem_ld32x2(taddr + c0, taddr + BN + c0, v, t);
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] += t[j];
                float u[32];
                tc::tmem_ld32x2(taddr + 2 * BN + c0, taddr + 3 * BN + c0, t, u);
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] += t[j] + u[j];
            } else {
                tc::tmem_ld32(taddr + c0, v);
            }
            if (p.splits == 1) {
                if (m0 + c0 >= mend) break;  // warp-uniform
                epi_chunk<32>(p.epi, nn, acc_ok && nn < p.w.rows, v, m0 + c0, 1, mend, p.post, nullptr, &bias_v);
            } else if (push) {
                if (c0 == 0) tc::cluster_wait();  // phase 1: every peer's rings may be written
                // columns of rank r go to slot `rank` of CTA r: remote 16-byte stores that
                // complete on r's recv_full, plain stores for this CTA's own columns
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    const int c = c0 + j, r = c / CW, q = c - r * CW;
                    float* dst = recv + ((size_t)rank * 128 + row) * CW + q;
                    const float4 val = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                    if (r == rank)
                        *reinterpret_cast<float4*>(dst) = val;
                    else if (!stall)
                        tc::st_async_f32x4((uint32_t)r, dst, val, recv_full);
                }
            } else if constexpr (!C::PUSH) {
                // wide tiles: the partial goes to L2 as [BN / 4][128 rows] float4 (a warp writes
                // 512 contiguous bytes per store); distributed shared memory is several times
                // slower per SM than L2 for a 128 KB partial
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    __stcg(gpart + (size_t)((c0 + j) >> 2) * 128 + row, make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
            }
        }
        if (push) {
            if (stall && threadIdx.x == 32) atomicExch(p.fault, 0);
            if (threadIdx.x == 32) tc_stamp(p, 13);
            const bool ok = acc_ok && (own_w == 0 || tc::mbar_wait_cluster(recv_full, 0, p.err));
            if (threadIdx.x == 32) tc_stamp(p, 14);
            __syncwarp();
            tc::cluster_arrive_relaxed();  // phase 2: everything sent to this CTA has landed
            // sum the splits in rank order (this thread's own row of each slot: its own slot was
            // written by itself), then the epilogue for this CTA's token columns
            for (int cb = 0; cb < own_w && m0 + rank * CW + cb < mend; cb += 4) {
                const int m = m0 + rank * CW + cb;
                float rp[4], acc[4] = {0.f, 0.f, 0.f, 0.f};
                if (resid) {
                    if (own_w <= RPRE) {
#pragma unroll
                        for (int j = 0; j < 4; ++j) rp[j] = (cb == 0) ? rpre[j] : rpre[4 + j];
                    } else {
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            rp[j] = (nn < p.w.rows && m + j < mend) ? p.epi.out[(size_t)(m + j) * p.epi.ldo + nn] : 0.f;
                    }
                }
#pragma unroll
                for (int sp = 0; sp < MAX_SPLITS; ++sp) {
                    if (sp < p.splits) {
                        const float4 x = *reinterpret_cast<const float4*>(recv + ((size_t)sp * 128 + row) * CW + cb);
                        acc[0] += x.x;
                        acc[1] += x.y;
                        acc[2] += x.z;
                        acc[3] += x.w;
                    }
                }
                epi_chunk<4>(p.epi, nn, ok && nn < p.w.rows, acc, m, 1, mend, p.post, resid ? rp : nullptr, &bias_v);
            }
        }
    }
    if (push && (warp == 0 || warp >= 5)) {
        __syncwarp();
        tc::cluster_wait();            // phase 0
        tc::cluster_arrive_relaxed();  // phase 1
        tc::cluster_wait();
        tc::cluster_arrive_relaxed();  // phase 2
    }
    tc::tc_fence_before();
    __syncthreads();
    if (!push && threadIdx.x == 32) tc_stamp(p, 12);
    if (push) {
        tc::cluster_wait();  // phase 2: no copy into or out of any CTA of the cluster is in flight
    } else if (!C::PUSH && p.splits > 1) {  // (PUSH tiles exchange by push whenever they split)
        // ---- epilogue part 2: split-K reduction of the partials in L2 ----
        tc::cluster_sync();  // every CTA's partial is written (release / acquire, cluster scope)
        if (threadIdx.x == 32) tc_stamp(p, 13);
        if (warp >= 1 && warp <= 4) {
            const int row = (warp & 3) * 32 + lane;
            const int nn = n0 + row;
            const int mend = min(p.M, m0 + BN);
            const float4* tile_part = p.part + (size_t)(blockIdx.x + gridDim.x * blockIdx.y) * p.splits * (BN / 4) * 128;
            // split s reduces and writes a contiguous block of CW columns (tokens). Every split's
            // loads of a block are issued before any is summed; the sums run in split order.
            const int CW = push_cw(BN, p.splits);
            const int cend = min(BN, (split + 1) * CW);
            constexpr int RJ = 16, RQ = RJ / 4;
            for (int cb = split * CW; cb < cend && m0 + cb < mend; cb += RJ) {
                float acc[RJ], rp[RJ];
                const bool resid = p.epi.kind == EPI_RESID;
                if (resid) {  // residual loads in flight together with the partial loads
#pragma unroll
                    for (int j = 0; j < RJ; ++j) {
                        const int m = m0 + cb + j;
                        rp[j] = (nn < p.w.rows && m < mend && cb + j < cend) ? p.epi.out[(size_t)m * p.epi.ldo + nn] : 0.f;
                    }
                }
                // unconditional loads from clamped (valid) addresses, masked afterwards: no branch
                // separates a load from the next one
                float4 x[MAX_SPLITS_PULL][RQ];
#pragma unroll
                for (int sp = 0; sp < MAX_SPLITS_PULL; ++sp) {
                    const int spc = min(sp, p.splits - 1);
#pragma unroll
                    for (int q = 0; q < RQ; ++q) {
                        const int c4 = min((cb >> 2) + q, (cend >> 2) - 1);
                        x[sp][q] = __ldcg(tile_part + ((size_t)spc * (BN / 4) + c4) * 128 + row);
                    }
                }
#pragma unroll
                for (int j = 0; j < RJ; ++j) acc[j] = 0.f;
#pragma unroll
                for (int sp = 0; sp < MAX_SPLITS_PULL; ++sp) {
                    const bool keep = sp < p.splits;  // an absent split adds +0: no value changes
#pragma unroll
                    for (int q = 0; q < RQ; ++q) {
                        acc[4 * q] += keep ? x[sp][q].x : 0.f;
                        acc[4 * q + 1] += keep ? x[sp][q].y : 0.f;
                        acc[4 * q + 2] += keep ? x[sp][q].z : 0.f;
                        acc[4 * q + 3] += keep ? x[sp][q].w : 0.f;
                    }
                }
                if (threadIdx.x == 32 && cb == split * CW) tc_stamp(p, 15);  // first block summed
                epi_chunk<RJ>(p.epi, nn, nn < p.w.rows, acc, m0 + cb, 1, min(mend, m0 + cend), p.post,
                              resid ? rp : nullptr);
            }
        }
        // no closing cluster barrier: the partials live in global memory, and the next launch
        // writes them only after its dependent-launch wait, when this grid has completed
        if (threadIdx.x == 32) tc_stamp(p, 14);
    }
    if (threadIdx.x == 0 && (C::PUSH || p.splits == 1)) tc_stamp(p, 15);  // (pull: see above)
    if (warp == 0) tc::tmem_dealloc(tmem, C::TMEM_COLS);
}

// ---------------------------------------------------------------- persistent prefill form
// Compute-bound prefill tiles (BN = 256, exact fp16 hi/lo weight copies, no split-K): one CTA
// per SM walks the tiles t = blockIdx.x, blockIdx.x + gridDim.x, ... (weight-row tiles
// fastest, so the CTAs running together share activation tiles in L2). The two operand rings
// run on across tiles, and the fp32 accumulator is double-buffered in TMEM (2 x 256 columns):
// the epilogue warps drain tile j while the MMAs of tile j + 1 run.
constexpr int PB_BN = 256, PB_OS = 2, PB_XS = 2;
constexpr int PB_A_BYTES = BM * 128, PB_B_BYTES = PB_BN * 128;
constexpr int PB_OFF_B = PB_OS * 2 * PB_A_BYTES;
constexpr int PB_OFF_BAR = PB_OFF_B + PB_XS * 2 * PB_B_BYTES;
constexpr int PB_N_BAR = 2 * PB_OS + 2 * PB_XS + 4;
constexpr int PB_SMEM = PB_OFF_BAR + PB_N_BAR * 8 + 16 + 1024;
static_assert(PB_SMEM <= 232448, "shared memory per CTA");

__global__ void __launch_bounds__(THREADS, 1)
    k_linear_tc_persistent(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_wlo,
                           const __grid_constant__ CUtensorMap tm_xhi, const __grid_constant__ CUtensorMap tm_xlo,
                           TcParams p, int n_row_tiles, int n_tiles) {
    extern __shared__ __align__(1024) uint8_t smem_raw_[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw_) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + PB_OFF_BAR);
    uint64_t* op_full = bars;
    uint64_t* op_empty = op_full + PB_OS;
    uint64_t* x_full = op_empty + PB_OS;
    uint64_t* x_empty = x_full + PB_XS;
    uint64_t* acc_full = x_empty + PB_XS;  // [2]
    uint64_t* acc_empty = acc_full + 2;    // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + PB_OFF_BAR + PB_N_BAR * 8);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nkb = p.nkb_total;

    if (threadIdx.x == 0) {
        for (int i = 0; i < PB_OS; ++i) {
            tc::mbar_init(&op_full[i], 1);
            tc::mbar_init(&op_empty[i], 1);
        }
        for (int i = 0; i < PB_XS; ++i) {
            tc::mbar_init(&x_full[i], 1);
            tc::mbar_init(&x_empty[i], 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&acc_full[b], 1);
            tc::mbar_init(&acc_empty[b], 128);
        }
        tc::fence_mbar_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(tmem_slot, 2 * PB_BN);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    tc::pdl_trigger();  // after the TMEM allocation (see k_linear_tc)

    if (warp == 0) {
        // ---------------- weight tiles (exact fp16 hi/lo copies) ----------------
        if (lane == 0) {
            tc::prefetch_tmap(&tm_w);
            tc::prefetch_tmap(&tm_wlo);
            int it = 0;
            for (int t = blockIdx.x; t < n_tiles; t += gridDim.x) {
                const int n0 = (t % n_row_tiles) * BM;
                for (int i = 0; i < nkb; ++i, ++it) {
                    const int s = it % PB_OS, use = it / PB_OS;
                    if (!tc::mbar_wait_spin(&op_empty[s], (use & 1) ^ 1, p.err)) break;
                    const bool wlo = p.products >= 2;
                    tc::mbar_arrive_expect_tx(&op_full[s], (wlo ? 2 : 1) * PB_A_BYTES);
                    uint8_t* a = smem + s * 2 * PB_A_BYTES;
                    tc::tma_load_2d(a, &tm_w, i * BK, n0, &op_full[s]);
                    if (wlo) tc::tma_load_2d(a + PB_A_BYTES, &tm_wlo, i * BK, n0, &op_full[s]);
                }
            }
        }
    } else if (warp == 6) {
        // ---------------- activation tiles ----------------
        if (lane == 0) {
            tc::prefetch_tmap(&tm_xhi);
            tc::prefetch_tmap(&tm_xlo);
            tc::pdl_wait();  // X was written by the previous kernel
            int it = 0;
            for (int t = blockIdx.x; t < n_tiles; t += gridDim.x) {
                const int m0 = (t / n_row_tiles) * PB_BN;
                for (int i = 0; i < nkb; ++i, ++it) {
                    const int s = it % PB_XS, use = it / PB_XS;
                    if (!tc::mbar_wait_spin(&x_empty[s], (use & 1) ^ 1, p.err)) break;
                    const bool xlo = p.products >= 3;
                    tc::mbar_arrive_expect_tx(&x_full[s], (xlo ? 2 : 1) * PB_B_BYTES);
                    uint8_t* b = smem + PB_OFF_B + s * 2 * PB_B_BYTES;
                    tc::tma_load_2d(b, &tm_xhi, i * BK, m0, &x_full[s]);
                    if (xlo) tc::tma_load_2d(b + PB_B_BYTES, &tm_xlo, i * BK, m0, &x_full[s]);
                }
            }
        }
    } else if (warp == 5) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_f16_f32(BM, PB_BN);
            int it = 0, j = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x, ++j) {
                const int buf = j & 1;
                // the epilogue has drained this accumulator (tile j - 2)
                ok = tc::mbar_wait_spin(&acc_empty[buf], ((j >> 1) & 1) ^ 1, p.err);
                tc::tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(buf * PB_BN);
                for (int i = 0; i < nkb && ok; ++i, ++it) {
                    const int s = it % PB_OS, use = it / PB_OS;
                    const int xs = it % PB_XS, xuse = it / PB_XS;
                    ok = tc::mbar_wait_spin(&op_full[s], use & 1, p.err) && tc::mbar_wait_spin(&x_full[xs], xuse & 1, p.err);
                    if (!ok) break;
                    tc::tc_fence_after();
                    const uint32_t a_hi = tc::smem_u32(smem + s * 2 * PB_A_BYTES), a_lo = a_hi + PB_A_BYTES;
                    const uint32_t b_hi = tc::smem_u32(smem + PB_OFF_B + xs * 2 * PB_B_BYTES), b_lo = b_hi + PB_B_BYTES;
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        const uint32_t ko = kk * 32;
                        const uint64_t dah = tc::desc_sw128(a_hi + ko), dal = tc::desc_sw128(a_lo + ko);
                        const uint64_t dbh = tc::desc_sw128(b_hi + ko), dbl = tc::desc_sw128(b_lo + ko);
                        tc::mma_f16(d, dah, dbh, idesc, (i > 0 || kk > 0) ? 1u : 0u);
                        if (p.products >= 3) tc::mma_f16(d, dah, dbl, idesc, 1u);
                        if (p.products >= 2) tc::mma_f16(d, dal, dbh, idesc, 1u);
                    }
                    tc::mma_commit(&op_empty[s]);
                    tc::mma_commit(&x_empty[xs]);
                }
                tc::mma_commit(&acc_full[buf]);
            }
        }
    } else {
        // ---------------- epilogue (warps 1-4): TMEM -> fused epilogue, one tile at a time ----------------
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16);
        tc::pdl_wait();  // outputs / residual inputs belong to earlier kernels
        int j = 0;
        for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++j) {
            const int buf = j & 1;
            const int n0 = (t % n_row_tiles) * BM, m0 = (t / n_row_tiles) * PB_BN;
            const int nn = n0 + row;
            const float bias_v = (p.epi.bias && nn < p.w.rows) ? __ldg(p.epi.bias + nn) : 0.f;
            const bool ok = tc::mbar_wait(&acc_full[buf], (uint32_t)((j >> 1) & 1), p.err);
            tc::tc_fence_after();
            const int mend = min(p.M, m0 + PB_BN);
#pragma unroll 1
            for (int c0 = 0; c0 < PB_BN; c0 += 32) {
                if (m0 + c0 >= mend) break;  // warp-uniform
                float v[32];
                tc::tmem_ld32(taddr + (uint32_t)(buf * PB_BN + c0), v);
                epi_chunk<32>(p.epi, nn, ok && nn < p.w.rows, v, m0 + c0, 1, mend, p.post, nullptr, &bias_v);
            }
            tc::tc_fence_before();
            tc::mbar_arrive(&acc_empty[buf]);  // this accumulator may be overwritten
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tmem, 2 * PB_BN);
}

// One-time exact split of a quantised weight for the prefill path: w' = deq(w) * 2^P,
// hi = f16(w'), lo = f16(w' - hi), both [rows][cols].
__global__ void k_presplit_weight(QW w, float pre, __half* __restrict__ hi, __half* __restrict__ lo) {
    const size_t n = (size_t)w.rows * w.cols;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float v = deq_elem(w, (int)(i / w.cols), (int)(i % w.cols)) * pre;
        const __half h = __float2half_rn(v);
        hi[i] = h;
        lo[i] = __float2half_rn(v - __half2float(h));
    }
}

// ---------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    });
    return fn;
}

bool make_map_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
                 uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t es[2] = {1, 1};
    return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int ATOM, int BN, bool PRESPLIT, bool DEEP>
cudaError_t launch_tc(const CUtensorMap& tw, const CUtensorMap& twlo, const CUtensorMap& txh, const CUtensorMap& txl,
                      const TcParams& tp, dim3 grid, cudaStream_t st) {
    auto kern = k_linear_tc<ATOM, BN, PRESPLIT, DEEP>;
    const int smem = Cfg<BN, PRESPLIT, DEEP>::SMEM;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attrs[2];
    int na = 0;
    if (pdl_enabled()) {
        attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attrs[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (grid.z > 8) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
    }
    if (grid.z > 1) {
        attrs[na].id = cudaLaunchAttributeClusterDimension;
        attrs[na].val.clusterDim.x = 1;
        attrs[na].val.clusterDim.y = 1;
        attrs[na].val.clusterDim.z = grid.z;
        ++na;
    }
    cfg.attrs = attrs;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, kern, tw, twlo, txh, txl, tp);
}

cudaError_t launch_persistent(const CUtensorMap& tw, const CUtensorMap& twlo, const CUtensorMap& txh,
                              const CUtensorMap& txl, const TcParams& tp, int n_row_tiles, int n_tiles, cudaStream_t st) {
    static int sms = [] {
        int dev = 0, n = 148;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        return n;
    }();
    cudaError_t e = cudaFuncSetAttribute(k_linear_tc_persistent, cudaFuncAttributeMaxDynamicSharedMemorySize, PB_SMEM);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(std::min(n_tiles, sms));
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = PB_SMEM;
    cfg.stream = st;
    cudaLaunchAttribute at;
    at.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &at;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_linear_tc_persistent, tw, twlo, txh, txl, tp, n_row_tiles, n_tiles);
}

// Clusters of `cs` CTAs of this kernel that the device holds at once (cached per size).
template <int ATOM, int BN, bool PRESPLIT, bool DEEP>
int resident_clusters(int cs) {
    static std::atomic<int> cache[MAX_SPLITS + 1];
    if (cs < 1 || cs > MAX_SPLITS) return 0;
    int v = cache[cs].load(std::memory_order_relaxed);
    if (v != 0) return v;
    auto kern = k_linear_tc<ATOM, BN, PRESPLIT, DEEP>;
    const int smem = Cfg<BN, PRESPLIT, DEEP>::SMEM;
    int n = 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) == cudaSuccess &&
        (cs <= 8 || cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess)) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(1, 1, cs);
        cfg.blockDim = dim3(THREADS, 1, 1);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = cs;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
    }
    cudaGetLastError();
    v = n > 0 ? n : -1;
    cache[cs].store(v, std::memory_order_relaxed);
    return v;
}

// Decode tiles (BN <= 64) run the deep configuration (one CTA per SM) only when the whole
// grid is resident at once in it; a second wave would start late and serialise.
template <int ATOM, int BN, bool PRESPLIT>
cudaError_t launch_small(const CUtensorMap& tw, const CUtensorMap& twlo, const CUtensorMap& txh,
                         const CUtensorMap& txl, const TcParams& tp, dim3 grid, cudaStream_t st) {
    // measured on GPT-2 small decode at 32 sequences: the shallow configuration is faster (the
    // MMA issue rate, not the weight stream, bounds these tiles), so deep is opt-in
    static const bool want_deep = [] {
        const char* e = getenv("GPT2Q_TC_DEEP");
        return e && e[0] == '1';
    }();
    const long clusters = (long)grid.x * grid.y;
    const bool deep = want_deep && clusters <= resident_clusters<ATOM, BN, PRESPLIT, true>((int)grid.z);
    if (deep) return launch_tc<ATOM, BN, PRESPLIT, true>(tw, twlo, txh, txl, tp, grid, st);
    return launch_tc<ATOM, BN, PRESPLIT, false>(tw, twlo, txh, txl, tp, grid, st);
}

template <int ATOM, bool PRESPLIT>
cudaError_t launch_bn(int BN, const CUtensorMap& tw, const CUtensorMap& twlo, const CUtensorMap& txh,
                      const CUtensorMap& txl, const TcParams& tp, dim3 grid, cudaStream_t st) {
    switch (BN) {
        case 32: return launch_small<ATOM, 32, PRESPLIT>(tw, twlo, txh, txl, tp, grid, st);
        case 64: return launch_small<ATOM, 64, PRESPLIT>(tw, twlo, txh, txl, tp, grid, st);
        case 128: return launch_tc<ATOM, 128, PRESPLIT, false>(tw, twlo, txh, txl, tp, grid, st);
        default: return launch_tc<ATOM, 256, PRESPLIT, false>(tw, twlo, txh, txl, tp, grid, st);
    }
}

// ---------------------------------------------------------------- int8 lm head for decode batches
// The tied head over 16..64 tokens on kind::i8. k_head_pieces splits the ln_f output of every
// token and 32-group exactly into three int8 pieces, x = 2^-S (p0 + p1 2^-7 + p2 2^-14) + r with
// |r| <= 2^-20 of the group's largest |x|, laid out as B operands. The int8 weights enter as they
// are stored, so one MMA of N = 3 MP per group gives the exact integer dot products of 128 rows
// with every piece of every token (four f16 MMAs per group on the hi/lo path). Groups carry
// their own scales (f16 per row for W, 2^-S per token for x), so each group's product lands in
// one of two TMEM buffers and the epilogue warps fold it in, v = d0 + d1 2^-7 + d2 2^-14,
// acc += (v 2^-S) s_w, while the next group's MMA runs.
constexpr int HI_RS = 4;  // raw weight stages of 128 rows x 64 bytes (two groups each)

template <int MP>
struct HeadCfg {
    static constexpr int N = 3 * MP;          // MMA columns: piece-major, then token
    static constexpr int B_GROUP = N * 32;    // bytes of one group's pieces
    static constexpr int A_STAGE = BM * 64;
    static constexpr int OFF_B = HI_RS * A_STAGE;
    static constexpr uint32_t TMEM_COLS = N <= 128 ? 256 : 512;  // two buffers of N columns
    static size_t smem(int G) {
        return (size_t)OFF_B + (size_t)G * B_GROUP + (size_t)MP * G * 4 + (2 * HI_RS + 5) * 8 + 16 + 1024;
    }
};

template <int MP>
__global__ void __launch_bounds__(THREADS, MP == 32 ? 2 : 1)
    k_head_i8(const __grid_constant__ CUtensorMap tm_w, const uint8_t* __restrict__ pieces,
              const float* __restrict__ xscale, QW w, int M, float* __restrict__ out, int ldo, int* err) {
    using C = HeadCfg<MP>;
    extern __shared__ __align__(1024) uint8_t smem_raw_[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw_) + 1023) & ~uintptr_t(1023));
    const int G = w.cols / 32, nkb = G / 2;
    float* sxs = reinterpret_cast<float*>(smem + C::OFF_B + (size_t)G * C::B_GROUP);  // [MP][G]: 2^-S
    uint64_t* full = reinterpret_cast<uint64_t*>(sxs + ((MP * G + 1) & ~1));
    uint64_t* empty = full + HI_RS;
    uint64_t* xbar = empty + HI_RS;  // pieces and scales landed
    uint64_t* mfull = xbar + 1;      // [2] a group's product is in TMEM buffer b
    uint64_t* tempty = mfull + 2;    // [2] the epilogue has read buffer b
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BM;

    if (threadIdx.x == 0) {
        for (int i = 0; i < HI_RS; ++i) {
            tc::mbar_init(&full[i], 1);
            tc::mbar_init(&empty[i], 1);
        }
        tc::mbar_init(xbar, 1);
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&mfull[b], 1);
            tc::mbar_init(&tempty[b], 128);
        }
        tc::fence_mbar_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(tmem_slot, C::TMEM_COLS);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    tc::pdl_trigger();  // after the TMEM allocation (see k_linear_tc)

    if (warp == 0) {
        // ---------------- weight tiles: 64 bytes of K (two groups) x 128 rows per stage ----------------
        if (lane == 0) {
            tc::prefetch_tmap(&tm_w);
            int issued = 0;
            for (int kb = 0; kb < nkb; ++kb) {
                const int st = kb % HI_RS, use = kb / HI_RS;
                if (!tc::mbar_wait_spin(&empty[st], (use & 1) ^ 1, err)) break;
                tc::mbar_arrive_expect_tx(&full[st], C::A_STAGE);
                tc::tma_load_2d(smem + st * C::A_STAGE, &tm_w, kb * 64, n0, &full[st]);
                issued = kb + 1;
            }
            for (int kb = (issued > HI_RS ? issued - HI_RS : 0); kb < issued; ++kb)
                tc::mbar_wait(&full[kb % HI_RS], (kb / HI_RS) & 1, err);  // nothing in flight at exit
        }
    } else if (warp == 6) {
        // ---------------- the pieces and scales of every token (written by k_head_pieces) ----------------
        if (lane == 0) {
            tc::pdl_wait();
            const uint32_t pb = (uint32_t)G * C::B_GROUP, sb = (uint32_t)(MP * G * 4);
            tc::mbar_arrive_expect_tx(xbar, pb + sb);
            tc::bulk_load_1d(smem + C::OFF_B, pieces, pb, xbar);
            tc::bulk_load_1d(sxs, xscale, sb, xbar);
            tc::mbar_wait(xbar, 0, err);
        }
    } else if (warp == 5) {
        // ---------------- MMA issuer: one kind::i8 MMA per group ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_s8_s32(BM, C::N);
            bool ok = tc::mbar_wait_spin(xbar, 0, err);
            for (int g = 0; g < G && ok; ++g) {
                const int kb = g >> 1, st = kb % HI_RS, use = kb / HI_RS;
                const int b = g & 1, bu = g >> 1;
                if ((g & 1) == 0) ok = tc::mbar_wait_spin(&full[st], use & 1, err);
                ok = ok && tc::mbar_wait_spin(&tempty[b], (bu & 1) ^ 1, err);
                if (!ok) break;
                tc::tc_fence_after();
                const uint64_t ad = tc::desc_sw64(tc::smem_u32(smem + st * C::A_STAGE) + (uint32_t)(g & 1) * 32);
                const uint64_t bd = tc::desc_noswz(tc::smem_u32(smem + C::OFF_B + (size_t)g * C::B_GROUP), 128, 256);
                tc::mma_i8(tmem + (uint32_t)(b * C::N), ad, bd, idesc, 0u);
                tc::mma_commit(&mfull[b]);
                if ((g & 1) == 1) tc::mma_commit(&empty[st]);
            }
        }
    } else {
        // ---------------- epilogue (warps 1-4): one weight row per thread ----------------
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const int nn = n0 + row;
        const bool row_ok = nn < w.rows;
        const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16);
        const __half* srow = w.s + (size_t)(row_ok ? nn : 0) * w.sstride;
        float acc[MP];
#pragma unroll
        for (int t = 0; t < MP; ++t) acc[t] = 0.f;
        // polled waits: a suspended try_wait resumes microseconds late, once per group here
        bool ok = tc::mbar_wait_spin(xbar, 0, err);
        float sw = row_ok ? __half2float(srow[0]) : 0.f;
        for (int g = 0; g < G && ok; ++g) {
            const int b = g & 1, bu = g >> 1;
            const float sw_next = (row_ok && g + 1 < G) ? __half2float(srow[g + 1]) : 0.f;
            ok = tc::mbar_wait_spin(&mfull[b], bu & 1, err);
            if (!ok) break;
            tc::tc_fence_after();
            float v[MP];
#pragma unroll
            for (int c = 0; c < MP / 32; ++c) {
                float d0[32], d1[32], d2[32];
                tc::tmem_ld32x2(taddr + b * C::N + c * 32, taddr + b * C::N + MP + c * 32, d0, d1);
                tc::tmem_ld32(taddr + b * C::N + 2 * MP + c * 32, d2);
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const float p0 = (float)__float_as_int(d0[j]);
                    const float p1 = (float)__float_as_int(d1[j]);
                    const float p2 = (float)__float_as_int(d2[j]);
                    v[c * 32 + j] = fmaf(p2, 1.0f / 16384.0f, fmaf(p1, 1.0f / 128.0f, p0));
                }
            }
            tc::tc_fence_before();
            tc::mbar_arrive(&tempty[b]);
#pragma unroll
            for (int t = 0; t < MP; ++t) acc[t] = fmaf(v[t] * sxs[t * G + g], sw, acc[t]);
            sw = sw_next;
        }
        if (row_ok && ok) {
#pragma unroll
            for (int t = 0; t < MP; ++t)
                if (t < M) out[(size_t)t * ldo + nn] = acc[t];
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tmem, C::TMEM_COLS);
}

template <int MP>
cudaError_t launch_head_i8_mp(const CUtensorMap& tw, const uint8_t* pieces, const float* xscale, const QW& w, int M,
                              float* out, int ldo, int* err, cudaStream_t st) {
    auto kern = k_head_i8<MP>;
    const size_t smem = HeadCfg<MP>::smem(w.cols / 32);
    if (smem > 232448) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((w.rows + BM - 1) / BM);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at;
    at.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &at;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, tw, pieces, xscale, w, M, out, ldo, err);
}

}  // namespace

struct WeightTc {
    CUtensorMap raw;         // int8 / int4 tiles
    CUtensorMap hi, lo;      // fp16 split copies (prefill)
    bool has_split = false;
    float pre = 1.f, post = 1.f;
};

struct XKey {
    const void* buf;
    int K, ld, BN;
    bool operator==(const XKey& o) const { return buf == o.buf && K == o.K && ld == o.ld && BN == o.BN; }
};
struct XKeyHash {
    size_t operator()(const XKey& k) const {
        return std::hash<const void*>()(k.buf) ^ ((size_t)k.K << 1) ^ ((size_t)k.ld << 17) ^ ((size_t)k.BN << 33);
    }
};

struct GemmState {
    std::unordered_map<const void*, WeightTc> w;                 // weight payload -> maps
    std::unordered_map<XKey, CUtensorMap, XKeyHash> xmaps;       // activation buffer -> map
    std::vector<void*> owned;                                     // split weight copies
    // phase trace of one launch (GPT2Q_TC_TRACE="rows x cols x M", e.g. 768x3072x32)
    unsigned long long* trace = nullptr;
    int trace_rows = 0, trace_cols = 0, trace_m = 0;
    bool traced = false;
    dim3 trace_grid;
};

bool GemmPlan::usable(const QW& w, int M) const {
    if (!enabled || M < min_m || M > Mmax) return false;
    if (w.atom != ATOM_Q8 && w.atom != ATOM_Q4) return false;
    if (w.cols % 32 != 0) return false;
    if (w.cols > Kmax || (w.qstride % 16) != 0) return false;
    return state->w.count(w.q) != 0;
}

int gemm_init(GemmPlan& p, int device, int Mmax, int Kmax) {
    p.enabled = false;
    p.Mmax = Mmax;
    p.Kmax = Kmax;
    int major = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
    if (major != 10 || !encode_fn()) return 0;  // the tensor-core path needs sm_100
    if (const char* e = std::getenv("GPT2Q_TC_DISABLE"))
        if (e[0] == '1') return 0;
    p.min_m = 16;
    if (const char* e = std::getenv("GPT2Q_TC_MIN_M")) p.min_m = std::max(1, std::atoi(e));
    p.presplit_min_m = 257;
    if (const char* e = std::getenv("GPT2Q_TC_PRESPLIT_MIN_M")) p.presplit_min_m = std::max(1, std::atoi(e));
    if (const char* e = std::getenv("GPT2Q_TC_PRODUCTS")) p.products = std::max(1, std::min(3, std::atoi(e)));
    if (cudaMalloc(&p.err, 8) != cudaSuccess || cudaMemset(p.err, 0, 8) != cudaSuccess) return -1;
    p.fault = p.err + 1;
    if (const char* e = std::getenv("GPT2Q_TEST_SPLITK_STALL")) {
        const int one = 1;
        if (e[0] == '1' && cudaMemcpy(p.fault, &one, 4, cudaMemcpyHostToDevice) != cudaSuccess) return -1;
    }
    if (Mmax > 64) {
        // split-K partials of the wide tiles (BN 128 / 256): fewer than 120 tiles, each split
        // ceil(148 / tiles) ways at most, so under 268 CTAs of 128 x 256 fp32
        p.part_floats = (size_t)268 * 128 * 256;
        if (cudaMalloc(&p.part, p.part_floats * 4) != cudaSuccess) return -1;
    }
    if (cudaDeviceSynchronize() != cudaSuccess) return -1;
    p.state = new GemmState();
    if (const char* e = std::getenv("GPT2Q_TC_TRACE")) {
        if (std::sscanf(e, "%dx%dx%d", &p.state->trace_rows, &p.state->trace_cols, &p.state->trace_m) == 3 &&
            cudaMalloc(&p.state->trace, (size_t)4096 * TC_TRACE * 8) == cudaSuccess)
            cudaMemset(p.state->trace, 0, (size_t)4096 * TC_TRACE * 8);
    }
    p.enabled = true;
    return 0;
}

void gemm_destroy(GemmPlan& p) {
    if (p.err) cudaFree(p.err);
    if (p.part) cudaFree(p.part);
    if (p.state && p.state->trace) cudaFree(p.state->trace);
    if (p.state)
        for (void* q : p.state->owned) cudaFree(q);
    delete p.state;
    p = GemmPlan();
}

// Power-of-two prescale so the fp16 lo part of every weight stays normal:
// max |q * scale| * 2^P <= 2^14.
static int prescale_exponent(float max_abs_w) {
    if (!(max_abs_w > 0.f) || !std::isfinite(max_abs_w)) return 0;
    int P = (int)std::floor(std::log2(16384.0 / (double)max_abs_w));
    return std::max(-30, std::min(30, P));
}

int gemm_register_weight(GemmPlan& p, const QW& w, float max_abs_w, bool presplit, cudaStream_t st) {
    if (!p.enabled || (w.atom != ATOM_Q8 && w.atom != ATOM_Q4)) return 0;
    if (w.cols % 32 != 0 || w.cols > p.Kmax) return 0;
    WeightTc wt;
    const int P = prescale_exponent(max_abs_w);
    wt.pre = std::ldexp(1.0f, P);
    wt.post = std::ldexp(1.0f, -P);
    const bool q8 = w.atom == ATOM_Q8;
    if (!make_map_2d(&wt.raw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.q, w.qstride, (uint64_t)w.rows, w.qstride,
                     q8 ? 64 : 32, BM, q8 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B))
        return -1;
    if (presplit) {
        const size_t n = (size_t)w.rows * w.cols;
        void *hi = nullptr, *lo = nullptr;
        if (cudaMalloc(&hi, n * 2) != cudaSuccess) return -2;
        p.state->owned.push_back(hi);
        if (cudaMalloc(&lo, n * 2) != cudaSuccess) return -2;
        p.state->owned.push_back(lo);
        k_presplit_weight<<<148 * 8, 256, 0, st>>>(w, wt.pre, reinterpret_cast<__half*>(hi),
                                                  reinterpret_cast<__half*>(lo));
        if (cudaGetLastError() != cudaSuccess) return -1;
        if (!make_map_2d(&wt.hi, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, hi, (uint64_t)w.cols, (uint64_t)w.rows,
                         (uint64_t)w.cols * 2, 64, BM, CU_TENSOR_MAP_SWIZZLE_128B) ||
            !make_map_2d(&wt.lo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, lo, (uint64_t)w.cols, (uint64_t)w.rows,
                         (uint64_t)w.cols * 2, 64, BM, CU_TENSOR_MAP_SWIZZLE_128B))
            return -1;
        wt.has_split = true;
        p.presplit_bytes += 4 * n;
    }
    p.state->w[w.q] = wt;
    return 0;
}

// Tensor map of one fp16 activation buffer [Mmax][ld] viewed as [Mmax][K], box 64 x BN.
static const CUtensorMap* xmap(const GemmPlan& p, const __half* buf, int K, int ld, int BN) {
    const XKey key{buf, K, ld, BN};
    auto it = p.state->xmaps.find(key);
    if (it != p.state->xmaps.end()) return &it->second;
    CUtensorMap m;
    if (!make_map_2d(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, buf, (uint64_t)K, (uint64_t)p.Mmax, (uint64_t)ld * 2, 64,
                     (uint32_t)BN, CU_TENSOR_MAP_SWIZZLE_128B))
        return nullptr;
    return &p.state->xmaps.emplace(key, m).first->second;
}

cudaError_t launch_linear_tc(const GemmPlan& p, const QW& w, const XSplit& x, int M, const Epi& e,
                             cudaStream_t st) {
    auto wi = p.state->w.find(w.q);
    if (wi == p.state->w.end()) return cudaErrorInvalidValue;
    const WeightTc& wt = wi->second;
    const int K = w.cols;
    const bool presplit = wt.has_split && M >= p.presplit_min_m;
    // tokens per tile; GPT2Q_TC_BN_MAX caps it (tuning)
    static const int bn_max = [] {
        const char* e = std::getenv("GPT2Q_TC_BN_MAX");
        const int v = e ? std::atoi(e) : 256;
        return v >= 256 ? 256 : (v >= 128 ? 128 : (v >= 64 ? 64 : 32));
    }();
    const int n_tiles = (w.rows + BM - 1) / BM;
    int BN = M <= 32 ? 32 : (M <= 64 ? 64 : (M <= 128 ? 128 : 256));
    if (M > 64 && !presplit && n_tiles * ((M + BN - 1) / BN) < 120) {
        // 65..256 tokens on raw weights, too few tiles for a wave: the wide tiles would split K
        // and exchange 64-128 KB partials per CTA. Measured on GPT-2 small at 256 tokens (µs per
        // launch, tile width 256 -> chosen): qkv 15.2 -> 14.4 and c_fc 28.2 -> 17.1 with 32-token
        // tiles (a wave of tiles, no split), attn c_proj 12.3 -> 9.0 and mlp c_proj 15.1 -> 12.3
        // with 128-token tiles (smaller partials); the tied head (393 x 1 tiles) keeps 256.
        BN = n_tiles * ((M + 31) / 32) >= 120 ? 32 : std::min(BN, 128);
    }
    BN = std::min(bn_max, BN);
    const int m_tiles = (M + BN - 1) / BN;
    const int nkb = (K + BK - 1) / BK;
    int splits = 1, kb_per = nkb;
    const int tiles = m_tiles * n_tiles;
    if (tiles < 120) {
        // about one wave of CTAs; decode tiles exchange partials in [splits][128][CW] areas
        // that hold splits * CW <= BN + 32 columns
        const int s0 = std::max(1, std::min(std::min(nkb, BN <= 64 ? MAX_SPLITS : MAX_SPLITS_PULL),
                                            (148 + tiles - 1) / tiles));
        for (int s = s0; s >= 1; --s) {
            kb_per = (nkb + s - 1) / s;
            splits = (nkb + kb_per - 1) / kb_per;
            if (BN > 64 || splits * push_cw(BN, splits) <= BN + 32) break;
        }
    }
    const CUtensorMap* xh = xmap(p, x.hi, K, x.ld, BN);
    const CUtensorMap* xl = xmap(p, x.lo, K, x.ld, BN);
    if (!xh || !xl) return cudaErrorInvalidValue;
    TcParams tp;
    tp.w = w;
    tp.M = M;
    tp.nkb_total = nkb;
    tp.kb_per_split = kb_per;
    tp.splits = splits;
    tp.pre = wt.pre;
    tp.post = wt.post;
    tp.epi = e;
    tp.err = p.err;
    tp.fault = p.fault;
    tp.part = reinterpret_cast<float4*>(p.part);
    tp.products = p.products;
    tp.trace = nullptr;
    dim3 grid(n_tiles, m_tiles, splits);
    if (splits > 1 && BN > 64 && (size_t)n_tiles * m_tiles * splits * 128 * BN > p.part_floats)
        return cudaErrorInvalidValue;  // cannot happen: tiles < 120 and splits <= ceil(148 / tiles)
    GemmState& gs = *p.state;
    if (gs.trace && !gs.traced && w.rows == gs.trace_rows && w.cols == gs.trace_cols && M == gs.trace_m &&
        (size_t)grid.x * grid.y * grid.z <= 4096) {
        tp.trace = gs.trace;
        gs.traced = true;
        gs.trace_grid = grid;
    }
    if (presplit && BN == PB_BN && splits == 1 && !tp.trace) {
        static const bool off = std::getenv("GPT2Q_TC_NO_PERSISTENT") != nullptr;  // tuning
        if (!off) return launch_persistent(wt.hi, wt.lo, *xh, *xl, tp, n_tiles, n_tiles * m_tiles, st);
    }
    if (presplit) {
        if (w.atom == ATOM_Q8) return launch_bn<ATOM_Q8, true>(BN, wt.hi, wt.lo, *xh, *xl, tp, grid, st);
        return launch_bn<ATOM_Q4, true>(BN, wt.hi, wt.lo, *xh, *xl, tp, grid, st);
    }
    if (w.atom == ATOM_Q8) return launch_bn<ATOM_Q8, false>(BN, wt.raw, wt.raw, *xh, *xl, tp, grid, st);
    return launch_bn<ATOM_Q4, false>(BN, wt.raw, wt.raw, *xh, *xl, tp, grid, st);
}

bool head_i8_usable(const GemmPlan& p, const QW& w, int M) {
    if (!p.enabled || w.atom != ATOM_Q8 || M < 1 || M > 64 || w.cols % 64 != 0) return false;
    if (p.state->w.find(w.q) == p.state->w.end()) return false;
    return (M <= 32 ? HeadCfg<32>::smem(w.cols / 32) : HeadCfg<64>::smem(w.cols / 32)) <= 232448;
}

cudaError_t launch_head_i8(const GemmPlan& p, const QW& w, const uint8_t* pieces, const float* xscale, int M,
                           float* out, int ldo, cudaStream_t st) {
    if (!head_i8_usable(p, w, M)) return cudaErrorInvalidValue;
    const WeightTc& wt = p.state->w.find(w.q)->second;
    if (M <= 32) return launch_head_i8_mp<32>(wt.raw, pieces, xscale, w, M, out, ldo, p.err, st);
    return launch_head_i8_mp<64>(wt.raw, pieces, xscale, w, M, out, ldo, p.err, st);
}

std::string gemm_trace_json(const GemmPlan& p) {
    if (!p.state || !p.state->trace || !p.state->traced) return "";
    const dim3 g = p.state->trace_grid;
    const size_t n = (size_t)g.x * g.y * g.z;
    std::vector<unsigned long long> t(n * TC_TRACE);
    if (cudaMemcpy(t.data(), p.state->trace, t.size() * 8, cudaMemcpyDeviceToHost) != cudaSuccess) return "";
    unsigned long long t0 = ~0ull;
    for (auto v : t)
        if (v && v < t0) t0 = v;
    std::string s = "{\"grid\": [" + std::to_string(g.x) + ", " + std::to_string(g.y) + ", " + std::to_string(g.z) +
                    "], \"stamps\": [";
    for (size_t c = 0; c < n; ++c) {
        s += c ? ", [" : "[";
        for (int k = 0; k < TC_TRACE; ++k) {
            const unsigned long long v = t[c * TC_TRACE + k];
            s += (k ? ", " : "") + std::to_string(v ? (long long)(v - t0) : -1);
        }
        s += "]";
    }
    return s + "]}";
}

int gemm_take_error(GemmPlan& p, cudaStream_t st) {
    if (!p.enabled || !p.err) return 0;
    int h = 0;
    if (cudaMemcpyAsync(&h, p.err, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess) return -1;
    if (cudaStreamSynchronize(st) != cudaSuccess) return -1;
    if (h != 0) cudaMemsetAsync(p.err, 0, 4, st);
    return h;
}

}  // namespace gpt2q
