// Backward kernels of the GPT-2 trunk, batched over positions (fp32, sm_100a).
//
// The reference runs one GEMV-shaped launch per position and per op (gpu_backward.rs:651-790
// over cu/backward.cu); here every op takes all T positions of a sequence at once:
// * k_bwd_linear: the transposed product dX = dY . W as an outer-product accumulation. A CTA
//   owns 128 columns x 16 positions and a contiguous range of W's rows; each warp walks rows
//   (coalesced 128-byte row segments of the quantised payload, dequantised exactly in
//   registers) and broadcasts the staged dY values from shared memory. Row ranges are split
//   across CTAs so the grid fills the 148 SMs; the last CTA of each tile sums the splits in
//   fixed order and applies the epilogue (store, add, or GELU backward): deterministic.
// * k_bwd_linear_tc: the same product on the tensor cores as 3xTF32 (mma.sync m16n8k8), used
//   for long reductions (the tied head's 50257 rows) at 16 or more positions.
// * k_bwd_ln_warp: one warp per row held in registers, shuffle reductions (k_bwd_ln, one CTA
//   per row, for rows wider than 1600).
// * attention: one CTA per (query row, head) recomputes the probability row, the row's dP and
//   dq; one CTA per (key row, head) recomputes the column of P and dS from the saved row
//   statistics and sums dk and dv over the later queries (strided over the CTA's thread groups,
//   parts added in fixed order). For head dim 64 a whole row goes to one warp (the _w64
//   kernels). No floating-point atomics anywhere.
#include <cuda_runtime.h>

#include <cmath>
#include <string>
#include <vector>

#include "backward.h"
#include "gpt2q.h"

namespace gpt2q {

void set_global_error(const std::string& msg);

namespace {

constexpr int BL_COLS = 128;  // columns per CTA (4 per lane)
constexpr int BL_TT = 16;     // positions per CTA
constexpr int BL_RCH = 128;   // rows of dY staged per chunk (double-buffered)
constexpr int BL_WARPS = 8;
constexpr int BL_PAD = 20;    // row stride of the staged dY tile (floats; 16-byte aligned rows)
constexpr int BL_RB = 8;      // weight rows in flight per warp
constexpr int BL_PRE = BL_RCH * BL_TT / 256;  // dY values each thread prefetches per chunk
constexpr int ATT_MAX_T = 1024;
constexpr int ATT_MAX_HD = 128;

struct BwdSplit {
    int splits, rows_per_split, col_tiles, t_tiles;
};

BwdSplit bwd_split(int T, int rows, int cols) {
    BwdSplit s;
    s.col_tiles = (cols + BL_COLS - 1) / BL_COLS;
    s.t_tiles = (T + BL_TT - 1) / BL_TT;
    const int chunks = (rows + BL_RCH - 1) / BL_RCH;
    int want = (2 * 148 + s.col_tiles * s.t_tiles - 1) / (s.col_tiles * s.t_tiles);
    want = want < 1 ? 1 : (want > 64 ? 64 : want);
    if (want > chunks) want = chunks;
    const int ch_per = (chunks + want - 1) / want;
    s.rows_per_split = ch_per * BL_RCH;
    s.splits = (rows + s.rows_per_split - 1) / s.rows_per_split;
    if (s.splits < 1) s.splits = 1;
    return s;
}

// Raw weight words of W[r][c..c+3] as loaded (dequantised later, so the next batch's loads can
// be in flight while the current batch is consumed).
template <int ATOM>
struct WRaw {
    uint32_t q;
    float s;
};
template <>
struct WRaw<ATOM_F16> {
    uint2 v;
};
template <>
struct WRaw<ATOM_F32> {
    float4 v;
};

template <int ATOM>
__device__ __forceinline__ void raw_load(const QW& w, int r, int c, WRaw<ATOM>& o) {
    const uint8_t* row = w.q + (size_t)r * w.qstride;
    if constexpr (ATOM == ATOM_F32) {
        o.v = __ldg(reinterpret_cast<const float4*>(row) + (c >> 2));
    } else if constexpr (ATOM == ATOM_F16) {
        o.v = __ldg(reinterpret_cast<const uint2*>(row) + (c >> 2));
    } else if constexpr (ATOM == ATOM_Q8) {
        o.q = __ldg(reinterpret_cast<const uint32_t*>(row) + (c >> 2));
        o.s = __half2float(w.s[(size_t)r * w.sstride + (c >> 5)]);
    } else {
        const int g = c >> 5, e = c & 31;
        o.q = __ldg(reinterpret_cast<const uint32_t*>(row + g * 16 + (e & 15)));
        o.s = __half2float(w.s[(size_t)r * w.sstride + g]);
    }
}

template <int ATOM>
__device__ __forceinline__ void raw_zero(WRaw<ATOM>& o) {
    if constexpr (ATOM == ATOM_F32) {
        o.v = make_float4(0.f, 0.f, 0.f, 0.f);
    } else if constexpr (ATOM == ATOM_F16) {
        o.v = make_uint2(0u, 0u);
    } else {
        o.q = 0u;
        o.s = 0.f;
    }
}

// Exactly (float)q * scale for the quantised atoms (as Engine::vec_f32).
template <int ATOM>
__device__ __forceinline__ void raw_deq(const WRaw<ATOM>& o, int c, float f[4]) {
    if constexpr (ATOM == ATOM_F32) {
        f[0] = o.v.x, f[1] = o.v.y, f[2] = o.v.z, f[3] = o.v.w;
    } else if constexpr (ATOM == ATOM_F16) {
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&o.v.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&o.v.y));
        f[0] = a.x, f[1] = a.y, f[2] = b.x, f[3] = b.y;
    } else if constexpr (ATOM == ATOM_Q8) {
        i8x4_to_f32(o.q, f);
#pragma unroll
        for (int j = 0; j < 4; ++j) f[j] *= o.s;
    } else {
        float lo[4], hi[4];
        i4x8_to_f32(o.q, lo, hi);
        const bool low = (c & 31) < 16;
#pragma unroll
        for (int j = 0; j < 4; ++j) f[j] = (low ? lo[j] : hi[j]) * o.s;
    }
}

__device__ __forceinline__ float gelu_grad(float v) {
    // d/dv of 0.5 v (1 + tanh(u)), u = c (v + 0.044715 v^3), in cu/backward.cu:124-130's order
    const float u = 0.7978845608028654f * (v + 0.044715f * v * v * v);
    const float th = tanhf(u);
    const float sech2 = 1.f - th * th;
    return 0.5f * (1.f + th) + 0.5f * v * sech2 * 0.7978845608028654f * (1.f + 3.f * 0.044715f * v * v);
}

__device__ __forceinline__ void bwd_epi(int epi, float s, float* out, int ldo, const float* xpre, int ldx, int t,
                                        int c) {
    float* o = out + (size_t)t * ldo + c;
    if (epi == BWD_ADD)
        *o += s;
    else if (epi == BWD_GELU_BWD)
        *o = s * gelu_grad(xpre[(size_t)t * ldx + c]);
    else
        *o = s;
}

// dX = dY . W for 128 columns x 16 positions over this CTA's row range. dY is staged chunk by
// chunk into shared memory, the next chunk prefetched into registers while the current one is
// consumed; each warp keeps 8 weight rows in flight. The warps' partials are summed in warp
// order. With several row splits every CTA stores its partial and the last CTA of the tile
// (atomic ticket after a fence) sums the splits in split order and applies the epilogue, so the
// result does not depend on which CTA finishes last.
template <int ATOM>
__global__ void __launch_bounds__(256, 2) k_bwd_linear(QW w, const float* __restrict__ dY, int ldy, int T,
                                                       int rows_per_split, float* part, unsigned* counters,
                                                       int epi, float* out, int ldo, const float* xpre, int ldx) {
    // dY double buffer, then (after the main loop) the warp partials
    constexpr int SM_FLOATS = 2 * BL_RCH * BL_PAD > BL_WARPS * 8 * BL_COLS ? 2 * BL_RCH * BL_PAD : BL_WARPS * 8 * BL_COLS;
    __shared__ __align__(16) float sm[SM_FLOATS];
    __shared__ bool is_last;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c0 = blockIdx.x * BL_COLS, t0 = blockIdx.y * BL_TT;
    const int r_begin = blockIdx.z * rows_per_split;
    const int r_end = min(w.rows, r_begin + rows_per_split);
    const int c = c0 + 4 * lane;
    const bool cok = c < w.cols;
    float acc[BL_TT][4];
#pragma unroll
    for (int t = 0; t < BL_TT; ++t)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[t][j] = 0.f;

    float pre[BL_PRE];
    auto load_chunk = [&](int rc, int nr) {
#pragma unroll
        for (int k = 0; k < BL_PRE; ++k) {
            const int i = tid + k * 256, t = i / BL_RCH, r = i - t * BL_RCH;
            pre[k] = (t0 + t < T && r < nr) ? dY[(size_t)(t0 + t) * ldy + rc + r] : 0.f;
        }
    };
    auto store_chunk = [&](float* buf) {
#pragma unroll
        for (int k = 0; k < BL_PRE; ++k) {
            const int i = tid + k * 256, t = i / BL_RCH, r = i - t * BL_RCH;
            buf[r * BL_PAD + t] = pre[k];
        }
    };
    const int nchunks = r_end > r_begin ? (r_end - r_begin + BL_RCH - 1) / BL_RCH : 0;
    if (nchunks > 0) {
        load_chunk(r_begin, min(BL_RCH, r_end - r_begin));
        store_chunk(sm);
    }
    __syncthreads();
    // weights of the next batch (8 rows per warp, possibly in the next chunk) are loaded while
    // the current batch is consumed
    WRaw<ATOM> nxt[BL_RB];
    auto load_batch = [&](int rbase) {
#pragma unroll
        for (int k = 0; k < BL_RB; ++k) {
            const int r = rbase + warp + k * BL_WARPS;
            if (cok && r < r_end)
                raw_load<ATOM>(w, r, c, nxt[k]);
            else
                raw_zero<ATOM>(nxt[k]);
        }
    };
    load_batch(r_begin);
    for (int ci = 0; ci < nchunks; ++ci) {
        const int rc = r_begin + ci * BL_RCH;
        const int nr = min(BL_RCH, r_end - rc);
        const float* cur = sm + (ci & 1) * BL_RCH * BL_PAD;
        const bool more = ci + 1 < nchunks;
        if (more) load_chunk(rc + BL_RCH, min(BL_RCH, r_end - rc - BL_RCH));
        for (int rb = 0; rb < nr; rb += BL_RB * BL_WARPS) {
            WRaw<ATOM> wr[BL_RB];
#pragma unroll
            for (int k = 0; k < BL_RB; ++k) wr[k] = nxt[k];
            load_batch(rc + rb + BL_RB * BL_WARPS);
#pragma unroll
            for (int k = 0; k < BL_RB; ++k) {
                // rows past the range carry zero weights; their staged dY row is any row in bounds
                const int r = min(rb + warp + k * BL_WARPS, BL_RCH - 1);
                float f[4];
                raw_deq<ATOM>(wr[k], c, f);
                const float4* dv = reinterpret_cast<const float4*>(cur + r * BL_PAD);
#pragma unroll
                for (int q = 0; q < BL_TT / 4; ++q) {
                    const float4 y = dv[q];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        acc[4 * q + 0][j] = fmaf(y.x, f[j], acc[4 * q + 0][j]);
                        acc[4 * q + 1][j] = fmaf(y.y, f[j], acc[4 * q + 1][j]);
                        acc[4 * q + 2][j] = fmaf(y.z, f[j], acc[4 * q + 2][j]);
                        acc[4 * q + 3][j] = fmaf(y.w, f[j], acc[4 * q + 3][j]);
                    }
                }
            }
        }
        if (more) store_chunk(sm + ((ci + 1) & 1) * BL_RCH * BL_PAD);
        __syncthreads();
    }
    // warp partials summed in warp order, 8 positions per pass
    const bool split = gridDim.z > 1;
    float* mine = part + (size_t)blockIdx.z * T * w.cols;
    float* red = sm;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        __syncthreads();
#pragma unroll
        for (int t = 0; t < 8; ++t)
            *reinterpret_cast<float4*>(red + (warp * 8 + t) * BL_COLS + 4 * lane) =
                make_float4(acc[half * 8 + t][0], acc[half * 8 + t][1], acc[half * 8 + t][2], acc[half * 8 + t][3]);
        __syncthreads();
        for (int i = tid; i < 8 * BL_COLS; i += blockDim.x) {
            const int t = i / BL_COLS, cc = i - t * BL_COLS;
            const int tg = t0 + half * 8 + t, cg = c0 + cc;
            if (tg < T && cg < w.cols) {
                float v = 0.f;
#pragma unroll
                for (int wp = 0; wp < BL_WARPS; ++wp) v += red[(wp * 8 + t) * BL_COLS + cc];
                if (split)
                    mine[(size_t)tg * w.cols + cg] = v;
                else
                    bwd_epi(epi, v, out, ldo, xpre, ldx, tg, cg);
            }
        }
    }
    if (!split) return;
    __threadfence();
    __syncthreads();
    unsigned* ticket = counters + blockIdx.y * gridDim.x + blockIdx.x;
    if (tid == 0) is_last = atomicAdd(ticket, 1u) == gridDim.z - 1;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    const int tn = min(BL_TT, T - t0);
    for (int i = tid; i < tn * BL_COLS; i += blockDim.x) {
        const int t = i / BL_COLS, cc = i - t * BL_COLS;
        const int tg = t0 + t, cg = c0 + cc;
        if (cg < w.cols) {
            float v = 0.f;
            for (int z = 0; z < (int)gridDim.z; ++z) v += __ldcg(part + ((size_t)z * T + tg) * w.cols + cg);
            bwd_epi(epi, v, out, ldo, xpre, ldx, tg, cg);
        }
    }
    if (tid == 0) *ticket = 0u;  // ready for the next launch
}

// ---- the same transposed product on the tensor cores (3xTF32, mma.sync m16n8k8) ----
// Each operand is split x = hi + lo with hi = tf32(x) and lo = tf32(x - hi) (both rounded to
// nearest); hi*hi + hi*lo + lo*hi keeps about 21 bits, the fp32-level accuracy of the CUDA-core
// product, with fp32's exponent range (no scaling needed for small gradients). A CTA owns 64
// positions x 128 columns and a range of W's rows; per 32-row chunk the dequantised W and dY
// tiles are staged (split) in shared memory, the next chunk's raw loads in flight meanwhile,
// and warp w computes rows 16 (w % 4) .. + 15 against columns 64 (w / 4) .. + 63.
constexpr int TB_M = 64, TB_N = 128, TB_K = 32;
constexpr int TB_WS = TB_N + 8;  // W tile row stride (words): bank = 8 k + n, conflict-free fragments
constexpr int TB_YS = TB_K + 4;  // dY tile row stride (words): bank = 4 t + k
constexpr int TB_SMEM = (2 * TB_K * TB_WS + 2 * TB_M * TB_YS) * 4;

struct TbSplit {
    int splits, rows_per_split, col_tiles, m_tiles;
};

TbSplit tb_split(int T, int rows, int cols) {
    TbSplit s;
    s.col_tiles = (cols + TB_N - 1) / TB_N;
    s.m_tiles = (T + TB_M - 1) / TB_M;
    const int chunks = (rows + TB_K - 1) / TB_K;
    int want = (2 * 148 + s.col_tiles * s.m_tiles - 1) / (s.col_tiles * s.m_tiles);
    want = want < 1 ? 1 : (want > 64 ? 64 : want);
    // at least 8 chunks per CTA: the last CTA of a tile sums every split's partial tile
    const int by_len = chunks / 8 > 1 ? chunks / 8 : 1;
    if (want > by_len) want = by_len;
    s.rows_per_split = ((chunks + want - 1) / want) * TB_K;
    s.splits = (rows + s.rows_per_split - 1) / s.rows_per_split;
    if (s.splits < 1) s.splits = 1;
    return s;
}

__device__ __forceinline__ void tf32_split(float x, uint32_t& hi, uint32_t& lo) {
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(hi) : "f"(x));
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(lo) : "f"(x - __uint_as_float(hi)));
}

__device__ __forceinline__ void mma_tf32(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int ATOM>
__global__ void __launch_bounds__(256, 2) k_bwd_linear_tc(QW w, const float* __restrict__ dY, int ldy, int T,
                                                          int rows_per_split, float* part, unsigned* counters, int epi,
                                                          float* out, int ldo, const float* xpre, int ldx) {
    extern __shared__ __align__(16) uint32_t tb_sm[];
    uint32_t* Wh = tb_sm;                    // [TB_K][TB_WS]
    uint32_t* Wl = Wh + TB_K * TB_WS;        // [TB_K][TB_WS]
    uint32_t* Yh = Wl + TB_K * TB_WS;        // [TB_M][TB_YS]
    uint32_t* Yl = Yh + TB_M * TB_YS;        // [TB_M][TB_YS]
    __shared__ bool is_last;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
    const int c0 = blockIdx.x * TB_N, m0 = blockIdx.y * TB_M;
    const int r_begin = blockIdx.z * rows_per_split;
    const int r_end = min(w.rows, r_begin + rows_per_split);
    // staging roles: W row tid / 8 (of 32), columns 16 (tid % 8) .. + 15 (four quads);
    // dY position tid / 4 (of 64), k 8 (tid % 4) .. + 7
    const int wr = tid >> 3, wc = 16 * (tid & 7);
    const int yt = tid >> 2, yk = 8 * (tid & 3);
    WRaw<ATOM> raw[4];
    float yv[8];
    auto load = [&](int rc) {
        const int r = rc + wr;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int c = c0 + wc + 4 * q;
            if (r < r_end && c < w.cols)
                raw_load<ATOM>(w, r, c, raw[q]);
            else
                raw_zero<ATOM>(raw[q]);
        }
        const int tg = m0 + yt;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int k = rc + yk + u;
            yv[u] = (tg < T && k < r_end) ? dY[(size_t)tg * ldy + k] : 0.f;
        }
    };
    auto stage = [&]() {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            float f[4];
            raw_deq<ATOM>(raw[q], c0 + wc + 4 * q, f);
            uint4 h, l;
            tf32_split(f[0], h.x, l.x);
            tf32_split(f[1], h.y, l.y);
            tf32_split(f[2], h.z, l.z);
            tf32_split(f[3], h.w, l.w);
            *reinterpret_cast<uint4*>(Wh + wr * TB_WS + wc + 4 * q) = h;
            *reinterpret_cast<uint4*>(Wl + wr * TB_WS + wc + 4 * q) = l;
        }
#pragma unroll
        for (int u = 0; u < 8; u += 4) {
            uint4 h, l;
            tf32_split(yv[u], h.x, l.x);
            tf32_split(yv[u + 1], h.y, l.y);
            tf32_split(yv[u + 2], h.z, l.z);
            tf32_split(yv[u + 3], h.w, l.w);
            *reinterpret_cast<uint4*>(Yh + yt * TB_YS + yk + u) = h;
            *reinterpret_cast<uint4*>(Yl + yt * TB_YS + yk + u) = l;
        }
    };
    float acc[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[nt][j] = 0.f;
    const int mrow = 16 * (warp & 3), ncol = 64 * (warp >> 2);
    if (r_begin < r_end) load(r_begin);
    for (int rc = r_begin; rc < r_end; rc += TB_K) {
        stage();
        __syncthreads();
        if (rc + TB_K < r_end) load(rc + TB_K);  // next chunk's loads fly during the MMAs
#pragma unroll
        for (int ks = 0; ks < TB_K / 8; ++ks) {
            const int kk = 8 * ks + t4;
            const uint32_t ah0 = Yh[(mrow + g) * TB_YS + kk], ah1 = Yh[(mrow + g + 8) * TB_YS + kk];
            const uint32_t ah2 = Yh[(mrow + g) * TB_YS + kk + 4], ah3 = Yh[(mrow + g + 8) * TB_YS + kk + 4];
            const uint32_t al0 = Yl[(mrow + g) * TB_YS + kk], al1 = Yl[(mrow + g + 8) * TB_YS + kk];
            const uint32_t al2 = Yl[(mrow + g) * TB_YS + kk + 4], al3 = Yl[(mrow + g + 8) * TB_YS + kk + 4];
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                const int n = ncol + 8 * nt + g;
                const uint32_t bh0 = Wh[kk * TB_WS + n], bh1 = Wh[(kk + 4) * TB_WS + n];
                const uint32_t bl0 = Wl[kk * TB_WS + n], bl1 = Wl[(kk + 4) * TB_WS + n];
                mma_tf32(acc[nt], al0, al1, al2, al3, bh0, bh1);
                mma_tf32(acc[nt], ah0, ah1, ah2, ah3, bl0, bl1);
                mma_tf32(acc[nt], ah0, ah1, ah2, ah3, bh0, bh1);
            }
        }
        __syncthreads();  // the tiles are restaged next
    }
    // C fragment: rows mrow + g (+ 8), columns ncol + 8 nt + 2 t4 (+ 1)
    const bool split = gridDim.z > 1;
    float* mine = part + (size_t)blockIdx.z * T * w.cols;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int tg = m0 + mrow + g + ((j & 2) ? 8 : 0);
            const int cg = c0 + ncol + 8 * nt + 2 * t4 + (j & 1);
            if (tg < T && cg < w.cols) {
                if (split)
                    mine[(size_t)tg * w.cols + cg] = acc[nt][j];
                else
                    bwd_epi(epi, acc[nt][j], out, ldo, xpre, ldx, tg, cg);
            }
        }
    if (!split) return;
    __threadfence();
    __syncthreads();
    unsigned* ticket = counters + blockIdx.y * gridDim.x + blockIdx.x;
    if (tid == 0) is_last = atomicAdd(ticket, 1u) == gridDim.z - 1;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    const int tn = min(TB_M, T - m0);
    for (int i = tid; i < tn * TB_N; i += blockDim.x) {
        const int tt = i / TB_N, cc = i - tt * TB_N;
        const int tg = m0 + tt, cg = c0 + cc;
        if (cg < w.cols) {
            float v = 0.f;
            for (int z = 0; z < (int)gridDim.z; ++z) v += __ldcg(part + ((size_t)z * T + tg) * w.cols + cg);
            bwd_epi(epi, v, out, ldo, xpre, ldx, tg, cg);
        }
    }
    if (tid == 0) *ticket = 0u;  // ready for the next launch
}


// Sum over the block in fixed order (warp shuffles, then warp 0 over the warps' sums).
__device__ float block_sum(float v, float* red) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    float s = 0.f;
    for (int i = 0; i < nw; ++i) s += red[i];
    return s;
}

__device__ float block_max(float v, float* red) {
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    float m = -1e30f;
    for (int i = 0; i < nw; ++i) m = fmaxf(m, red[i]);
    return m;
}

// LayerNorm backward of one row per CTA (cu/backward.cu:38-115): mean and population variance
// recomputed from the saved input, then
// dx = rstd * (dy*g - mean(dy*g) - xhat * mean(dy*g*xhat)).
__global__ void __launch_bounds__(256) k_bwd_ln(const float* __restrict__ dY, int ldy, const float* __restrict__ X,
                                                int ldx, const float* __restrict__ g, float eps, int n, int epi,
                                                float* __restrict__ out, int ldo, float* dg, float* db) {
    __shared__ float red[32];
    const int t = blockIdx.x;
    const float* x = X + (size_t)t * ldx;
    const float* dy = dY + (size_t)t * ldy;
    float s = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s += x[i];
    const float mean = block_sum(s, red) / (float)n;
    float sq = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = x[i] - mean;
        sq = fmaf(v, v, sq);
    }
    const float rstd = 1.0f / sqrtf(block_sum(sq, red) / (float)n + eps);
    float a = 0.f, cc = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float dh = dy[i] * g[i];
        a += dh;
        cc = fmaf(dh, (x[i] - mean) * rstd, cc);
    }
    const float mdxh = block_sum(a, red) / (float)n;
    const float mdxh_xh = block_sum(cc, red) / (float)n;
    float* o = out + (size_t)t * ldo;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float xh = (x[i] - mean) * rstd;
        const float dh = dy[i] * g[i];
        const float v = rstd * (dh - mdxh - xh * mdxh_xh);
        if (epi == BWD_ADD)
            o[i] += v;
        else
            o[i] = v;
        if (dg) dg[i] += dy[i] * xh;
        if (db) db[i] += dy[i];
    }
}

// The same LayerNorm backward with one warp per row (rows of up to 32 * NPL features held in
// registers, reductions by shuffles only), one single-warp CTA per row so the rows spread over
// the SMs.
template <int NPL>
__global__ void __launch_bounds__(32) k_bwd_ln_warp(const float* __restrict__ dY, int ldy,
                                                     const float* __restrict__ X, int ldx,
                                                     const float* __restrict__ g, float eps, int n, int T, int epi,
                                                     float* __restrict__ out, int ldo, float* dg, float* db) {
    const int t = blockIdx.x, lane = threadIdx.x;
    if (t >= T) return;
    const float* x = X + (size_t)t * ldx;
    const float* dy = dY + (size_t)t * ldy;
    auto wsum = [](float v) {
#pragma unroll
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        return v;
    };
    float xv[NPL], dh[NPL];
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < NPL; ++k) {
        const int i = lane + 32 * k;
        xv[k] = i < n ? x[i] : 0.f;
        dh[k] = i < n ? dy[i] * g[i] : 0.f;
        s += xv[k];
    }
    const float mean = wsum(s) / (float)n;
    float sq = 0.f;
#pragma unroll
    for (int k = 0; k < NPL; ++k) {
        const float v = lane + 32 * k < n ? xv[k] - mean : 0.f;
        sq = fmaf(v, v, sq);
    }
    const float rstd = 1.0f / sqrtf(wsum(sq) / (float)n + eps);
    float a = 0.f, cc = 0.f;
#pragma unroll
    for (int k = 0; k < NPL; ++k) {
        if (lane + 32 * k < n) {
            a += dh[k];
            cc = fmaf(dh[k], (xv[k] - mean) * rstd, cc);
        }
    }
    const float mdxh = wsum(a) / (float)n;
    const float mdxh_xh = wsum(cc) / (float)n;
    float* o = out + (size_t)t * ldo;
#pragma unroll
    for (int k = 0; k < NPL; ++k) {
        const int i = lane + 32 * k;
        if (i < n) {
            const float xh = (xv[k] - mean) * rstd;
            const float v = rstd * (dh[k] - mdxh - xh * mdxh_xh);
            if (epi == BWD_ADD)
                o[i] += v;
            else
                o[i] = v;
            if (dg) dg[i] += dy[i] * xh;
            if (db) db[i] += dy[i];
        }
    }
}

__global__ void k_gelu_fwd(const float* __restrict__ x, float* __restrict__ out, __half* ohi, __half* olo, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float g = gelu_tanh(x[i]);
        out[i] = g;
        if (ohi) split_hl(g, ohi[i], olo[i]);
    }
}

__global__ void k_gelu_bwd(const float* __restrict__ x, const float* __restrict__ dy, float* __restrict__ dx,
                           size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dx[i] = dy[i] * gelu_grad(x[i]);
}

// Scaled score and dot products shared by the attention kernels (same operands, same order,
// so the probability recomputed by the key-row kernel equals the query-row kernel's).
// HD > 0 fixes the head dim at compile time (loads batched by full unrolling); HD == 0 reads hd.
template <int HD>
__device__ __forceinline__ float dot_hd(const float* a, const float* b, int hd) {
    float d = 0.f;
    if (HD > 0) {
#pragma unroll
        for (int t = 0; t < HD; ++t) d = fmaf(a[t], b[t], d);
    } else {
        for (int t = 0; t < hd; ++t) d = fmaf(a[t], b[t], d);
    }
    return d;
}

// Query row i of head h: P row (causal, j <= i), out_i = sum_j P_ij v_j.
template <int HD>
__global__ void __launch_bounds__(128) k_attn_fwd_train(const float* __restrict__ q, int ldq,
                                                        const float* __restrict__ k, int ldk,
                                                        const float* __restrict__ v, int ldv, int hd, float scale,
                                                        float* __restrict__ out, int ldo, __half* ohi, __half* olo) {
    __shared__ float qs[ATT_MAX_HD];
    __shared__ float sc[ATT_MAX_T];
    __shared__ float red[32];
    __shared__ float pp[128];  // per-part partial sums (blockDim floats)
    const int i = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
    const size_t base = (size_t)h * hd;
    for (int t = tid; t < hd; t += blockDim.x) qs[t] = q[(size_t)i * ldq + base + t];
    __syncthreads();
    float mx = -1e30f;
    for (int j = tid; j <= i; j += blockDim.x) {
        const float s = dot_hd<HD>(qs, k + (size_t)j * ldk + base, hd) * scale;
        sc[j] = s;
        mx = fmaxf(mx, s);
    }
    const float m = block_max(mx, red);
    float ls = 0.f;
    for (int j = tid; j <= i; j += blockDim.x) {
        const float e = expf(sc[j] - m);
        sc[j] = e;
        ls += e;
    }
    const float L = block_sum(ls, red);
    for (int j = tid; j <= i; j += blockDim.x) sc[j] = sc[j] / L;
    __syncthreads();
    // out_t = sum_j P_j v_j[t]: the blockDim / hd thread groups take j = part, part + parts, ...
    // (more loads in flight), then the parts are added in part order
    const int parts = blockDim.x / hd, t = tid % hd, part = tid / hd;
    if (part < parts) {
        float o = 0.f;
#pragma unroll 8
        for (int j = part; j <= i; j += parts) o = fmaf(sc[j], v[(size_t)j * ldv + base + t], o);
        pp[part * hd + t] = o;
    }
    __syncthreads();
    if (tid < hd) {
        float o = 0.f;
        for (int q = 0; q < parts; ++q) o += pp[q * hd + tid];
        out[(size_t)i * ldo + base + tid] = o;
        if (ohi) split_hl(o, ohi[(size_t)i * ldo + base + tid], olo[(size_t)i * ldo + base + tid]);
    }
}

// Query row i of head h: P row, dP_j = dy_i . v_j, rs = sum_j dP_j P_j,
// dS_j = (dP_j - rs) P_j scale, dq_i = sum_j dS_j k_j. Saves (m, L, rs) for the key-row pass.
template <int HD>
__global__ void __launch_bounds__(128) k_attn_bwd_rows(const float* __restrict__ q, int ldq,
                                                       const float* __restrict__ k, int ldk,
                                                       const float* __restrict__ v, int ldv,
                                                       const float* __restrict__ dy, int lddy, int T, int hd,
                                                       float scale, float* __restrict__ dq, int lddq,
                                                       float* __restrict__ stats) {
    __shared__ float qs[ATT_MAX_HD], dys[ATT_MAX_HD];
    __shared__ float sc[ATT_MAX_T], dp[ATT_MAX_T];
    __shared__ float red[32];
    __shared__ float pp[128];  // per-part partial sums (blockDim floats)
    const int i = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
    const size_t base = (size_t)h * hd;
    for (int t = tid; t < hd; t += blockDim.x) {
        qs[t] = q[(size_t)i * ldq + base + t];
        dys[t] = dy[(size_t)i * lddy + base + t];
    }
    __syncthreads();
    float mx = -1e30f;
    for (int j = tid; j <= i; j += blockDim.x) {
        const float s = dot_hd<HD>(qs, k + (size_t)j * ldk + base, hd) * scale;
        sc[j] = s;
        mx = fmaxf(mx, s);
    }
    const float m = block_max(mx, red);
    float ls = 0.f;
    for (int j = tid; j <= i; j += blockDim.x) {
        const float e = expf(sc[j] - m);
        sc[j] = e;
        ls += e;
    }
    const float L = block_sum(ls, red);
    float rsp = 0.f;
    for (int j = tid; j <= i; j += blockDim.x) {
        const float p = sc[j] / L;
        sc[j] = p;
        const float d = dot_hd<HD>(dys, v + (size_t)j * ldv + base, hd);
        dp[j] = d;
        rsp = fmaf(d, p, rsp);
    }
    const float rs = block_sum(rsp, red);
    for (int j = tid; j <= i; j += blockDim.x) dp[j] = (dp[j] - rs) * sc[j] * scale;
    __syncthreads();
    const int parts = blockDim.x / hd, t = tid % hd, part = tid / hd;
    if (part < parts) {
        float a = 0.f;
#pragma unroll 8
        for (int j = part; j <= i; j += parts) a = fmaf(dp[j], k[(size_t)j * ldk + base + t], a);
        pp[part * hd + t] = a;
    }
    __syncthreads();
    if (tid < hd) {
        float a = 0.f;
        for (int q = 0; q < parts; ++q) a += pp[q * hd + tid];
        dq[(size_t)i * lddq + base + tid] = a;
    }
    if (tid == 0) {
        float* st = stats + ((size_t)h * T + i) * 3;
        st[0] = m;
        st[1] = L;
        st[2] = rs;
    }
}

// Key row j of head h: P_ij and dS_ij for i >= j from the saved row statistics, then
// dk_j = sum_i dS_ij q_i and dv_j = sum_i P_ij dy_i (thread groups take interleaved i; their
// partial sums are added in group order).
template <int HD>
__global__ void __launch_bounds__(128) k_attn_bwd_keys(const float* __restrict__ q, int ldq,
                                                       const float* __restrict__ k, int ldk,
                                                       const float* __restrict__ v, int ldv,
                                                       const float* __restrict__ dy, int lddy, int T, int hd,
                                                       float scale, const float* __restrict__ stats, float* dk,
                                                       int lddk, float* dv, int lddv, int accumulate) {
    __shared__ float ks[ATT_MAX_HD], vs[ATT_MAX_HD];
    __shared__ float pv[ATT_MAX_T], dsv[ATT_MAX_T];
    __shared__ float pp[128], pb[128];  // per-part partial sums of dk and dv
    const int j = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
    const size_t base = (size_t)h * hd;
    for (int t = tid; t < hd; t += blockDim.x) {
        ks[t] = k[(size_t)j * ldk + base + t];
        vs[t] = v[(size_t)j * ldv + base + t];
    }
    __syncthreads();
    for (int i = j + tid; i < T; i += blockDim.x) {
        const float* st = stats + ((size_t)h * T + i) * 3;
        const float s = dot_hd<HD>(q + (size_t)i * ldq + base, ks, hd) * scale;
        const float p = expf(s - st[0]) / st[1];
        const float d = dot_hd<HD>(dy + (size_t)i * lddy + base, vs, hd);
        pv[i] = p;
        dsv[i] = (d - st[2]) * p * scale;
    }
    __syncthreads();
    const int parts = blockDim.x / hd, t = tid % hd, part = tid / hd;
    if (part < parts) {
        float a = 0.f, b = 0.f;
#pragma unroll 8
        for (int i = j + part; i < T; i += parts) {
            a = fmaf(dsv[i], q[(size_t)i * ldq + base + t], a);
            b = fmaf(pv[i], dy[(size_t)i * lddy + base + t], b);
        }
        pp[part * hd + t] = a;
        pb[part * hd + t] = b;
    }
    __syncthreads();
    if (tid < hd) {
        float* dkp = dk + (size_t)j * lddk + base + tid;
        float* dvp = dv + (size_t)j * lddv + base + tid;
        float a = 0.f, b = 0.f;
        for (int q2 = 0; q2 < parts; ++q2) {
            a += pp[q2 * hd + tid];
            b += pb[q2 * hd + tid];
        }
        *dkp = accumulate ? *dkp + a : a;
        *dvp = accumulate ? *dvp + b : b;
    }
}

// ---- head dim 64: a warp takes a whole row (lane l: dimensions 2l, 2l+1), so a row is one
// coalesced 256-byte load; dot products reduce by an xor shuffle tree whose result every lane
// holds. The query-row and key-row kernels call wdot64 with the same operands in the same
// order, so the probabilities and dS the key-row kernel recomputes are the query-row kernel's.
__device__ __forceinline__ float wdot64(float2 a, float2 b) {
    float s = fmaf(a.y, b.y, a.x * b.x);
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    return s;
}

__device__ __forceinline__ float2 ld2(const float* p) { return *reinterpret_cast<const float2*>(p); }

__global__ void __launch_bounds__(128) k_attn_fwd_w64(const float* __restrict__ q, int ldq,
                                                      const float* __restrict__ k, int ldk,
                                                      const float* __restrict__ v, int ldv, float scale,
                                                      float* __restrict__ out, int ldo, __half* ohi, __half* olo) {
    __shared__ float sc[ATT_MAX_T];
    __shared__ float red[32];
    __shared__ float2 part[4][32];
    const int i = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const size_t base = (size_t)blockIdx.y * 64 + 2 * lane;
    const float2 qv = ld2(q + (size_t)i * ldq + base);
    float mx = -1e30f;
#pragma unroll 4
    for (int j = warp; j <= i; j += 4) {
        const float s = wdot64(qv, ld2(k + (size_t)j * ldk + base)) * scale;
        if (lane == 0) sc[j] = s;
        mx = fmaxf(mx, s);
    }
    const float m = block_max(mx, red);
    float ls = 0.f;
    for (int j = tid; j <= i; j += blockDim.x) {
        const float e = expf(sc[j] - m);
        sc[j] = e;
        ls += e;
    }
    const float L = block_sum(ls, red);
    for (int j = tid; j <= i; j += blockDim.x) sc[j] = sc[j] / L;
    __syncthreads();
    float2 o = make_float2(0.f, 0.f);
#pragma unroll 4
    for (int j = warp; j <= i; j += 4) {
        const float2 vv = ld2(v + (size_t)j * ldv + base);
        const float p = sc[j];
        o.x = fmaf(p, vv.x, o.x);
        o.y = fmaf(p, vv.y, o.y);
    }
    part[warp][lane] = o;
    __syncthreads();
    if (warp == 0) {
        float2 r = part[0][lane];
#pragma unroll
        for (int w = 1; w < 4; ++w) {
            r.x += part[w][lane].x;
            r.y += part[w][lane].y;
        }
        const size_t oi = (size_t)i * ldo + base;
        *reinterpret_cast<float2*>(out + oi) = r;
        if (ohi) {
            split_hl(r.x, ohi[oi], olo[oi]);
            split_hl(r.y, ohi[oi + 1], olo[oi + 1]);
        }
    }
}

__global__ void __launch_bounds__(128) k_attn_bwd_rows_w64(const float* __restrict__ q, int ldq,
                                                           const float* __restrict__ k, int ldk,
                                                           const float* __restrict__ v, int ldv,
                                                           const float* __restrict__ dy, int lddy, int T, float scale,
                                                           float* __restrict__ dq, int lddq,
                                                           float* __restrict__ stats) {
    __shared__ float sc[ATT_MAX_T], dp[ATT_MAX_T];
    __shared__ float red[32];
    __shared__ float2 part[4][32];
    const int i = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const size_t base = (size_t)h * 64 + 2 * lane;
    const float2 qv = ld2(q + (size_t)i * ldq + base);
    const float2 dyv = ld2(dy + (size_t)i * lddy + base);
    float mx = -1e30f;
#pragma unroll 4
    for (int j = warp; j <= i; j += 4) {
        const float s = wdot64(qv, ld2(k + (size_t)j * ldk + base)) * scale;
        if (lane == 0) sc[j] = s;
        mx = fmaxf(mx, s);
    }
    const float m = block_max(mx, red);
    float ls = 0.f;
    for (int j = tid; j <= i; j += blockDim.x) {
        const float e = expf(sc[j] - m);
        sc[j] = e;
        ls += e;
    }
    const float L = block_sum(ls, red);
    for (int j = tid; j <= i; j += blockDim.x) sc[j] = sc[j] / L;
    __syncthreads();
    float rsp = 0.f;
#pragma unroll 4
    for (int j = warp; j <= i; j += 4) {
        const float d = wdot64(dyv, ld2(v + (size_t)j * ldv + base));
        if (lane == 0) dp[j] = d;
        rsp = fmaf(d, sc[j], rsp);
    }
    const float rs = block_sum(lane == 0 ? rsp : 0.f, red);
    for (int j = tid; j <= i; j += blockDim.x) dp[j] = (dp[j] - rs) * sc[j] * scale;
    __syncthreads();
    float2 a = make_float2(0.f, 0.f);
#pragma unroll 4
    for (int j = warp; j <= i; j += 4) {
        const float2 kv = ld2(k + (size_t)j * ldk + base);
        const float ds = dp[j];
        a.x = fmaf(ds, kv.x, a.x);
        a.y = fmaf(ds, kv.y, a.y);
    }
    part[warp][lane] = a;
    __syncthreads();
    if (warp == 0) {
        float2 r = part[0][lane];
#pragma unroll
        for (int w = 1; w < 4; ++w) {
            r.x += part[w][lane].x;
            r.y += part[w][lane].y;
        }
        *reinterpret_cast<float2*>(dq + (size_t)i * lddq + base) = r;
    }
    if (tid == 0) {
        float* st = stats + ((size_t)h * T + i) * 3;
        st[0] = m;
        st[1] = L;
        st[2] = rs;
    }
}

__global__ void __launch_bounds__(128) k_attn_bwd_keys_w64(const float* __restrict__ q, int ldq,
                                                           const float* __restrict__ k, int ldk,
                                                           const float* __restrict__ v, int ldv,
                                                           const float* __restrict__ dy, int lddy, int T, float scale,
                                                           const float* __restrict__ stats, float* dk, int lddk,
                                                           float* dv, int lddv, int accumulate) {
    __shared__ float2 pk[4][32], pv[4][32];
    const int j = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const size_t base = (size_t)h * 64 + 2 * lane;
    const float2 kj = ld2(k + (size_t)j * ldk + base);
    const float2 vj = ld2(v + (size_t)j * ldv + base);
    float2 a = make_float2(0.f, 0.f), b = make_float2(0.f, 0.f);
#pragma unroll 4
    for (int i = j + warp; i < T; i += 4) {
        const float* st = stats + ((size_t)h * T + i) * 3;
        const float2 qv = ld2(q + (size_t)i * ldq + base);
        const float2 dyv = ld2(dy + (size_t)i * lddy + base);
        const float s = wdot64(qv, kj) * scale;
        const float p = expf(s - st[0]) / st[1];
        const float d = wdot64(dyv, vj);
        const float ds = (d - st[2]) * p * scale;
        a.x = fmaf(ds, qv.x, a.x);
        a.y = fmaf(ds, qv.y, a.y);
        b.x = fmaf(p, dyv.x, b.x);
        b.y = fmaf(p, dyv.y, b.y);
    }
    pk[warp][lane] = a;
    pv[warp][lane] = b;
    __syncthreads();
    if (warp == 0) {
        float2 ra = pk[0][lane], rb = pv[0][lane];
#pragma unroll
        for (int w = 1; w < 4; ++w) {
            ra.x += pk[w][lane].x;
            ra.y += pk[w][lane].y;
            rb.x += pv[w][lane].x;
            rb.y += pv[w][lane].y;
        }
        float2* dkp = reinterpret_cast<float2*>(dk + (size_t)j * lddk + base);
        float2* dvp = reinterpret_cast<float2*>(dv + (size_t)j * lddv + base);
        if (accumulate) {
            const float2 ok = *dkp, ov = *dvp;
            ra.x += ok.x;
            ra.y += ok.y;
            rb.x += ov.x;
            rb.y += ov.y;
        }
        *dkp = ra;
        *dvp = rb;
    }
}

int grid_1d(size_t n, int block) {
    size_t g = (n + block - 1) / block;
    if (g > 148 * 16) g = 148 * 16;
    return g < 1 ? 1 : (int)g;
}

}  // namespace

// The tensor-core kernel serves T >= 16 positions over long reductions (W with at least 8192
// rows: the tied head). Measured at 64 positions: head 404 -> 207 us; on the per-layer weights
// (768 .. 3072 rows) it was slower than the CUDA-core kernel (c_fc 34 -> 66 us with 2 chunks per
// CTA, 58 us with 8), its per-chunk staging and mma.sync issue costing more than the CUDA-core
// kernel's whole pass.
constexpr int BWD_TC_MIN_T = 16, BWD_TC_MIN_ROWS = 8192;

bool use_tc(int T, int rows) { return T >= BWD_TC_MIN_T && rows >= BWD_TC_MIN_ROWS; }

size_t bwd_linear_part_floats(int T, int rows, int cols) {
    const BwdSplit s = bwd_split(T, rows, cols);
    const TbSplit b = tb_split(T, rows, cols);
    const int splits = use_tc(T, rows) ? b.splits : s.splits;
    return splits > 1 ? (size_t)splits * T * cols : 1;
}

size_t bwd_linear_counters(int T, int cols) {
    const size_t simt = (size_t)((cols + BL_COLS - 1) / BL_COLS) * ((T + BL_TT - 1) / BL_TT);
    const size_t tc = (size_t)((cols + TB_N - 1) / TB_N) * ((T + TB_M - 1) / TB_M);
    return simt > tc ? simt : tc;
}

template <int ATOM>
cudaError_t launch_bwd_tc(const QW& w, const float* dY, int ldy, int T, float* part, unsigned* counters, int epi,
                          float* out, int ldo, const float* xpre, int ldx, cudaStream_t st) {
    static bool attr[64] = {};  // the attribute is per device: once per instantiation and device
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64 || !attr[dev]) {
        e = cudaFuncSetAttribute(k_bwd_linear_tc<ATOM>, cudaFuncAttributeMaxDynamicSharedMemorySize, TB_SMEM);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr[dev] = true;
    }
    const TbSplit s = tb_split(T, w.rows, w.cols);
    k_bwd_linear_tc<ATOM><<<dim3(s.col_tiles, s.m_tiles, s.splits), 256, TB_SMEM, st>>>(
        w, dY, ldy, T, s.rows_per_split, part, counters, epi, out, ldo, xpre, ldx);
    return cudaGetLastError();
}

cudaError_t launch_bwd_linear(const QW& w, const float* dY, int ldy, int T, float* part, unsigned* counters, int epi,
                              float* out, int ldo, const float* xpre, int ldx, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (w.cols % 4 != 0) return cudaErrorInvalidValue;
    if (use_tc(T, w.rows)) {
        switch (w.atom) {
            case ATOM_Q8: return launch_bwd_tc<ATOM_Q8>(w, dY, ldy, T, part, counters, epi, out, ldo, xpre, ldx, st);
            case ATOM_Q4: return launch_bwd_tc<ATOM_Q4>(w, dY, ldy, T, part, counters, epi, out, ldo, xpre, ldx, st);
            case ATOM_F16: return launch_bwd_tc<ATOM_F16>(w, dY, ldy, T, part, counters, epi, out, ldo, xpre, ldx, st);
            default: return launch_bwd_tc<ATOM_F32>(w, dY, ldy, T, part, counters, epi, out, ldo, xpre, ldx, st);
        }
    }
    const BwdSplit s = bwd_split(T, w.rows, w.cols);
    const dim3 grid(s.col_tiles, s.t_tiles, s.splits), block(256);
    switch (w.atom) {
        case ATOM_Q8:
            k_bwd_linear<ATOM_Q8><<<grid, block, 0, st>>>(w, dY, ldy, T, s.rows_per_split, part, counters, epi, out,
                                                          ldo, xpre, ldx);
            break;
        case ATOM_Q4:
            k_bwd_linear<ATOM_Q4><<<grid, block, 0, st>>>(w, dY, ldy, T, s.rows_per_split, part, counters, epi, out,
                                                          ldo, xpre, ldx);
            break;
        case ATOM_F16:
            k_bwd_linear<ATOM_F16><<<grid, block, 0, st>>>(w, dY, ldy, T, s.rows_per_split, part, counters, epi, out,
                                                           ldo, xpre, ldx);
            break;
        default:
            k_bwd_linear<ATOM_F32><<<grid, block, 0, st>>>(w, dY, ldy, T, s.rows_per_split, part, counters, epi, out,
                                                           ldo, xpre, ldx);
            break;
    }
    return cudaGetLastError();
}

cudaError_t launch_bwd_ln(const float* dY, int ldy, const float* x, int ldx, const float* g, float eps, int n, int T,
                          int epi, float* out, int ldo, float* dg, float* db, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if ((dg || db) && T != 1) return cudaErrorInvalidValue;
    if (n <= 256)
        k_bwd_ln_warp<8><<<T, 32, 0, st>>>(dY, ldy, x, ldx, g, eps, n, T, epi, out, ldo, dg, db);
    else if (n <= 768)
        k_bwd_ln_warp<24><<<T, 32, 0, st>>>(dY, ldy, x, ldx, g, eps, n, T, epi, out, ldo, dg, db);
    else if (n <= 1024)
        k_bwd_ln_warp<32><<<T, 32, 0, st>>>(dY, ldy, x, ldx, g, eps, n, T, epi, out, ldo, dg, db);
    else if (n <= 1600)
        k_bwd_ln_warp<50><<<T, 32, 0, st>>>(dY, ldy, x, ldx, g, eps, n, T, epi, out, ldo, dg, db);
    else
        k_bwd_ln<<<T, 256, 0, st>>>(dY, ldy, x, ldx, g, eps, n, epi, out, ldo, dg, db);
    return cudaGetLastError();
}

cudaError_t launch_gelu_fwd(const float* x, float* out, __half* ohi, __half* olo, size_t n, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    k_gelu_fwd<<<grid_1d(n, 256), 256, 0, st>>>(x, out, ohi, olo, n);
    return cudaGetLastError();
}

cudaError_t launch_gelu_bwd(const float* x, const float* dy, float* dx, size_t n, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    k_gelu_bwd<<<grid_1d(n, 256), 256, 0, st>>>(x, dy, dx, n);
    return cudaGetLastError();
}

cudaError_t launch_attn_fwd_train(const float* q, int ldq, const float* k, int ldk, const float* v, int ldv, int T,
                                  int n_head, int hd, float* out, int ldo, __half* ohi, __half* olo, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (T > ATT_MAX_T || hd > ATT_MAX_HD || hd <= 0 || n_head <= 0) return cudaErrorInvalidValue;
    const float scale = 1.0f / sqrtf((float)hd);
    const bool even = ((ldq | ldk | ldv | ldo) & 1) == 0 &&
                      (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) & 7) == 0;
    if (hd == 64 && even)
        k_attn_fwd_w64<<<dim3(T, n_head), 128, 0, st>>>(q, ldq, k, ldk, v, ldv, scale, out, ldo, ohi, olo);
    else if (hd == 64)
        k_attn_fwd_train<64><<<dim3(T, n_head), 128, 0, st>>>(q, ldq, k, ldk, v, ldv, hd, scale, out, ldo, ohi, olo);
    else
        k_attn_fwd_train<0><<<dim3(T, n_head), 128, 0, st>>>(q, ldq, k, ldk, v, ldv, hd, scale, out, ldo, ohi, olo);
    return cudaGetLastError();
}

cudaError_t launch_attn_bwd_train(const float* q, int ldq, const float* k, int ldk, const float* v, int ldv,
                                  const float* dy, int lddy, int T, int n_head, int hd, float* dq, int lddq, float* dk,
                                  int lddk, float* dv, int lddv, int accumulate, float* stats, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (T > ATT_MAX_T || hd > ATT_MAX_HD || hd <= 0 || n_head <= 0) return cudaErrorInvalidValue;
    const float scale = 1.0f / sqrtf((float)hd);
    const dim3 grid(T, n_head);
    const bool even = ((ldq | ldk | ldv | lddy | lddq | lddk | lddv) & 1) == 0 &&
                      (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)dy | (uintptr_t)dq | (uintptr_t)dk |
                        (uintptr_t)dv) & 7) == 0;
    if (hd == 64 && even) {
        k_attn_bwd_rows_w64<<<grid, 128, 0, st>>>(q, ldq, k, ldk, v, ldv, dy, lddy, T, scale, dq, lddq, stats);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        k_attn_bwd_keys_w64<<<grid, 128, 0, st>>>(q, ldq, k, ldk, v, ldv, dy, lddy, T, scale, stats, dk, lddk, dv,
                                                  lddv, accumulate);
        return cudaGetLastError();
    }
    if (hd == 64)
        k_attn_bwd_rows<64><<<grid, 128, 0, st>>>(q, ldq, k, ldk, v, ldv, dy, lddy, T, hd, scale, dq, lddq, stats);
    else
        k_attn_bwd_rows<0><<<grid, 128, 0, st>>>(q, ldq, k, ldk, v, ldv, dy, lddy, T, hd, scale, dq, lddq, stats);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if (hd == 64)
        k_attn_bwd_keys<64><<<grid, 128, 0, st>>>(q, ldq, k, ldk, v, ldv, dy, lddy, T, hd, scale, stats, dk, lddk, dv,
                                                  lddv, accumulate);
    else
        k_attn_bwd_keys<0><<<grid, 128, 0, st>>>(q, ldq, k, ldk, v, ldv, dy, lddy, T, hd, scale, stats, dk, lddk, dv,
                                                 lddv, accumulate);
    return cudaGetLastError();
}

}  // namespace gpt2q

// =================================================================== per-op C-ABI
// Host-slice operations with the BwdOps signatures (gpu_backward.rs:69-93): every call uploads
// its inputs, runs the kernel on `device` and downloads the outputs, like GpuBackward's
// trait methods (gpu_backward.rs:307-377).
using namespace gpt2q;

namespace {

struct Scratch {
    std::vector<void*> ptrs;
    cudaStream_t st = nullptr;
    cudaError_t err = cudaSuccess;
    ~Scratch() {
        if (st) cudaStreamSynchronize(st);
        for (void* p : ptrs) cudaFree(p);
        if (st) cudaStreamDestroy(st);
    }
    float* up(const float* h, size_t n) {
        float* d = alloc(n);
        if (d && h && n) err = cudaMemcpyAsync(d, h, n * 4, cudaMemcpyHostToDevice, st);
        return err == cudaSuccess ? d : nullptr;
    }
    float* alloc(size_t n) {
        if (err != cudaSuccess) return nullptr;
        void* p = nullptr;
        err = cudaMalloc(&p, n ? n * 4 : 16);
        if (err != cudaSuccess) return nullptr;
        ptrs.push_back(p);
        return static_cast<float*>(p);
    }
    int down(float* h, const float* d, size_t n) {
        if (err == cudaSuccess && n) err = cudaMemcpyAsync(h, d, n * 4, cudaMemcpyDeviceToHost, st);
        if (err == cudaSuccess) err = cudaStreamSynchronize(st);
        return err == cudaSuccess ? GPT2Q_OK : GPT2Q_ECUDA;
    }
};

int open_scratch(int device, Scratch& s, const char* fn) {
    if ((s.err = cudaSetDevice(device)) != cudaSuccess ||
        (s.err = cudaStreamCreateWithFlags(&s.st, cudaStreamNonBlocking)) != cudaSuccess) {
        set_global_error(std::string(fn) + ": " + cudaGetErrorString(s.err));
        return GPT2Q_ECUDA;
    }
    return GPT2Q_OK;
}

int finish(Scratch& s, int rc, const char* fn) {
    if (rc != GPT2Q_OK || s.err != cudaSuccess) {
        set_global_error(std::string(fn) + ": " + cudaGetErrorString(s.err));
        return GPT2Q_ECUDA;
    }
    return GPT2Q_OK;
}

}  // namespace

extern "C" {

int gpt2q_bwd_lin_input_grad(int device, const float* w, const float* dy, int rows, int cols, float* dx) {
    if (!w || !dy || !dx || rows <= 0 || cols <= 0 || cols % 4 != 0) {
        set_global_error("gpt2q_bwd_lin_input_grad: null pointer, or rows/cols not positive, or cols % 4 != 0");
        return GPT2Q_EARG;
    }
    Scratch s;
    if (open_scratch(device, s, "gpt2q_bwd_lin_input_grad") != GPT2Q_OK) return GPT2Q_ECUDA;
    QW q{};
    q.q = reinterpret_cast<const uint8_t*>(s.up(w, (size_t)rows * cols));
    q.rows = rows;
    q.cols = cols;
    q.atom = ATOM_F32;
    q.qstride = (size_t)cols * 4;
    const float* ddy = s.up(dy, rows);
    float* part = s.alloc(bwd_linear_part_floats(1, rows, cols));
    unsigned* counters = reinterpret_cast<unsigned*>(s.alloc(bwd_linear_counters(1, cols)));
    if (s.err == cudaSuccess) s.err = cudaMemsetAsync(counters, 0, bwd_linear_counters(1, cols) * 4, s.st);
    float* ddx = s.alloc(cols);
    if (s.err == cudaSuccess)
        s.err = launch_bwd_linear(q, ddy, rows, 1, part, counters, BWD_STORE, ddx, cols, nullptr, 0, s.st);
    return finish(s, s.down(dx, ddx, cols), "gpt2q_bwd_lin_input_grad");
}

int gpt2q_bwd_ln_backward(int device, const float* dy, const float* x, const float* g, const float* b, float eps,
                          int n, float* dx, float* dg, float* db) {
    (void)b;  // the bias does not enter the Jacobian (cu/backward.cu:114)
    if (!dy || !x || !g || !dx || !dg || !db || n <= 0) {
        set_global_error("gpt2q_bwd_ln_backward: null pointer or n <= 0");
        return GPT2Q_EARG;
    }
    Scratch s;
    if (open_scratch(device, s, "gpt2q_bwd_ln_backward") != GPT2Q_OK) return GPT2Q_ECUDA;
    const float* ddy = s.up(dy, n);
    const float* dxs = s.up(x, n);
    const float* dgm = s.up(g, n);
    float* ddx = s.alloc(n);
    float* ddg = s.up(dg, n);
    float* ddb = s.up(db, n);
    if (s.err == cudaSuccess)
        s.err = launch_bwd_ln(ddy, n, dxs, n, dgm, eps, n, 1, BWD_STORE, ddx, n, ddg, ddb, s.st);
    int rc = s.down(dx, ddx, n);
    if (rc == GPT2Q_OK) rc = s.down(dg, ddg, n);
    if (rc == GPT2Q_OK) rc = s.down(db, ddb, n);
    return finish(s, rc, "gpt2q_bwd_ln_backward");
}

int gpt2q_bwd_gelu(int device, const float* x_pre, const float* dy, int n, float* dx) {
    if (!x_pre || !dy || !dx || n <= 0) {
        set_global_error("gpt2q_bwd_gelu: null pointer or n <= 0");
        return GPT2Q_EARG;
    }
    Scratch s;
    if (open_scratch(device, s, "gpt2q_bwd_gelu") != GPT2Q_OK) return GPT2Q_ECUDA;
    const float* dxp = s.up(x_pre, n);
    const float* ddy = s.up(dy, n);
    float* ddx = s.alloc(n);
    if (s.err == cudaSuccess) s.err = launch_gelu_bwd(dxp, ddy, ddx, (size_t)n, s.st);
    return finish(s, s.down(dx, ddx, n), "gpt2q_bwd_gelu");
}

int gpt2q_bwd_attn_train(int device, const float* q, const float* k, const float* v, const float* dy, int t, int hd,
                         int stride, float* dq, float* dk, float* dv) {
    if (!q || !k || !v || !dy || !dq || !dk || !dv || t <= 0 || hd <= 0 || stride <= 0 || stride % hd != 0 ||
        t > ATT_MAX_T || hd > ATT_MAX_HD) {
        set_global_error("gpt2q_bwd_attn_train: null pointer, or t/hd/stride out of range (t <= 1024, hd <= 128, "
                         "stride a multiple of hd)");
        return GPT2Q_EARG;
    }
    Scratch s;
    if (open_scratch(device, s, "gpt2q_bwd_attn_train") != GPT2Q_OK) return GPT2Q_ECUDA;
    const size_t total = (size_t)t * stride;
    const int heads = stride / hd;
    const float* d_q = s.up(q, total);
    const float* d_k = s.up(k, total);
    const float* d_v = s.up(v, total);
    const float* d_dy = s.up(dy, total);
    float* d_dq = s.alloc(total);
    float* d_dk = s.up(dk, total);
    float* d_dv = s.up(dv, total);
    float* stats = s.alloc((size_t)3 * heads * t);
    if (s.err == cudaSuccess)
        s.err = launch_attn_bwd_train(d_q, stride, d_k, stride, d_v, stride, d_dy, stride, t, heads, hd, d_dq, stride,
                                      d_dk, stride, d_dv, stride, 1, stats, s.st);
    int rc = s.down(dq, d_dq, total);
    if (rc == GPT2Q_OK) rc = s.down(dk, d_dk, total);
    if (rc == GPT2Q_OK) rc = s.down(dv, d_dv, total);
    return finish(s, rc, "gpt2q_bwd_attn_train");
}

}  // extern "C"
