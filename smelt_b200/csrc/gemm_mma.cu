// Batched-decode linear on the warp-level tensor cores: y[m][n] = sum_k W[n][k] x[m][k] for a
// handful of tokens (M <= 64), W int8 or int4 with fp16 group scales (one per 32 along K).
//
// Why not the tcgen05 GEMM at this size: with 16-64 tokens the work per weight tile is tiny, so a
// launch is bound by fixed latencies (TMEM allocation, single-thread MMA issue and commit, the
// split-K exchange), not by HBM or the tensor pipe. mma.sync keeps operands and accumulators in
// registers, so a CTA's warps can each take a sliver of K and meet in shared memory.
//
// Exactness (the same ~22 bits as the tcgen05 path): every weight w = q * s is split as
// hi + lo in fp16 with hi = fp16(q * s') and lo = fma(q, s', -hi) = the exact residual, where
// s' = s * 2^P is the group scale times a per-matrix power of two; both are computed in fp16
// with one rounding (q is an exact fp16 integer, the residual has at most 7 significant bits on
// the grid of ulp(s')). Activations arrive split the same way by their producer (x = x_hi + x_lo).
// Each 16 x 8 x 16 step issues W_hi x_hi, W_hi x_lo and W_lo x_hi into fp32 accumulators; the
// dropped W_lo x_lo is below 2^-22 of the product.
//
// K permutation: a dot product does not depend on the order of its terms, so the k-slots of an
// mma fragment are fed any permutation of K, the same for both operands. Thread (g, t) of a warp
// takes the 8 contiguous weights 8t..8t+7 of a 32-group (int4: bytes 4t..4t+3, i.e. elements
// 4t..4t+3 and 16+4t..16+4t+3) and the matching 16 contiguous bytes of each token's activation
// row, so both operands load as plain vectors with no shuffles.
//
// Work layout: grid (16-row tiles, S), clusters of the S CTAs of a tile. A CTA stages the
// activations of its K range ([NB*8 tokens][K/S], hi and lo) by bulk copies, its warps take
// consecutive group ranges of that range, and the warp partials meet in shared memory (fixed
// order). With S > 1 the other CTAs of the cluster store their tile partials into CTA 0's shared
// memory, and after one cluster barrier CTA 0 sums them in rank order and runs the epilogue, so
// results do not depend on scheduling.
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

#include "common.cuh"
#include "gemm_mma.h"
#include "kernels.h"
#include "tcgen05.cuh"

namespace gpt2q {
namespace {

constexpr int TILE = 16;  // weight rows per warp tile (the mma M)
constexpr int PF = 2;     // groups of weights a warp holds in registers ahead of use (warps take 1-2 groups)
constexpr int EP = 2;     // epilogue outputs per thread (2 * NB <= warps keeps 16 * NB * 8 <= 2 * threads)

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// Two small biased integers (bytes sel of u, each value + bias in [0, 255]) -> exact fp16 pair:
// 0x64bb is 1024 + bb, so subtracting 1024 + bias leaves the integer.
__device__ __forceinline__ __half2 bytes_to_h2(uint32_t u, uint32_t sel, uint32_t magic2) {
    return __hsub2(u2h(__byte_perm(u, 0x64646464u, sel)), u2h(magic2));
}

// hi/lo split of two weights q * s' (see the file comment).
__device__ __forceinline__ void split_w(__half2 q, __half2 s, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __hmul2(q, s);
    hi = h2u(h);
    lo = h2u(__hfma2(q, s, __hneg2(h)));
}

// A fragments (hi and lo, two k16 steps) of one 32-group from the thread's raw weight bytes of
// rows g (ra) and g + 8 (rb): step 0 takes K 8t..8t+3 (int4: 4t..4t+3), step 1 K 8t+4..8t+7
// (int4: 16+4t..16+4t+3). Register order of m16n8k16's A: {row g, slots 2t,2t+1},
// {row g+8, 2t,2t+1}, {row g, 2t+8,2t+9}, {row g+8, 2t+8,2t+9}.
template <int ATOM>
__device__ __forceinline__ void dequant_group(uint2 ra, uint2 rb, __half sa, __half sb, __half pre,
                                              uint32_t (&hi)[2][4], uint32_t (&lo)[2][4]) {
    const __half2 s0 = __half2half2(__hmul(sa, pre)), s1 = __half2half2(__hmul(sb, pre));
    if constexpr (ATOM == ATOM_Q8) {
        const uint32_t m = 0x64806480u;  // 1152 = 1024 + 128
        const uint32_t a0 = ra.x ^ 0x80808080u, a1 = ra.y ^ 0x80808080u;
        const uint32_t b0 = rb.x ^ 0x80808080u, b1 = rb.y ^ 0x80808080u;
        split_w(bytes_to_h2(a0, 0x4140u, m), s0, hi[0][0], lo[0][0]);
        split_w(bytes_to_h2(b0, 0x4140u, m), s1, hi[0][1], lo[0][1]);
        split_w(bytes_to_h2(a0, 0x4342u, m), s0, hi[0][2], lo[0][2]);
        split_w(bytes_to_h2(b0, 0x4342u, m), s1, hi[0][3], lo[0][3]);
        split_w(bytes_to_h2(a1, 0x4140u, m), s0, hi[1][0], lo[1][0]);
        split_w(bytes_to_h2(b1, 0x4140u, m), s1, hi[1][1], lo[1][1]);
        split_w(bytes_to_h2(a1, 0x4342u, m), s0, hi[1][2], lo[1][2]);
        split_w(bytes_to_h2(b1, 0x4342u, m), s1, hi[1][3], lo[1][3]);
    } else {
        const uint32_t m = 0x64086408u;  // 1032 = 1024 + 8
        // ra.x: bytes 4t..4t+3 of row g's group; low nibbles are elements 4t+i, high 16+4t+i
        const uint32_t al = (ra.x & 0x0F0F0F0Fu) ^ 0x08080808u, ah = ((ra.x >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
        const uint32_t bl = (rb.x & 0x0F0F0F0Fu) ^ 0x08080808u, bh = ((rb.x >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
        split_w(bytes_to_h2(al, 0x4140u, m), s0, hi[0][0], lo[0][0]);
        split_w(bytes_to_h2(bl, 0x4140u, m), s1, hi[0][1], lo[0][1]);
        split_w(bytes_to_h2(al, 0x4342u, m), s0, hi[0][2], lo[0][2]);
        split_w(bytes_to_h2(bl, 0x4342u, m), s1, hi[0][3], lo[0][3]);
        split_w(bytes_to_h2(ah, 0x4140u, m), s0, hi[1][0], lo[1][0]);
        split_w(bytes_to_h2(bh, 0x4140u, m), s1, hi[1][1], lo[1][1]);
        split_w(bytes_to_h2(ah, 0x4342u, m), s0, hi[1][2], lo[1][2]);
        split_w(bytes_to_h2(bh, 0x4342u, m), s1, hi[1][3], lo[1][3]);
    }
}

// B fragments of one token row for the two k16 steps of a group, from the staged activations
// (row = the token's row at the group's first K): {b0, b1} of step 0, then of step 1, at the K
// positions the A fragments use.
template <int ATOM>
__device__ __forceinline__ uint4 load_x(const __half* row, int t) {
    if constexpr (ATOM == ATOM_Q8) {
        return *reinterpret_cast<const uint4*>(row + 8 * t);
    } else {
        const uint2 a = *reinterpret_cast<const uint2*>(row + 4 * t);
        const uint2 b = *reinterpret_cast<const uint2*>(row + 16 + 4 * t);
        return make_uint4(a.x, a.y, b.x, b.y);
    }
}

// Staged activation row stride in halves for a K range of kg groups: the row bytes padded so that
// the fragment loads of one load phase hit distinct banks (16-byte loads, 8 lanes = rows g, g+1:
// stride = 64 mod 128 bytes; int4's 8-byte loads, 16 lanes = rows g..g+3: stride = 32 mod 128).
template <int ATOM>
__host__ __device__ __forceinline__ int staged_stride(int kg) {
    const int bytes = kg * 64;
    const int want = (ATOM == ATOM_Q8) ? 64 : 32;
    return (bytes + ((want - bytes % 128) + 128) % 128) / 2;
}

// Optional phase stamps of one traced launch: [CTA][MMA_TRACE] globaltimer values, thread 0.
constexpr int MMA_TRACE = 8;
__device__ __forceinline__ void mma_stamp(unsigned long long* trace, int k) {
    if (trace && threadIdx.x == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        trace[(blockIdx.x + (size_t)gridDim.x * blockIdx.y) * MMA_TRACE + k] = t;
    }
}

// Bounded wait by non-blocking polls (a suspended try_wait resumes only after a time slice).
__device__ __forceinline__ void wait_staged(uint64_t* bar, int* err) {
    for (uint32_t i = 0; i < (1u << 26); ++i)
        if (tc::mbar_test_wait(bar, 0)) return;
    atomicExch(err, tc::ERR_WAIT_TIMEOUT);
}

__device__ __forceinline__ float lane_sum(float v) {  // butterfly: the same order on every lane
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <int ATOM, int NB>
__global__ void __launch_bounds__(MMA_MAX_WARPS * 32, 1)
k_linear_mma(const QW w, const __half* xhi, const __half* xlo, int ldx, int M, int gps, int gpw, __half pre,
             float post, int* err, unsigned long long* trace, Epi e, LnFold ln) {
    constexpr int NC = NB * 8;
    constexpr int N_OUT = TILE * NC;
    constexpr int GB = (ATOM == ATOM_Q8) ? 32 : 16;  // payload bytes per row and group
    extern __shared__ __align__(16) uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t xbar;
    tc::pdl_trigger();
    mma_stamp(trace, 0);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int G = w.cols / 32;
    const int tile = blockIdx.x, split = blockIdx.y, S = gridDim.y;
    const int kg0 = split * gps, kg1 = min(G, kg0 + gps);
    // A CTA that covers whole activation rows stages them with one bulk copy per operand
    // (rows dense, stride ldx); otherwise one copy per token row at a bank-spread stride. One
    // layout for every CTA of a cluster (CTA 0's partial slots are addressed by the others): the
    // stride of the nominal range, even where the last split holds fewer groups.
    const bool fold = ln.stats != nullptr;  // X = g * x of a LayerNorm folded into the epilogue
    const bool whole = S == 1 && G * 32 == ldx;
    const int xs = whole ? ldx : staged_stride<ATOM>(gps);
    __half* sxh = reinterpret_cast<__half*>(smem_raw);
    __half* sxl = sxh + (size_t)NC * xs;
    // warp partials [nw][NC][TILE] reuse the staged activations once every warp's MMAs are done;
    // the cluster's tile partials [S][N_OUT] (CTA 0) have their own space after the activations
    float* red = reinterpret_cast<float*>(smem_raw);
    const size_t staged_bytes = max((size_t)2 * NC * xs * 2, (size_t)nw * N_OUT * 4);
    float* recv = reinterpret_cast<float*>(smem_raw + staged_bytes);
    // folded LayerNorm: each token's mean and 1 / sqrt(var + eps)
    float* smean = recv + (S > 1 ? (size_t)S * N_OUT : 0);
    float* srstd = smean + NC;
    const int g0 = min(kg1, kg0 + warp * gpw), g1 = min(kg1, g0 + gpw);

    // ---- before the previous kernel finishes: this warp's first weights, the epilogue's bias ----
    uint2 wa[PF], wb[PF];
    __half ws_a[PF], ws_b[PF];
    const int ra = min(tile * TILE + g, w.rows - 1), rb = min(tile * TILE + g + 8, w.rows - 1);
    const uint8_t* qa = w.q + (size_t)ra * w.qstride;
    const uint8_t* qb = w.q + (size_t)rb * w.qstride;
    auto load_slot = [&](int u, int gr) {
        if constexpr (ATOM == ATOM_Q8) {
            wa[u] = __ldg(reinterpret_cast<const uint2*>(qa + (size_t)gr * GB + 8 * t));
            wb[u] = __ldg(reinterpret_cast<const uint2*>(qb + (size_t)gr * GB + 8 * t));
        } else {
            wa[u] = make_uint2(__ldg(reinterpret_cast<const uint32_t*>(qa + (size_t)gr * GB + 4 * t)), 0u);
            wb[u] = make_uint2(__ldg(reinterpret_cast<const uint32_t*>(qb + (size_t)gr * GB + 4 * t)), 0u);
        }
        ws_a[u] = __ldg(w.s + (size_t)ra * w.sstride + gr);
        ws_b[u] = __ldg(w.s + (size_t)rb * w.sstride + gr);
    };
#pragma unroll
    for (int u = 0; u < PF; ++u)
        if (g0 + u < g1) load_slot(u, g0 + u);
    // epilogue outputs of this thread: i = threadIdx.x + k * blockDim.x -> token i / 16, row i % 16
    const bool epi_cta = split == 0;
    int em[EP], en[EP];
    bool eok[EP];
    float eb[EP], er[EP];
    int esl[EP], eps[EP];
    float ec1[EP];  // folded LayerNorm: sum_k W[n][k] g[k]; eb then holds sum_k W[n][k] b[k] + bias[n]
#pragma unroll
    for (int k = 0; k < EP; ++k) {
        const int i = threadIdx.x + k * (int)blockDim.x;
        em[k] = i / TILE;
        en[k] = tile * TILE + i % TILE;
        eok[k] = epi_cta && i < N_OUT && em[k] < M && en[k] < w.rows;
        eb[k] = 0.f;
        ec1[k] = 0.f;
        if (eok[k]) {
            if (fold) {
                ec1[k] = __ldg(ln.c1 + en[k]);
                eb[k] = __ldg(ln.c2b + en[k]);
            } else if (e.bias) {
                eb[k] = __ldg(e.bias + en[k]);
            }
        }
        er[k] = 0.f;
        esl[k] = eps[k] = 0;
    }
    if (threadIdx.x == 0) {
        tc::mbar_init(&xbar, 1);
        tc::fence_mbar_init();
    }
    __syncthreads();
    mma_stamp(trace, 1);
    tc::pdl_wait();
    mma_stamp(trace, 2);
    // ---- the activations of tokens 0..M-1 (staged rows M..NC-1 hold leftovers; the outputs of
    // those token columns are never stored) ----
    if (warp == 0) {
        if (whole) {
            const uint32_t bytes = (uint32_t)M * (uint32_t)ldx * 2u;
            if (lane == 0) {
                tc::mbar_arrive_expect_tx(&xbar, 2u * bytes);
                tc::bulk_load_1d(sxh, xhi, bytes, &xbar);
                tc::bulk_load_1d(sxl, xlo, bytes, &xbar);
            }
        } else {
            const uint32_t row_bytes = (uint32_t)(kg1 - kg0) * 64;
            if (lane == 0) tc::mbar_arrive_expect_tx(&xbar, 2u * (uint32_t)M * row_bytes);
            __syncwarp();
            for (int i = lane; i < 2 * M; i += 32) {
                const int tok = i % M;
                const __half* src = (i < M ? xhi : xlo) + (size_t)tok * ldx + (size_t)kg0 * 32;
                tc::bulk_load_1d((i < M ? sxh : sxl) + (size_t)tok * xs, src, row_bytes, &xbar);
            }
        }
    }
    // the epilogue's inputs written by earlier kernels fly while the activations arrive
#pragma unroll
    for (int k = 0; k < EP; ++k) {
        if (!eok[k]) continue;
        if (e.kind == EPI_RESID) er[k] = e.out[(size_t)em[k] * e.ldo + en[k]];
        if (e.kind == EPI_QKV && en[k] >= e.d_local) {
            esl[k] = e.slot[em[k]];
            eps[k] = e.pos[em[k]];
        }
    }
    if (fold && epi_cta) {
        // each token's LayerNorm statistics from the (mean_t, M2_t) of the T 16-element tiles of
        // its row, in a fixed order: mean = sum(mean_t) / T, M2 = sum(M2_t + 16 (mean_t - mean)^2)
        // (exact identities); rstd = 1 / sqrt(M2 / (16 T) + eps) as k_layernorm computes it.
        // Every load of a warp's tokens is issued first; they fly with the activation copy.
        constexpr int TPW = 4;  // tokens per warp (M <= 64, at least 16 warps when M > 32)
        const int T = ln.n_tiles;
        float2 st[TPW][4];
#pragma unroll
        for (int r = 0; r < TPW; ++r) {
            const int m = warp + r * nw;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int t = lane + 32 * u;
                st[r][u] = (m < M && t < T) ? __ldcg(ln.stats + (size_t)m * ln.stats_ld + t) : make_float2(0.f, 0.f);
            }
        }
#pragma unroll
        for (int r = 0; r < TPW; ++r) {
            const int m = warp + r * nw;
            const float mean = lane_sum(st[r][0].x + st[r][1].x + st[r][2].x + st[r][3].x) / (float)T;
            float q = 0.f;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float dm = st[r][u].x - mean;
                if (lane + 32 * u < T) q += st[r][u].y + 16.f * dm * dm;
            }
            const float var = lane_sum(q) / (float)(16 * T);
            if (lane == 0 && m < M) {
                smean[m] = mean;
                srstd[m] = __frcp_rn(sqrtf(var + ln.eps));
            }
        }
    }
    wait_staged(&xbar, err);
    mma_stamp(trace, 3);

    // ---- MMAs: up to 32 tokens, two accumulator sets (x_hi products; x_lo and w_lo products)
    // halve the dependent chains; more tokens have chains enough and keep the registers ----
    constexpr bool TWO = NB <= 4;
    float acc[NB][4], acd[NB][4];
#pragma unroll
    for (int j = 0; j < NB; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[j][q] = acd[j][q] = 0.f;
    for (int base = g0; base < g1; base += PF) {
#pragma unroll
        for (int u = 0; u < PF; ++u) {
            const int gr = base + u;
            if (gr < g1) {
                uint32_t ahi[2][4], alo[2][4];
                dequant_group<ATOM>(wa[u], wb[u], ws_a[u], ws_b[u], pre, ahi, alo);
                if (gr + PF < g1) load_slot(u, gr + PF);  // slot u holds the groups = g0 + u mod PF
                const int kofs = (gr - kg0) * 32;
                uint4 xh[NB], xl[NB];
#pragma unroll
                for (int j = 0; j < NB; ++j) {
                    xh[j] = load_x<ATOM>(sxh + (size_t)(8 * j + g) * xs + kofs, t);
                    xl[j] = load_x<ATOM>(sxl + (size_t)(8 * j + g) * xs + kofs, t);
                }
#pragma unroll
                for (int j = 0; j < NB; ++j) {
                    mma16816(acc[j], ahi[0], xh[j].x, xh[j].y);
                    mma16816(TWO ? acd[j] : acc[j], ahi[0], xl[j].x, xl[j].y);
                    mma16816(acc[j], ahi[1], xh[j].z, xh[j].w);
                    mma16816(TWO ? acd[j] : acc[j], alo[0], xh[j].x, xh[j].y);
                    mma16816(TWO ? acd[j] : acc[j], ahi[1], xl[j].z, xl[j].w);
                    mma16816(TWO ? acd[j] : acc[j], alo[1], xh[j].z, xh[j].w);
                }
            }
        }
    }
    mma_stamp(trace, 4);
    __syncthreads();  // the staged activations are dead: their space takes the warp partials
    // C fragment: {row g, tokens 2t, 2t+1}, {row g+8, tokens 2t, 2t+1} of each n8 block
    float* mine = red + (size_t)warp * N_OUT;
#pragma unroll
    for (int j = 0; j < NB; ++j) {
        mine[(8 * j + 2 * t) * TILE + g] = TWO ? acc[j][0] + acd[j][0] : acc[j][0];
        mine[(8 * j + 2 * t + 1) * TILE + g] = TWO ? acc[j][1] + acd[j][1] : acc[j][1];
        mine[(8 * j + 2 * t) * TILE + g + 8] = TWO ? acc[j][2] + acd[j][2] : acc[j][2];
        mine[(8 * j + 2 * t + 1) * TILE + g + 8] = TWO ? acc[j][3] + acd[j][3] : acc[j][3];
    }
    __syncthreads();
    // the CTA's partial, warps summed in order
    float v[EP];
#pragma unroll
    for (int k = 0; k < EP; ++k) {
        const int i = threadIdx.x + k * (int)blockDim.x;
        v[k] = 0.f;
        if (i < N_OUT)
            for (int wq = 0; wq < nw; ++wq) v[k] += red[(size_t)wq * N_OUT + i];
    }
    mma_stamp(trace, 5);
    if (S > 1) {
        // the cluster's partials meet in CTA 0, which sums them in rank order
        if (split > 0) {
#pragma unroll
            for (int k = 0; k < EP; ++k) {
                const int i = threadIdx.x + k * (int)blockDim.x;
                if (i < N_OUT) {
                    const uint32_t dst = tc::map_cluster(tc::smem_u32(recv + (size_t)split * N_OUT + i), 0);
                    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(dst), "f"(v[k]) : "memory");
                }
            }
        }
        tc::cluster_sync();
        if (split > 0) return;
#pragma unroll
        for (int k = 0; k < EP; ++k) {
            const int i = threadIdx.x + k * (int)blockDim.x;
            if (i < N_OUT)
                for (int s2 = 1; s2 < S; ++s2) v[k] += recv[(size_t)s2 * N_OUT + i];
        }
        mma_stamp(trace, 6);
    }
    // ---- epilogue: every input is already in registers ----
    float res[EP];
#pragma unroll
    for (int k = 0; k < EP; ++k) {
        res[k] = 0.f;
        if (!eok[k]) continue;
        // folded LayerNorm: W (g (x - mean) rstd + b) + bias = rstd (W (g x) - mean W g) + W b + bias
        const float x = fold ? srstd[em[k]] * (v[k] * post - smean[em[k]] * ec1[k]) + eb[k] : v[k] * post + eb[k];
        const size_t o = (size_t)em[k] * e.ldo + en[k];
        switch (e.kind) {
            case EPI_STORE:
                e.out[o] = x;
                break;
            case EPI_RESID:
                res[k] = er[k] + x;
                e.out[o] = res[k];
                if (e.stats) {  // g * x of the next LayerNorm, the next linear's activations
                    __half h, l;
                    split_hl(e.ln_g[en[k]] * res[k], h, l);
                    e.out_hi[o] = h;
                    e.out_lo[o] = l;
                }
                break;
            case EPI_GELU: {
                const float gv = gelu_tanh(x);
                if (e.out) e.out[o] = gv;  // null: the consumer reads only the hi/lo pair
                if (e.out_hi) {
                    const __half h = __float2half_rn(gv);
                    e.out_hi[o] = h;
                    e.out_lo[o] = __float2half_rn(gv - __half2float(h));
                }
                break;
            }
            default: {  // EPI_QKV: q to out, k/v into the cache at (slot, pos)
                if (en[k] < e.d_local) {
                    e.out[o] = x;
                } else {
                    const int sel = en[k] / e.d_local - 1;
                    const int c = en[k] - (sel + 1) * e.d_local;
                    const int head = c / e.hd, i = c - head * e.hd;
                    e.kv[(size_t)esl[k] * e.slot_stride + e.layer_off + (size_t)sel * e.sel_stride +
                         (size_t)head * e.head_stride + (size_t)eps[k] * e.hd + i] = x;
                }
            }
        }
    }
    if (e.kind == EPI_RESID && e.stats) {
        // the tile's 16 new residual values of a token sit in 16 consecutive threads: their mean
        // and sum of squared deviations (fixed butterfly order), for the next LayerNorm
#pragma unroll
        for (int k = 0; k < EP; ++k) {
            const int i = threadIdx.x + k * (int)blockDim.x;
            if (i - (threadIdx.x & 31) >= N_OUT) break;  // warp-uniform: no outputs left
            float s = res[k];
#pragma unroll
            for (int o = 1; o < TILE; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            const float mean = s * (1.0f / TILE);
            const float dv = eok[k] ? res[k] - mean : 0.f;
            float q = dv * dv;
#pragma unroll
            for (int o = 1; o < TILE; o <<= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
            if (eok[k] && i % TILE == 0) e.stats[(size_t)em[k] * e.stats_ld + tile] = make_float2(mean, q);
        }
    }
    mma_stamp(trace, 7);
}

// The launch traced when GPT2Q_MMA_TRACE=<rows>x<cols>x<M> is set: the first one of that shape.
constexpr size_t MMA_TRACE_CTAS = 4096;
struct MmaTraceState {
    unsigned long long* buf = nullptr;
    int rows = 0, cols = 0, m = 0;
    bool traced = false;
    dim3 grid;
};
MmaTraceState& trace_state() {
    static MmaTraceState st;
    static bool init = false;
    if (!init) {
        init = true;
        if (const char* e = std::getenv("GPT2Q_MMA_TRACE"))
            if (std::sscanf(e, "%dx%dx%d", &st.rows, &st.cols, &st.m) == 3 &&
                cudaMalloc(&st.buf, MMA_TRACE_CTAS * MMA_TRACE * 8) == cudaSuccess)
                cudaMemset(st.buf, 0, MMA_TRACE_CTAS * MMA_TRACE * 8);
    }
    return st;
}

int num_sms() {
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!cached[dev]) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        cached[dev] = v > 0 ? v : 148;
    }
    return cached[dev];
}

struct Plan {
    int S = 1, warps = 1, gps = 0, gpw = 0;
    size_t smem = 0;
};

size_t smem_bytes(int atom, int NB, int kgroups, int warps, int S, bool ln) {
    const int NC = NB * 8;
    const int xs = atom == ATOM_Q8 ? staged_stride<ATOM_Q8>(kgroups) : staged_stride<ATOM_Q4>(kgroups);
    const size_t staged = std::max((size_t)2 * NC * xs * 2, (size_t)warps * TILE * NC * 4);
    // folded LayerNorm: each token's mean and rstd
    const size_t lnb = ln ? (size_t)2 * NC * 4 : 0;
    return staged + (S > 1 ? (size_t)S * TILE * NC * 4 : 0) + lnb;
}

// Work layout: K split over a cluster of S CTAs only where the row tiles alone leave most SMs
// idle (or the staged activations of the whole K would not fit); warps of 1-2 groups each.
bool plan(const QW& w, int M, Plan& p, bool ln) {
    const int tiles = (w.rows + TILE - 1) / TILE;
    const int G = w.cols / 32;
    const int NB = (M + 7) / 8;
    const int sms = num_sms();
    // whole rows per CTA (one bulk copy per operand) unless that leaves more than 1 - 1 / F of the
    // SMs idle (F = 4; GPT2Q_MMA_SPLIT_F overrides it for tuning) or does not fit
    static const int F = [] {
        const char* e = std::getenv("GPT2Q_MMA_SPLIT_F");
        return e ? std::max(1, std::atoi(e)) : 4;
    }();
    int S = tiles >= sms / F ? 1 : std::max(1, std::min({MMA_MAX_SPLITS, (sms - 8 + tiles - 1) / tiles, G / 2}));
    for (; S <= MMA_MAX_SPLITS && S <= G; ++S) {
        const int gps = (G + S - 1) / S;
        const int Sx = (G + gps - 1) / gps;  // no empty split
        // more row tiles than SMs: CTAs of 8 warps, two per SM (registers), all resident at once
        const int wmax = tiles > sms ? MMA_MAX_WARPS / 2 : MMA_MAX_WARPS;
        const int warps = std::max(2 * NB, std::min(wmax, gps));  // 2 epilogue outputs per thread
        const int gpw = (gps + warps - 1) / warps;
        const size_t smem = smem_bytes(w.atom, NB, gps, warps, Sx, ln);
        if (smem <= (size_t)MMA_MAX_SMEM) {
            p.S = Sx;
            p.warps = warps;
            p.gps = gps;
            p.gpw = gpw;
            p.smem = smem;
            return true;
        }
    }
    return false;
}

template <int ATOM, int NB>
cudaError_t launch_nb(const QW& w, const __half* xhi, const __half* xlo, int ldx, int M, const Plan& p, __half pre,
                      float post, int* err, const Epi& e, const LnFold& ln, cudaStream_t st) {
    auto kern = k_linear_mma<ATOM, NB>;
    // the dynamic shared-memory limit is raised once per device for each instantiation
    static unsigned long long raised = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(raised & bit)) {
        const cudaError_t ae = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, MMA_MAX_SMEM);
        if (ae != cudaSuccess) return ae;
        raised |= bit;
    }
    const dim3 grid((w.rows + TILE - 1) / TILE, p.S);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(32 * p.warps);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    int na = 0;
    if (pdl_enabled()) {
        at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (p.S > 1) {
        at[na].id = cudaLaunchAttributeClusterDimension;
        at[na].val.clusterDim.x = 1;
        at[na].val.clusterDim.y = p.S;
        at[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = at;
    cfg.numAttrs = na;
    unsigned long long* tr = nullptr;
    MmaTraceState& ts = trace_state();
    if (ts.buf && !ts.traced && w.rows == ts.rows && w.cols == ts.cols && M == ts.m &&
        (size_t)grid.x * grid.y <= MMA_TRACE_CTAS) {
        tr = ts.buf;
        ts.traced = true;
        ts.grid = grid;
    }
    return cudaLaunchKernelEx(&cfg, kern, w, xhi, xlo, ldx, M, p.gps, p.gpw, pre, post, err, tr, e, ln);
}

template <int ATOM>
cudaError_t launch_atom(int NB, const QW& w, const __half* xhi, const __half* xlo, int ldx, int M, const Plan& p,
                        __half pre, float post, int* err, const Epi& e, const LnFold& ln, cudaStream_t st) {
    switch (NB) {
        case 1: return launch_nb<ATOM, 1>(w, xhi, xlo, ldx, M, p, pre, post, err, e, ln, st);
        case 2: return launch_nb<ATOM, 2>(w, xhi, xlo, ldx, M, p, pre, post, err, e, ln, st);
        case 3: return launch_nb<ATOM, 3>(w, xhi, xlo, ldx, M, p, pre, post, err, e, ln, st);
        case 4: return launch_nb<ATOM, 4>(w, xhi, xlo, ldx, M, p, pre, post, err, e, ln, st);
        case 5: return launch_nb<ATOM, 5>(w, xhi, xlo, ldx, M, p, pre, post, err, e, ln, st);
        case 6: return launch_nb<ATOM, 6>(w, xhi, xlo, ldx, M, p, pre, post, err, e, ln, st);
        case 7: return launch_nb<ATOM, 7>(w, xhi, xlo, ldx, M, p, pre, post, err, e, ln, st);
        default: return launch_nb<ATOM, 8>(w, xhi, xlo, ldx, M, p, pre, post, err, e, ln, st);
    }
}

}  // namespace

bool mma_usable(const QW& w, int M) {
    // matrices of many row tiles (the tied head) stay on the tcgen05 GEMM
    return M >= 1 && M <= MMA_MAX_M && (w.atom == ATOM_Q8 || w.atom == ATOM_Q4) && w.cols % 32 == 0 &&
           w.rows >= 1 && (w.rows + TILE - 1) / TILE <= MMA_MAX_TILES;
}

int mma_prescale_exp(float max_abs_w) {
    // largest |hi| at most 1024: hi and lo stay normal fp16 for scales within 2^10 of the largest
    if (!(max_abs_w > 0.f) || !std::isfinite(max_abs_w)) return 0;
    const int p = (int)std::floor(std::log2(1024.0 / (double)max_abs_w));
    return std::max(-14, std::min(15, p));
}

void mma_init() {
    trace_state();  // the trace buffer, if any, is allocated here, never during a graph capture
    num_sms();
}

bool mma_fits(const QW& w, int M, bool ln) {
    Plan p;
    return mma_usable(w, M) && plan(w, M, p, ln);
}

cudaError_t launch_linear_mma(const QW& w, const __half* xhi, const __half* xlo, int ldx, int M, int pexp, int* err,
                              const Epi& e, cudaStream_t st, const LnFold* ln) {
    if (M <= 0) return cudaSuccess;
    Plan p;
    if (!mma_usable(w, M) || ldx % 8 != 0 || !err || !plan(w, M, p, ln != nullptr)) return cudaErrorInvalidValue;
    LnFold lf{};
    if (ln) {
        // the row's statistics in at most 128 tiles of 16; four tokens per warp at most
        const int warps = p.warps;
        if (!ln->stats || !ln->c1 || !ln->c2b || ln->n_tiles * 16 != w.cols || ln->n_tiles > 128 ||
            ln->stats_ld < ln->n_tiles || 4 * warps < M)
            return cudaErrorInvalidValue;
        lf = *ln;
    }
    if (e.kind == EPI_RESID && e.stats && (w.rows % TILE != 0 || e.stats_ld * TILE < w.rows || !e.ln_g || !e.out_hi || !e.out_lo))
        return cudaErrorInvalidValue;
    const __half pre = __float2half_rn(std::ldexp(1.0f, pexp));
    const float post = std::ldexp(1.0f, -pexp);
    const int NB = (M + 7) / 8;
    if (w.atom == ATOM_Q8) return launch_atom<ATOM_Q8>(NB, w, xhi, xlo, ldx, M, p, pre, post, err, e, lf, st);
    return launch_atom<ATOM_Q4>(NB, w, xhi, xlo, ldx, M, p, pre, post, err, e, lf, st);
}

std::string mma_trace_json() {
    MmaTraceState& ts = trace_state();
    if (!ts.buf || !ts.traced) return "";
    const size_t n = (size_t)ts.grid.x * ts.grid.y;
    std::vector<unsigned long long> t(n * MMA_TRACE);
    if (cudaMemcpy(t.data(), ts.buf, t.size() * 8, cudaMemcpyDeviceToHost) != cudaSuccess) return "";
    unsigned long long t0 = ~0ull;
    for (auto v : t)
        if (v && v < t0) t0 = v;
    std::string s = "{\"grid\": [" + std::to_string(ts.grid.x) + ", " + std::to_string(ts.grid.y) + "], \"stamps\": [";
    for (size_t c = 0; c < n; ++c) {
        s += c ? ", [" : "[";
        for (int k = 0; k < MMA_TRACE; ++k) {
            const unsigned long long v = t[c * MMA_TRACE + k];
            s += (k ? ", " : "") + std::to_string(v ? (long long)(v - t0) : -1);
        }
        s += "]";
    }
    return s + "]}";
}

}  // namespace gpt2q
