// Batched-decode linear on the warp-level tensor cores: y[m][n] = sum_k W[n][k] x[m][k] for a
// handful of tokens (M <= 64), W int8 or int4 with fp16 group scales (one per 32 along K).
//
// Why not the tcgen05 GEMM at this size: with 16-64 tokens the work per weight tile is tiny, so a
// launch is bound by fixed latencies (TMEM allocation, single-thread MMA issue and commit, the
// split-K exchange), not by HBM or the tensor pipe. mma.sync keeps operands and accumulators in
// registers, so a CTA's warps can each take a sliver of K and meet in shared memory.
//
// Exactness: the integer weights q (|q| <= 128) are exact fp16 values, and the activations
// arrive from their producer as an fp16 pair x = x_hi + x_lo (~22 bits). For each 32-group a
// warp issues q x_hi and q x_lo (products exact in the fp32 accumulators) and then adds s times
// the group's sum to its fp32 accumulator, s the group's fp16 scale: one rounding per group, no
// product dropped. Four 16 x 8 x 16 MMAs per group and 8 tokens; splitting q s into an fp16
// hi/lo pair instead (three products, W_lo x_lo dropped) took six and was 4 % slower per decode
// step at 32 sequences.
//
// K permutation: a dot product does not depend on the order of its terms, so the k-slots of an
// mma fragment are fed any permutation of K, the same for both operands. Thread (g, t) of a warp
// takes the 8 contiguous weights 8t..8t+7 of a 32-group (int4: bytes 4t..4t+3, i.e. elements
// 4t..4t+3 and 16+4t..16+4t+3) and the matching 16 contiguous bytes of each token's activation
// row, so both operands load as plain vectors with no shuffles.
//
// Work layout: grid (tile groups of T consecutive 16-row tiles, S), clusters of the S CTAs of a
// tile group. A CTA stages the activations of its K range ([NB*8 tokens][K/S], hi and lo) by bulk
// copies once for its T tiles; each tile is a team of warps / T warps taking consecutive group
// ranges of that range, and a team's warp partials meet in shared memory (fixed order). With
// S > 1 the other CTAs of the cluster store their partials into CTA 0's shared memory, and after
// one cluster barrier CTA 0 sums them in rank order and runs the epilogue, so results do not
// depend on scheduling. T > 1 serves matrices of more tiles than SMs, or whose one-tile layout
// would need a second wave of CTAs (plan()).
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
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

// A fragments (two k16 steps) of one 32-group as exact fp16 integers q, from the thread's raw
// weight bytes of rows g (ra) and g + 8 (rb): step 0 takes K 8t..8t+3 (int4: 4t..4t+3), step 1
// K 8t+4..8t+7 (int4: 16+4t..16+4t+3). Register order of m16n8k16's A: {row g, slots 2t,2t+1},
// {row g+8, 2t,2t+1}, {row g, 2t+8,2t+9}, {row g+8, 2t+8,2t+9}.
template <int ATOM>
__device__ __forceinline__ void dequant_q(uint2 ra, uint2 rb, uint32_t (&aq)[2][4]) {
    if constexpr (ATOM == ATOM_Q8) {
        const uint32_t m = 0x64806480u;  // 1152 = 1024 + 128
        const uint32_t a0 = ra.x ^ 0x80808080u, a1 = ra.y ^ 0x80808080u;
        const uint32_t b0 = rb.x ^ 0x80808080u, b1 = rb.y ^ 0x80808080u;
        aq[0][0] = h2u(bytes_to_h2(a0, 0x4140u, m));
        aq[0][1] = h2u(bytes_to_h2(b0, 0x4140u, m));
        aq[0][2] = h2u(bytes_to_h2(a0, 0x4342u, m));
        aq[0][3] = h2u(bytes_to_h2(b0, 0x4342u, m));
        aq[1][0] = h2u(bytes_to_h2(a1, 0x4140u, m));
        aq[1][1] = h2u(bytes_to_h2(b1, 0x4140u, m));
        aq[1][2] = h2u(bytes_to_h2(a1, 0x4342u, m));
        aq[1][3] = h2u(bytes_to_h2(b1, 0x4342u, m));
    } else {
        const uint32_t m = 0x64086408u;  // 1032 = 1024 + 8
        // ra.x: bytes 4t..4t+3 of row g's group; low nibbles are elements 4t+i, high 16+4t+i
        const uint32_t al = (ra.x & 0x0F0F0F0Fu) ^ 0x08080808u, ah = ((ra.x >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
        const uint32_t bl = (rb.x & 0x0F0F0F0Fu) ^ 0x08080808u, bh = ((rb.x >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
        aq[0][0] = h2u(bytes_to_h2(al, 0x4140u, m));
        aq[0][1] = h2u(bytes_to_h2(bl, 0x4140u, m));
        aq[0][2] = h2u(bytes_to_h2(al, 0x4342u, m));
        aq[0][3] = h2u(bytes_to_h2(bl, 0x4342u, m));
        aq[1][0] = h2u(bytes_to_h2(ah, 0x4140u, m));
        aq[1][1] = h2u(bytes_to_h2(bh, 0x4140u, m));
        aq[1][2] = h2u(bytes_to_h2(ah, 0x4342u, m));
        aq[1][3] = h2u(bytes_to_h2(bh, 0x4342u, m));
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
k_linear_mma(const QW w, const __half* xhi, const __half* xlo, int ldx, int M, int T, int gps, int gpw, int* err,
             unsigned long long* trace, Epi e, LnFold ln) {
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
    // T consecutive 16-row tiles per CTA, one team of nw / T warps each (left-over warps idle in
    // the MMA phase); every team reads the same staged activations
    const int tile0 = blockIdx.x * T, split = blockIdx.y, S = gridDim.y;
    const int n_out = T * N_OUT;  // the CTA's outputs
    const int wt = nw / T, team = warp / wt, wr = warp - team * wt;
    const int mytile = tile0 + min(team, T - 1);
    const bool active = team < T && mytile * TILE < w.rows;
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
    float* smean = recv + (S > 1 ? (size_t)S * n_out : 0);
    float* srstd = smean + NC;
    const int g0 = active ? min(kg1, kg0 + wr * gpw) : kg1, g1 = min(kg1, g0 + gpw);

    // ---- before the previous kernel finishes: this warp's first weights, the epilogue's bias ----
    uint2 wa[PF], wb[PF];
    __half ws_a[PF], ws_b[PF];
    const int ra = min(mytile * TILE + g, w.rows - 1), rb = min(mytile * TILE + g + 8, w.rows - 1);
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
    // epilogue outputs of this thread: i = threadIdx.x + k * blockDim.x -> tile i / N_OUT, token
    // (i % N_OUT) / 16, row i % 16
    const bool epi_cta = split == 0;
    int em[EP], en[EP];
    bool eok[EP];
    float eb[EP], er[EP];
    int esl[EP], eps[EP];
    float ec1[EP];  // folded LayerNorm: sum_k W[n][k] g[k]; eb then holds sum_k W[n][k] b[k] + bias[n]
#pragma unroll
    for (int k = 0; k < EP; ++k) {
        const int i = threadIdx.x + k * (int)blockDim.x;
        em[k] = (i % N_OUT) / TILE;
        en[k] = (tile0 + i / N_OUT) * TILE + i % TILE;
        eok[k] = epi_cta && i < n_out && em[k] < M && en[k] < w.rows;
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

    // ---- MMAs: up to 32 tokens, the x_hi and x_lo sums of a group in two accumulator sets
    // (halving the dependent chains); more tokens have chains enough and keep the registers ----
    constexpr bool TWO = NB <= 4;
    float acc[NB][4];
#pragma unroll
    for (int j = 0; j < NB; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[j][q] = 0.f;
    for (int base = g0; base < g1; base += PF) {
#pragma unroll
        for (int u = 0; u < PF; ++u) {
            const int gr = base + u;
            if (gr < g1) {
                uint32_t aq[2][4];
                dequant_q<ATOM>(wa[u], wb[u], aq);
                const float sa = __half2float(ws_a[u]), sb = __half2float(ws_b[u]);
                if (gr + PF < g1) load_slot(u, gr + PF);  // slot u holds the groups = g0 + u mod PF
                const int kofs = (gr - kg0) * 32;
#pragma unroll
                for (int j = 0; j < NB; ++j) {
                    const uint4 xh = load_x<ATOM>(sxh + (size_t)(8 * j + g) * xs + kofs, t);
                    const uint4 xl = load_x<ATOM>(sxl + (size_t)(8 * j + g) * xs + kofs, t);
                    // the group's q x_hi and q x_lo sums (exact products), then its scale
                    float th[4] = {0.f, 0.f, 0.f, 0.f}, tl[4] = {0.f, 0.f, 0.f, 0.f};
                    mma16816(th, aq[0], xh.x, xh.y);
                    mma16816(TWO ? tl : th, aq[0], xl.x, xl.y);
                    mma16816(th, aq[1], xh.z, xh.w);
                    mma16816(TWO ? tl : th, aq[1], xl.z, xl.w);
                    acc[j][0] = fmaf(sa, TWO ? th[0] + tl[0] : th[0], acc[j][0]);
                    acc[j][1] = fmaf(sa, TWO ? th[1] + tl[1] : th[1], acc[j][1]);
                    acc[j][2] = fmaf(sb, TWO ? th[2] + tl[2] : th[2], acc[j][2]);
                    acc[j][3] = fmaf(sb, TWO ? th[3] + tl[3] : th[3], acc[j][3]);
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
        mine[(8 * j + 2 * t) * TILE + g] = acc[j][0];
        mine[(8 * j + 2 * t + 1) * TILE + g] = acc[j][1];
        mine[(8 * j + 2 * t) * TILE + g + 8] = acc[j][2];
        mine[(8 * j + 2 * t + 1) * TILE + g + 8] = acc[j][3];
    }
    __syncthreads();
    // the CTA's partials, each tile's team summed in warp order
    float v[EP];
#pragma unroll
    for (int k = 0; k < EP; ++k) {
        const int i = threadIdx.x + k * (int)blockDim.x;
        v[k] = 0.f;
        if (i < n_out) {
            const int tt = i / N_OUT, j = i - tt * N_OUT;
            for (int wq = tt * wt; wq < tt * wt + wt; ++wq) v[k] += red[(size_t)wq * N_OUT + j];
        }
    }
    mma_stamp(trace, 5);
    if (S > 1) {
        // the cluster's partials meet in CTA 0, which sums them in rank order
        if (split > 0) {
#pragma unroll
            for (int k = 0; k < EP; ++k) {
                const int i = threadIdx.x + k * (int)blockDim.x;
                if (i < n_out) {
                    const uint32_t dst = tc::map_cluster(tc::smem_u32(recv + (size_t)split * n_out + i), 0);
                    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(dst), "f"(v[k]) : "memory");
                }
            }
        }
        tc::cluster_sync();
        if (split > 0) return;
#pragma unroll
        for (int k = 0; k < EP; ++k) {
            const int i = threadIdx.x + k * (int)blockDim.x;
            if (i < n_out)
                for (int s2 = 1; s2 < S; ++s2) v[k] += recv[(size_t)s2 * n_out + i];
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
        const float x = fold ? srstd[em[k]] * (v[k] - smean[em[k]] * ec1[k]) + eb[k] : v[k] + eb[k];
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
            if (i - (threadIdx.x & 31) >= n_out) break;  // warp-uniform: no outputs left
            float s = res[k];
#pragma unroll
            for (int o = 1; o < TILE; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            const float mean = s * (1.0f / TILE);
            const float dv = eok[k] ? res[k] - mean : 0.f;
            float q = dv * dv;
#pragma unroll
            for (int o = 1; o < TILE; o <<= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
            if (eok[k] && i % TILE == 0)
                e.stats[(size_t)em[k] * e.stats_ld + tile0 + i / N_OUT] = make_float2(mean, q);
        }
    }
    mma_stamp(trace, 7);
}

// The tied lm head for 1..64 tokens: logits[m][n] = sum_k W[n][k] x[m][k] over the vocabulary's
// 16-row tiles. Unlike the layer linears, the head has thousands of tiles (3142 for GPT-2), so
// one CTA per SM stages the activations once (one bulk copy per operand) and every warp then
// runs whole tiles over the full K, storing each tile's outputs straight from its accumulator
// fragments: no cross-warp reduction and one staging per SM. Same arithmetic as k_linear_mma:
// exact integer weights against x_hi and x_lo, the group's fp32 sum scaled once. Measured on
// GPT-2 small: 22 us at 8 tokens against 35 + 1.3 us for the int8 head (kind::i8, one TMEM
// drain per group), but 36 us at 32 tokens against 28.7 us for the tcgen05 f16 hi/lo tile, so
// it serves the batches the tcgen05 head does not take (fewer than 16 rows). Its weights stream
// at under 2 TB/s whether or not each load asks L2 for the 256 bytes around it.
// CTA c owns tiles [c * tpc, (c + 1) * tpc); warp w takes tiles w, w + warps, ... of them, as
// one stream of (tile, group) units with HPF units of weights in registers ahead of use.
template <int ATOM, int NB>
__global__ void __launch_bounds__(MMA_MAX_WARPS * 32, 1)
k_head_mma(const QW w, const __half* xhi, const __half* xlo, int ldx, int M, int tpc, float* out, int ldo,
           int* err) {
    constexpr int NC = NB * 8;
    constexpr int GB = (ATOM == ATOM_Q8) ? 32 : 16;  // payload bytes per row and group
    constexpr int HPF = 4;                           // units of weights in flight per warp
    extern __shared__ __align__(16) uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t xbar;
    tc::pdl_trigger();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int G = w.cols / 32;
    const int tiles = (w.rows + TILE - 1) / TILE;
    const int t0 = blockIdx.x * tpc, t1 = min(tiles, t0 + tpc);
    const int my_tiles = t0 + warp < t1 ? (t1 - t0 - warp + nw - 1) / nw : 0;
    const int units = my_tiles * G;
    __half* sxh = reinterpret_cast<__half*>(smem_raw);
    __half* sxl = sxh + (size_t)NC * ldx;

    // ---- before the previous kernel finishes: this warp's first weights ----
    uint2 wa[HPF], wb[HPF];
    __half ws_a[HPF], ws_b[HPF];
    auto load_unit = [&](int slot, int u) {
        const int k = u / G, gr = u - k * G;
        const int tile = t0 + warp + k * nw;
        const int ra = min(tile * TILE + g, w.rows - 1), rb = min(tile * TILE + g + 8, w.rows - 1);
        const uint8_t* qa = w.q + (size_t)ra * w.qstride + (size_t)gr * GB;
        const uint8_t* qb = w.q + (size_t)rb * w.qstride + (size_t)gr * GB;
        if constexpr (ATOM == ATOM_Q8) {
            wa[slot] = __ldg(reinterpret_cast<const uint2*>(qa + 8 * t));
            wb[slot] = __ldg(reinterpret_cast<const uint2*>(qb + 8 * t));
        } else {
            wa[slot] = make_uint2(__ldg(reinterpret_cast<const uint32_t*>(qa + 4 * t)), 0u);
            wb[slot] = make_uint2(__ldg(reinterpret_cast<const uint32_t*>(qb + 4 * t)), 0u);
        }
        ws_a[slot] = __ldg(w.s + (size_t)ra * w.sstride + gr);
        ws_b[slot] = __ldg(w.s + (size_t)rb * w.sstride + gr);
    };
#pragma unroll
    for (int s = 0; s < HPF; ++s)
        if (s < units) load_unit(s, s);
    if (threadIdx.x == 0) {
        tc::mbar_init(&xbar, 1);
        tc::fence_mbar_init();
    }
    __syncthreads();
    tc::pdl_wait();
    // ---- the activations of tokens 0..M-1, rows dense at stride ldx ----
    if (threadIdx.x == 0) {
        const uint32_t bytes = (uint32_t)M * (uint32_t)ldx * 2u;
        tc::mbar_arrive_expect_tx(&xbar, 2u * bytes);
        tc::bulk_load_1d(sxh, xhi, bytes, &xbar);
        tc::bulk_load_1d(sxl, xlo, bytes, &xbar);
    }
    wait_staged(&xbar, err);

    // ---- units: 4 MMAs per group and 8 tokens into two accumulator sets (x_hi, x_lo) ----
    constexpr bool TWO = NB <= 4;
    float acc[NB][4];
    for (int base = 0; base < units; base += HPF) {
#pragma unroll
        for (int s = 0; s < HPF; ++s) {
            const int u = base + s;
            if (u < units) {
                const int k = u / G, gr = u - k * G;
                if (gr == 0) {
#pragma unroll
                    for (int j = 0; j < NB; ++j)
#pragma unroll
                        for (int q = 0; q < 4; ++q) acc[j][q] = 0.f;
                }
                uint32_t aq[2][4];
                dequant_q<ATOM>(wa[s], wb[s], aq);
                const float sa = __half2float(ws_a[s]), sb = __half2float(ws_b[s]);
                if (u + HPF < units) load_unit(s, u + HPF);  // slot s holds the units = s mod HPF
                const int kofs = gr * 32;
#pragma unroll
                for (int j = 0; j < NB; ++j) {
                    const uint4 xh = load_x<ATOM>(sxh + (size_t)(8 * j + g) * ldx + kofs, t);
                    const uint4 xl = load_x<ATOM>(sxl + (size_t)(8 * j + g) * ldx + kofs, t);
                    float th[4] = {0.f, 0.f, 0.f, 0.f}, tl[4] = {0.f, 0.f, 0.f, 0.f};
                    mma16816(th, aq[0], xh.x, xh.y);
                    mma16816(TWO ? tl : th, aq[0], xl.x, xl.y);
                    mma16816(th, aq[1], xh.z, xh.w);
                    mma16816(TWO ? tl : th, aq[1], xl.z, xl.w);
                    acc[j][0] = fmaf(sa, TWO ? th[0] + tl[0] : th[0], acc[j][0]);
                    acc[j][1] = fmaf(sa, TWO ? th[1] + tl[1] : th[1], acc[j][1]);
                    acc[j][2] = fmaf(sb, TWO ? th[2] + tl[2] : th[2], acc[j][2]);
                    acc[j][3] = fmaf(sb, TWO ? th[3] + tl[3] : th[3], acc[j][3]);
                }
                if (gr == G - 1) {
                    // C fragment: {row g, tokens 2t, 2t+1}, {row g+8, tokens 2t, 2t+1} of each n8 block
                    const int tile = t0 + warp + k * nw;
                    const int na = tile * TILE + g, nb = na + 8;
#pragma unroll
                    for (int j = 0; j < NB; ++j) {
                        const int m0 = 8 * j + 2 * t, m1 = m0 + 1;
                        if (na < w.rows) {
                            if (m0 < M) out[(size_t)m0 * ldo + na] = acc[j][0];
                            if (m1 < M) out[(size_t)m1 * ldo + na] = acc[j][1];
                        }
                        if (nb < w.rows) {
                            if (m0 < M) out[(size_t)m0 * ldo + nb] = acc[j][2];
                            if (m1 < M) out[(size_t)m1 * ldo + nb] = acc[j][3];
                        }
                    }
                }
            }
        }
    }
}

// The launch traced when GPT2Q_MMA_TRACE=<rows>x<cols>x<M>[x<skip>] is set: the first one of that
// shape after `skip` others.
constexpr size_t MMA_TRACE_CTAS = 4096;
struct MmaTraceState {
    unsigned long long* buf = nullptr;
    int rows = 0, cols = 0, m = 0, skip = 0;
    bool traced = false;
    dim3 grid;
};
MmaTraceState& trace_state() {
    static MmaTraceState st;
    static bool init = false;
    if (!init) {
        init = true;
        if (const char* e = std::getenv("GPT2Q_MMA_TRACE"))
            if (std::sscanf(e, "%dx%dx%dx%d", &st.rows, &st.cols, &st.m, &st.skip) >= 3 &&
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
    int T = 1, S = 1, warps = 1, gps = 0, gpw = 0;
    size_t smem = 0;
};

size_t smem_bytes(int atom, int NB, int kgroups, int warps, int S, bool ln, int T = 1) {
    const int NC = NB * 8;
    const int xs = atom == ATOM_Q8 ? staged_stride<ATOM_Q8>(kgroups) : staged_stride<ATOM_Q4>(kgroups);
    const size_t staged = std::max((size_t)2 * NC * xs * 2, (size_t)warps * TILE * NC * 4);
    // folded LayerNorm: each token's mean and rstd
    const size_t lnb = ln ? (size_t)2 * NC * 4 : 0;
    return staged + (S > 1 ? (size_t)S * T * TILE * NC * 4 : 0) + lnb;
}

// Residency of this kernel (at most 128 registers a thread): one 16-warp CTA or two 8-warp CTAs
// per SM, fewer where shared memory runs out; clusters of S CTAs fit in a GPC, so how many run
// at once is asked of the runtime when a handle is created (never during a graph capture).
struct Residency {
    bool init = false;
    int smem_per_sm = 228 * 1024;
    int clusters[3][MMA_MAX_SPLITS + 1] = {};  // [CTAs per SM][S]: clusters resident at once
};
Residency g_res[64];

Residency& residency() {
    int dev = 0;
    cudaGetDevice(&dev);
    return g_res[dev & 63];
}

void init_residency() {
    Residency& r = residency();
    if (r.init) return;
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) == cudaSuccess && v > 0)
        r.smem_per_sm = v;
    const int sms = num_sms();
    auto kern = k_linear_mma<ATOM_Q8, 4>;
    const bool raised = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, MMA_MAX_SMEM) ==
                        cudaSuccess;
    for (int per_sm = 1; per_sm <= 2; ++per_sm) {
        for (int S = 2; S <= MMA_MAX_SPLITS; ++S) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(1, S);
            cfg.blockDim = dim3(32 * MMA_MAX_WARPS / per_sm);
            cfg.dynamicSmemBytes = per_sm == 1 ? 150 * 1024 : 100 * 1024;
            cudaLaunchAttribute at;
            at.id = cudaLaunchAttributeClusterDimension;
            at.val.clusterDim.x = 1;
            at.val.clusterDim.y = S;
            at.val.clusterDim.z = 1;
            cfg.attrs = &at;
            cfg.numAttrs = 1;
            int n = 0;
            if (!raised || cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
                cudaGetLastError();
                n = sms * per_sm / S;
            }
            r.clusters[per_sm][S] = n;
        }
    }
    r.init = true;
}

// Modelled time of a work layout, in ns, used only to choose among layouts. The constants come
// from the measured phases of one launch:
//  - ~10 ns of an SM's issue for one group of one tile and 8 tokens (six 16x8x16 MMAs, their
//    dequantisation and operand loads from shared memory);
//  - ~100 ns per group on one warp's dependent chain;
//  - ~12 ns per KB of activations staged into one SM;
//  - ~1.5 us of launch, reduction and epilogue per wave;
//  - ~0.4 us per CTA of a split-K cluster exchange.
int ctas_per_sm(const Plan& p) {
    const int by_smem = (int)(residency().smem_per_sm / (p.smem + 1024));  // 1 KB reserved per CTA
    return std::max(1, std::min(p.warps > MMA_MAX_WARPS / 2 ? 1 : 2, by_smem));
}

long wave_capacity(const Plan& p) {  // CTAs resident at once
    const Residency& r = residency();
    const int sms = num_sms(), per_sm = ctas_per_sm(p);
    if (p.S == 1) return (long)sms * per_sm;
    return (long)std::max(1, r.init ? r.clusters[per_sm][p.S] : sms * per_sm / p.S) * p.S;
}

double plan_cost(const Plan& p, int tiles, int M, int NB) {
    const int sms = num_sms(), per_sm = ctas_per_sm(p);
    const long cap = wave_capacity(p);
    const long ctas = (long)((tiles + p.T - 1) / p.T) * p.S;
    const long waves = (ctas + cap - 1) / cap;
    const long cps = std::min<long>(per_sm, (std::min(ctas, cap) + sms - 1) / sms);
    const double mma = 10.0 * p.T * p.gps * NB, chain = 100.0 * p.gpw;
    const double stage = 12.0 * (double)M * p.gps * 128 / 1024;
    return (double)waves * (1500.0 + std::max((double)cps * mma, chain) + (double)cps * stage +
                            (p.S > 1 ? 400.0 * p.S : 0.0));
}

// Work layout with one 16-row tile per CTA: K split over a cluster of S CTAs only where the row
// tiles alone leave most SMs idle (or the staged activations of the whole K would not fit); warps
// of 1-2 groups each.
bool plan_one_tile(const QW& w, int M, Plan& p, bool ln) {
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
            p.T = 1;
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

int env_int(const char* name, int dflt) {
    const char* e = std::getenv(name);
    return e && *e ? std::atoi(e) : dflt;
}

// Where one tile per CTA needs more than one wave of CTAs, or more tiles than SMs (two CTAs per
// SM then stage the same activations twice), T tiles per CTA share one staged copy: the layout
// (T, S, warps) of least modelled time among those that fit. GPT2Q_MMA_MULTI=0 keeps one tile;
// GPT2Q_MMA_TILES=<T> takes the best layout of exactly T tiles per CTA where one fits (tests and
// tuning). Both are read at every plan, so a handle created after a change sees it.
bool plan(const QW& w, int M, Plan& p, bool ln) {
    const bool multi = env_int("GPT2Q_MMA_MULTI", 1) != 0;
    const int force_t = std::min(8, std::max(0, env_int("GPT2Q_MMA_TILES", 0)));
    Plan base;
    const bool have = plan_one_tile(w, M, base, ln);
    const int tiles = (w.rows + TILE - 1) / TILE, G = w.cols / 32, NB = (M + 7) / 8;
    const int sms = num_sms();
    if (!force_t && (!multi || (have && tiles <= sms && (long)tiles * base.S <= wave_capacity(base)))) {
        if (!have) return false;
        p = base;
        return true;
    }
    Plan best = base;
    double best_cost = have && !force_t ? plan_cost(base, tiles, M, NB) : 1e30;
    for (int T = force_t ? force_t : 1; T <= (force_t ? force_t : 8); ++T) {
        for (int S = 1; S <= MMA_MAX_SPLITS && S <= G; ++S) {
            const int gps = (G + S - 1) / S;
            if ((G + gps - 1) / gps != S) continue;  // no empty split
            for (int warps = MMA_MAX_WARPS; warps >= MMA_MAX_WARPS / 2; warps -= MMA_MAX_WARPS / 2) {
                const int wt = warps / T;
                if (wt < 1 || 2 * NB * T > warps || (ln && 4 * warps < M)) continue;
                Plan c;
                c.T = T;
                c.S = S;
                c.warps = warps;
                c.gps = gps;
                c.gpw = (gps + wt - 1) / wt;
                c.smem = smem_bytes(w.atom, NB, gps, warps, S, ln, T);
                if (c.smem > (size_t)MMA_MAX_SMEM) continue;
                const double cost = plan_cost(c, tiles, M, NB);
                if (cost < best_cost) {
                    best_cost = cost;
                    best = c;
                }
            }
        }
    }
    if (best_cost >= 1e30) {  // no layout of the forced T fits
        if (!have) return false;
        best = base;
    }
    p = best;
    return true;
}

template <int ATOM, int NB>
cudaError_t launch_nb(const QW& w, const __half* xhi, const __half* xlo, int ldx, int M, const Plan& p, int* err,
                      const Epi& e, const LnFold& ln, cudaStream_t st) {
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
    const dim3 grid(((w.rows + TILE - 1) / TILE + p.T - 1) / p.T, p.S);
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
        (size_t)grid.x * grid.y <= MMA_TRACE_CTAS && ts.skip-- <= 0) {
        tr = ts.buf;
        ts.traced = true;
        ts.grid = grid;
    }
    return cudaLaunchKernelEx(&cfg, kern, w, xhi, xlo, ldx, M, p.T, p.gps, p.gpw, err, tr, e, ln);
}

template <int ATOM>
cudaError_t launch_atom(int NB, const QW& w, const __half* xhi, const __half* xlo, int ldx, int M, const Plan& p,
                        int* err, const Epi& e, const LnFold& ln, cudaStream_t st) {
    switch (NB) {
        case 1: return launch_nb<ATOM, 1>(w, xhi, xlo, ldx, M, p, err, e, ln, st);
        case 2: return launch_nb<ATOM, 2>(w, xhi, xlo, ldx, M, p, err, e, ln, st);
        case 3: return launch_nb<ATOM, 3>(w, xhi, xlo, ldx, M, p, err, e, ln, st);
        case 4: return launch_nb<ATOM, 4>(w, xhi, xlo, ldx, M, p, err, e, ln, st);
        case 5: return launch_nb<ATOM, 5>(w, xhi, xlo, ldx, M, p, err, e, ln, st);
        case 6: return launch_nb<ATOM, 6>(w, xhi, xlo, ldx, M, p, err, e, ln, st);
        case 7: return launch_nb<ATOM, 7>(w, xhi, xlo, ldx, M, p, err, e, ln, st);
        default: return launch_nb<ATOM, 8>(w, xhi, xlo, ldx, M, p, err, e, ln, st);
    }
}

}  // namespace

bool mma_usable(const QW& w, int M) {
    // matrices of many row tiles (the tied head) stay on the tcgen05 GEMM
    return M >= 1 && M <= MMA_MAX_M && (w.atom == ATOM_Q8 || w.atom == ATOM_Q4) && w.cols % 32 == 0 &&
           w.rows >= 1 && (w.rows + TILE - 1) / TILE <= MMA_MAX_TILES;
}

bool head_mma_usable(const QW& w, int M, int ldx) {
    const size_t staged = (size_t)((M + 7) / 8) * 8 * (size_t)ldx * 4;  // hi and lo rows of NB * 8 tokens
    return M >= 1 && M <= MMA_MAX_M && (w.atom == ATOM_Q8 || w.atom == ATOM_Q4) && w.cols % 32 == 0 &&
           w.rows >= 1 && ldx % 8 == 0 && ldx >= w.cols && staged <= (size_t)MMA_MAX_SMEM;
}

namespace {
template <int ATOM, int NB>
cudaError_t launch_head_nb(const QW& w, const __half* xhi, const __half* xlo, int ldx, int M, float* out, int ldo,
                           int* err, cudaStream_t st) {
    auto kern = k_head_mma<ATOM, NB>;
    static unsigned long long raised = 0;  // dynamic shared-memory limit raised once per device
    int dev = 0;
    cudaGetDevice(&dev);
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(raised & bit)) {
        const cudaError_t ae = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, MMA_MAX_SMEM);
        if (ae != cudaSuccess) return ae;
        raised |= bit;
    }
    const int tiles = (w.rows + TILE - 1) / TILE;
    const int tpc = (tiles + num_sms() - 1) / num_sms();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((tiles + tpc - 1) / tpc);
    cfg.blockDim = dim3(32 * MMA_MAX_WARPS);
    cfg.dynamicSmemBytes = (size_t)NB * 8 * ldx * 4;
    cfg.stream = st;
    cudaLaunchAttribute at;
    at.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &at;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, w, xhi, xlo, ldx, M, tpc, out, ldo, err);
}

template <int ATOM>
cudaError_t launch_head_atom(int NB, const QW& w, const __half* xhi, const __half* xlo, int ldx, int M, float* out,
                             int ldo, int* err, cudaStream_t st) {
    switch (NB) {
        case 1: return launch_head_nb<ATOM, 1>(w, xhi, xlo, ldx, M, out, ldo, err, st);
        case 2: return launch_head_nb<ATOM, 2>(w, xhi, xlo, ldx, M, out, ldo, err, st);
        case 3: return launch_head_nb<ATOM, 3>(w, xhi, xlo, ldx, M, out, ldo, err, st);
        case 4: return launch_head_nb<ATOM, 4>(w, xhi, xlo, ldx, M, out, ldo, err, st);
        case 5: return launch_head_nb<ATOM, 5>(w, xhi, xlo, ldx, M, out, ldo, err, st);
        case 6: return launch_head_nb<ATOM, 6>(w, xhi, xlo, ldx, M, out, ldo, err, st);
        case 7: return launch_head_nb<ATOM, 7>(w, xhi, xlo, ldx, M, out, ldo, err, st);
        default: return launch_head_nb<ATOM, 8>(w, xhi, xlo, ldx, M, out, ldo, err, st);
    }
}
}  // namespace

cudaError_t launch_head_mma(const QW& w, const __half* xhi, const __half* xlo, int ldx, int M, float* out, int ldo,
                            int* err, cudaStream_t st) {
    if (M <= 0) return cudaSuccess;
    if (!head_mma_usable(w, M, ldx) || !xhi || !xlo || !out || !err || ldo < w.rows) return cudaErrorInvalidValue;
    const int NB = (M + 7) / 8;
    if (w.atom == ATOM_Q8) return launch_head_atom<ATOM_Q8>(NB, w, xhi, xlo, ldx, M, out, ldo, err, st);
    return launch_head_atom<ATOM_Q4>(NB, w, xhi, xlo, ldx, M, out, ldo, err, st);
}

std::atomic<int> g_tiles_max{0};

void mma_init() {
    trace_state();  // the trace buffer, if any, is allocated here, never during a graph capture
    num_sms();
    init_residency();
    g_tiles_max = 0;
}

int mma_tiles_per_cta_max() { return g_tiles_max.load(); }

bool mma_fits(const QW& w, int M, bool ln) {
    Plan p;
    return mma_usable(w, M) && plan(w, M, p, ln);
}

cudaError_t launch_linear_mma(const QW& w, const __half* xhi, const __half* xlo, int ldx, int M, int* err,
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
    for (int cur = g_tiles_max.load(); p.T > cur && !g_tiles_max.compare_exchange_weak(cur, p.T);) {
    }
    const int NB = (M + 7) / 8;
    if (w.atom == ATOM_Q8) return launch_atom<ATOM_Q8>(NB, w, xhi, xlo, ldx, M, p, err, e, lf, st);
    return launch_atom<ATOM_Q4>(NB, w, xhi, xlo, ldx, M, p, err, e, lf, st);
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
