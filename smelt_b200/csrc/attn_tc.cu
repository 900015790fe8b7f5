// Causal prefill attention on the tensor cores (tcgen05 / TMEM), one CTA of 256 threads per
// (128-query tile, head), two CTAs per SM (98 KB shared memory, 256 TMEM columns each), so
// one CTA's softmax and operand conversion overlap the other's MMAs.
//
// Per key block of 64 positions:
//   S  = (Q * 2^-3) K^T          tcgen05.mma kind::f16, M = 128 queries, N = 64 keys, K = 64
//   P  = exp(S - m_new)          two threads per query row (TMEM lane), online softmax in fp32
//   PV = P V                     tcgen05.mma, M = 128, N = 64 (head dim), K = 64 keys
//   O  = O * exp(m_old - m_new) + PV   (O in registers, 32 dimensions per thread)
// Both products use the fp16x3 split of gemm.cu: every fp32 operand x is held as
// x_hi + x_lo (fp16 pair, ~22 bits) and A_hi B_hi + A_hi B_lo + A_lo B_hi accumulate in fp32
// TMEM, so scores and outputs keep fp32-class accuracy (the dropped lo*lo term is ~2^-22
// relative). B_hi and B_lo sit next to each other, so A_hi [B_hi; B_lo] is one MMA of twice
// the width and each k-step issues two MMAs instead of three (the MMA issue rate, not its
// width, bounds these tiles). The pair only keeps 22 bits while lo is a normal fp16, so every
// operand is first scaled by a power of two that brings its largest magnitude to
// [2^13, 2^14): Q per query row, K and V per key block, P by 2^14. The scales are undone
// exactly on S and PV, together with the attention scale 1/sqrt(64) = 2^-3.
//
// Operands are tiles with the 128-byte swizzle (rows of 64 fp16; 8-row groups 1024 bytes
// apart), as in gemm.cu: Q [128 q][64], K [64 keys][64] and P [128 q][64 keys] K-major, V
// [64 keys][64 dims] the same bytes read as an MN-major B operand. The raw fp32 rows of a key
// block (16 KB each for K and V, contiguous in the cache) arrive by one 1-D bulk copy into the
// very area their hi/lo tiles occupy, issued as soon as that area is free: K's after the S MMAs
// of the previous block, V's after its PV MMAs. A block's conversion then reads shared memory
// (four threads per key row), holds its values in registers across the block maximum's barrier
// and writes the tiles in place. Reference semantics: gpt2.rs:261-291 (softmax(q.K^T / sqrt(hd))
// . V over positions 0..t), per query position t of the prompt.
#include <cuda_fp16.h>

#include <cstdlib>
#include <string>
#include <vector>

#include "kernels.h"
#include "tcgen05.cuh"

namespace gpt2q {
namespace {

constexpr int QT = 128;  // queries per CTA (TMEM lanes)
constexpr int KB = 64;   // keys per block
constexpr int HD = 64;
constexpr int THREADS = 256;  // two threads per query row
constexpr int TILE_Q = QT * 128;   // bytes of one [128][64] fp16 tile
constexpr int TILE_K = KB * 128;   // bytes of one [64][64] fp16 tile
constexpr int OFF_QH = 0, OFF_QL = OFF_QH + TILE_Q;
// K_hi and K_lo adjacent: [K_hi; K_lo] is one 128-row B operand; same for V^T
constexpr int OFF_KH = OFF_QL + TILE_Q, OFF_KL = OFF_KH + TILE_K;
constexpr int OFF_VH = OFF_KL + TILE_K, OFF_VL = OFF_VH + TILE_K;
constexpr int OFF_PH = OFF_VL + TILE_K, OFF_PL = OFF_PH + TILE_Q;
constexpr int OFF_BAR = OFF_PL + TILE_Q;
constexpr int OFF_XCH = OFF_BAR + 128;              // [2][QT] floats: the halves of a query row
constexpr int SMEM = OFF_XCH + 2 * QT * 4 + 1024;  // + alignment slack
static_assert(SMEM <= 232448 / 2 - 1024, "two CTAs per SM");
// S: columns 0..127 (Q_hi K_hi | Q_hi K_lo, Q_lo K_hi added to the first half);
// PV: 128..255 (P_hi V_hi | P_hi V_lo, P_lo V_hi added to the first half)
constexpr uint32_t TMEM_COLS = 256;

// Phase trace of one launch (GPT2Q_ATTN_TRACE set at the first launch): globaltimer stamps of
// thread 0 of the first ATR_CTAS CTAs: start, Q staged, then per key block kb < 8: iteration
// start (its K converted, S issued), S ready, P and V staged, PV ready (the next block's K
// converted and S issued meanwhile).
constexpr int ATR_CTAS = 128, ATR_N = 2 + 4 * 8;
__device__ unsigned long long g_attn_trace[ATR_CTAS * ATR_N];

__device__ __forceinline__ void atr_stamp(bool on, int k) {
    const int cta = blockIdx.y * gridDim.x + blockIdx.x;
    if (on && threadIdx.x == 0 && cta < ATR_CTAS && k < ATR_N) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        g_attn_trace[cta * ATR_N + k] = t;
    }
}

// Byte offset of 16-byte chunk c (8 fp16) of row r in a 128-byte-swizzled K-major tile.
__device__ __forceinline__ uint32_t sw_off(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ uint32_t pack_h2(__half a, __half b) {
    return (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
}

// 2^e as a float, e in [-126, 127].
__device__ __forceinline__ float pow2f(int e) { return __int_as_float((e + 127) << 23); }

// Exponent e with m * 2^e in [2^13, 2^14) for m > 0 (0 for m == 0 or subnormal), in [-60, 60].
__device__ __forceinline__ int scale_exp(float m) {
    const int b = (__float_as_int(m) >> 23) & 0xff;
    if (b == 0) return 0;
    return max(-60, min(60, 13 - (b - 127)));
}

// Maximum over the THREADS threads of the CTA (red: 8 floats of shared memory).
__device__ __forceinline__ float block_max(float a, float* red) {
#pragma unroll
    for (int o = 16; o; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = a;
    __syncthreads();
    float r = red[0];
#pragma unroll
    for (int w = 1; w < THREADS / 32; ++w) r = fmaxf(r, red[w]);
    __syncthreads();  // red is reused by the next call
    return r;
}

__global__ void __launch_bounds__(THREADS, 2)
    k_attn_prefill_tc(const float* q, int ldq, KVGeom g, size_t layer_off,
                      const AttnTile* __restrict__ tiles, float* __restrict__ out, __half* __restrict__ ohi,
                      __half* __restrict__ olo, int ldo, int* err, bool trace) {
    extern __shared__ __align__(1024) uint8_t smem_raw_[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw_) + 1023) & ~uintptr_t(1023));
    uint64_t* bar_s = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint64_t* bar_pv = bar_s + 1;
    uint64_t* bar_k = bar_s + 2;  // raw K rows of a block landed in the K area
    uint64_t* bar_v = bar_s + 3;  // raw V rows landed in the V area
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_s + 4);
    float* red = reinterpret_cast<float*>(bar_s + 6);        // [8] block maxima
    float* xch = reinterpret_cast<float*>(smem + OFF_XCH);   // [2][QT]: the two halves of a query row
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // query row r (TMEM lane) of this thread, and its half: keys 32h..32h+31 of each block in
    // the softmax, head dimensions 32h..32h+31 of the output (a warp reads only its own lane
    // quarter of TMEM: warps w and w + 4 share lanes 32 (w % 4) ..)
    const int quarter = warp & 3, half = warp >> 2;
    const int r = quarter * 32 + lane;

    if (tid == 0) {
        tc::mbar_init(bar_s, 1);
        tc::mbar_init(bar_pv, 1);
        tc::mbar_init(bar_k, 1);
        tc::mbar_init(bar_v, 1);
        tc::fence_mbar_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(tmem_slot, TMEM_COLS);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    tc::pdl_trigger();  // after the TMEM allocation: dependents never hold columns this CTA waits for
    const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);  // this warp's TMEM lanes

    tc::pdl_wait();  // q and the K/V rows were written by the preceding kernels
    atr_stamp(trace, 0);
    const AttnTile tile = tiles[blockIdx.y];
    const int head = blockIdx.x;
    const float* Kc = g.base + (size_t)tile.slot * g.slot_stride + layer_off + (size_t)head * g.head_stride;
    const float* Vc = Kc + g.sel_stride;
    const int qpos = tile.q0 + r;  // this thread's query position
    const bool qvalid = qpos < tile.T;
    const int kend = min(tile.T, tile.q0 + QT);  // keys past the last query of the tile are masked
    const int nkb = (kend + KB - 1) / KB;
    // raw fp32 K (or V) rows of key block kb into the K (V) operand area: 64 rows x 256 bytes =
    // the 16 KB of its hi/lo tiles, contiguous in the cache
    auto fetch = [&](uint64_t* bar, int area, const float* src, int kb) {
        const uint32_t bytes = (uint32_t)min(KB, kend - kb * KB) * HD * 4;
        tc::mbar_arrive_expect_tx(bar, bytes);
        tc::bulk_load_1d(smem + area, src + (size_t)kb * KB * HD, bytes, bar);
    };
    if (tid == 0 && nkb > 0) {
        fetch(bar_k, OFF_KH, Kc, 0);
        fetch(bar_v, OFF_VH, Vc, 0);
    }

    // ---- Q tile, row scaled by 2^eq (the row maximum over both halves) ----
    int eq;
    {
        float v[32];
        const float* src = q + (size_t)(tile.row0 + (qvalid ? qpos : 0)) * ldq + head * HD + half * 32;
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
            // coherent loads: q comes from the preceding kernel, and a non-coherent (__ldg) load
            // could be scheduled above griddepcontrol.wait
            const float4 x = qvalid ? __ldcg(reinterpret_cast<const float4*>(src + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
            v[i] = x.x;
            v[i + 1] = x.y;
            v[i + 2] = x.z;
            v[i + 3] = x.w;
        }
        float am = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) am = fmaxf(am, fabsf(v[i]));
        xch[half * QT + r] = am;
        __syncthreads();
        eq = scale_exp(fmaxf(xch[r], xch[QT + r]));
        __syncthreads();  // xch is reused
        const float sq = pow2f(eq);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            uint32_t h[4], lo[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                __half2 h2, l2;
                split_hl2(v[8 * c + 2 * j] * sq, v[8 * c + 2 * j + 1] * sq, h2, l2);
                h[j] = *reinterpret_cast<uint32_t*>(&h2);
                lo[j] = *reinterpret_cast<uint32_t*>(&l2);
            }
            const uint32_t o = sw_off(r, 4 * half + c);
            *reinterpret_cast<uint4*>(smem + OFF_QH + o) = make_uint4(h[0], h[1], h[2], h[3]);
            *reinterpret_cast<uint4*>(smem + OFF_QL + o) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
    }
    atr_stamp(trace, 1);

    constexpr uint32_t idesc_s2 = tc::idesc_f16_f32(QT, 2 * KB);  // Q_hi [K_hi; K_lo]
    constexpr uint32_t idesc_s = tc::idesc_f16_f32(QT, KB);
    // V tiles are [keys][64 dims] rows, an MN-major B operand; V_lo follows V_hi as a second
    // 64-wide atom along N: P_hi [V_hi | V_lo] is one MMA of N = 128
    constexpr uint32_t idesc_pv2 = tc::idesc_f16_f32_bmn(QT, 2 * HD);
    constexpr uint32_t idesc_pv = tc::idesc_f16_f32_bmn(QT, HD);
    float o[32];  // output dimensions 32 half .. 32 half + 31 of query row r
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] = 0.f;
    float m = -INFINITY, l = 0.f;  // l: this half's share of the row sum
    // block conversion: four threads per key row, 16 values each
    const int krow = tid >> 2, kq = tid & 3;
    bool ok = true;
    // ---- K of block kb: raw rows (prefetched) -> scaled by 2^ek of the block -> hi/lo tiles in
    // place (every thread holds its values before the block maximum's barrier); returns ek ----
    auto convert_k = [&](int kb) {
        const bool kvalid = kb * KB + krow < kend;
        ok = tc::mbar_wait_spin(bar_k, (uint32_t)(kb & 1), err) && ok;
        float v[16];
        const float* src = reinterpret_cast<const float*>(smem + OFF_KH) + krow * HD + kq * 16;
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
            const float4 x = kvalid ? *reinterpret_cast<const float4*>(src + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            v[i] = x.x;
            v[i + 1] = x.y;
            v[i + 2] = x.z;
            v[i + 3] = x.w;
        }
        float am = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) am = fmaxf(am, fabsf(v[i]));
        const int e = scale_exp(block_max(am, red));
        const float sk = pow2f(e);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            uint32_t h[4], lo[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                __half2 h2, l2;
                split_hl2(v[8 * c + 2 * j] * sk, v[8 * c + 2 * j + 1] * sk, h2, l2);
                h[j] = *reinterpret_cast<uint32_t*>(&h2);
                lo[j] = *reinterpret_cast<uint32_t*>(&l2);
            }
            const uint32_t off = sw_off(krow, 2 * kq + c);
            *reinterpret_cast<uint4*>(smem + OFF_KH + off) = make_uint4(h[0], h[1], h[2], h[3]);
            *reinterpret_cast<uint4*>(smem + OFF_KL + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
        tc::fence_proxy_async_smem();
        tc::tc_fence_before();
        __syncthreads();
        return e;
    };
    // ---- S = Q K^T of the block in the K area (one thread issues) ----
    auto issue_s = [&]() {
        if (tid == 0) {
            tc::tc_fence_after();
            const uint32_t qh = tc::smem_u32(smem + OFF_QH), ql = tc::smem_u32(smem + OFF_QL);
            const uint32_t kh = tc::smem_u32(smem + OFF_KH);
#pragma unroll
            for (int ks = 0; ks < HD / 16; ++ks) {
                const uint32_t ko = ks * 32;
                tc::mma_f16(tmem, tc::desc_sw128(qh + ko), tc::desc_sw128(kh + ko), idesc_s2, ks > 0 ? 1u : 0u);
                tc::mma_f16(tmem, tc::desc_sw128(ql + ko), tc::desc_sw128(kh + ko), idesc_s, 1u);
            }
            tc::mma_commit(bar_s);
        }
    };
    int ek = 0;
    if (nkb > 0) {
        ek = convert_k(0);
        issue_s();
    }
    for (int kb = 0; kb < nkb; ++kb) {
        const int k0 = kb * KB;
        const bool kvalid = k0 + krow < kend;
        atr_stamp(trace, 2 + 4 * kb);
        ok = tc::mbar_wait_spin(bar_s, (uint32_t)(kb & 1), err) && ok;
        tc::tc_fence_after();
        // the K area is free until the next block's conversion: its raw rows fly meanwhile
        if (tid == 0 && kb + 1 < nkb) fetch(bar_k, OFF_KH, Kc, kb + 1);
        atr_stamp(trace, 3 + 4 * kb);
        // ---- online softmax: keys 32 half .. 32 half + 31 of query row r ----
        float s[32];
        {
            float u[32];
            tc::tmem_ld32x2(t_lane + 32 * half, t_lane + KB + 32 * half, s, u);
#pragma unroll
            for (int j = 0; j < 32; ++j) s[j] += u[j];
        }
        const float s_unscale = pow2f(-(eq + ek) - 3);  // operand scales and 1/sqrt(64)
        float bmax = -INFINITY;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const int kp = k0 + 32 * half + j;
            s[j] = (kp > qpos || kp >= tile.T) ? -INFINITY : s[j] * s_unscale;
            bmax = fmaxf(bmax, s[j]);
        }
        xch[half * QT + r] = bmax;  // the row maximum over both halves
        __syncthreads();
        const float mnew = fmaxf(m, fmaxf(xch[r], xch[QT + r]));
        const float alpha = (mnew == -INFINITY) ? 1.f : __expf(m - mnew);
        float psum = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {  // 4 chunks of 8 keys
            uint32_t h[4], lo[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float p0 = (mnew == -INFINITY) ? 0.f : __expf(s[8 * c + 2 * j] - mnew);
                const float p1 = (mnew == -INFINITY) ? 0.f : __expf(s[8 * c + 2 * j + 1] - mnew);
                psum += p0 + p1;
                __half2 h2, l2;
                split_hl2(p0 * 16384.0f, p1 * 16384.0f, h2, l2);  // P * 2^14
                h[j] = *reinterpret_cast<uint32_t*>(&h2);
                lo[j] = *reinterpret_cast<uint32_t*>(&l2);
            }
            const uint32_t off = sw_off(r, 4 * half + c);
            *reinterpret_cast<uint4*>(smem + OFF_PH + off) = make_uint4(h[0], h[1], h[2], h[3]);
            *reinterpret_cast<uint4*>(smem + OFF_PL + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
        l = l * alpha + psum;
        m = mnew;
        // ---- V of the block: raw rows (prefetched) -> scaled by 2^ev -> hi/lo tiles in place, rows
        // of keys as for K ----
        int ev;
        {
            ok = tc::mbar_wait_spin(bar_v, (uint32_t)(kb & 1), err) && ok;
            float v[16];
            const float* src = reinterpret_cast<const float*>(smem + OFF_VH) + krow * HD + kq * 16;
#pragma unroll
            for (int i = 0; i < 16; i += 4) {
                const float4 x = kvalid ? *reinterpret_cast<const float4*>(src + i) : make_float4(0.f, 0.f, 0.f, 0.f);
                v[i] = x.x;
                v[i + 1] = x.y;
                v[i + 2] = x.z;
                v[i + 3] = x.w;
            }
            float am = 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) am = fmaxf(am, fabsf(v[i]));
            ev = scale_exp(block_max(am, red));  // its first barrier also orders xch's reads above
            const float sv = pow2f(ev);
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t h[4], lo[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    __half2 h2, l2;
                    split_hl2(v[8 * c + 2 * j] * sv, v[8 * c + 2 * j + 1] * sv, h2, l2);
                    h[j] = *reinterpret_cast<uint32_t*>(&h2);
                    lo[j] = *reinterpret_cast<uint32_t*>(&l2);
                }
                const uint32_t off = sw_off(krow, 2 * kq + c);
                *reinterpret_cast<uint4*>(smem + OFF_VH + off) = make_uint4(h[0], h[1], h[2], h[3]);
                *reinterpret_cast<uint4*>(smem + OFF_VL + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            }
        }
        tc::fence_proxy_async_smem();
        tc::tc_fence_before();
        __syncthreads();
        atr_stamp(trace, 4 + 4 * kb);
        // ---- PV = P V (columns 128..255) ----
        if (tid == 0) {
            tc::tc_fence_after();
            const uint32_t ph = tc::smem_u32(smem + OFF_PH), pl = tc::smem_u32(smem + OFF_PL);
            const uint32_t vh = tc::smem_u32(smem + OFF_VH);
#pragma unroll
            for (int ks = 0; ks < KB / 16; ++ks) {
                const uint32_t ko = ks * 32;           // 16 keys of P's K-major rows
                const uint32_t vo = ks * 16 * 128;     // 16 key rows of V (two 8-row groups)
                const uint64_t dv = tc::desc_sw128_mn(vh + vo, OFF_VL - OFF_VH);
                tc::mma_f16(tmem + 128, tc::desc_sw128(ph + ko), dv, idesc_pv2, ks > 0 ? 1u : 0u);
                tc::mma_f16(tmem + 128, tc::desc_sw128(pl + ko), dv, idesc_pv, 1u);
            }
            tc::mma_commit(bar_pv);
        }
        // the next block's K conversion and S MMAs run while this block's PV MMAs do (S and PV
        // accumulate in disjoint TMEM columns)
        if (kb + 1 < nkb) {
            ek = convert_k(kb + 1);
            issue_s();
        }
        ok = tc::mbar_wait_spin(bar_pv, (uint32_t)(kb & 1), err) && ok;
        tc::tc_fence_after();
        if (tid == 0 && kb + 1 < nkb) fetch(bar_v, OFF_VH, Vc, kb + 1);  // the V area is free now
        atr_stamp(trace, 5 + 4 * kb);
        float pv[32];
        {
            float u[32];
            tc::tmem_ld32x2(t_lane + 128 + 32 * half, t_lane + 128 + HD + 32 * half, pv, u);
#pragma unroll
            for (int j = 0; j < 32; ++j) pv[j] += u[j];
        }
        const float pv_unscale = pow2f(-14 - ev);
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = fmaf(o[i], alpha, pv[i] * pv_unscale);
    }
    // ---- out = O / l, l the sum of both halves' shares (fp32 and the fp16 hi/lo copy for the
    // c_proj GEMM) ----
    xch[half * QT + r] = l;
    __syncthreads();
    l = xch[r] + xch[QT + r];
    if (qvalid && ok) {
        const size_t base = (size_t)(tile.row0 + qpos) * ldo + head * HD + half * 32;
        const float inv = 1.0f / l;
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
            float rr[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) rr[j] = o[i + j] * inv;
            if (out) *reinterpret_cast<float4*>(out + base + i) = make_float4(rr[0], rr[1], rr[2], rr[3]);
            if (ohi) {
                __half h[4], lo[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) split_hl(rr[j], h[j], lo[j]);
                *reinterpret_cast<uint2*>(ohi + base + i) = make_uint2(pack_h2(h[0], h[1]), pack_h2(h[2], h[3]));
                *reinterpret_cast<uint2*>(olo + base + i) = make_uint2(pack_h2(lo[0], lo[1]), pack_h2(lo[2], lo[3]));
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tmem, TMEM_COLS);
}

}  // namespace

cudaError_t launch_attn_prefill_tc(const float* q, int ldq, const KVGeom& g, size_t layer_off, const AttnTile* tiles,
                                   int n_tiles, float* out, __half* ohi, __half* olo, int ldo, int n_head, int* err,
                                   cudaStream_t st) {
    if (n_tiles <= 0) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(k_attn_prefill_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_head, n_tiles);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = SMEM;
    cfg.stream = st;
    cudaLaunchAttribute at;
    at.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &at;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    static bool trace_pending = std::getenv("GPT2Q_ATTN_TRACE") != nullptr;
    const bool trace = trace_pending;
    trace_pending = false;
    return cudaLaunchKernelEx(&cfg, k_attn_prefill_tc, q, ldq, g, layer_off, tiles, out, ohi, olo, ldo, err, trace);
}

std::string attn_tc_trace_json() {
    if (!std::getenv("GPT2Q_ATTN_TRACE")) return "";
    std::vector<unsigned long long> t(ATR_CTAS * ATR_N);
    if (cudaMemcpyFromSymbol(t.data(), g_attn_trace, t.size() * 8) != cudaSuccess) return "";
    unsigned long long t0 = ~0ull;
    for (auto v : t)
        if (v && v < t0) t0 = v;
    std::string s = "[";
    for (int c = 0; c < ATR_CTAS; ++c) {
        s += c ? ", [" : "[";
        for (int k = 0; k < ATR_N; ++k) {
            const unsigned long long v = t[c * ATR_N + k];
            s += (k ? ", " : "") + std::to_string(v ? (long long)(v - t0) : -1);
        }
        s += "]";
    }
    return s + "]";
}

}  // namespace gpt2q
