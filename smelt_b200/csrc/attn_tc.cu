// Causal prefill attention on the tensor cores (tcgen05 / TMEM), one CTA per
// (128-query tile, head), two CTAs per SM (97 KB shared memory, 256 TMEM columns each), so
// one CTA's softmax and operand conversion overlap the other's MMAs.
//
// Per key block of 64 positions:
//   S  = (Q * 2^-3) K^T          tcgen05.mma kind::f16, M = 128 queries, N = 64 keys, K = 64
//   P  = exp(S - m_new)          one thread per query row (TMEM lane), online softmax in fp32
//   PV = P V                     tcgen05.mma, M = 128, N = 64 (head dim), K = 64 keys
//   O  = O * exp(m_old - m_new) + PV   (O in registers)
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
// Operands are K-major tiles with the 128-byte swizzle (rows of 64 fp16; 8-row groups 1024
// bytes apart), as in gemm.cu: Q [128 q][64], K [64 keys][64], P [128 q][64 keys] and
// V^T [64 dims][64 keys] (V is transposed while it is converted). Threads 0-63 convert the K
// rows, threads 64-127 the V rows of a block. Reference semantics: gpt2.rs:261-291
// (softmax(q.K^T / sqrt(hd)) . V over positions 0..t), per query position t of the prompt.
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
constexpr int THREADS = 128;
constexpr int TILE_Q = QT * 128;   // bytes of one [128][64] fp16 tile
constexpr int TILE_K = KB * 128;   // bytes of one [64][64] fp16 tile
constexpr int OFF_QH = 0, OFF_QL = OFF_QH + TILE_Q;
// K_hi and K_lo adjacent: [K_hi; K_lo] is one 128-row B operand; same for V^T
constexpr int OFF_KH = OFF_QL + TILE_Q, OFF_KL = OFF_KH + TILE_K;
constexpr int OFF_VH = OFF_KL + TILE_K, OFF_VL = OFF_VH + TILE_K;
constexpr int OFF_PH = OFF_VL + TILE_K, OFF_PL = OFF_PH + TILE_Q;
constexpr int OFF_BAR = OFF_PL + TILE_Q;
constexpr int SMEM = OFF_BAR + 64 + 1024;  // barriers, TMEM slot, block-max scratch, alignment slack
static_assert(SMEM <= 232448 / 2 - 1024, "two CTAs per SM");
// S: columns 0..127 (Q_hi K_hi | Q_hi K_lo, Q_lo K_hi added to the first half);
// PV: 128..255 (P_hi V_hi | P_hi V_lo, P_lo V_hi added to the first half)
constexpr uint32_t TMEM_COLS = 256;

// Phase trace of one launch (GPT2Q_ATTN_TRACE set at the first launch): globaltimer stamps of
// thread 0 of the first ATR_CTAS CTAs: start, Q staged, then per key block kb < 8: K/V staged,
// S ready, P staged, PV ready.
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

// Row r of a [rows][64] tile from 64 fp32 values (times `mul`, a power of two): hi and lo.
__device__ __forceinline__ void put_row64(uint8_t* hi, uint8_t* lo, int r, const float* v, float mul) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        uint32_t h[4], l[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            __half2 h2, l2;
            split_hl2(v[8 * c + 2 * j] * mul, v[8 * c + 2 * j + 1] * mul, h2, l2);
            h[j] = *reinterpret_cast<uint32_t*>(&h2);
            l[j] = *reinterpret_cast<uint32_t*>(&l2);
        }
        const uint32_t o = sw_off(r, c);
        *reinterpret_cast<uint4*>(hi + o) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4*>(lo + o) = make_uint4(l[0], l[1], l[2], l[3]);
    }
}

// 2^e as a float, e in [-126, 127].
__device__ __forceinline__ float pow2f(int e) { return __int_as_float((e + 127) << 23); }

// Exponent e with m * 2^e in [2^13, 2^14) for m > 0 (0 for m == 0 or subnormal), in [-60, 60].
__device__ __forceinline__ int scale_exp(float m) {
    const int b = (__float_as_int(m) >> 23) & 0xff;
    if (b == 0) return 0;
    return max(-60, min(60, 13 - (b - 127)));
}

__device__ __forceinline__ float row_absmax(const float* v) {
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < 64; ++i) m = fmaxf(m, fabsf(v[i]));
    return m;
}

// Maxima over the 128 threads of the CTA of two values at once (red: 8 floats of shared memory).
__device__ __forceinline__ float2 block_max2(float a, float b, float* red) {
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
        b = fmaxf(b, __shfl_xor_sync(0xffffffffu, b, o));
    }
    if ((threadIdx.x & 31) == 0) {
        red[threadIdx.x >> 5] = a;
        red[4 + (threadIdx.x >> 5)] = b;
    }
    __syncthreads();
    const float2 r = make_float2(fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3])),
                                 fmaxf(fmaxf(red[4], red[5]), fmaxf(red[6], red[7])));
    __syncthreads();  // red is reused by the next call
    return r;
}

__device__ __forceinline__ void load_row64(const float* src, bool ok, float* v) {
#pragma unroll
    for (int i = 0; i < 64; i += 4) {
        // coherent loads: q and K/V come from the preceding kernel, and a non-coherent (__ldg)
        // load could be scheduled above griddepcontrol.wait
        float4 x = ok ? __ldcg(reinterpret_cast<const float4*>(src + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
        v[i] = x.x;
        v[i + 1] = x.y;
        v[i + 2] = x.z;
        v[i + 3] = x.w;
    }
}

__global__ void __launch_bounds__(THREADS, 2)
    k_attn_prefill_tc(const float* q, int ldq, KVGeom g, size_t layer_off,
                      const AttnTile* __restrict__ tiles, float* __restrict__ out, __half* __restrict__ ohi,
                      __half* __restrict__ olo, int ldo, int* err, bool trace) {
    extern __shared__ __align__(1024) uint8_t smem_raw_[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw_) + 1023) & ~uintptr_t(1023));
    uint64_t* bar_s = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint64_t* bar_pv = bar_s + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_s + 2);
    float* red = reinterpret_cast<float*>(bar_s + 3);  // [8]
    const int tid = threadIdx.x, warp = tid >> 5;

    if (tid == 0) {
        tc::mbar_init(bar_s, 1);
        tc::mbar_init(bar_pv, 1);
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
    const uint32_t t_lane = tmem + ((uint32_t)(warp * 32) << 16);  // this warp's TMEM lanes

    tc::pdl_wait();  // q and the K/V rows were written by the preceding kernels
    atr_stamp(trace, 0);
    const AttnTile tile = tiles[blockIdx.y];
    const int head = blockIdx.x;
    const float* Kc = g.base + (size_t)tile.slot * g.slot_stride + layer_off + (size_t)head * g.head_stride;
    const float* Vc = Kc + g.sel_stride;
    const int qpos = tile.q0 + tid;  // this thread's query position (TMEM lane tid)
    const bool qvalid = qpos < tile.T;

    // ---- Q tile, row scaled by 2^eq ----
    int eq;
    {
        float v[64];
        load_row64(q + (size_t)(tile.row0 + (qvalid ? qpos : 0)) * ldq + head * HD, qvalid, v);
        eq = scale_exp(row_absmax(v));
        put_row64(smem + OFF_QH, smem + OFF_QL, tid, v, pow2f(eq));
    }
    atr_stamp(trace, 1);

    constexpr uint32_t idesc_s2 = tc::idesc_f16_f32(QT, 2 * KB);  // Q_hi [K_hi; K_lo]
    constexpr uint32_t idesc_s = tc::idesc_f16_f32(QT, KB);
    constexpr uint32_t idesc_pv2 = tc::idesc_f16_f32(QT, 2 * HD);  // P_hi [V^T_hi; V^T_lo]
    constexpr uint32_t idesc_pv = tc::idesc_f16_f32(QT, HD);
    float o[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) o[i] = 0.f;
    float m = -INFINITY, l = 0.f;
    const int kend = min(tile.T, tile.q0 + QT);  // keys past the last query of the tile are masked
    const int nkb = (kend + KB - 1) / KB;
    const bool is_k = tid < KB;        // threads 0-63: K row tid; 64-127: V row tid - 64
    const int krow = tid & (KB - 1);
    bool ok = true;
    for (int kb = 0; kb < nkb; ++kb) {
        const int k0 = kb * KB;
        // ---- K tile and V^T tile of keys k0..k0+63, each scaled by 2^ek / 2^ev of the block ----
        int ek, ev;
        {
            const int kp = k0 + krow;
            const bool kvalid = kp < kend;
            float v[64];
            load_row64((is_k ? Kc : Vc) + (size_t)(kvalid ? kp : 0) * HD, kvalid, v);
            const float am = row_absmax(v);
            const float2 mx = block_max2(is_k ? am : 0.f, is_k ? 0.f : am, red);
            ek = scale_exp(mx.x);
            ev = scale_exp(mx.y);
            if (is_k) {
                put_row64(smem + OFF_KH, smem + OFF_KL, krow, v, pow2f(ek));
            } else {
                // V^T column krow: element (dim d, key) -> row d
                const float sv = pow2f(ev);
#pragma unroll
                for (int dd = 0; dd < 64; dd += 2) {
                    __half2 h, lo;
                    split_hl2(v[dd] * sv, v[dd + 1] * sv, h, lo);
                    const uint32_t off0 = sw_off(dd, krow >> 3) + (uint32_t)((krow & 7) * 2);
                    const uint32_t off1 = sw_off(dd + 1, krow >> 3) + (uint32_t)((krow & 7) * 2);
                    *reinterpret_cast<__half*>(smem + OFF_VH + off0) = __low2half(h);
                    *reinterpret_cast<__half*>(smem + OFF_VL + off0) = __low2half(lo);
                    *reinterpret_cast<__half*>(smem + OFF_VH + off1) = __high2half(h);
                    *reinterpret_cast<__half*>(smem + OFF_VL + off1) = __high2half(lo);
                }
            }
        }
        tc::fence_proxy_async_smem();
        tc::tc_fence_before();
        __syncthreads();
        atr_stamp(trace, 2 + 4 * kb);
        // ---- S = Q K^T ----
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
        ok = tc::mbar_wait_spin(bar_s, (uint32_t)(kb & 1), err) && ok;
        tc::tc_fence_after();
        atr_stamp(trace, 3 + 4 * kb);
        // ---- online softmax of this thread's query row ----
        float s[KB];
        {
            float u[32];
            tc::tmem_ld32x2(t_lane, t_lane + KB, *reinterpret_cast<float(*)[32]>(s), u);
#pragma unroll
            for (int j = 0; j < 32; ++j) s[j] += u[j];
            tc::tmem_ld32x2(t_lane + 32, t_lane + KB + 32, *reinterpret_cast<float(*)[32]>(s + 32), u);
#pragma unroll
            for (int j = 0; j < 32; ++j) s[32 + j] += u[j];
        }
        const float s_unscale = pow2f(-(eq + ek) - 3);  // operand scales and 1/sqrt(64)
        float bmax = -INFINITY;
#pragma unroll
        for (int j = 0; j < KB; ++j) {
            const int kp = k0 + j;
            s[j] = (kp > qpos || kp >= tile.T) ? -INFINITY : s[j] * s_unscale;
            bmax = fmaxf(bmax, s[j]);
        }
        const float mnew = fmaxf(m, bmax);
        const float alpha = (mnew == -INFINITY) ? 1.f : __expf(m - mnew);
        float psum = 0.f;
#pragma unroll
        for (int c = 0; c < KB / 8; ++c) {  // 8 chunks of 8 keys
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
            const uint32_t off = sw_off(tid, c);
            *reinterpret_cast<uint4*>(smem + OFF_PH + off) = make_uint4(h[0], h[1], h[2], h[3]);
            *reinterpret_cast<uint4*>(smem + OFF_PL + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
        l = l * alpha + psum;
        m = mnew;
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
                const uint32_t ko = ks * 32;
                tc::mma_f16(tmem + 128, tc::desc_sw128(ph + ko), tc::desc_sw128(vh + ko), idesc_pv2, ks > 0 ? 1u : 0u);
                tc::mma_f16(tmem + 128, tc::desc_sw128(pl + ko), tc::desc_sw128(vh + ko), idesc_pv, 1u);
            }
            tc::mma_commit(bar_pv);
        }
        ok = tc::mbar_wait_spin(bar_pv, (uint32_t)(kb & 1), err) && ok;
        tc::tc_fence_after();
        atr_stamp(trace, 5 + 4 * kb);
        float pv[HD];
        {
            float u[32];
            tc::tmem_ld32x2(t_lane + 128, t_lane + 128 + HD, *reinterpret_cast<float(*)[32]>(pv), u);
#pragma unroll
            for (int j = 0; j < 32; ++j) pv[j] += u[j];
            tc::tmem_ld32x2(t_lane + 160, t_lane + 160 + HD, *reinterpret_cast<float(*)[32]>(pv + 32), u);
#pragma unroll
            for (int j = 0; j < 32; ++j) pv[32 + j] += u[j];
        }
        const float pv_unscale = pow2f(-14 - ev);
#pragma unroll
        for (int i = 0; i < HD; ++i) o[i] = fmaf(o[i], alpha, pv[i] * pv_unscale);
    }
    // ---- out = O / l (fp32 and the fp16 hi/lo copy for the c_proj GEMM) ----
    if (qvalid && ok) {
        const size_t base = (size_t)(tile.row0 + qpos) * ldo + head * HD;
        const float inv = 1.0f / l;
#pragma unroll
        for (int i = 0; i < HD; i += 4) {
            float r[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) r[j] = o[i + j] * inv;
            *reinterpret_cast<float4*>(out + base + i) = make_float4(r[0], r[1], r[2], r[3]);
            if (ohi) {
                __half h[4], lo[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) split_hl(r[j], h[j], lo[j]);
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
