// Shared device-side definitions for the gpt2q kernels (sm_100a).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gpt2q {

// Weight atoms as stored in HBM after upload (see repack kernels).
enum Atom : int {
    ATOM_F32 = 0,  // fp32 [rows][cols]
    ATOM_F16 = 1,  // fp16 [rows][cols]
    ATOM_Q8 = 2,   // int8 [rows][cols] + fp16 scale [rows][sstride] (one per 32 along K)
    ATOM_Q4 = 3,   // packed nibbles [rows][cols/2] (per 32-group: byte j = elem j | elem j+16 << 4)
                   // + fp16 scale [rows][sstride]
};

// Device view of one weight matrix W[rows=out][cols=in].
struct QW {
    const uint8_t* q;  // payload (see Atom)
    const __half* s;   // group scales (Q8/Q4), row stride sstride
    int rows, cols;
    int sstride;       // scales per row, padded to a multiple of 8 (16 B rows)
    int atom;
    size_t qstride;    // bytes per row of q
};

// Epilogue kinds of the linear kernels.
enum EpiKind : int {
    EPI_STORE = 0,  // out[m][n] = acc (+ bias)
    EPI_RESID = 1,  // out[m][n] += acc + bias          (residual stream, gpt2.rs:297-299)
    EPI_GELU = 2,   // out[m][n] = gelu(acc + bias)      (gpt2.rs:310-314)
    EPI_QKV = 3,    // q -> out, k/v -> KV cache at (slot[m], pos[m])   (gpt2.rs:250-259)
};

struct Epi {
    int kind;
    const float* bias;  // may be null
    float* out;
    int ldo;
    // EPI_GELU: optional fp16 hi/lo copies of the output (x = hi + lo), row stride ldo,
    // read by the tensor-core linear that consumes this activation
    __half* out_hi;
    __half* out_lo;
    // EPI_QKV
    float* kv;             // KV arena base
    const int* slot;       // per row m
    const int* pos;        // per row m
    int d_local;           // width of q (= width of k = width of v) in this handle
    int hd;                // head dim
    size_t slot_stride;    // floats per slot
    size_t layer_off;      // floats to this layer inside a slot
    size_t sel_stride;     // floats from K to V block inside a layer
    size_t head_stride;    // floats per head (n_ctx * hd)
    // EPI_RESID, warp-level linear only (optional): per token and 16-row tile, the mean and the
    // sum of squared deviations of the tile's new residual values, [token][stats_ld], and
    // ln_g * (new value) split into out_hi / out_lo, for the LayerNorm that the next linear folds
    // into its epilogue
    float2* stats;
    int stats_ld;
    const float* ln_g;
};

__device__ __forceinline__ float gelu_tanh(float v) {
    // 0.5 v (1 + tanh(0.7978845608028654 (v + 0.044715 v^3))), same operation order as gpt2.rs:313.
    return 0.5f * v * (1.0f + tanhf(0.7978845608028654f * (v + 0.044715f * v * v * v)));
}

__device__ __forceinline__ void epi_apply(const Epi& e, int m, int n, float acc) {
    float v = acc;
    switch (e.kind) {
        case EPI_STORE:
            if (e.bias) v += e.bias[n];
            e.out[(size_t)m * e.ldo + n] = v;
            break;
        case EPI_RESID: {
            float b = e.bias ? e.bias[n] : 0.f;
            float* p = e.out + (size_t)m * e.ldo + n;
            *p = *p + (v + b);
            break;
        }
        case EPI_GELU: {
            if (e.bias) v += e.bias[n];
            const float gv = gelu_tanh(v);
            const size_t o = (size_t)m * e.ldo + n;
            if (e.out) e.out[o] = gv;  // null: the consumer reads only the hi/lo pair
            if (e.out_hi) {
                const __half h = __float2half_rn(gv);
                e.out_hi[o] = h;
                e.out_lo[o] = __float2half_rn(gv - __half2float(h));
            }
            break;
        }
        default: {  // EPI_QKV
            if (e.bias) v += e.bias[n];
            if (n < e.d_local) {
                e.out[(size_t)m * e.ldo + n] = v;
            } else {
                int sel = n / e.d_local - 1;  // 0 = K, 1 = V
                int c = n - (sel + 1) * e.d_local;
                int head = c / e.hd, i = c - head * e.hd;
                size_t off = (size_t)e.slot[m] * e.slot_stride + e.layer_off + (size_t)sel * e.sel_stride +
                             (size_t)head * e.head_stride + (size_t)e.pos[m] * e.hd + i;
                e.kv[off] = v;
            }
        }
    }
}

// ---- exact small-integer -> fp32 conversion with one PRMT + one FADD ----
// Places a biased byte (value + bias, in [0,255]) in the low mantissa bits of 2^23:
// float(0x4B0000bb) = 8388608 + bb. Subtracting 8388608 + bias gives the integer exactly.
__device__ __forceinline__ float byte_to_f(uint32_t biased_word, int j, float magic) {
    uint32_t sel = 0x7440u | (uint32_t)j;
    return __uint_as_float(__byte_perm(biased_word, 0x4B000000u, sel)) - magic;
}

// 4 signed int8 (little-endian in w) -> 4 floats.
__device__ __forceinline__ void i8x4_to_f32(uint32_t w, float* f) {
    uint32_t u = w ^ 0x80808080u;
    const float magic = 8388736.0f;  // 2^23 + 128
    f[0] = byte_to_f(u, 0, magic);
    f[1] = byte_to_f(u, 1, magic);
    f[2] = byte_to_f(u, 2, magic);
    f[3] = byte_to_f(u, 3, magic);
}

// 8 signed nibbles of w: low nibbles of bytes 0..3 -> lo[0..3], high nibbles -> hi[0..3].
__device__ __forceinline__ void i4x8_to_f32(uint32_t w, float* lo, float* hi) {
    uint32_t ul = (w & 0x0F0F0F0Fu) ^ 0x08080808u;
    uint32_t uh = ((w >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
    const float magic = 8388616.0f;  // 2^23 + 8
    lo[0] = byte_to_f(ul, 0, magic);
    lo[1] = byte_to_f(ul, 1, magic);
    lo[2] = byte_to_f(ul, 2, magic);
    lo[3] = byte_to_f(ul, 3, magic);
    hi[0] = byte_to_f(uh, 0, magic);
    hi[1] = byte_to_f(uh, 1, magic);
    hi[2] = byte_to_f(uh, 2, magic);
    hi[3] = byte_to_f(uh, 3, magic);
}

// Dequantised element (row r, column c): exactly (float)q * f16(scale) as Engine::vec_f32.
__device__ __forceinline__ float deq_elem(const QW& w, int r, int c) {
    switch (w.atom) {
        case ATOM_F32:
            return reinterpret_cast<const float*>(w.q + (size_t)r * w.qstride)[c];
        case ATOM_F16:
            return __half2float(reinterpret_cast<const __half*>(w.q + (size_t)r * w.qstride)[c]);
        case ATOM_Q8: {
            int8_t q = (int8_t)w.q[(size_t)r * w.qstride + c];
            return (float)q * __half2float(w.s[(size_t)r * w.sstride + c / 32]);
        }
        default: {
            int g = c >> 5, e = c & 31;
            uint8_t b = w.q[(size_t)r * w.qstride + g * 16 + (e & 15)];
            int nib = (e < 16) ? (b & 0xf) : (b >> 4);
            return (float)((nib ^ 8) - 8) * __half2float(w.s[(size_t)r * w.sstride + g]);
        }
    }
}

// IEEE total-order key (Rust f32::total_cmp): larger key == larger in total order.
__device__ __forceinline__ int total_key(float f) {
    int b = __float_as_int(f);
    return b ^ (int)(((unsigned)(b >> 31)) >> 1);
}

// (total-order key, index) packed so that unsigned 64-bit max picks the largest value
// and, among equal values, the LAST index (Iterator::max_by, gpt2.rs:390-396).
__device__ __forceinline__ unsigned long long argmax_pack(float v, int idx) {
    const unsigned k = (unsigned)total_key(v) ^ 0x80000000u;
    return ((unsigned long long)k << 32) | (unsigned)idx;
}

// fp32 -> fp16 pair with x ~= hi + lo (about 22 significant bits).
__device__ __forceinline__ void split_hl(float x, __half& hi, __half& lo) {
    hi = __float2half_rn(x);
    lo = __float2half_rn(x - __half2float(hi));
}

// split_hl of two values with paired conversions (same roundings): hi = (hi(a), hi(b)).
__device__ __forceinline__ void split_hl2(float a, float b, __half2& hi, __half2& lo) {
    hi = __floats2half2_rn(a, b);
    const float2 h = __half22float2(hi);
    lo = __floats2half2_rn(a - h.x, b - h.y);
}

}  // namespace gpt2q
