// CPU oracle for the quantized GPT-2 forward. TEST INFRASTRUCTURE ONLY: the
// checker for the CUDA path, never part of the product. Build with
// -ffp-contract=off (see oracle.h); every function cites the reference
// (LukasParke/smelt) lines it restates.
#include "oracle.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <string>
#include <thread>
#include <vector>

#if defined(__AVX2__) && defined(__FMA__)
#include <immintrin.h>
#endif

static const char* ATOM_F16 = "core.f16";              // atoms.rs:5
static const char* ATOM_Q8 = "core.i8.b32.f16scale";   // atoms.rs:6
static const char* ATOM_Q4 = "core.i4.b32.f16scale";   // int4 atom (18 B / 32 values)
static const char* ATOM_F32 = "core.f32";              // oracle extension (fp32 weights)

// ---------------------------------------------------------------- f16 codec
// atoms.rs:10-37 (round-to-nearest-even encode).
extern "C" uint16_t orc_f32_to_f16(float x) {
    uint32_t b;
    std::memcpy(&b, &x, 4);
    uint16_t sign = (uint16_t)((b >> 16) & 0x8000u);
    int32_t exp = (int32_t)((b >> 23) & 0xffu) - 127 + 15;
    uint32_t man = b & 0x007fffffu;
    if (((b >> 23) & 0xffu) == 0xffu) return (uint16_t)(sign | 0x7c00u | ((man != 0) << 8));
    if (exp >= 0x1f) return (uint16_t)(sign | 0x7c00u);
    if (exp <= 0) {
        if (exp < -10) return sign;
        uint32_t m2 = man | 0x00800000u;
        uint32_t shift = (uint32_t)(14 - exp);
        uint32_t hm = m2 >> shift;
        uint32_t rem = m2 & ((1u << shift) - 1);
        uint32_t mid = 1u << (shift - 1);
        uint16_t round = (uint16_t)((rem > mid) || (rem == mid && (hm & 1u) == 1u));
        return (uint16_t)(sign | (uint16_t)((uint16_t)hm + round));
    }
    uint32_t hm = man >> 13;
    uint32_t rem = man & 0x1fffu;
    uint32_t round = (uint32_t)((rem > 0x1000u) || (rem == 0x1000u && (hm & 1u) == 1u));
    return (uint16_t)(sign | (uint16_t)(((uint32_t)exp << 10) + hm + round));
}

// atoms.rs:39-61 (exact decode incl. subnormals).
extern "C" float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)(h & 0x8000u)) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x03ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            uint32_t e = 127 - 15 + 1;
            uint32_t m = man;
            while ((m & 0x0400u) == 0) {
                m <<= 1;
                e -= 1;
            }
            m &= 0x03ffu;
            bits = sign | (e << 23) | (m << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

static inline float rust_max(float a, float b) {  // f32::max: NaN-ignoring
    if (std::isnan(a)) return b;
    if (std::isnan(b)) return a;
    return a > b ? a : b;
}
static inline float rust_clamp(float v, float lo, float hi) {
    if (v < lo) v = lo;
    if (v > hi) v = hi;
    return v;
}
// Rust `f as i8`: saturating, NaN -> 0 (a scale that underflows to 0 gives 0/0).
static inline int8_t rust_as_i8(float v) {
    if (std::isnan(v)) return 0;
    if (v <= -128.f) return -128;
    if (v >= 127.f) return 127;
    return (int8_t)v;
}

// ---------------------------------------------------------------- Q8 encode
// atoms.rs:65-78: s = amax/127 in f32 (unrounded) is used to quantise; f16(s) is stored.
extern "C" void orc_q8_encode(const float* x, size_t n, uint8_t* out) {
    for (size_t b = 0; b < n / 32; ++b) {
        const float* blk = x + b * 32;
        float amax = 0.f;
        for (int i = 0; i < 32; ++i) amax = rust_max(amax, std::fabs(blk[i]));
        float s = (amax == 0.f) ? 1.0f : amax / 127.0f;
        uint16_t h = orc_f32_to_f16(s);
        uint8_t* o = out + b * 34;
        o[0] = (uint8_t)(h & 0xff);
        o[1] = (uint8_t)(h >> 8);
        for (int i = 0; i < 32; ++i) {
            o[2 + i] = (uint8_t)rust_as_i8(rust_clamp(std::round(blk[i] / s), -127.0f, 127.0f));
        }
    }
}

// ---------------------------------------------------------------- Q4 encode
// Math: perf-lab/src/bin/atoms.rs:89-99 (d = f16_round(amax/7) is used to quantise,
// q = clamp(round(v/d), +-7)). Packing (the reference has none): 18 B per group,
// [f16 d LE][16 B], byte j = (q[j] & 0xF) | (q[j+16] & 0xF) << 4, two's-complement nibbles.
extern "C" void orc_q4_encode(const float* x, size_t n, uint8_t* out) {
    for (size_t b = 0; b < n / 32; ++b) {
        const float* blk = x + b * 32;
        float amax = 0.f;
        for (int i = 0; i < 32; ++i) amax = rust_max(amax, std::fabs(blk[i]));
        uint16_t h = orc_f32_to_f16(amax == 0.f ? 1.0f : amax / 7.0f);
        float d = orc_f16_to_f32(h);
        int8_t q[32];
        for (int i = 0; i < 32; ++i) q[i] = rust_as_i8(rust_clamp(std::round(blk[i] / d), -7.0f, 7.0f));
        uint8_t* o = out + b * 18;
        o[0] = (uint8_t)(h & 0xff);
        o[1] = (uint8_t)(h >> 8);
        for (int j = 0; j < 16; ++j)
            o[2 + j] = (uint8_t)(((uint8_t)q[j] & 0xfu) | (((uint8_t)q[j + 16] & 0xfu) << 4));
    }
}

static inline float q4_elem(const uint8_t* grp16, int e) {  // grp16 -> the 16 packed bytes
    uint8_t byte = grp16[e & 15];
    int nib = (e < 16) ? (byte & 0xf) : (byte >> 4);
    return (float)((nib ^ 8) - 8);
}

static inline float blk_scale(const uint8_t* p) {
    return orc_f16_to_f32((uint16_t)(p[0] | (p[1] << 8)));
}

// ---------------------------------------------------------------- GEMV kernels
// atoms.rs:89-132 (4 interleaved fp32 FMA accumulators, 4 blocks at a time).
extern "C" void orc_gemv_q8(const uint8_t* w, const float* x, float* y, size_t rows, size_t cols,
                            size_t r0, size_t r_end) {
    (void)rows;
    size_t nblk = cols / 32;
    for (size_t r = r0; r < r_end; ++r) {
        const uint8_t* row = w + r * nblk * 34;
        float acc = 0.f, acc2 = 0.f, acc3 = 0.f, acc4 = 0.f;
        size_t b = 0;
        while (b + 4 <= nblk) {
            float scales[4] = {blk_scale(row + b * 34), blk_scale(row + (b + 1) * 34),
                               blk_scale(row + (b + 2) * 34), blk_scale(row + (b + 3) * 34)};
            size_t j = b * 32;
            for (size_t bi = 0; bi < 4; ++bi) {
                float s = scales[bi];
                size_t xb = j + bi * 32;
                size_t ob = (b + bi) * 34 + 2;
                for (size_t t = 0; t < 8; ++t) {
                    size_t o = ob + t * 4;
                    acc = std::fma((float)(int8_t)row[o] * s, x[xb + t * 4], acc);
                    acc2 = std::fma((float)(int8_t)row[o + 1] * s, x[xb + t * 4 + 1], acc2);
                    acc3 = std::fma((float)(int8_t)row[o + 2] * s, x[xb + t * 4 + 2], acc3);
                    acc4 = std::fma((float)(int8_t)row[o + 3] * s, x[xb + t * 4 + 3], acc4);
                }
            }
            b += 4;
        }
        while (b < nblk) {
            float s = blk_scale(row + b * 34);
            size_t base = b * 34 + 2;
            size_t j = b * 32;
            for (size_t t = 0; t < 32; ++t) acc = std::fma((float)(int8_t)row[base + t] * s, x[j + t], acc);
            b += 1;
        }
        y[r - r0] += acc + acc2 + acc3 + acc4;
    }
}

// int4 twin of gemv_q8 (same accumulator order; the reference has no int4 GEMV).
extern "C" void orc_gemv_q4(const uint8_t* w, const float* x, float* y, size_t rows, size_t cols,
                            size_t r0, size_t r_end) {
    (void)rows;
    size_t nblk = cols / 32;
    for (size_t r = r0; r < r_end; ++r) {
        const uint8_t* row = w + r * nblk * 18;
        float acc = 0.f, acc2 = 0.f, acc3 = 0.f, acc4 = 0.f;
        size_t b = 0;
        while (b + 4 <= nblk) {
            for (size_t bi = 0; bi < 4; ++bi) {
                const uint8_t* g = row + (b + bi) * 18;
                float s = blk_scale(g);
                size_t xb = (b + bi) * 32;
                for (int t = 0; t < 8; ++t) {
                    acc = std::fma(q4_elem(g + 2, t * 4) * s, x[xb + t * 4], acc);
                    acc2 = std::fma(q4_elem(g + 2, t * 4 + 1) * s, x[xb + t * 4 + 1], acc2);
                    acc3 = std::fma(q4_elem(g + 2, t * 4 + 2) * s, x[xb + t * 4 + 2], acc3);
                    acc4 = std::fma(q4_elem(g + 2, t * 4 + 3) * s, x[xb + t * 4 + 3], acc4);
                }
            }
            b += 4;
        }
        while (b < nblk) {
            const uint8_t* g = row + b * 18;
            float s = blk_scale(g);
            for (int t = 0; t < 32; ++t) acc = std::fma(q4_elem(g + 2, t) * s, x[b * 32 + t], acc);
            b += 1;
        }
        y[r - r0] += acc + acc2 + acc3 + acc4;
    }
}

// atoms.rs:135-164.
extern "C" void orc_gemv_f16(const uint8_t* w, const float* x, float* y, size_t rows, size_t cols,
                             size_t r0, size_t r_end) {
    (void)rows;
    for (size_t r = r0; r < r_end; ++r) {
        const uint8_t* row = w + r * cols * 2;
        auto hv = [&](size_t j) { return orc_f16_to_f32((uint16_t)(row[j * 2] | (row[j * 2 + 1] << 8))); };
        float acc = 0.f, acc2 = 0.f, acc3 = 0.f, acc4 = 0.f;
        size_t j = 0;
        while (j + 4 <= cols) {
            acc = std::fma(hv(j), x[j], acc);
            acc2 = std::fma(hv(j + 1), x[j + 1], acc2);
            acc3 = std::fma(hv(j + 2), x[j + 2], acc3);
            acc4 = std::fma(hv(j + 3), x[j + 3], acc4);
            j += 4;
        }
        while (j < cols) {
            acc += hv(j) * x[j];
            j += 1;
        }
        y[r - r0] += acc + acc2 + acc3 + acc4;
    }
}

// fp32-weight twin of gemv_f16 (the reference has no f32 atom; oracle extension).
extern "C" void orc_gemv_f32(const uint8_t* w, const float* x, float* y, size_t rows, size_t cols,
                             size_t r0, size_t r_end) {
    (void)rows;
    for (size_t r = r0; r < r_end; ++r) {
        const float* row = reinterpret_cast<const float*>(w) + r * cols;
        float acc = 0.f, acc2 = 0.f, acc3 = 0.f, acc4 = 0.f;
        size_t j = 0;
        while (j + 4 <= cols) {
            acc = std::fma(row[j], x[j], acc);
            acc2 = std::fma(row[j + 1], x[j + 1], acc2);
            acc3 = std::fma(row[j + 2], x[j + 2], acc3);
            acc4 = std::fma(row[j + 3], x[j + 3], acc4);
            j += 4;
        }
        while (j < cols) {
            acc += row[j] * x[j];
            j += 1;
        }
        y[r - r0] += acc + acc2 + acc3 + acc4;
    }
}

// ---------------------------------------------------------------- converter
// pack.rs:47-66 (transpose of the four Conv1D weights) and :68-84 (atom policy).
static bool is_conv1d(const std::string& name) {
    static const char* suf[] = {"attn.c_attn.weight", "attn.c_proj.weight", "mlp.c_fc.weight",
                                "mlp.c_proj.weight"};
    for (const char* s : suf) {
        size_t L = std::strlen(s);
        if (name.size() >= L && name.compare(name.size() - L, L, s) == 0) return true;
    }
    return false;
}

static std::string pick_atom(int ndim, size_t numel, const std::string& policy) {
    if (policy == "f32") return ATOM_F32;
    if (policy == "auto" && numel >= 4096 && ndim == 2) return ATOM_Q8;
    if (policy == "q4auto" && numel >= 4096 && ndim == 2) return ATOM_Q4;
    if (policy == "auto" || policy == "q4auto" || policy == ATOM_F16) return ATOM_F16;
    if (policy == ATOM_Q8 && ndim == 2) return ATOM_Q8;
    return ATOM_F16;
}

extern "C" size_t orc_pack_size(const char* name, int ndim, const int64_t* hf_shape, const char* policy) {
    (void)name;
    size_t numel = 1;
    for (int i = 0; i < ndim; ++i) numel *= (size_t)hf_shape[i];
    std::string a = pick_atom(ndim, numel, policy);
    if (a == ATOM_Q8) return numel / 32 * 34;
    if (a == ATOM_Q4) return numel / 32 * 18;
    if (a == ATOM_F32) return numel * 4;
    return numel * 2;
}

extern "C" int orc_pack_tensor(const char* name, int ndim, const int64_t* hf_shape, const float* data,
                               const char* policy, int64_t* shape_out, char* atom_out, size_t atom_cap,
                               uint8_t* out_bytes) {
    std::string nm(name);
    size_t numel = 1;
    for (int i = 0; i < ndim; ++i) numel *= (size_t)hf_shape[i];
    std::vector<float> f(data, data + numel);
    std::vector<int64_t> shape(hf_shape, hf_shape + ndim);
    if (ndim == 2 && is_conv1d(nm)) {
        size_t a = (size_t)shape[0], b = (size_t)shape[1];
        std::vector<float> t(a * b);
        for (size_t i = 0; i < a; ++i)
            for (size_t j = 0; j < b; ++j) t[j * a + i] = f[i * b + j];
        f.swap(t);
        shape = {(int64_t)b, (int64_t)a};
    }
    std::string atom = pick_atom(ndim, numel, policy);
    if ((atom == ATOM_Q8 || atom == ATOM_Q4) && numel % 32 != 0) return -1;
    if (atom.size() + 1 > atom_cap) return -2;
    std::memcpy(atom_out, atom.c_str(), atom.size() + 1);
    for (int i = 0; i < ndim; ++i) shape_out[i] = shape[i];
    if (atom == ATOM_Q8) {
        orc_q8_encode(f.data(), numel, out_bytes);
    } else if (atom == ATOM_Q4) {
        orc_q4_encode(f.data(), numel, out_bytes);
    } else if (atom == ATOM_F32) {
        std::memcpy(out_bytes, f.data(), numel * 4);
    } else {
        for (size_t i = 0; i < numel; ++i) {
            uint16_t h = orc_f32_to_f16(f[i]);
            out_bytes[2 * i] = (uint8_t)(h & 0xff);
            out_bytes[2 * i + 1] = (uint8_t)(h >> 8);
        }
    }
    return 0;
}

// ---------------------------------------------------------------- RNG
// gpu_backward.rs:835-856: Rng::new(seed) = seed ^ 0x9E3779B97F4A7C15; xorshift64*.
extern "C" uint64_t orc_rng_new(uint64_t seed) { return seed ^ 0x9E3779B97F4A7C15ull; }

static inline uint64_t xs64star(uint64_t* s) {
    uint64_t x = *s;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *s = x;
    return x * 0x2545F4914F6CDD1Dull;
}

// Box-Muller as perf-lab/src/bin/atoms.rs:75-83, uniform from the xorshift64* stream.
extern "C" void orc_rng_normal_f32(uint64_t* state, float* out, size_t n, double stdv) {
    const double TAU = 6.283185307179586;
    for (size_t i = 0; i < n; ++i) {
        double u1 = (double)(xs64star(state) >> 11) / 9007199254740992.0;
        double u2 = (double)(xs64star(state) >> 11) / 9007199254740992.0;
        if (u1 < 1e-12) u1 = 1e-12;
        double z = std::sqrt(-2.0 * std::log(u1)) * std::cos(TAU * u2);
        out[i] = (float)(z * stdv);
    }
}

// gpu_backward.rs:851-853 Rng::below.
extern "C" void orc_rng_below(uint64_t* state, uint32_t* out, size_t n, uint64_t bound) {
    for (size_t i = 0; i < n; ++i) out[i] = (uint32_t)(xs64star(state) % bound);
}

// ---------------------------------------------------------------- perf-lab atoms experiment
// perf-lab/src/bin/atoms.rs: the xorshift (13,7,17) RNG :65-84, the atoms :57-155, metrics
// :159-175 and main :177-209.
namespace perf {
struct Rng {
    uint64_t s;
    uint64_t next_u() {
        uint64_t x = s;
        x ^= x << 13;
        x ^= x >> 7;
        x ^= x << 17;
        s = x;
        return x;
    }
    double uniform() { return (double)(next_u() >> 11) / 9007199254740992.0; }
    double normal() {
        double u1 = uniform();
        if (u1 < 1e-12) u1 = 1e-12;
        double u2 = uniform();
        return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
    }
};
static inline double signum(double v) { return std::signbit(v) ? -1.0 : 1.0; }
static inline float signumf(float v) { return std::signbit(v) ? -1.0f : 1.0f; }

static float bf16_rne(float x) {
    uint32_t b;
    std::memcpy(&b, &x, 4);
    uint32_t r = b + (0x7fffu + ((b >> 16) & 1u));
    r &= 0xffff0000u;
    float f;
    std::memcpy(&f, &r, 4);
    return f;
}
static void q4_sym(const std::vector<float>& x, std::vector<float>& q, size_t blk) {
    for (size_t b = 0; b < x.size() / blk; ++b) {
        float amax = 0.f;
        for (size_t i = 0; i < blk; ++i) amax = rust_max(amax, std::fabs(x[b * blk + i]));
        float d = orc_f16_to_f32(orc_f32_to_f16(amax == 0.f ? 1.0f : amax / 7.0f));
        for (size_t i = 0; i < blk; ++i) {
            float v = x[b * blk + i];
            q[b * blk + i] = rust_clamp(std::round(v / d), -7.0f, 7.0f) * d;
        }
    }
}
static void mxfp4(const std::vector<float>& x, std::vector<float>& q) {
    static const float L[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
    for (size_t b = 0; b < x.size() / 32; ++b) {
        float amax = 0.f;
        for (int i = 0; i < 32; ++i) amax = rust_max(amax, std::fabs(x[b * 32 + i]));
        int e = (amax == 0.f) ? -126 : (int)std::floor(std::log2(amax)) - 2;
        float inv = std::exp2(-(float)e);
        for (int i = 0; i < 32; ++i) {
            float v = x[b * 32 + i];
            float r = std::min(std::fabs(v * inv), 6.0f);
            size_t k = 0;
            while (k + 1 < 8 && r > L[k + 1]) k++;
            float lo = L[k];
            float hi = (k + 1 < 8) ? L[k + 1] : lo;
            size_t pick;
            if (r - lo < hi - r) pick = k;
            else if (r - lo > hi - r) pick = k + 1;
            else if (k % 2 == 0) pick = k;
            else pick = k + 1;
            q[b * 32 + i] = (signumf(v) * L[std::min<size_t>(pick, 7)]) * std::exp2((float)e);
        }
    }
}
static void metrics(const std::vector<float>& o, const std::vector<float>& q, double* rel, double* cs) {
    double n = (double)o.size(), se = 0, dot = 0, no = 0, nq = 0;
    for (size_t i = 0; i < o.size(); ++i) {
        double d = (double)(o[i] - q[i]);
        se += d * d;
        dot += (double)o[i] * (double)q[i];
        no += (double)o[i] * (double)o[i];
        nq += (double)q[i] * (double)q[i];
    }
    *rel = std::sqrt(se / n) / std::sqrt(no / n);
    *cs = dot / (std::sqrt(no) * std::sqrt(nq));
}
}  // namespace perf

extern "C" void orc_perf_atoms(double* out40, size_t n) {
    perf::Rng rng{0xDEADBEEF12345678ull};
    std::vector<float> xs(n), q(n);
    int k = 0;
    for (int dist = 0; dist < 5; ++dist) {
        for (size_t i = 0; i < n; ++i) {
            double v;
            if (dist == 0) {
                v = rng.normal();
            } else if (dist == 1) {
                double u = rng.uniform() - 0.5;
                v = -perf::signum(u) * std::log(1.0 - 2.0 * std::fabs(u));
            } else if (dist == 2) {
                v = (rng.uniform() < 0.01) ? rng.normal() * 25.0 : rng.normal();
            } else if (dist == 3) {
                v = (rng.uniform() - 0.5) * 6.0;
            } else {
                v = rng.normal() * 1e-3;
            }
            xs[i] = (float)v;
        }
        for (int atom = 0; atom < 4; ++atom) {
            if (atom == 0) for (size_t i = 0; i < n; ++i) q[i] = perf::bf16_rne(xs[i]);
            if (atom == 1) perf::q4_sym(xs, q, 32);
            if (atom == 2) perf::mxfp4(xs, q);
            if (atom == 3) perf::q4_sym(xs, q, 16);  // two_level_sub16: 256-superblocks of 16-subblocks
            perf::metrics(xs, q, &out40[k], &out40[k + 1]);
            k += 2;
        }
    }
}

// ---------------------------------------------------------------- engine
struct Tensor {
    std::string atom;
    std::vector<int64_t> shape;
    std::vector<uint8_t> data;
};

struct orc_engine {
    int n_embd, n_layer, n_head, n_ctx, vocab;
    float ln_eps;
    int threads;
    std::map<std::string, Tensor> t;
    // plastic adapter on the post-ln_f state (gpu.rs:188-194, 364-367): h += B (A h)
    int ad_r = 0;
    std::vector<float> ad_a, ad_b;  // A [r][d], B [d][r]
    const Tensor& get(const std::string& n) const { return t.at(n); }
};

extern "C" orc_engine* orc_engine_new(int n_embd, int n_layer, int n_head, int n_ctx, int vocab,
                                      float ln_eps, int threads) {
    auto* e = new orc_engine();
    e->n_embd = n_embd;
    e->n_layer = n_layer;
    e->n_head = n_head;
    e->n_ctx = n_ctx;
    e->vocab = vocab;
    e->ln_eps = ln_eps;
    e->threads = threads > 0 ? threads : 8;
    return e;
}

extern "C" int orc_engine_add(orc_engine* e, const char* name, const char* atom, int ndim,
                              const int64_t* shape, const uint8_t* data, uint64_t len) {
    Tensor t;
    t.atom = atom;
    t.shape.assign(shape, shape + ndim);
    t.data.assign(data, data + len);
    e->t[name] = std::move(t);
    return 0;
}

extern "C" void orc_engine_free(orc_engine* e) { delete e; }

extern "C" size_t orc_kv_floats(const orc_engine* e) {
    return (size_t)e->n_layer * 2 * (size_t)e->n_ctx * (size_t)e->n_embd;
}

static size_t numel_of(const Tensor& t) {
    size_t n = 1;
    for (auto s : t.shape) n *= (size_t)s;
    return n;
}

// gpt2.rs:121-142 (plus the int4 and f32 atoms).
static std::vector<float> vec_f32(const orc_engine* e, const std::string& name) {
    const Tensor& t = e->get(name);
    size_t n = numel_of(t);
    std::vector<float> out;
    out.reserve(n);
    const uint8_t* p = t.data.data();
    if (t.atom == ATOM_F16) {
        for (size_t i = 0; i < n; ++i) out.push_back(orc_f16_to_f32((uint16_t)(p[2 * i] | (p[2 * i + 1] << 8))));
    } else if (t.atom == ATOM_Q8) {
        for (size_t b = 0; b < t.data.size() / 34; ++b) {
            float s = blk_scale(p + b * 34);
            for (int i = 0; i < 32; ++i) out.push_back((float)(int8_t)p[b * 34 + 2 + i] * s);
        }
        out.resize(n);
    } else if (t.atom == ATOM_Q4) {
        for (size_t b = 0; b < t.data.size() / 18; ++b) {
            float s = blk_scale(p + b * 18);
            for (int i = 0; i < 32; ++i) out.push_back(q4_elem(p + b * 18 + 2, i) * s);
        }
        out.resize(n);
    } else if (t.atom == ATOM_F32) {
        out.resize(n);
        std::memcpy(out.data(), p, n * 4);
    }
    return out;
}

// gpt2.rs:187-220.
static std::vector<float> vec_row(const orc_engine* e, const std::string& name, uint32_t row) {
    const Tensor& t = e->get(name);
    size_t cols = (size_t)t.shape[1];
    std::vector<float> out;
    out.reserve(cols);
    const uint8_t* p = t.data.data();
    if (t.atom == ATOM_F16) {
        const uint8_t* r = p + (size_t)row * cols * 2;
        for (size_t i = 0; i < cols; ++i) out.push_back(orc_f16_to_f32((uint16_t)(r[2 * i] | (r[2 * i + 1] << 8))));
    } else if (t.atom == ATOM_F32) {
        const float* r = reinterpret_cast<const float*>(p) + (size_t)row * cols;
        out.assign(r, r + cols);
    } else if (t.atom == ATOM_Q4) {
        const uint8_t* r = p + (size_t)row * (cols / 32 * 18);
        for (size_t b = 0; b < cols / 32; ++b) {
            float s = blk_scale(r + b * 18);
            for (int i = 0; i < 32; ++i) out.push_back(q4_elem(r + b * 18 + 2, i) * s);
        }
    } else {
        const uint8_t* r = p + (size_t)row * (cols / 32 * 34);
        for (size_t b = 0; b < cols / 32; ++b) {
            float s = blk_scale(r + b * 34);
            for (int i = 0; i < 32; ++i) out.push_back((float)(int8_t)r[b * 34 + 2 + i] * s);
        }
    }
    return out;
}

// gpt2.rs:145-176: out = W @ x with min(threads, rows) scoped threads over row chunks.
static void matmul(const orc_engine* e, const std::string& wname, const float* x, float* out) {
    const Tensor& t = e->get(wname);
    size_t rows = (size_t)t.shape[0], cols = (size_t)t.shape[1];
    std::fill(out, out + rows, 0.f);
    auto kern = [&](size_t lo, size_t hi) {
        const uint8_t* w = t.data.data();
        if (t.atom == ATOM_Q8) orc_gemv_q8(w, x, out + lo, rows, cols, lo, hi);
        else if (t.atom == ATOM_Q4) orc_gemv_q4(w, x, out + lo, rows, cols, lo, hi);
        else if (t.atom == ATOM_F16) orc_gemv_f16(w, x, out + lo, rows, cols, lo, hi);
        else orc_gemv_f32(w, x, out + lo, rows, cols, lo, hi);
    };
    size_t threads = std::min<size_t>((size_t)e->threads, rows);
    size_t per = (rows + threads - 1) / threads;
    if (threads <= 1) {
        kern(0, rows);
        return;
    }
    std::vector<std::thread> hs;
    for (size_t lo = 0; lo < rows; lo += per) hs.emplace_back(kern, lo, std::min(rows, lo + per));
    for (auto& h : hs) h.join();
}

// gpt2.rs:178-185.
static void layernorm(float* x, size_t d, const float* w, const float* b, float eps) {
    float sum = 0.f;
    for (size_t i = 0; i < d; ++i) sum += x[i];
    float mean = sum / (float)d;
    float vs = 0.f;
    for (size_t i = 0; i < d; ++i) vs += (x[i] - mean) * (x[i] - mean);
    float var = vs / (float)d;
    for (size_t i = 0; i < d; ++i) x[i] = (x[i] - mean) / std::sqrt(var + eps) * w[i] + b[i];
}

static std::string L(int layer, const char* suffix) { return "h." + std::to_string(layer) + "." + suffix; }

// gpt2.rs:227-332: one decoder step at `pos`, writing K/V rows into kv, returning logits.
extern "C" int orc_engine_step(const orc_engine* e, uint32_t tok, int pos, float* kv, float* logits) {
    const size_t d = (size_t)e->n_embd;
    const size_t hd = d / (size_t)e->n_head;
    const size_t ctxd = (size_t)e->n_ctx * d;
    if (pos < 0 || pos >= e->n_ctx || (int)tok >= e->vocab) return -1;
    std::vector<float> x = vec_row(e, "wte.weight", tok);
    std::vector<float> wpe = vec_row(e, "wpe.weight", (uint32_t)pos);
    for (size_t i = 0; i < d; ++i) x[i] += wpe[i];

    for (int layer = 0; layer < e->n_layer; ++layer) {
        float* kc = kv + (size_t)layer * 2 * ctxd;
        float* vc = kc + ctxd;
        std::vector<float> gw = vec_f32(e, L(layer, "ln_1.weight"));
        std::vector<float> gb = vec_f32(e, L(layer, "ln_1.bias"));
        std::vector<float> h = x;
        layernorm(h.data(), d, gw.data(), gb.data(), e->ln_eps);

        std::string qkv_name = L(layer, "attn.c_attn.weight");
        size_t inter3 = (size_t)e->get(qkv_name).shape[0];
        std::vector<float> qkv(inter3);
        matmul(e, qkv_name, h.data(), qkv.data());
        std::vector<float> qb = vec_f32(e, L(layer, "attn.c_attn.bias"));
        for (size_t i = 0; i < inter3; ++i) qkv[i] += qb[i];

        size_t row = (size_t)pos * d;
        std::memcpy(kc + row, qkv.data() + d, d * 4);
        std::memcpy(vc + row, qkv.data() + 2 * d, d * 4);

        float scale = 1.0f / std::sqrt((float)hd);
        std::vector<float> attn_out(d, 0.f);
        for (int head = 0; head < e->n_head; ++head) {
            size_t o = (size_t)head * hd;
            const float* q = qkv.data() + o;
            std::vector<float> scores((size_t)pos + 1, 0.f);
            float maxs = -3.40282347e+38f;  // f32::MIN
            for (int p = 0; p <= pos; ++p) {
                const float* kp = kc + (size_t)p * d + o;
                float dot = 0.f;
                for (size_t tt = 0; tt < hd; ++tt) dot += q[tt] * kp[tt];
                scores[p] = dot * scale;
                maxs = rust_max(maxs, scores[p]);
            }
            float sum = 0.f;
            for (auto& s : scores) {
                s = std::exp(s - maxs);
                sum += s;
            }
            for (auto& s : scores) s /= sum;
            for (int p = 0; p <= pos; ++p) {
                const float* vp = vc + (size_t)p * d + o;
                for (size_t tt = 0; tt < hd; ++tt) attn_out[o + tt] += scores[p] * vp[tt];
            }
        }

        std::vector<float> proj(d);
        matmul(e, L(layer, "attn.c_proj.weight"), attn_out.data(), proj.data());
        std::vector<float> pb = vec_f32(e, L(layer, "attn.c_proj.bias"));
        for (size_t i = 0; i < d; ++i) x[i] += proj[i] + pb[i];

        std::vector<float> gw2 = vec_f32(e, L(layer, "ln_2.weight"));
        std::vector<float> gb2 = vec_f32(e, L(layer, "ln_2.bias"));
        std::vector<float> h2 = x;
        layernorm(h2.data(), d, gw2.data(), gb2.data(), e->ln_eps);
        std::string fc_name = L(layer, "mlp.c_fc.weight");
        size_t inter = (size_t)e->get(fc_name).shape[0];
        std::vector<float> fc(inter);
        matmul(e, fc_name, h2.data(), fc.data());
        std::vector<float> fb = vec_f32(e, L(layer, "mlp.c_fc.bias"));
        for (size_t i = 0; i < inter; ++i) {
            float v = fc[i] + fb[i];
            fc[i] = 0.5f * v * (1.0f + std::tanh(0.7978845608028654f * (v + 0.044715f * v * v * v)));
        }
        std::vector<float> mo(d);
        matmul(e, L(layer, "mlp.c_proj.weight"), fc.data(), mo.data());
        std::vector<float> mb = vec_f32(e, L(layer, "mlp.c_proj.bias"));
        for (size_t i = 0; i < d; ++i) x[i] += mo[i] + mb[i];
    }
    std::vector<float> wf = vec_f32(e, "ln_f.weight");
    std::vector<float> bf = vec_f32(e, "ln_f.bias");
    layernorm(x.data(), d, wf.data(), bf.data(), e->ln_eps);
    if (e->ad_r > 0) {
        // k_adapter_apply (cu/gpt2.cu:196-215): ah[j] = sum_i A[j][i] h[i], then
        // h[i] += sum_j B[i][j] ah[j], both sums sequential fused multiply-adds
        const int r = e->ad_r;
        std::vector<float> ah(r);
        for (int j = 0; j < r; ++j) {
            float acc = 0.f;
            const float* ar = e->ad_a.data() + (size_t)j * d;
            for (size_t i = 0; i < d; ++i) acc = std::fma(ar[i], x[i], acc);
            ah[j] = acc;
        }
        for (size_t i = 0; i < d; ++i) {
            float acc = 0.f;
            const float* br = e->ad_b.data() + i * r;
            for (int j = 0; j < r; ++j) acc = std::fma(br[j], ah[j], acc);
            x[i] += acc;
        }
    }
    matmul(e, "wte.weight", x.data(), logits);
    return 0;
}

// ---------------------------------------------------------------- batched prefill
// T consecutive Engine::step calls (gpt2.rs:227-332, driven by the prompt loop gpt2.rs:373-381)
// computed layer by layer over all T positions, so that long prompts check in seconds. Every
// value goes through the same operations in the same order as in orc_engine_step; only the loop
// nest differs (positions are SIMD lanes), so the results are bit-identical (tested against the
// per-token step on every atom).
namespace {

// Weight row r as the fp32 values the GEMV multiplies: (float)q * f16(s) for the group atoms
// (exact in fp32: 8 x 11 significant bits), the decoded half, or the float itself.
void deq_row(const Tensor& t, size_t r, size_t cols, float* out) {
    const uint8_t* p = t.data.data();
    if (t.atom == ATOM_Q8) {
        const uint8_t* row = p + r * (cols / 32) * 34;
        for (size_t b = 0; b < cols / 32; ++b) {
            float s = blk_scale(row + b * 34);
            for (int i = 0; i < 32; ++i) out[b * 32 + i] = (float)(int8_t)row[b * 34 + 2 + i] * s;
        }
    } else if (t.atom == ATOM_Q4) {
        const uint8_t* row = p + r * (cols / 32) * 18;
        for (size_t b = 0; b < cols / 32; ++b) {
            float s = blk_scale(row + b * 18);
            for (int i = 0; i < 32; ++i) out[b * 32 + i] = q4_elem(row + b * 18 + 2, i) * s;
        }
    } else if (t.atom == ATOM_F16) {
        const uint8_t* row = p + r * cols * 2;
        for (size_t j = 0; j < cols; ++j) out[j] = orc_f16_to_f32((uint16_t)(row[2 * j] | (row[2 * j + 1] << 8)));
    } else {
        std::memcpy(out, reinterpret_cast<const float*>(p) + r * cols, cols * 4);
    }
}

// Accumulation order of the GEMVs (atoms.rs:89-164): element j goes to accumulator j % 4 for
// j < main_end, in increasing j; the rest goes to accumulator 0, by FMA in the group kernels
// (gemv_q8's single-block tail) and by an unfused multiply-add in the element kernels
// (gemv_f16's `acc += w * x` tail). The result is ((acc0 + acc1) + acc2) + acc3, added to 0.
struct GemvOrder {
    size_t main_end;
    bool tail_fused;
};
GemvOrder order_of(const Tensor& t, size_t cols) {
    if (t.atom == ATOM_Q8 || t.atom == ATOM_Q4) return {cols / 128 * 128, true};
    return {cols / 4 * 4, false};
}

template <class F>
void parallel_for(int threads, size_t n, F&& f) {
    size_t nt = std::min<size_t>((size_t)std::max(threads, 1), std::max<size_t>(n, 1));
    if (nt <= 1) {
        f(0, 0, n);
        return;
    }
    std::vector<std::thread> hs;
    size_t per = (n + nt - 1) / nt;
    for (size_t i = 0; i < nt; ++i) {
        size_t lo = i * per, hi = std::min(n, lo + per);
        if (lo < hi) hs.emplace_back(f, i, lo, hi);
    }
    for (auto& h : hs) h.join();
}

constexpr int TB = 8;  // positions per SIMD vector

// Y[t][r] = matmul(W, X[t])[r] for t in [0, T): bit-identical to T calls of matmul(). X is
// staged block-major (Xb[block][j][lane], 8 positions per block) so that a row's pass over one
// block streams contiguous memory; two weight rows share every activation load.
void matmul_batched(const orc_engine* e, const std::string& wname, const float* X, int T, float* Y) {
    const Tensor& w = e->get(wname);
    const size_t rows = (size_t)w.shape[0], cols = (size_t)w.shape[1];
    const size_t nb = (size_t)(T + TB - 1) / TB;
    std::vector<float> Xb(nb * cols * TB, 0.f);
    for (int t = 0; t < T; ++t)
        for (size_t j = 0; j < cols; ++j) Xb[((size_t)t / TB * cols + j) * TB + (size_t)t % TB] = X[(size_t)t * cols + j];
    const GemvOrder ord = order_of(w, cols);
    auto store = [&](size_t b, size_t r, const float* lanes) {
        for (size_t p = 0; p < (size_t)TB && b * TB + p < (size_t)T; ++p) Y[(b * TB + p) * rows + r] = 0.f + lanes[p];
    };
    const size_t pairs = (rows + 1) / 2;
    parallel_for(e->threads, pairs, [&](size_t, size_t lo, size_t hi) {
        std::vector<float> w0(cols), w1(cols);
        alignas(32) float out0[TB], out1[TB];
        for (size_t pr = lo; pr < hi; ++pr) {
            const size_t r0 = 2 * pr, r1 = r0 + 1;
            const bool two = r1 < rows;
            deq_row(w, r0, cols, w0.data());
            if (two) deq_row(w, r1, cols, w1.data());
            else std::fill(w1.begin(), w1.end(), 0.f);
            for (size_t b = 0; b < nb; ++b) {
                const float* xb = Xb.data() + b * cols * TB;
#if defined(__AVX2__) && defined(__FMA__)
                __m256 a0 = _mm256_setzero_ps(), a1 = a0, a2 = a0, a3 = a0;
                __m256 c0 = a0, c1 = a0, c2 = a0, c3 = a0;
                size_t j = 0;
                for (; j < ord.main_end; j += 4) {
                    const __m256 x0 = _mm256_loadu_ps(xb + j * TB), x1 = _mm256_loadu_ps(xb + (j + 1) * TB);
                    const __m256 x2 = _mm256_loadu_ps(xb + (j + 2) * TB), x3 = _mm256_loadu_ps(xb + (j + 3) * TB);
                    a0 = _mm256_fmadd_ps(_mm256_set1_ps(w0[j]), x0, a0);
                    a1 = _mm256_fmadd_ps(_mm256_set1_ps(w0[j + 1]), x1, a1);
                    a2 = _mm256_fmadd_ps(_mm256_set1_ps(w0[j + 2]), x2, a2);
                    a3 = _mm256_fmadd_ps(_mm256_set1_ps(w0[j + 3]), x3, a3);
                    c0 = _mm256_fmadd_ps(_mm256_set1_ps(w1[j]), x0, c0);
                    c1 = _mm256_fmadd_ps(_mm256_set1_ps(w1[j + 1]), x1, c1);
                    c2 = _mm256_fmadd_ps(_mm256_set1_ps(w1[j + 2]), x2, c2);
                    c3 = _mm256_fmadd_ps(_mm256_set1_ps(w1[j + 3]), x3, c3);
                }
                for (; j < cols; ++j) {
                    const __m256 xv = _mm256_loadu_ps(xb + j * TB);
                    const __m256 v0 = _mm256_set1_ps(w0[j]), v1 = _mm256_set1_ps(w1[j]);
                    if (ord.tail_fused) {
                        a0 = _mm256_fmadd_ps(v0, xv, a0);
                        c0 = _mm256_fmadd_ps(v1, xv, c0);
                    } else {
                        a0 = _mm256_add_ps(a0, _mm256_mul_ps(v0, xv));
                        c0 = _mm256_add_ps(c0, _mm256_mul_ps(v1, xv));
                    }
                }
                _mm256_store_ps(out0, _mm256_add_ps(_mm256_add_ps(_mm256_add_ps(a0, a1), a2), a3));
                _mm256_store_ps(out1, _mm256_add_ps(_mm256_add_ps(_mm256_add_ps(c0, c1), c2), c3));
#else
                for (int k = 0; k < 2; ++k) {
                    const float* wr = k ? w1.data() : w0.data();
                    float acc[4][TB] = {};
                    size_t j = 0;
                    for (; j < ord.main_end; ++j)
                        for (int p = 0; p < TB; ++p) acc[j & 3][p] = std::fma(wr[j], xb[j * TB + p], acc[j & 3][p]);
                    for (; j < cols; ++j)
                        for (int p = 0; p < TB; ++p)
                            acc[0][p] = ord.tail_fused ? std::fma(wr[j], xb[j * TB + p], acc[0][p])
                                                       : acc[0][p] + wr[j] * xb[j * TB + p];
                    float* o = k ? out1 : out0;
                    for (int p = 0; p < TB; ++p) o[p] = acc[0][p] + acc[1][p] + acc[2][p] + acc[3][p];
                }
#endif
                store(b, r0, out0);
                if (two) store(b, r1, out1);
            }
        }
    });
}

}  // namespace

// T positions pos0..pos0+T-1 of one sequence (kv rows 0..pos0-1 already written by earlier
// steps); writes their K/V rows and the logits of the last position.
extern "C" int orc_engine_prefill(const orc_engine* e, const uint32_t* ids, int T, int pos0, float* kv,
                                  float* logits_last) {
    const size_t d = (size_t)e->n_embd;
    const size_t hd = d / (size_t)e->n_head;
    const size_t ctxd = (size_t)e->n_ctx * d;
    if (T <= 0 || pos0 < 0 || pos0 + T > e->n_ctx) return -1;
    for (int t = 0; t < T; ++t)
        if ((int)ids[t] >= e->vocab) return -1;
    std::vector<float> X((size_t)T * d);
    for (int t = 0; t < T; ++t) {
        std::vector<float> x = vec_row(e, "wte.weight", ids[t]);
        std::vector<float> wpe = vec_row(e, "wpe.weight", (uint32_t)(pos0 + t));
        for (size_t i = 0; i < d; ++i) X[t * d + i] = x[i] + wpe[i];
    }
    std::vector<float> Hn((size_t)T * d), ATT((size_t)T * d), PR((size_t)T * d);
    for (int layer = 0; layer < e->n_layer; ++layer) {
        float* kc = kv + (size_t)layer * 2 * ctxd;
        float* vc = kc + ctxd;
        std::vector<float> gw = vec_f32(e, L(layer, "ln_1.weight"));
        std::vector<float> gb = vec_f32(e, L(layer, "ln_1.bias"));
        Hn = X;
        for (int t = 0; t < T; ++t) layernorm(Hn.data() + t * d, d, gw.data(), gb.data(), e->ln_eps);
        std::string qkv_name = L(layer, "attn.c_attn.weight");
        const size_t inter3 = (size_t)e->get(qkv_name).shape[0];
        std::vector<float> QKV((size_t)T * inter3);
        matmul_batched(e, qkv_name, Hn.data(), T, QKV.data());
        std::vector<float> qb = vec_f32(e, L(layer, "attn.c_attn.bias"));
        for (int t = 0; t < T; ++t) {
            float* qkv = QKV.data() + t * inter3;
            for (size_t i = 0; i < inter3; ++i) qkv[i] += qb[i];
            size_t row = (size_t)(pos0 + t) * d;
            std::memcpy(kc + row, qkv + d, d * 4);
            std::memcpy(vc + row, qkv + 2 * d, d * 4);
        }
        // attention of every (position, head), the loops of orc_engine_step; the scores of 8 keys
        // are one vector (each lane sums q[tt] * k[tt] over tt in order, unfused, as the step does)
        const float scale = 1.0f / std::sqrt((float)hd);
        std::fill(ATT.begin(), ATT.end(), 0.f);
        const size_t npos = (size_t)pos0 + (size_t)T, npos8 = (npos + 7) / 8 * 8;
        std::vector<float> Kt((size_t)e->n_head * hd * npos8, 0.f);  // Kt[head][tt][p]
        for (size_t p = 0; p < npos; ++p)
            for (size_t i = 0; i < d; ++i) Kt[((i / hd) * hd + i % hd) * npos8 + p] = kc[p * d + i];
        const size_t pairs = (size_t)T * (size_t)e->n_head;
        const int nth = std::max(1, e->threads);
        parallel_for(nth, (size_t)nth, [&](size_t th, size_t, size_t) {
            std::vector<float> scores(npos8);
            for (size_t k = th; k < pairs; k += (size_t)nth) {  // interleaved: cost grows with the position
                const int t = (int)(k / (size_t)e->n_head), head = (int)(k % (size_t)e->n_head);
                const int pos = pos0 + t;
                const size_t o = (size_t)head * hd;
                const float* q = QKV.data() + t * inter3 + o;
                const float* kt = Kt.data() + (size_t)head * hd * npos8;
                float* attn_out = ATT.data() + t * d;
                float maxs = -3.40282347e+38f;  // f32::MIN
                for (int p0 = 0; p0 <= pos; p0 += 8) {
#if defined(__AVX2__) && defined(__FMA__)
                    __m256 dot = _mm256_setzero_ps();
                    for (size_t tt = 0; tt < hd; ++tt)
                        dot = _mm256_add_ps(dot, _mm256_mul_ps(_mm256_set1_ps(q[tt]), _mm256_loadu_ps(kt + tt * npos8 + p0)));
                    _mm256_storeu_ps(scores.data() + p0, _mm256_mul_ps(dot, _mm256_set1_ps(scale)));
#else
                    for (int p = p0; p < p0 + 8; ++p) {
                        float dot = 0.f;
                        for (size_t tt = 0; tt < hd; ++tt) dot += q[tt] * kt[tt * npos8 + p];
                        scores[p] = dot * scale;
                    }
#endif
                }
                for (int p = 0; p <= pos; ++p) maxs = rust_max(maxs, scores[p]);
                float sum = 0.f;
                for (int p = 0; p <= pos; ++p) {
                    scores[p] = std::exp(scores[p] - maxs);
                    sum += scores[p];
                }
                for (int p = 0; p <= pos; ++p) scores[p] /= sum;
                for (int p = 0; p <= pos; ++p) {
                    const float* vp = vc + (size_t)p * d + o;
                    for (size_t tt = 0; tt < hd; ++tt) attn_out[o + tt] += scores[p] * vp[tt];
                }
            }
        });
        matmul_batched(e, L(layer, "attn.c_proj.weight"), ATT.data(), T, PR.data());
        std::vector<float> pb = vec_f32(e, L(layer, "attn.c_proj.bias"));
        for (int t = 0; t < T; ++t)
            for (size_t i = 0; i < d; ++i) X[t * d + i] += PR[t * d + i] + pb[i];

        std::vector<float> gw2 = vec_f32(e, L(layer, "ln_2.weight"));
        std::vector<float> gb2 = vec_f32(e, L(layer, "ln_2.bias"));
        Hn = X;
        for (int t = 0; t < T; ++t) layernorm(Hn.data() + t * d, d, gw2.data(), gb2.data(), e->ln_eps);
        std::string fc_name = L(layer, "mlp.c_fc.weight");
        const size_t inter = (size_t)e->get(fc_name).shape[0];
        std::vector<float> FC((size_t)T * inter);
        matmul_batched(e, fc_name, Hn.data(), T, FC.data());
        std::vector<float> fb = vec_f32(e, L(layer, "mlp.c_fc.bias"));
        for (int t = 0; t < T; ++t) {
            float* fc = FC.data() + t * inter;
            for (size_t i = 0; i < inter; ++i) {
                float v = fc[i] + fb[i];
                fc[i] = 0.5f * v * (1.0f + std::tanh(0.7978845608028654f * (v + 0.044715f * v * v * v)));
            }
        }
        matmul_batched(e, L(layer, "mlp.c_proj.weight"), FC.data(), T, PR.data());
        std::vector<float> mb = vec_f32(e, L(layer, "mlp.c_proj.bias"));
        for (int t = 0; t < T; ++t)
            for (size_t i = 0; i < d; ++i) X[t * d + i] += PR[t * d + i] + mb[i];
    }
    // the tail of the last position's step (earlier positions' logits are not needed)
    std::vector<float> x(X.end() - (long)d, X.end());
    std::vector<float> wf = vec_f32(e, "ln_f.weight");
    std::vector<float> bf = vec_f32(e, "ln_f.bias");
    layernorm(x.data(), d, wf.data(), bf.data(), e->ln_eps);
    if (e->ad_r > 0) {
        const int r = e->ad_r;
        std::vector<float> ah(r);
        for (int j = 0; j < r; ++j) {
            float acc = 0.f;
            const float* ar = e->ad_a.data() + (size_t)j * d;
            for (size_t i = 0; i < d; ++i) acc = std::fma(ar[i], x[i], acc);
            ah[j] = acc;
        }
        for (size_t i = 0; i < d; ++i) {
            float acc = 0.f;
            const float* br = e->ad_b.data() + i * r;
            for (int j = 0; j < r; ++j) acc = std::fma(br[j], ah[j], acc);
            x[i] += acc;
        }
    }
    matmul(e, "wte.weight", x.data(), logits_last);
    return 0;
}

// Gpu::set_adapter / clear_adapter (gpu.rs:188-194): r = 0 clears.
extern "C" int orc_set_adapter(orc_engine* e, const float* a, const float* b, int r) {
    if (r < 0) return -1;
    e->ad_r = r;
    e->ad_a.assign(a ? a : nullptr, a ? a + (size_t)r * e->n_embd : nullptr);
    e->ad_b.assign(b ? b : nullptr, b ? b + (size_t)r * e->n_embd : nullptr);
    if (r > 0 && (!a || !b)) e->ad_r = 0;
    return 0;
}

extern "C" int orc_vec_f32(const orc_engine* e, const char* name, float* out, uint64_t n) {
    auto it = e->t.find(name);
    if (it == e->t.end()) return -1;
    std::vector<float> v = vec_f32(e, name);
    if (v.size() != n) return -2;
    std::memcpy(out, v.data(), n * 4);
    return 0;
}

extern "C" int orc_vec_row(const orc_engine* e, const char* name, uint32_t row, float* out, uint64_t n) {
    auto it = e->t.find(name);
    if (it == e->t.end()) return -1;
    std::vector<float> v = vec_row(e, name, row);
    if (v.size() != n) return -2;
    std::memcpy(out, v.data(), n * 4);
    return 0;
}

// gpt2.rs:390-396: Iterator::max_by(total_cmp) keeps the LAST maximal element.
static inline int32_t total_key(float f) {
    int32_t b;
    std::memcpy(&b, &f, 4);
    return b ^ (int32_t)(((uint32_t)(b >> 31)) >> 1);
}
extern "C" uint32_t orc_argmax(const float* v, size_t n) {
    size_t best = 0;
    int32_t bk = total_key(v[0]);
    for (size_t i = 1; i < n; ++i) {
        int32_t k = total_key(v[i]);
        if (k >= bk) {
            bk = k;
            best = i;
        }
    }
    return (uint32_t)best;
}

// gpt2.rs:367-388.
extern "C" int orc_generate_greedy(const orc_engine* e, const uint32_t* prompt, int n_prompt, int steps,
                                   uint32_t* out) {
    if (n_prompt <= 0) return -1;
    std::vector<float> kv(orc_kv_floats(e), 0.f);
    std::vector<float> logits((size_t)e->vocab);
    int n_out = 0;
    uint32_t next = 0;
    int max_pos = e->n_ctx - 1;
    for (int pos = 0; pos < n_prompt + steps; ++pos) {
        if (pos > max_pos) break;
        uint32_t tok = pos < n_prompt ? prompt[pos] : next;
        orc_engine_step(e, tok, pos, kv.data(), logits.data());
        if (pos + 1 >= n_prompt) {
            next = orc_argmax(logits.data(), logits.size());
            out[n_out++] = next;
            if (n_out == steps) break;
        }
    }
    return n_out;
}

// gpt2.rs:348-364.
extern "C" double orc_nll_per_token(const orc_engine* e, const uint32_t* ids, int n) {
    if (n < 2) return NAN;
    std::vector<float> kv(orc_kv_floats(e), 0.f);
    std::vector<float> logits((size_t)e->vocab);
    double total = 0.0;
    for (int pos = 0; pos < n - 1; ++pos) {
        orc_engine_step(e, ids[pos], pos, kv.data(), logits.data());
        size_t target = ids[pos + 1];
        float mx = -3.40282347e+38f;
        for (float l : logits) mx = rust_max(mx, l);
        double s = 0.0;
        for (float l : logits) s += std::exp((double)(l - mx));
        double lse = std::log(s);
        total -= (double)(logits[target] - mx) - lse;
    }
    return total / (double)(n - 1);
}

// bwparity.rs:215-305: independent full-sequence causal forward in f64.
extern "C" int orc_forward_f64(const orc_engine* e, const uint32_t* ids, int T, double* logits_out) {
    const size_t d = (size_t)e->n_embd, H = (size_t)e->n_head, hd = d / H;
    auto deq = [&](const std::string& n) {
        std::vector<float> f = vec_f32(e, n);
        return std::vector<double>(f.begin(), f.end());
    };
    auto gemv = [&](const std::vector<double>& W, const std::vector<double>& x, size_t rows) {
        size_t cols = x.size();
        std::vector<double> y(rows, 0.0);
        for (size_t r = 0; r < rows; ++r) {
            double a = 0.0;
            for (size_t c = 0; c < cols; ++c) a += W[r * cols + c] * x[c];
            y[r] = a;
        }
        return y;
    };
    auto ln = [&](const std::vector<double>& x, const std::vector<double>& w, const std::vector<double>& b) {
        double mean = 0.0;
        for (double v : x) mean += v;
        mean /= (double)d;
        double var = 0.0;
        for (double v : x) var += (v - mean) * (v - mean);
        var /= (double)d;
        std::vector<double> o(d);
        for (size_t i = 0; i < d; ++i) o[i] = (x[i] - mean) / std::sqrt(var + (double)e->ln_eps) * w[i] + b[i];
        return o;
    };
    std::vector<double> wte = deq("wte.weight");
    std::vector<std::vector<double>> x(T, std::vector<double>(d));
    for (int p = 0; p < T; ++p) {
        std::vector<float> pr = vec_row(e, "wpe.weight", (uint32_t)p);
        for (size_t i = 0; i < d; ++i) x[p][i] = wte[(size_t)ids[p] * d + i] + (double)pr[i];
    }
    const double scale = 1.0 / std::sqrt((double)hd);
    for (int l = 0; l < e->n_layer; ++l) {
        auto g1 = deq(L(l, "ln_1.weight")), b1 = deq(L(l, "ln_1.bias"));
        auto wca = deq(L(l, "attn.c_attn.weight")), bca = deq(L(l, "attn.c_attn.bias"));
        auto wap = deq(L(l, "attn.c_proj.weight")), bap = deq(L(l, "attn.c_proj.bias"));
        auto g2 = deq(L(l, "ln_2.weight")), b2 = deq(L(l, "ln_2.bias"));
        auto wfc = deq(L(l, "mlp.c_fc.weight")), bfc = deq(L(l, "mlp.c_fc.bias"));
        auto wmp = deq(L(l, "mlp.c_proj.weight")), bmp = deq(L(l, "mlp.c_proj.bias"));
        std::vector<std::vector<double>> qkv(T);
        for (int p = 0; p < T; ++p) {
            qkv[p] = gemv(wca, ln(x[p], g1, b1), bca.size());
            for (size_t i = 0; i < bca.size(); ++i) qkv[p][i] += bca[i];
        }
        for (int p = 0; p < T; ++p) {
            std::vector<double> ao(d, 0.0);
            for (size_t h = 0; h < H; ++h) {
                size_t o = h * hd;
                std::vector<double> sc((size_t)p + 1);
                double mx = -1.79769313486231570e+308;
                for (int j = 0; j <= p; ++j) {
                    double dd = 0.0;
                    for (size_t t = 0; t < hd; ++t) dd += qkv[p][o + t] * qkv[j][d + o + t];
                    sc[j] = dd * scale;
                    mx = std::max(mx, sc[j]);
                }
                double sum = 0.0;
                for (auto& s : sc) {
                    s = std::exp(s - mx);
                    sum += s;
                }
                for (auto& s : sc) s /= sum;
                for (int j = 0; j <= p; ++j)
                    for (size_t t = 0; t < hd; ++t) ao[o + t] += sc[j] * qkv[j][2 * d + o + t];
            }
            auto pr = gemv(wap, ao, d);
            for (size_t i = 0; i < d; ++i) x[p][i] += pr[i] + bap[i];
        }
        for (int p = 0; p < T; ++p) {
            auto fc = gemv(wfc, ln(x[p], g2, b2), bfc.size());
            for (size_t i = 0; i < fc.size(); ++i) {
                double v = fc[i] + bfc[i];
                fc[i] = 0.5 * v * (1.0 + std::tanh(0.7978845608028654 * (v + 0.044715 * v * v * v)));
            }
            auto mo = gemv(wmp, fc, d);
            for (size_t i = 0; i < d; ++i) x[p][i] += mo[i] + bmp[i];
        }
    }
    auto wf = deq("ln_f.weight"), bf = deq("ln_f.bias");
    for (int p = 0; p < T; ++p) {
        auto lg = gemv(wte, ln(x[p], wf, bf), (size_t)e->vocab);
        std::memcpy(logits_out + (size_t)p * e->vocab, lg.data(), (size_t)e->vocab * 8);
    }
    return 0;
}
