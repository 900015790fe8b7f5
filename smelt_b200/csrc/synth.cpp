// Seeded synthetic workload generator (host only): the xorshift64* Rng of
// LukasParke/smelt experiments/model-lab/src/gpu_backward.rs:835-856 and the
// Box-Muller normal of experiments/perf-lab/src/bin/atoms.rs:78-83. The uniform
// pairs are drawn sequentially; the transcendental transform runs on host threads
// (each output depends only on its own pair, so results equal the serial loop).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <thread>
#include <vector>

#include "gpt2q.h"

static inline uint64_t next_u64(uint64_t* s) {
    uint64_t x = *s;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *s = x;
    return x * 0x2545F4914F6CDD1Dull;
}

extern "C" uint64_t gpt2q_rng_new(uint64_t seed) { return seed ^ 0x9E3779B97F4A7C15ull; }

extern "C" void gpt2q_rng_normal_f32(uint64_t* state, float* out, size_t n, double stdv) {
    const size_t chunk = 1 << 20;
    std::vector<uint64_t> u(2 * std::min(n, chunk));
    unsigned hw = std::thread::hardware_concurrency();
    const size_t nthreads = hw == 0 ? 1 : (hw > 16 ? 16 : hw);
    for (size_t base = 0; base < n; base += chunk) {
        const size_t m = std::min(chunk, n - base);
        for (size_t i = 0; i < 2 * m; ++i) u[i] = next_u64(state) >> 11;
        auto work = [&](size_t lo, size_t hi) {
            for (size_t i = lo; i < hi; ++i) {
                double u1 = (double)u[2 * i] / 9007199254740992.0;
                double u2 = (double)u[2 * i + 1] / 9007199254740992.0;
                if (u1 < 1e-12) u1 = 1e-12;
                double z = std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
                out[base + i] = (float)(z * stdv);
            }
        };
        if (m < 65536 || nthreads == 1) {
            work(0, m);
        } else {
            std::vector<std::thread> ts;
            const size_t per = (m + nthreads - 1) / nthreads;
            for (size_t t = 0; t < nthreads; ++t) {
                const size_t lo = t * per, hi = std::min(m, lo + per);
                if (lo < hi) ts.emplace_back(work, lo, hi);
            }
            for (auto& t : ts) t.join();
        }
    }
}

extern "C" void gpt2q_rng_below(uint64_t* state, uint32_t* out, size_t n, uint64_t bound) {
    for (size_t i = 0; i < n; ++i) out[i] = (uint32_t)(next_u64(state) % bound);
}

// ---------------------------------------------------------------- converter (host)
// Group quantisers of the SMT atoms, multithreaded over 32-value groups:
//   Q8 (experiments/model-lab/src/atoms.rs:65-78): s = amax/127 in fp32 (1.0 when amax == 0)
//      quantises with the unrounded s; f16(s) is stored; q = clamp(round(v/s), +-127).
//   Q4 (experiments/perf-lab/src/bin/atoms.rs:89-99 math): d = f16(amax/7) quantises;
//      q = clamp(round(v/d), +-7); byte j = q[j] & 0xF | (q[j+16] & 0xF) << 4.
// round() is ties-away-from-zero like Rust's f32::round; NaN quotients (a scale that
// underflows to 0 gives 0/0) become 0 like Rust's `as i8`.
#include <cstring>

namespace {

uint16_t f32_to_f16_rne(float x) {
    uint32_t b;
    std::memcpy(&b, &x, 4);
    const uint16_t sign = (uint16_t)((b >> 16) & 0x8000u);
    const int32_t exp = (int32_t)((b >> 23) & 0xffu) - 127 + 15;
    const uint32_t man = b & 0x007fffffu;
    if (((b >> 23) & 0xffu) == 0xffu) return (uint16_t)(sign | 0x7c00u | ((man != 0) << 8));
    if (exp >= 0x1f) return (uint16_t)(sign | 0x7c00u);
    if (exp <= 0) {
        if (exp < -10) return sign;
        const uint32_t m2 = man | 0x00800000u;
        const uint32_t shift = (uint32_t)(14 - exp);
        const uint32_t hm = m2 >> shift;
        const uint32_t rem = m2 & ((1u << shift) - 1);
        const uint32_t mid = 1u << (shift - 1);
        const uint16_t round = (uint16_t)((rem > mid) || (rem == mid && (hm & 1u)));
        return (uint16_t)(sign | (uint16_t)((uint16_t)hm + round));
    }
    const uint32_t hm = man >> 13, rem = man & 0x1fffu;
    const uint32_t round = (uint32_t)((rem > 0x1000u) || (rem == 0x1000u && (hm & 1u)));
    return (uint16_t)(sign | (uint16_t)(((uint32_t)exp << 10) + hm + round));
}

float f16_bits_to_f32(uint16_t h) {
    const uint32_t sign = ((uint32_t)(h & 0x8000u)) << 16;
    uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu, bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            uint32_t e = 113;
            while ((man & 0x400u) == 0) {
                man <<= 1;
                e -= 1;
            }
            bits = sign | (e << 23) | ((man & 0x3ffu) << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

inline int8_t q_clamp(float v, float lim) {
    float r = std::round(v);
    if (std::isnan(r)) return 0;
    if (r < -lim) r = -lim;
    if (r > lim) r = lim;
    return (int8_t)r;
}

inline float max_abs32(const float* b) {
    float a = 0.f;
    for (int i = 0; i < 32; ++i) {
        const float v = std::fabs(b[i]);
        if (v > a) a = v;  // NaN-ignoring like f32::max
    }
    return a;
}

template <class F>
void parallel_groups(size_t groups, F&& f) {
    unsigned hw = std::thread::hardware_concurrency();
    const size_t nt = (groups < 4096 || hw <= 1) ? 1 : std::min<size_t>(hw, 32);
    if (nt == 1) {
        f(0, groups);
        return;
    }
    std::vector<std::thread> ts;
    const size_t per = (groups + nt - 1) / nt;
    for (size_t t = 0; t < nt; ++t) {
        const size_t lo = t * per, hi = std::min(groups, lo + per);
        if (lo < hi) ts.emplace_back(f, lo, hi);
    }
    for (auto& t : ts) t.join();
}

}  // namespace

extern "C" int gpt2q_quantize_q8(const float* x, size_t n, uint8_t* out) {
    if (!x || !out || n % 32) return GPT2Q_EARG;
    parallel_groups(n / 32, [&](size_t lo, size_t hi) {
        for (size_t g = lo; g < hi; ++g) {
            const float* b = x + g * 32;
            const float amax = max_abs32(b);
            const float s = amax == 0.f ? 1.0f : amax / 127.0f;
            const uint16_t h = f32_to_f16_rne(s);
            uint8_t* o = out + g * 34;
            o[0] = (uint8_t)(h & 0xff);
            o[1] = (uint8_t)(h >> 8);
            for (int i = 0; i < 32; ++i) o[2 + i] = (uint8_t)q_clamp(b[i] / s, 127.f);
        }
    });
    return GPT2Q_OK;
}

extern "C" int gpt2q_quantize_q4(const float* x, size_t n, uint8_t* out) {
    if (!x || !out || n % 32) return GPT2Q_EARG;
    parallel_groups(n / 32, [&](size_t lo, size_t hi) {
        for (size_t g = lo; g < hi; ++g) {
            const float* b = x + g * 32;
            const float amax = max_abs32(b);
            const uint16_t h = f32_to_f16_rne(amax == 0.f ? 1.0f : amax / 7.0f);
            const float d = f16_bits_to_f32(h);
            int8_t q[32];
            for (int i = 0; i < 32; ++i) q[i] = q_clamp(b[i] / d, 7.f);
            uint8_t* o = out + g * 18;
            o[0] = (uint8_t)(h & 0xff);
            o[1] = (uint8_t)(h >> 8);
            for (int j = 0; j < 16; ++j)
                o[2 + j] = (uint8_t)(((uint8_t)q[j] & 0xfu) | (((uint8_t)q[j + 16] & 0xfu) << 4));
        }
    });
    return GPT2Q_OK;
}
