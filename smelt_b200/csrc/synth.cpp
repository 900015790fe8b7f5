// Seeded synthetic workload generator (host only): the xorshift64* Rng of
// LukasParke/smelt experiments/model-lab/src/gpu_backward.rs:835-856 and the
// Box-Muller normal of experiments/perf-lab/src/bin/atoms.rs:78-83. The uniform
// pairs are drawn sequentially; the transcendental transform runs on host threads
// (each output depends only on its own pair, so results equal the serial loop).
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
