// BLAKE3, portable scalar form of the published specification (see blake3.h).
#include "blake3.h"

#include <cstring>
#include <thread>

namespace gpt2q {

namespace {

constexpr uint32_t IV[8] = {0x6A09E667u, 0xBB67AE85u, 0x3C6EF372u, 0xA54FF53Au,
                            0x510E527Fu, 0x9B05688Cu, 0x1F83D9ABu, 0x5BE0CD19u};
constexpr uint8_t PERM[16] = {2, 6, 3, 10, 7, 0, 4, 13, 1, 11, 12, 5, 9, 14, 15, 8};
constexpr uint32_t CHUNK_START = 1, CHUNK_END = 2, PARENT = 4, ROOT = 8;
constexpr size_t CHUNK_LEN = 1024, BLOCK_LEN = 64;

inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

inline void g(uint32_t* s, int a, int b, int c, int d, uint32_t mx, uint32_t my) {
    s[a] = s[a] + s[b] + mx;
    s[d] = rotr(s[d] ^ s[a], 16);
    s[c] = s[c] + s[d];
    s[b] = rotr(s[b] ^ s[c], 12);
    s[a] = s[a] + s[b] + my;
    s[d] = rotr(s[d] ^ s[a], 8);
    s[c] = s[c] + s[d];
    s[b] = rotr(s[b] ^ s[c], 7);
}

// The compression function: 16-word state after 7 rounds, before the feed-forward.
void compress(const uint32_t cv[8], const uint32_t block[16], uint64_t counter, uint32_t block_len, uint32_t flags,
              uint32_t out[16]) {
    uint32_t s[16] = {cv[0], cv[1], cv[2], cv[3], cv[4], cv[5], cv[6], cv[7],
                      IV[0], IV[1], IV[2], IV[3], (uint32_t)counter, (uint32_t)(counter >> 32), block_len, flags};
    uint32_t m[16];
    std::memcpy(m, block, sizeof(m));
    for (int r = 0; r < 7; ++r) {
        g(s, 0, 4, 8, 12, m[0], m[1]);
        g(s, 1, 5, 9, 13, m[2], m[3]);
        g(s, 2, 6, 10, 14, m[4], m[5]);
        g(s, 3, 7, 11, 15, m[6], m[7]);
        g(s, 0, 5, 10, 15, m[8], m[9]);
        g(s, 1, 6, 11, 12, m[10], m[11]);
        g(s, 2, 7, 8, 13, m[12], m[13]);
        g(s, 3, 4, 9, 14, m[14], m[15]);
        if (r < 6) {
            uint32_t p[16];
            for (int i = 0; i < 16; ++i) p[i] = m[PERM[i]];
            std::memcpy(m, p, sizeof(m));
        }
    }
    for (int i = 0; i < 8; ++i) {
        out[i] = s[i] ^ s[i + 8];
        out[i + 8] = s[i + 8] ^ cv[i];
    }
}

inline void load_block(const uint8_t* b, uint32_t w[16]) {
    for (int i = 0; i < 16; ++i)
        w[i] = (uint32_t)b[4 * i] | ((uint32_t)b[4 * i + 1] << 8) | ((uint32_t)b[4 * i + 2] << 16) |
               ((uint32_t)b[4 * i + 3] << 24);
}

void parent_cv(const uint32_t l[8], const uint32_t r[8], uint32_t flags, uint32_t out[8]) {
    uint32_t block[16], o[16];
    std::memcpy(block, l, 32);
    std::memcpy(block + 8, r, 32);
    compress(IV, block, 0, (uint32_t)BLOCK_LEN, PARENT | flags, o);
    std::memcpy(out, o, 32);
}

// Chaining value of one chunk (len <= 1024 bytes) at chunk index `counter`; with `root`, the
// first 8 output words of the root compression instead.
void chunk_cv(const uint8_t* p, size_t len, uint64_t counter, bool root, uint32_t out[8]) {
    uint32_t cv[8], w[16], o[16];
    std::memcpy(cv, IV, sizeof(cv));
    size_t done = 0;
    uint32_t flags = CHUNK_START;
    while (len - done > BLOCK_LEN) {
        load_block(p + done, w);
        compress(cv, w, counter, (uint32_t)BLOCK_LEN, flags, o);
        std::memcpy(cv, o, 32);
        done += BLOCK_LEN;
        flags = 0;
    }
    uint8_t last[64] = {0};
    std::memcpy(last, p + done, len - done);
    load_block(last, w);
    compress(cv, w, counter, (uint32_t)(len - done), flags | CHUNK_END | (root ? ROOT : 0), o);
    std::memcpy(out, o, 32);
}

// The left-complete tree over `len` bytes starting at chunk `counter`: the left subtree holds
// the largest power-of-two number of chunks that leaves at least one chunk on the right.
// The two halves of the top `par_depth` levels are hashed on two threads.
void subtree(const uint8_t* p, size_t len, uint64_t counter, bool root, int par_depth, uint32_t out[8]) {
    const size_t n_chunks = len == 0 ? 1 : (len + CHUNK_LEN - 1) / CHUNK_LEN;
    if (n_chunks == 1) return chunk_cv(p, len, counter, root, out);
    size_t left_chunks = 1;
    while (left_chunks * 2 < n_chunks) left_chunks *= 2;
    const size_t left_len = left_chunks * CHUNK_LEN;
    uint32_t l[8], r[8];
    if (par_depth > 0 && len >= ((size_t)1 << 20)) {
        std::thread t([&] { subtree(p, left_len, counter, false, par_depth - 1, l); });
        subtree(p + left_len, len - left_len, counter + left_chunks, false, par_depth - 1, r);
        t.join();
    } else {
        subtree(p, left_len, counter, false, 0, l);
        subtree(p + left_len, len - left_len, counter + left_chunks, false, 0, r);
    }
    parent_cv(l, r, root ? ROOT : 0, out);
}

}  // namespace

void blake3(const void* data, size_t len, uint8_t out[32], int threads) {
    int depth = 0;
    while ((1 << (depth + 1)) <= threads && depth < 8) ++depth;
    uint32_t w[8];
    subtree(static_cast<const uint8_t*>(data), len, 0, true, depth, w);
    for (int i = 0; i < 8; ++i) {
        out[4 * i] = (uint8_t)w[i];
        out[4 * i + 1] = (uint8_t)(w[i] >> 8);
        out[4 * i + 2] = (uint8_t)(w[i] >> 16);
        out[4 * i + 3] = (uint8_t)(w[i] >> 24);
    }
}

}  // namespace gpt2q
