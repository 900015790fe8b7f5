// BLAKE3 hash (default 32-byte output, unkeyed), written from the published BLAKE3
// specification (J. O'Connor, J.-P. Aumasson, S. Neves, Z. Wilcox-O'Hearn, 2020): 1 KiB
// chunks of 64-byte blocks compressed with the 7-round ChaCha-style function, chunk chaining
// values merged into a left-complete binary tree, ROOT flag on the final compression.
// Used to verify SMT containers (per-section digests, merkle content_id, per-tensor digests).
#pragma once
#include <stddef.h>
#include <stdint.h>

namespace gpt2q {

// Hash (32-byte output) over the recursive form of the tree; `threads` > 1 hashes the top
// levels' subtrees of inputs of 1 MiB and more on that many threads (same result for any value).
void blake3(const void* data, size_t len, uint8_t out[32], int threads = 1);

}  // namespace gpt2q
