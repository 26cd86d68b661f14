// Attention dropout without a random-number state: every keep / drop decision is a pure function of
// (seed, batch * heads + query head, query row l, key s), so the forward and the backward recompute
// the same decisions wherever the element is handled, in any kernel, in any order.
//
// The mixing function is "lowbias32", the 32-bit integer hash published by Chris Wellons
// ("Prospecting for Hash Functions", 2018: xorshift-multiply rounds with the constants 0x7feb352d and
// 0x846ca68b). Keys are chained: head key = h(seed_hi ^ h(seed_lo ^ bh)), row key = h(head key ^ l),
// element = h(row key + s); the element is kept when its hash is >= threshold = floor(p * 2^32), so
// it is dropped with probability p (to 2^-32). Kept probabilities are scaled by 1 / (1 - p), as the
// reference's dropout on the attention probabilities does (gguf_train/nn/functional.py:750-767, with
// torch's inverted dropout). The reference draws its mask from a sequential generator instead, so the
// masks differ; tests compare against a restatement of this function.
#pragma once

#include <stdint.h>

namespace gtb {

__host__ __device__ __forceinline__ uint32_t lowbias32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

__host__ __device__ __forceinline__ uint32_t drop_head_key(uint64_t seed, uint32_t bh) {
    return lowbias32((uint32_t)(seed >> 32) ^ lowbias32((uint32_t)seed ^ bh));
}

__host__ __device__ __forceinline__ uint32_t drop_row_key(uint32_t head_key, uint32_t l) { return lowbias32(head_key ^ l); }

__host__ __device__ __forceinline__ bool drop_keep(uint32_t row_key, uint32_t s, uint32_t threshold) {
    return lowbias32(row_key + s) >= threshold;
}

// threshold of a drop probability p in [0, 1)
inline uint32_t drop_threshold(float p) {
    const double t = (double)p * 4294967296.0;
    return t <= 0.0 ? 0u : t >= 4294967295.0 ? 4294967295u : (uint32_t)t;
}

}  // namespace gtb
