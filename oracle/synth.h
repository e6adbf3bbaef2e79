/*
 * Seeded synthetic inputs shared by the oracle, the reference harness and the
 * tests.  TEST INFRASTRUCTURE: nothing in the product path includes this file;
 * the product carries its own device implementation of the same generator
 * (mini_llama_b200/csrc/synth.cu) and a test checks the two agree bit for bit.
 *
 * Generator: a counter-based splitmix64 stream per (seed, stream id).  A normal
 * value is the Irwin-Hall sum of twelve uniform 32-bit integers (six splitmix64
 * outputs, both halves), centred and scaled:
 *
 *     s  = sum of 12 uint32            (exact in uint64, < 2^36)
 *     z  = s * 2^-32 - 6               (exact in double)
 *     v  = (float)(z * sigma)          (two IEEE roundings)
 *
 * Only integer arithmetic and correctly rounded IEEE operations are involved,
 * so every platform (glibc, CUDA, any compiler without FMA contraction of the
 * single multiply) produces identical fp32 values.  Box-Muller would need log
 * and cos, whose last-ulp behaviour differs between libm and CUDA.
 *
 * Synthetic weight tensors are N(0, sigma) with this generator; stream ids for a
 * transformer are fixed by synth_stream_layer()/SYNTH_STREAM_* below.
 */
#ifndef MLB_ORACLE_SYNTH_H
#define MLB_ORACLE_SYNTH_H

#include <stdint.h>
#include <stddef.h>

#define SYNTH_GAMMA 0x9E3779B97F4A7C15ULL

static inline uint64_t synth_mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

/* Stream key for (seed, stream). */
static inline uint64_t synth_key(uint64_t seed, uint64_t stream) {
    return synth_mix64(seed * SYNTH_GAMMA + stream * 0xD1B54A32D192ED03ULL + 1ULL);
}

/* k-th raw 64-bit output of the stream (k >= 0). */
static inline uint64_t synth_u64(uint64_t key, uint64_t k) {
    return synth_mix64(key + (k + 1ULL) * SYNTH_GAMMA);
}

/* i-th N(0, sigma) value of the stream. */
static inline float synth_normal(uint64_t key, uint64_t i, double sigma) {
    uint64_t s = 0;
    for (uint64_t j = 0; j < 6; ++j) {
        uint64_t r = synth_u64(key, i * 6ULL + j);
        s += (r & 0xFFFFFFFFULL) + (r >> 32);
    }
    volatile double z = (double)s * (1.0 / 4294967296.0) - 6.0;
    volatile double v = z * sigma;
    return (float)v;
}

/* i-th integer uniform in [0, n). */
static inline uint32_t synth_index(uint64_t key, uint64_t i, uint32_t n) {
    uint64_t r = synth_u64(key, i) >> 32;
    return (uint32_t)((r * (uint64_t)n) >> 32);
}

/* Stream ids of a transformer's tensors. */
enum {
    SYNTH_KIND_WQ = 0,
    SYNTH_KIND_WK = 1,
    SYNTH_KIND_WV = 2,
    SYNTH_KIND_WO = 3,
    SYNTH_KIND_GATE = 4,
    SYNTH_KIND_UP = 5,
    SYNTH_KIND_DOWN = 6,
    SYNTH_KIND_BQ = 7,
    SYNTH_KIND_BK = 8,
    SYNTH_KIND_BV = 9,
};
#define SYNTH_STREAM_EMBEDDING 1ULL
#define SYNTH_STREAM_LM_HEAD 2ULL
#define SYNTH_STREAM_PROMPT 3ULL
#define SYNTH_STREAM_X 4ULL
#define SYNTH_STREAM_Q 5ULL
#define SYNTH_STREAM_K 6ULL
#define SYNTH_STREAM_V 7ULL
#define SYNTH_STREAM_W 8ULL

static inline uint64_t synth_stream_layer(int layer, int kind) {
    return ((uint64_t)(layer + 1) << 8) | (uint64_t)kind;
}

static inline void synth_fill_normal(float* out, size_t n, uint64_t seed, uint64_t stream,
                                     double sigma) {
    uint64_t key = synth_key(seed, stream);
    for (size_t i = 0; i < n; ++i) out[i] = synth_normal(key, (uint64_t)i, sigma);
}

#endif
