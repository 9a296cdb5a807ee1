/*
 * infernt_seed.h — counter-based, seed-reproducible synthetic inputs.
 *
 * Every synthetic weight, prompt token and KV prefill value used by the
 * decode path, its tests and its benchmark is a pure function of
 * (seed, stream, index).  The same inline functions compile for the host
 * (the CPU oracle, the reference runner) and for the device (the GPU
 * initialiser), and they use only integer arithmetic plus exact float
 * conversions and one IEEE multiply, so host and device produce
 * bit-identical values without moving gigabytes over PCIe.
 *
 * Generator: splitmix64 (S. Vigna, "Further scramblings of Marsaglia's
 * xorshift generators", 2014; the finaliser of Java's SplittableRandom),
 * used as a stateless hash of a 64-bit counter.
 *
 * Normal deviates: Irwin–Hall sum of twelve uniforms minus six (mean 0,
 * variance 1, support ±6).  Each uniform is a 16-bit integer k read as
 * (k + 0.5) / 65536, so the sum is an integer numerator over 65536 that
 * a float holds exactly; the only rounding is the final multiply by the
 * standard deviation.  Box–Muller would need log/cos, whose last-ulp
 * results differ between libm and the device math library.
 *
 * Stream ids used by the decode path (one stream per tensor):
 *   embedding 1, lm_head 2, prompt 7, KV prefill K 8 / V 9, logits 10,
 *   layer l matrix m: 100 + 16*l + m with m = q 0, k 1, v 2, o 3,
 *   gate 4, up 5, down 6.  Norm weights are the constant 1.0.
 */
#ifndef INFERNT_SEED_H
#define INFERNT_SEED_H

#include <stdint.h>

#if defined(__CUDACC__)
#define INFERNT_HD __host__ __device__ __forceinline__
#else
#define INFERNT_HD static inline
#endif

#define INFERNT_STREAM_EMBEDDING 1ull
#define INFERNT_STREAM_LM_HEAD 2ull
#define INFERNT_STREAM_PROMPT 7ull
#define INFERNT_STREAM_KV_K 8ull
#define INFERNT_STREAM_KV_V 9ull
#define INFERNT_STREAM_LOGITS 10ull
#define INFERNT_STREAM_LAYER(l, m) (100ull + 16ull * (uint64_t)(l) + (uint64_t)(m))

INFERNT_HD uint64_t infernt_splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

/* Key of one tensor stream. */
INFERNT_HD uint64_t infernt_stream_key(uint64_t seed, uint64_t stream) {
    return infernt_splitmix64(infernt_splitmix64(seed) ^ (stream * 0xD1B54A32D192ED03ull));
}

/* Standard normal (Irwin–Hall 12) for element i of a stream; exact in float. */
INFERNT_HD float infernt_normal(uint64_t key, uint64_t i) {
    uint32_t s = 0;
    for (uint64_t j = 0; j < 3; ++j) {
        uint64_t h = infernt_splitmix64(key + 3ull * i + j);
        s += (uint32_t)(h & 0xFFFFu) + (uint32_t)((h >> 16) & 0xFFFFu) +
             (uint32_t)((h >> 32) & 0xFFFFu) + (uint32_t)(h >> 48);
    }
    /* sum of (k+0.5)/65536 over 12 draws, minus 6  ==  (s - 393210) / 65536 */
    return (float)((int32_t)s - 393210) * (1.0f / 65536.0f);
}

/* Normal deviate with standard deviation `std` (one IEEE multiply). */
INFERNT_HD float infernt_normal_std(uint64_t key, uint64_t i, float std_dev) {
    return infernt_normal(key, i) * std_dev;
}

/* Uniform integer in [lo, hi) for element i (modulo bias < 2^-40 here). */
INFERNT_HD int32_t infernt_uniform_int(uint64_t key, uint64_t i, int32_t lo, int32_t hi) {
    uint64_t h = infernt_splitmix64(key + i);
    return lo + (int32_t)(h % (uint64_t)(hi - lo));
}

/* Round a float to the nearest bf16 value (ties to even), returned as float. */
INFERNT_HD float infernt_round_bf16(float f) {
    union { float f; uint32_t u; } v;
    v.f = f;
    if ((v.u & 0x7F800000u) == 0x7F800000u) return f; /* inf / nan unchanged */
    uint32_t lsb = (v.u >> 16) & 1u;
    v.u = (v.u + 0x7FFFu + lsb) & 0xFFFF0000u;
    return v.f;
}

#endif /* INFERNT_SEED_H */
