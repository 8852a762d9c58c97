/* Seeded synthetic data for Qwen3-shaped test and benchmark workloads.
 *
 * The same definition runs on the host (C99) and on the device (CUDA), and
 * gives bit-identical values on both: every step is integer arithmetic except
 * one exact int->float conversion and one IEEE f32 multiply.
 *
 *   key(seed, stream)   = mix64(seed ^ mix64(stream))
 *   bits(key, i)        = mix64(key + i * 0xD1B54A32D192ED03)
 *   normal(key, i, k)   = (float)(sum of the four 16-bit lanes of bits - 131070) * k
 *
 * mix64 is the splitmix64 finaliser (Steele, Lea, Flood, "Fast splittable
 * pseudorandom number generators", OOPSLA 2014). The sum of four independent
 * uniform 16-bit integers is an Irwin-Hall(4) variate: mean 131070, standard
 * deviation sqrt((65536^2 - 1) / 3) = 37837.2266. `k` = wanted std / 37837.2266,
 * rounded to f32 on the host, so `normal` has the wanted standard deviation and
 * a bounded (+-3.46 sigma) near-Gaussian shape. The bounded shape is a stated
 * choice: it keeps host and device bit-exact without transcendental functions.
 *
 * Streams name tensors: global tensors use stream = code, layer tensors use
 * stream = ((layer + 1) << 8) | code, with the codes below.
 */
#ifndef ZYNFER_SYNTH_RNG_H
#define ZYNFER_SYNTH_RNG_H

#include <stdint.h>

#if defined(__CUDACC__)
#define ZS_HD __host__ __device__ __forceinline__
#else
#define ZS_HD static inline
#endif

#define ZS_IH4_SIGMA 37837.2266

enum {
    /* global tensors */
    ZS_EMBED = 1,
    ZS_FINAL_NORM = 2,
    ZS_TOKENS = 3,
    ZS_PROMPT_LENS = 4,
    ZS_ACTIVATIONS = 5,
    /* per-layer tensors (stream = ((layer + 1) << 8) | code) */
    ZS_INPUT_LN = 1,
    ZS_Q_NORM = 2,
    ZS_K_NORM = 3,
    ZS_WQ = 4,
    ZS_WK = 5,
    ZS_WV = 6,
    ZS_WO = 7,
    ZS_POST_LN = 8,
    ZS_WG = 9,
    ZS_WU = 10,
    ZS_WD = 11,
};

ZS_HD uint64_t zs_mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

ZS_HD uint64_t zs_key(uint64_t seed, uint64_t stream) { return zs_mix64(seed ^ zs_mix64(stream)); }

ZS_HD uint64_t zs_layer_stream(uint32_t layer, uint32_t code) {
    return ((uint64_t)(layer + 1u) << 8) | (uint64_t)code;
}

ZS_HD uint64_t zs_bits(uint64_t key, uint64_t index) {
    return zs_mix64(key + index * 0xD1B54A32D192ED03ull);
}

ZS_HD int32_t zs_ih4(uint64_t h) {
    return (int32_t)((h & 0xFFFFu) + ((h >> 16) & 0xFFFFu) + ((h >> 32) & 0xFFFFu) + (h >> 48)) - 131070;
}

/* One near-normal f32 sample; k = std / ZS_IH4_SIGMA rounded to f32. */
ZS_HD float zs_normal(uint64_t key, uint64_t index, float k) {
#if defined(__CUDA_ARCH__)
    return __fmul_rn((float)zs_ih4(zs_bits(key, index)), k); /* never contracted into an FMA */
#else
    return (float)zs_ih4(zs_bits(key, index)) * k;
#endif
}

/* Sampling draws of one sequence slot: stream ZS_SAMPLE_STREAM(slot); the
 * token at position pos uses indices pos * (vocab + 1) + v (one draw per
 * vocabulary entry) and pos * (vocab + 1) + vocab (the row's single draw). */
#define ZS_SAMPLE_STREAM(slot) (0x5A5A000000000000ull | (uint64_t)(slot))

/* Uniform in (0, 1) from 23 random bits: (u + 1/2) 2^-23, every step exact in f32. */
ZS_HD float zs_uniform01(uint64_t key, uint64_t index) {
#if defined(__CUDA_ARCH__)
    return __fmul_rn(__fadd_rn((float)(zs_bits(key, index) >> 41), 0.5f), 1.1920928955078125e-07f);
#else
    return ((float)(zs_bits(key, index) >> 41) + 0.5f) * 1.1920928955078125e-07f;
#endif
}

/* Uniform integer in [0, n). */
ZS_HD uint32_t zs_uniform_u32(uint64_t key, uint64_t index, uint32_t n) {
    return (uint32_t)(zs_bits(key, index) % (uint64_t)n);
}

#endif
