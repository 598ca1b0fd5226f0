/*
 * synth.c -- seeded synthetic inputs for random-init Q8_0 models (libqq3synth.so).
 *
 * No model files exist on these machines, so every benchmark and parity run builds
 * its weights from a seed.  Each value is a pure function of (seed, index): a
 * splitmix64 finaliser (Steele, Lea & Flood, "Fast splittable pseudorandom number
 * generators", OOPSLA 2014) over a counter, so any slice can be produced on any
 * thread in any order with identical bytes.
 *
 * Q8_0 blocks are written in the GGUF layout read by the reference
 * (tensor.js:1-2, gguf.js:307-309): fp16 little-endian scale d, then 32 int8 qs.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static inline uint64_t draw(uint64_t seed, uint64_t stream, uint64_t i) {
    return mix64(mix64(seed ^ (stream * 0xD1B54A32D192ED03ull)) + i);
}

/* uniform in (0, 1] from the top 53 bits */
static inline double unit(uint64_t r) { return ((double)(r >> 11) + 1.0) * (1.0 / 9007199254740992.0); }

/* standard normal by Box-Muller on two independent draws */
static inline double normal(uint64_t seed, uint64_t stream, uint64_t i) {
    const double u1 = unit(draw(seed, stream, 2 * i)), u2 = unit(draw(seed, stream, 2 * i + 1));
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}

/* float -> IEEE binary16 bits, round to nearest even, from the format definition. */
static uint16_t f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds past 65504 */
    if (ax < 0x38800000u) {                                    /* half subnormal or zero */
        if (ax < 0x33000000u) return (uint16_t)sign;           /* below half of the smallest subnormal */
        /* value = m * 2^(E-150); in units of the half subnormal step 2^-24 that is m >> (126-E) */
        const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        const int s = 126 - (int)(ax >> 23); /* 14..24 here */
        uint32_t q = m >> s;
        const uint32_t rem = m & ((1u << s) - 1), halfw = 1u << (s - 1);
        if (rem > halfw || (rem == halfw && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (ax >> 23) - 112; /* rebias 127 -> 15 */
    uint32_t m = ax & 0x7fffffu;
    uint32_t q = (e << 10) | (m >> 13);
    const uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    return (uint16_t)(sign | q);
}

/*
 * Fill n_blocks Q8_0 blocks.  qs ~ U{-127..127}.  Scale d (converted to fp16):
 *   mode 0: d = a/127 * |1 + b*z|   (model weights: 0.02/127 x |N(1, 0.1)|, a=0.02, b=0.1)
 *   mode 1: d = |a*z| / 127          (matmul sweep: |N(0, 0.02)|/127, a=0.02)
 * with z ~ N(0, 1).  Block i depends only on (seed, block0 + i).
 */
void qq_synth_q8_0(uint8_t* out, int64_t n_blocks, int64_t block0, uint64_t seed, int mode, double a, double b) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n_blocks; i++) {
        const uint64_t bi = (uint64_t)(block0 + i);
        const double z = normal(seed, 1, bi);
        const double d = mode == 0 ? a / 127.0 * fabs(1.0 + b * z) : fabs(a * z) / 127.0;
        const uint16_t h = f32_to_f16((float)d);
        uint8_t* blk = out + i * 34;
        blk[0] = (uint8_t)(h & 0xff);
        blk[1] = (uint8_t)(h >> 8);
        for (int j = 0; j < 16; j++) {
            const uint64_t r = draw(seed, 2, bi * 16 + (uint64_t)j);
            const uint32_t lo = (uint32_t)r, hi = (uint32_t)(r >> 32);
            blk[2 + 2 * j] = (uint8_t)(int8_t)((int)(((uint64_t)lo * 255u) >> 32) - 127);
            blk[3 + 2 * j] = (uint8_t)(int8_t)((int)(((uint64_t)hi * 255u) >> 32) - 127);
        }
    }
}

/* n floats ~ N(mean, std), element i = f(seed, i0 + i). */
void qq_synth_normal_f32(float* out, int64_t n, int64_t i0, uint64_t seed, double mean, double std) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) out[i] = (float)(mean + std * normal(seed, 3, (uint64_t)(i0 + i)));
}

/* n ints uniform in [lo, hi). */
void qq_synth_uniform_i32(int32_t* out, int64_t n, uint64_t seed, int64_t lo, int64_t hi) {
    const uint64_t span = (uint64_t)(hi - lo);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
        const uint64_t r = draw(seed, 4, (uint64_t)i);
        out[i] = (int32_t)(lo + (int64_t)(((unsigned __int128)r * span) >> 64));
    }
}

uint16_t qq_synth_f32_to_f16(float f) { return f32_to_f16(f); }
