/* Seeded synthetic generator; see phonon_synth.h for the draw rules. */
#include "phonon_synth.h"

#include <math.h>
#include <string.h>

static uint64_t splitmix64(uint64_t *state) {
    uint64_t z = (*state += 0x9e3779b97f4a7c15ull);
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

static uint64_t rotl64(uint64_t v, int k) {
    return (v << k) | (v >> (64 - k));
}

void phonon_rng_seed(PhononRng *rng, uint64_t seed) {
    memset(rng, 0, sizeof(*rng));
    uint64_t state = seed;
    for (int i = 0; i < 4; i++)
        rng->s[i] = splitmix64(&state);
    if (!(rng->s[0] | rng->s[1] | rng->s[2] | rng->s[3]))
        rng->s[0] = 1;
}

/* xoshiro256** (Blackman & Vigna, 2018). */
uint64_t phonon_rng_next(PhononRng *rng) {
    uint64_t *s = rng->s;
    uint64_t result = rotl64(s[1] * 5, 7) * 9;
    uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl64(s[3], 45);
    return result;
}

void phonon_rng_normal(PhononRng *rng, float *out, size_t n) {
    const double unit = 1.0 / 9007199254740992.0; /* 2^-53 */
    for (size_t i = 0; i < n; i++) {
        if (rng->has_spare) {
            rng->has_spare = 0;
            out[i] = rng->spare;
            continue;
        }
        double u1 = ((double)(phonon_rng_next(rng) >> 11) + 0.5) * unit;
        double u2 = ((double)(phonon_rng_next(rng) >> 11) + 0.5) * unit;
        double radius = sqrt(-2.0 * log(u1)), angle = 6.283185307179586476925286766559 * u2;
        rng->spare = (float)(radius * sin(angle));
        rng->has_spare = 1;
        out[i] = (float)(radius * cos(angle));
    }
}

void phonon_rng_uniform(PhononRng *rng, float lo, float hi, float *out, size_t n) {
    for (size_t i = 0; i < n; i++) {
        float unit = (float)(phonon_rng_next(rng) >> 40) * (1.0f / 16777216.0f);
        out[i] = lo + (hi - lo) * unit;
    }
}

static uint32_t f2u(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    return u;
}

uint16_t phonon_float_to_bf16(float x) {
    uint32_t u = f2u(x);
    if ((u & 0x7fffffffu) > 0x7f800000u) /* NaN stays a quiet NaN */
        return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

/* IEEE binary32 -> binary16, round to nearest even, subnormals and overflow
 * to infinity included. */
uint16_t phonon_float_to_half(float x) {
    uint32_t u = f2u(x);
    uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    uint32_t abs = u & 0x7fffffffu;
    if (abs > 0x7f800000u)
        return sign | 0x7e00u;
    if (abs >= 0x477ff000u) /* rounds to >= 65520 -> inf */
        return sign | 0x7c00u;
    int exponent = (int)(abs >> 23) - 127;
    uint32_t mantissa = (abs & 0x7fffffu) | 0x800000u;
    if (abs < 0x33000001u) /* below half the smallest subnormal */
        return sign;
    int shift;
    uint32_t base;
    if (exponent < -14) { /* subnormal half: value = m * 2^-24 */
        shift = -exponent - 14 + 13;
        base = 0;
    } else {
        shift = 13;
        base = (uint32_t)(exponent + 15) << 10;
        mantissa &= 0x7fffffu;
    }
    uint32_t kept = mantissa >> shift, rest = mantissa & ((1u << shift) - 1u);
    uint32_t halfway = 1u << (shift - 1);
    if (rest > halfway || (rest == halfway && (kept & 1u)))
        kept++;
    return (uint16_t)(sign | (base + kept)); /* carry into the exponent is correct */
}

void phonon_synth_q8_linear(PhononRng *rng, size_t rows, size_t cols, int scale_mode,
                            uint8_t *blocks) {
    uint16_t scale = 0;
    if (scale_mode == PHONON_SYNTH_SCALE_PER_LINEAR) {
        float u;
        phonon_rng_uniform(rng, 0.5f, 1.5f, &u, 1);
        scale = phonon_float_to_half(u / (127.0f * sqrtf((float)cols)));
    }
    for (size_t r = 0; r < rows; r++) {
        if (scale_mode == PHONON_SYNTH_SCALE_PER_ROW) {
            float u;
            phonon_rng_uniform(rng, 0.5f, 1.5f, &u, 1);
            scale = phonon_float_to_half(u / 127.0f);
        }
        for (size_t b = 0; b < cols / 32; b++) {
            uint8_t *blk = blocks + (r * (cols / 32) + b) * 34;
            blk[0] = (uint8_t)(scale & 0xffu);
            blk[1] = (uint8_t)(scale >> 8);
            for (int i = 0; i < 32; i++)
                blk[2 + i] = (uint8_t)(int8_t)((int)(phonon_rng_next(rng) % 255u) - 127);
        }
    }
}

void phonon_synth_bf16_normal(PhononRng *rng, float mean, float std, uint16_t *out, size_t n) {
    for (size_t i = 0; i < n; i++) {
        float z;
        phonon_rng_normal(rng, &z, 1);
        out[i] = phonon_float_to_bf16(mean + std * z);
    }
}

void phonon_synth_layer(PhononRng *rng, int scale_mode, uint8_t *qkv, uint8_t *out, uint8_t *up,
                        uint8_t *down, uint16_t *norm1_w, uint16_t *norm1_b, uint16_t *norm2_w,
                        uint16_t *norm2_b) {
    phonon_synth_q8_linear(rng, 1536, 512, scale_mode, qkv);
    phonon_synth_q8_linear(rng, 512, 512, scale_mode, out);
    phonon_synth_q8_linear(rng, 2048, 512, scale_mode, up);
    phonon_synth_q8_linear(rng, 512, 2048, scale_mode, down);
    phonon_synth_bf16_normal(rng, 1.0f, 0.02f, norm1_w, 512);
    phonon_synth_bf16_normal(rng, 0.0f, 0.02f, norm1_b, 512);
    phonon_synth_bf16_normal(rng, 1.0f, 0.02f, norm2_w, 512);
    phonon_synth_bf16_normal(rng, 0.0f, 0.02f, norm2_b, 512);
}
