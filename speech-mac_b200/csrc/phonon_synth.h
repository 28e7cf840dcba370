/* Seeded synthetic weights and inputs for the Flow-transformer benchmarks.
 *
 * The generator is the one speech-mac uses for its flow-head noise
 * (src/phonon_sampler.c:9-84): splitmix64 seeds a xoshiro256** state and
 * normals come from a double-precision Box-Muller pair. Weights are drawn
 * once on the host, so the CPU oracle and the GPU read identical bits.
 *
 * Draw rules:
 *   uniform int8      (next % 255) - 127                     in [-127, 127]
 *   uniform U(a, b)   a + (b - a) * ((next >> 40) * 2^-24)
 *   normal N(0, 1)    Box-Muller on two open-interval 53-bit uniforms
 *   fp16 / bf16       round to nearest even of the fp32 draw
 */
#ifndef PHONON_SYNTH_H
#define PHONON_SYNTH_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    uint64_t s[4];
    int has_spare;
    float spare;
} PhononRng;

/* Scale drawing modes for a Q8_0 linear. */
#define PHONON_SYNTH_SCALE_PER_LINEAR 0 /* one U(0.5,1.5)/(127*sqrt(cols)) per linear */
#define PHONON_SYNTH_SCALE_PER_ROW 1    /* one U(0.5,1.5)/127 per row */

void phonon_rng_seed(PhononRng *rng, uint64_t seed);
uint64_t phonon_rng_next(PhononRng *rng);
void phonon_rng_normal(PhononRng *rng, float *out, size_t n);
void phonon_rng_uniform(PhononRng *rng, float lo, float hi, float *out, size_t n);
uint16_t phonon_float_to_half(float x);
uint16_t phonon_float_to_bf16(float x);
/* rows x cols Q8_0 blocks (34 bytes per 32 weights, row-major). */
void phonon_synth_q8_linear(PhononRng *rng, size_t rows, size_t cols, int scale_mode,
                            uint8_t *blocks);
/* n bf16 values of N(mean, std). */
void phonon_synth_bf16_normal(PhononRng *rng, float mean, float std, uint16_t *out, size_t n);
/* One Flow layer in draw order qkv, out, mlp_in, mlp_out, norm1 w/b, norm2 w/b. */
void phonon_synth_layer(PhononRng *rng, int scale_mode, uint8_t *qkv, uint8_t *out, uint8_t *up,
                        uint8_t *down, uint16_t *norm1_w, uint16_t *norm1_b, uint16_t *norm2_w,
                        uint16_t *norm2_b);

#ifdef __cplusplus
}
#endif
#endif
