/* Replacement for speech-mac src/phonon_math.c (NEON + generated SLEEF) when
 * the reference is compiled on x86 for the oracle/_ref build.
 *
 * TEST INFRASTRUCTURE ONLY (oracle/_ref). Same three entry points and the
 * same split as src/phonon_math.c:18-45: full four-element groups go through
 * SLEEF u10 (here the portable restatement in ../sleef_u10.c), scalar tails
 * go through the system libm. */
#include "../sleef_u10.h"

#include <math.h>
#include <stddef.h>

void phonon_math_silu(float *values, size_t count);
void phonon_math_sincos(const float *input, size_t count, float *cosines, float *sines);
void phonon_math_exp4(float values[4]);

void phonon_math_silu(float *values, size_t count) {
    size_t vector_end = count - count % 4;
    for (size_t i = 0; i < vector_end; i += 4)
        for (size_t lane = 0; lane < 4; lane++) {
            float x = values[i + lane];
            values[i + lane] = x / (1.0f + oracle_sleef_expf(-x));
        }
    for (size_t i = vector_end; i < count; i++)
        values[i] = values[i] / (1.0f + expf(-values[i]));
}

void phonon_math_sincos(const float *input, size_t count, float *cosines, float *sines) {
    size_t vector_end = count - count % 4;
    for (size_t i = 0; i < vector_end; i += 4)
        oracle_sleef_sincosf4(input + i, cosines + i, sines + i);
    for (size_t i = vector_end; i < count; i++) {
        cosines[i] = cosf(input[i]);
        sines[i] = sinf(input[i]);
    }
}

void phonon_math_exp4(float values[4]) {
    oracle_sleef_expf4(values);
}
