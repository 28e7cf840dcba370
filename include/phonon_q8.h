/* Q8_0 matvec API, served by libphonon_transformer_cuda (drop-in header).
 *
 * Same block type and prototypes as speech-mac src/phonon_q8.h:12-21. */
#ifndef PHONON_Q8_H
#define PHONON_Q8_H

#include <stddef.h>
#include <stdint.h>

/* GGML Q8_0: a little-endian binary16 scale, then 32 int8 values (34 bytes). */
typedef struct {
    uint16_t scale_bits;
    int8_t values[32];
} PhononQ8Block;

_Static_assert(sizeof(PhononQ8Block) == 34, "Q8_0 blocks are 34 packed bytes");

/* Return 1 on success, 0 on bad sizes, overlap or any non-finite value. */
int phonon_q8_dot(const PhononQ8Block *blocks, const float *input, size_t elements, float *result);
int phonon_q8_matvec(const PhononQ8Block *weights, const float *input, size_t rows, size_t columns,
                     float *output);

#endif
