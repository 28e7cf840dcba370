/* Tensor-view ABI shared with speech-mac's pack reader (drop-in header).
 *
 * Same types and prototypes as speech-mac src/phonon_pack.h:1-40 so that engine
 * sources compile unchanged against libphonon_transformer_cuda; the pack
 * functions themselves stay in the reference's src/phonon_pack.c. */
#ifndef PHONON_PACK_H
#define PHONON_PACK_H

#include <stddef.h>
#include <stdint.h>

#define PHONON_PACK_MAX_RANK 8

typedef enum { PHONON_PACK_Q8_0 = 1, PHONON_PACK_BF16 = 2 } PhononPackDType;

/* A borrowed tensor: Q8_0 blocks or bf16 values, row-major. linear_data is an
 * optional exact fp32 copy; its presence marks a prepared, immutable pack. */
typedef struct {
    PhononPackDType dtype;
    unsigned int rank;
    uint64_t shape[PHONON_PACK_MAX_RANK];
    const void *data;
    size_t byte_count;
    const float *linear_data;
} PhononTensorView;

typedef struct PhononPack PhononPack;

int phonon_pack_open(const char *path, PhononPack **pack);
void phonon_pack_close(PhononPack *pack);
int phonon_pack_prepare_linears(PhononPack *pack);
int phonon_tensor_expand_linear(const PhononTensorView *view, float **output);
size_t phonon_pack_tensor_count(const PhononPack *pack);
int phonon_pack_tensor(const PhononPack *pack, const char *name, PhononTensorView *view);
int phonon_pack_tensor_at(const PhononPack *pack, size_t index, const char **name,
                          size_t *name_length, PhononTensorView *view);
int phonon_bf16_to_float(const uint16_t *values, size_t count, float *output);

#endif
