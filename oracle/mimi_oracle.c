/* CPU oracle for the Mimi latent transformer (the two-layer transformer that
 * turns each 32-wide latent frame into 16 feature rows of 512): a plain-C
 * restatement of speech-mac src/phonon_mimi.c:108-283.
 *
 * TEST INFRASTRUCTURE ONLY: loaded by tests/ as the checker, never by the
 * CUDA product path. Linears reduce sequentially (oracle_linear_batch) where
 * the reference calls cblas_sgemm; the attention is oracle_attention (the
 * flow attention's softmax, which the Mimi attention repeats for up to 250
 * keys); everything else follows the reference's operation order, compiled
 * with -ffp-contract=off. */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "phonon_oracle.h"

#define MIMI_CONTEXT 250
#define MIMI_STRIDE 16

int oracle_mimi_state_init(OracleMimiState *s) {
    if (!s)
        return 0;
    memset(s, 0, sizeof(*s));
    s->keys = calloc((size_t)2 * MIMI_CONTEXT * 512, sizeof(float));
    s->values = calloc((size_t)2 * MIMI_CONTEXT * 512, sizeof(float));
    if (!s->keys || !s->values) {
        oracle_mimi_state_free(s);
        return 0;
    }
    return 1;
}

void oracle_mimi_state_free(OracleMimiState *s) {
    if (!s)
        return;
    free(s->keys);
    free(s->values);
    s->keys = s->values = NULL;
}

/* src/phonon_mimi.c:98-104: position and failure cleared, previous zeroed
 * (cache rows become visible only once their position is written again). */
void oracle_mimi_state_reset(OracleMimiState *s) {
    if (!s)
        return;
    s->position = 0;
    s->failed = 0;
    memset(s->previous, 0, sizeof(s->previous));
}

static int bf16_vector(const uint16_t *bits, size_t n, float *out) {
    if (!bits)
        return 0;
    for (size_t i = 0; i < n; i++) {
        uint32_t wide = (uint32_t)bits[i] << 16;
        memcpy(&out[i], &wide, 4);
        if (!isfinite(out[i]))
            return 0;
    }
    return 1;
}

/* Depthwise causal transposed convolution (src/phonon_mimi.c:108-131):
 * out[o][c] = previous[c] * k[c][stride + o] + input[c] * k[c][o]. */
int oracle_mimi_upsample_frame(const uint16_t *weight, const float *input, const float *previous,
                               size_t channels, size_t stride, float *output) {
    if (!weight || !input || !previous || !output || !channels || channels > 512 || !stride ||
        stride > 16)
        return 0;
    float kernel[512 * 32];
    if (!bf16_vector(weight, channels * 2 * stride, kernel))
        return 0;
    for (size_t c = 0; c < channels; c++) {
        if (!isfinite(input[c]) || !isfinite(previous[c]))
            return 0;
        for (size_t o = 0; o < stride; o++) {
            float current = input[c] * kernel[c * 2 * stride + o];
            float old = previous[c] * kernel[c * 2 * stride + stride + o];
            output[o * channels + c] = old + current;
            if (!isfinite(output[o * channels + c]))
                return 0;
        }
    }
    return 1;
}

/* Sixteen queries of one frame, inserted one by one into the 250-slot ring
 * (src/phonon_mimi.c:136-193). */
static int attention(OracleMimiState *s, size_t layer, float qkv[16][1536], float attended[16][512],
                     float theta) {
    float *keys = s->keys + layer * MIMI_CONTEXT * 512, *values = s->values + layer * MIMI_CONTEXT * 512;
    static float gk[MIMI_CONTEXT][64], gv[MIMI_CONTEXT][64];
    for (size_t row = 0; row < 16; row++) {
        size_t position = s->position + row, slot = position % MIMI_CONTEXT;
        float *q = qkv[row];
        if (!oracle_rope_interleaved(q, 512, 8, position, theta) ||
            !oracle_rope_interleaved(q + 512, 512, 8, position, theta))
            return 0;
        memcpy(keys + slot * 512, q + 512, 512 * sizeof(float));
        memcpy(values + slot * 512, q + 1024, 512 * sizeof(float));
        size_t count = position < MIMI_CONTEXT - 1 ? position + 1 : MIMI_CONTEXT;
        size_t first = position + 1 - count;
        for (size_t head = 0; head < 8; head++) {
            for (size_t key = 0; key < count; key++) {
                size_t index = (first + key) % MIMI_CONTEXT;
                memcpy(gk[key], keys + index * 512 + head * 64, 64 * sizeof(float));
                memcpy(gv[key], values + index * 512 + head * 64, 64 * sizeof(float));
            }
            if (!oracle_attention(q + head * 64, &gk[0][0], &gv[0][0], count, 64, attended[row] + head * 64))
                return 0;
        }
    }
    return 1;
}

static int linear16(const OracleLinear *w, const float *input, float *output) {
    return oracle_linear_batch(w, input, 16, NULL, output);
}

/* One layer over the frame's 16 rows (src/phonon_mimi.c:194-245). */
static int layer_forward(const OracleMimi *m, OracleMimiState *s, size_t layer, float hidden[16][512]) {
    static float normalized[16][512], qkv[16][1536], projected[16][512], attended[16][512], mlp[16][2048];
    float nw[512], nb[512], scale[512];
    if (!bf16_vector(m->norm1_w[layer], 512, nw) || !bf16_vector(m->norm1_b[layer], 512, nb))
        return 0;
    for (size_t row = 0; row < 16; row++)
        if (!oracle_layer_norm(hidden[row], nw, nb, 512, 1e-5f, normalized[row]))
            return 0;
    for (size_t part = 0; part < 3; part++) {
        OracleLinear view = m->in_proj[layer];
        view.rows = 512;
        view.data = (const uint16_t *)view.data + part * 512 * 512;
        if (!linear16(&view, &normalized[0][0], &projected[0][0]))
            return 0;
        for (size_t row = 0; row < 16; row++)
            memcpy(qkv[row] + part * 512, projected[row], 512 * sizeof(float));
    }
    if (!attention(s, layer, qkv, attended, m->rope_theta) ||
        !linear16(&m->out_proj[layer], &attended[0][0], &projected[0][0]) ||
        !bf16_vector(m->scale1[layer], 512, scale))
        return 0;
    for (size_t row = 0; row < 16; row++)
        for (size_t i = 0; i < 512; i++)
            hidden[row][i] += scale[i] * projected[row][i];
    if (!bf16_vector(m->norm2_w[layer], 512, nw) || !bf16_vector(m->norm2_b[layer], 512, nb))
        return 0;
    for (size_t row = 0; row < 16; row++)
        if (!oracle_layer_norm(hidden[row], nw, nb, 512, 1e-5f, normalized[row]))
            return 0;
    if (!oracle_linear_batch(&m->linear1[layer], &normalized[0][0], 16, NULL, &mlp[0][0]) ||
        !oracle_erf_gelu(&mlp[0][0], 16 * 2048) ||
        !oracle_linear_batch(&m->linear2[layer], &mlp[0][0], 16, NULL, &projected[0][0]) ||
        !bf16_vector(m->scale2[layer], 512, scale))
        return 0;
    for (size_t row = 0; row < 16; row++)
        for (size_t i = 0; i < 512; i++) {
            hidden[row][i] += scale[i] * projected[row][i];
            if (!isfinite(hidden[row][i]))
                return 0;
        }
    return 1;
}

/* phonon_mimi_process (src/phonon_mimi.c:246-283) without the pointer-range
 * checks: latents [frames][32] -> features [frames * 16][512]. */
int oracle_mimi_process(const OracleMimi *m, OracleMimiState *s, const float *latents, size_t frames,
                        float *features) {
    if (!m || !s || s->failed || !latents || !features || !frames || frames > 8192 ||
        s->position / 16 > 8192 - frames)
        return 0;
    for (size_t i = 0; i < frames * 32; i++)
        if (!isfinite(latents[i]))
            return 0;
    static float hidden[16][512];
    for (size_t frame = 0; frame < frames; frame++) {
        float projected[512];
        OracleLinear projection = m->projection;
        if (!oracle_linear_batch(&projection, latents + frame * 32, 1, NULL, projected) ||
            !oracle_mimi_upsample_frame(m->upsample, projected, s->previous, 512, MIMI_STRIDE, &hidden[0][0]) ||
            !layer_forward(m, s, 0, hidden) || !layer_forward(m, s, 1, hidden)) {
            s->failed = 1;
            return 0;
        }
        memcpy(s->previous, projected, sizeof(projected));
        memcpy(features + frame * 16 * 512, hidden, sizeof(hidden));
        s->position += 16;
    }
    return 1;
}
