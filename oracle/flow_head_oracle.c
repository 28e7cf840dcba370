/* CPU oracle for the Phonon flow head (the MLP that turns a Flow-transformer
 * output row into a 32-wide latent): a plain-C restatement of speech-mac
 * src/phonon_sampler.c:220-393.
 *
 * TEST INFRASTRUCTURE ONLY: loaded by tests/ as the checker, never by the
 * CUDA product path. Linears reduce sequentially (oracle_linear_batch) where
 * the reference calls cblas_sgemm; everything else follows the reference's
 * operation order, compiled with -ffp-contract=off. */
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "phonon_oracle.h"
#include "sleef_u10.h"

/* bf16 is the top half of a binary32 (src/phonon_pack.c:320-341); a
 * non-finite value fails the call. */
static int head_vector(const uint16_t *bits, float *out, size_t count) {
    if (!bits)
        return 0;
    for (size_t i = 0; i < count; i++) {
        uint32_t wide = (uint32_t)bits[i] << 16;
        memcpy(&out[i], &wide, 4);
        if (!isfinite(out[i]))
            return 0;
    }
    return 1;
}

/* y = W x + b with a bf16 [rows, cols] W and a bf16 [rows] b
 * (src/phonon_sampler.c:220-224). */
static int affine(const OracleAffine *a, const float *input, size_t rows, size_t cols, float *output) {
    float b[1536];
    if (!a || rows > 1536 || a->w.rows != rows || a->w.cols != cols || a->w.dtype != ORACLE_BF16 ||
        !head_vector(a->b, b, rows))
        return 0;
    return oracle_linear_batch(&a->w, input, 1, b, output);
}

/* x / (1 + exp(-x)): SLEEF u10 exp on full groups of four, libm on the tail
 * (src/phonon_math.c:18-28). */
static void silu(float *values, size_t count) {
    size_t vector_end = count - count % 4;
    for (size_t i = 0; i < vector_end; i += 4) {
        float e[4] = {-values[i], -values[i + 1], -values[i + 2], -values[i + 3]};
        oracle_sleef_expf4(e);
        for (size_t lane = 0; lane < 4; lane++)
            values[i + lane] = values[i + lane] / (1.0f + e[lane]);
    }
    for (size_t i = vector_end; i < count; i++)
        values[i] = values[i] / (1.0f + expf(-values[i]));
}

/* Mean of 512 values in PyTorch's SumKernel order as the reference restates
 * it: four interleaved four-lane vectors, two cascade chunks of 16 groups
 * (src/phonon_sampler.c:229-248). */
static float mean_512(const float input[512]) {
    float sums[4][4] = {{0}};
    for (size_t chunk = 0; chunk < 2; chunk++) {
        float partial[4][4] = {{0}};
        for (size_t group = 0; group < 16; group++)
            for (size_t v = 0; v < 4; v++)
                for (size_t lane = 0; lane < 4; lane++)
                    partial[v][lane] += input[chunk * 256 + group * 16 + v * 4 + lane];
        for (size_t v = 0; v < 4; v++)
            for (size_t lane = 0; lane < 4; lane++)
                sums[v][lane] += partial[v][lane];
    }
    for (size_t v = 1; v < 4; v++)
        for (size_t lane = 0; lane < 4; lane++)
            sums[0][lane] += sums[v][lane];
    float sum = 0.0f;
    for (size_t lane = 0; lane < 4; lane++)
        sum += sums[0][lane];
    return sum / 512.0f;
}

/* LayerNorm with eps 1e-6: float mean by mean_512, variance from double
 * centred squares rounded once, optional affine (src/phonon_sampler.c:250-278). */
static int head_layer_norm(const float *input, const float *weight, const float *bias, float output[512]) {
    for (size_t i = 0; i < 512; i++)
        if (!isfinite(input[i]) || (weight && !isfinite(weight[i])) || (bias && !isfinite(bias[i])))
            return 0;
    float mean = mean_512(input);
    double variance_sum = 0.0;
    for (size_t i = 0; i < 512; i++) {
        double centered = (double)input[i] - mean;
        variance_sum += centered * centered;
    }
    float variance = (float)(variance_sum / 512.0);
    float inverse = 1.0f / sqrtf(variance + 1e-6f);
    for (size_t i = 0; i < 512; i++) {
        float normalized = (input[i] - mean) * inverse;
        if (weight)
            normalized = normalized * weight[i];
        if (bias)
            normalized = normalized + bias[i];
        output[i] = normalized;
        if (!isfinite(output[i]))
            return 0;
    }
    return 1;
}

/* Sinusoidal embedding of a flow time through a two-layer MLP and an RMS
 * normalisation with a learned gain (src/phonon_sampler.c:280-305). */
static int time_embedding(const OracleFlowHead *h, size_t which, float value, float out[512]) {
    float freqs[128], phase[128], embedding[256], hidden[512], alpha[512], squares[512];
    if (!isfinite(value) || !head_vector(h->time_freqs[which], freqs, 128))
        return 0;
    for (size_t i = 0; i < 128; i++)
        phase[i] = value * freqs[i];
    for (size_t i = 0; i < 128; i += 4)  /* cosines first, then sines */
        oracle_sleef_sincosf4(phase + i, embedding + i, embedding + 128 + i);
    if (!affine(&h->time[which][0], embedding, 512, 256, hidden))
        return 0;
    silu(hidden, 512);
    if (!affine(&h->time[which][1], hidden, 512, 512, out) || !head_vector(h->time_alpha[which], alpha, 512))
        return 0;
    for (size_t i = 0; i < 512; i++)
        squares[i] = out[i] * out[i];
    float inverse = 1.0f / sqrtf(mean_512(squares) + 1e-5f);
    for (size_t i = 0; i < 512; i++) {
        float weighted = alpha[i] * out[i];
        out[i] = weighted * inverse;
    }
    return 1;
}

/* out = h * (1 + scale) + shift, scale/shift from the modulation row. */
static void modulate(float h[512], const float *shift, const float *scale) {
    for (size_t i = 0; i < 512; i++) {
        float one_plus_scale = 1.0f + scale[i];
        float scaled = h[i] * one_plus_scale;
        h[i] = scaled + shift[i];
    }
}

/* src/phonon_sampler.c:307-359 (head_forward_cancel without the cancel poll). */
int oracle_flow_head_forward(const OracleFlowHead *h, const float condition[512], const float state[32],
                             float s, float t, float velocity[32]) {
    float x[512], y[512], time_s[512], time_t[512], modulation[1536], norm_w[512], norm_b[512];
    float hh[512], first[512], second[512], normalized[512];
    if (!h || !condition || !state || !velocity || !isfinite(s) || !isfinite(t) ||
        !affine(&h->input, state, 512, 32, x) || !affine(&h->cond, condition, 512, 512, y) ||
        !time_embedding(h, 0, s, time_s) || !time_embedding(h, 1, t, time_t))
        return 0;
    for (size_t i = 0; i < 512; i++)
        y[i] += 0.5f * (time_s[i] + time_t[i]);
    for (size_t block = 0; block < ORACLE_HEAD_BLOCKS; block++) {
        memcpy(normalized, y, sizeof(normalized));
        silu(normalized, 512);
        if (!affine(&h->block_ada[block], normalized, 1536, 512, modulation) ||
            !head_vector(h->block_norm_w[block], norm_w, 512) || !head_vector(h->block_norm_b[block], norm_b, 512) ||
            !head_layer_norm(x, norm_w, norm_b, hh))
            return 0;
        modulate(hh, modulation, modulation + 512);
        if (!affine(&h->block_mlp[block][0], hh, 512, 512, first))
            return 0;
        silu(first, 512);
        if (!affine(&h->block_mlp[block][1], first, 512, 512, second))
            return 0;
        for (size_t i = 0; i < 512; i++) {
            float gated = modulation[1024 + i] * second[i];
            x[i] = x[i] + gated;
        }
    }
    memcpy(normalized, y, sizeof(normalized));
    silu(normalized, 512);
    if (!affine(&h->final_ada, normalized, 1024, 512, modulation) || !head_layer_norm(x, NULL, NULL, hh))
        return 0;
    modulate(hh, modulation, modulation + 512);
    return affine(&h->final_out, hh, 32, 512, velocity);
}

/* One Euler step of the flow from scaled noise (src/phonon_sampler.c:366-393). */
int oracle_flow_lsd_one_step(const OracleFlowHead *h, const float condition[512], const float raw_noise[32],
                             float temperature, float output[32]) {
    float noise[32], velocity[32];
    if (!h || !condition || !raw_noise || !output || !isfinite(temperature) || temperature <= 0)
        return 0;
    float scale = sqrtf(temperature);
    for (size_t i = 0; i < 32; i++) {
        if (!isfinite(raw_noise[i]))
            return 0;
        noise[i] = raw_noise[i] * scale;
    }
    if (!oracle_flow_head_forward(h, condition, noise, 0.0f, 1.0f, velocity))
        return 0;
    for (size_t i = 0; i < 32; i++) {
        output[i] = noise[i] + velocity[i];
        if (!isfinite(output[i]))
            return 0;
    }
    return 1;
}
