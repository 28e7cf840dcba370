/* CPU oracle: restatement of the speech-mac Flow-transformer decode step.
 *
 * TEST INFRASTRUCTURE ONLY (see phonon_oracle.h). Built with
 * -ffp-contract=off so that every multiply and add rounds separately, as the
 * reference's `#pragma STDC FP_CONTRACT OFF` regions require; the fused steps
 * the reference spells out with fmaf() are fmaf() here too.
 *
 * Reference files cited below are paths inside the speech-mac project.
 */
#include "phonon_oracle.h"
#include "sleef_u10.h"

#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- decoding */

/* Exact IEEE binary16 -> binary32, subnormals/inf/NaN included
 * (src/phonon_q8.c:7-34, duplicated at src/phonon_pack.c:343-370). */
float oracle_half_to_float(uint16_t bits) {
    uint32_t sign = (uint32_t)(bits >> 15) << 31;
    uint32_t exponent = (bits >> 10) & 0x1fu, mantissa = bits & 0x3ffu;
    float magnitude;
    if (exponent == 0x1fu) {
        uint32_t out = sign | 0x7f800000u | (mantissa << 13);
        memcpy(&magnitude, &out, 4);
        return magnitude;
    }
    if (exponent == 0)
        magnitude = ldexpf((float)mantissa, -24); /* exact: mantissa < 2^10 */
    else
        magnitude = ldexpf((float)(mantissa | 0x400u), (int)exponent - 25);
    return sign ? -magnitude : magnitude;
}

/* bf16 is the top half of a binary32 (src/phonon_pack.c:320-341). */
static float bf16_to_float(uint16_t bits) {
    uint32_t wide = (uint32_t)bits << 16;
    float f;
    memcpy(&f, &wide, 4);
    return f;
}

/* Round to the nearest bf16 (ties to even), returned widened to fp32. */
static float round_bf16(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    u += 0x7fffu + ((u >> 16) & 1u);
    u &= 0xffff0000u;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static int bf16_vector(const uint16_t *bits, float *out, size_t count) {
    if (!bits)
        return 0;
    for (size_t i = 0; i < count; i++) {
        out[i] = bf16_to_float(bits[i]);
        if (!isfinite(out[i]))
            return 0;
    }
    return 1;
}

static int ranges_overlap(const void *a, size_t a_bytes, const void *b, size_t b_bytes) {
    uintptr_t x = (uintptr_t)a, y = (uintptr_t)b;
    return x < y + b_bytes && y < x + a_bytes;
}

/* ------------------------------------------------------------------ Q8_0 */

/* One 34-byte Q8_0 block: little-endian binary16 scale + 32 int8
 * (src/phonon_q8.h:12-17). */
static uint16_t block_scale(const unsigned char *block) {
    return (uint16_t)(block[0] | (block[1] << 8));
}

/* Per-block fp32 partial sum, then sum += scale * partial
 * (src/phonon_q8.c:36-62). */
int oracle_q8_dot(const void *blocks, const float *input, size_t elements, float *result) {
    if (!blocks || !input || !result || !elements || elements % 32)
        return 0;
    const unsigned char *p = blocks;
    float sum = 0.0f;
    for (size_t b = 0; b < elements / 32; b++, p += 34) {
        float scale = oracle_half_to_float(block_scale(p));
        if (!isfinite(scale))
            return 0;
        float partial = 0.0f;
        for (size_t i = 0; i < 32; i++) {
            float x = input[b * 32 + i];
            if (!isfinite(x))
                return 0;
            partial += (float)(int8_t)p[2 + i] * x;
        }
        sum += scale * partial;
    }
    if (!isfinite(sum))
        return 0;
    *result = sum;
    return 1;
}

/* Row-wise q8_dot with the reference's size and overlap checks
 * (src/phonon_q8.c:64-92). */
int oracle_q8_matvec(const void *weights, const float *input, size_t rows, size_t columns,
                     float *output) {
    if (!weights || !input || !output || !rows || !columns || columns % 32)
        return 0;
    size_t weight_bytes = rows * (columns / 32) * 34;
    if (ranges_overlap(input, columns * sizeof(float), output, rows * sizeof(float)) ||
        ranges_overlap(weights, weight_bytes, output, rows * sizeof(float)))
        return 0;
    const unsigned char *w = weights;
    for (size_t r = 0; r < rows; r++)
        if (!oracle_q8_dot(w + r * (columns / 32) * 34, input, columns, output + r))
            return 0;
    return 1;
}

/* Exact expansion of a linear to fp32: W = fp16(scale) * q for Q8_0, plain
 * widening for BF16 (src/phonon_pack.c:372-411). */
static float *expand_linear(const OracleLinear *w) {
    size_t n = w->rows * w->cols;
    float *out = malloc(n * sizeof(float));
    if (!out)
        return NULL;
    if (w->dtype == ORACLE_BF16) {
        if (!bf16_vector(w->data, out, n)) {
            free(out);
            return NULL;
        }
        return out;
    }
    const unsigned char *p = w->data;
    for (size_t b = 0; b < n / 32; b++, p += 34) {
        float scale = oracle_half_to_float(block_scale(p));
        if (!isfinite(scale)) {
            free(out);
            return NULL;
        }
        for (size_t i = 0; i < 32; i++)
            out[b * 32 + i] = scale * (float)(int8_t)p[2 + i];
    }
    return out;
}

/* Y[b,r] = sum_c X[b,c] * W[r,c] (+ bias[r]). The reference reduces with
 * cblas_sgemm(RowMajor, NoTrans, Trans) (src/phonon_transformer.c:253-313);
 * the oracle reduces sequentially over c. */
int oracle_linear_batch(const OracleLinear *w, const float *input, size_t batch, const float *bias,
                        float *output) {
    if (!w || !w->data || !input || !output || !w->rows || !w->cols || !batch)
        return 0;
    if (w->dtype == ORACLE_Q8_0) {
        if (w->cols % 32 ||
            ranges_overlap(input, batch * w->cols * 4, output, batch * w->rows * 4) ||
            ranges_overlap(w->data, w->rows * w->cols / 32 * 34, output, batch * w->rows * 4))
            return 0;
    } else if (w->dtype != ORACLE_BF16) {
        return 0;
    }
    for (size_t i = 0; i < batch * w->cols; i++)
        if (!isfinite(input[i]))
            return 0;
    float *expanded = expand_linear(w);
    if (!expanded)
        return 0;
    for (size_t r = 0; r < w->rows; r++)
        if (bias && !isfinite(bias[r])) {
            free(expanded);
            return 0;
        }
    for (size_t b = 0; b < batch; b++)
        for (size_t r = 0; r < w->rows; r++) {
            const float *x = input + b * w->cols, *row = expanded + r * w->cols;
            float acc = 0.0f;
            for (size_t c = 0; c < w->cols; c++)
                acc += x[c] * row[c];
            output[b * w->rows + r] = bias ? acc + bias[r] : acc;
        }
    free(expanded);
    for (size_t i = 0; i < batch * w->rows; i++)
        if (!isfinite(output[i]))
            return 0;
    return 1;
}

/* ------------------------------------------------------------- LayerNorm */

/* Welford moments for width 512 in the exact order of PyTorch 2.7.1
 * RowwiseMoments<float> as the reference restates it
 * (src/phonon_transformer.c:87-151): eight 64-element chunks, each chunk four
 * interleaved lanes of 16 sequential Welford updates; chunk results merge into
 * a three-level binary cascade; the four lanes merge last with a fused mean
 * update and a fused M2 term. */
typedef struct {
    float mean[4], m2[4];
    size_t count;
} LaneMoments;

/* Merge `add` samples with moments (a_mean, a_m2) into (mean, m2) holding
 * `n` samples; unfused, in the reference's evaluation order
 * (src/phonon_transformer.c:90-98). */
static void merge_lane(size_t n, size_t add, float a_mean, float a_m2, float *mean, float *m2) {
    size_t total = n + add;
    float c = total ? (float)add / (float)total : 0.0f;
    float delta = a_mean - *mean;
    *mean += c * delta;
    *m2 += a_m2 + delta * delta * c * (float)n;
}

static void merge_level(const LaneMoments *from, LaneMoments *into) {
    for (int lane = 0; lane < 4; lane++)
        merge_lane(into->count, from->count, from->mean[lane], from->m2[lane], &into->mean[lane],
                   &into->m2[lane]);
    into->count += from->count;
}

static void moments_512(const float *x, float *mean_out, float *variance_out) {
    LaneMoments level[3];
    memset(level, 0, sizeof(level));
    for (size_t chunk = 0; chunk < 8; chunk++) {
        LaneMoments fresh;
        memset(&fresh, 0, sizeof(fresh));
        for (size_t j = 0; j < 16; j++)
            for (int lane = 0; lane < 4; lane++) {
                float v = x[chunk * 64 + j * 4 + lane], delta = v - fresh.mean[lane];
                fresh.mean[lane] += delta * (1.0f / (float)(j + 1));
                fresh.m2[lane] += delta * (v - fresh.mean[lane]);
            }
        fresh.count = 16;
        merge_level(&fresh, &level[0]);
        /* Binary carry: after chunk k, promote every level whose carry bit
         * of (k+1) is clear, lowest first. */
        size_t carry = chunk + 1;
        for (int l = 1; l < 3 && (carry & 1) == 0; l++, carry >>= 1) {
            merge_level(&level[l - 1], &level[l]);
            memset(&level[l - 1], 0, sizeof(level[l - 1]));
        }
    }
    for (int l = 1; l < 3; l++)
        merge_level(&level[l], &level[0]);
    float mean = 0.0f, m2 = 0.0f;
    size_t n = 0;
    for (int lane = 0; lane < 4; lane++) {
        size_t total = n + 128;
        float c = 128.0f / (float)total;
        float delta = level[0].mean[lane] - mean;
        mean = fmaf(c, delta, mean);
        m2 += fmaf(delta * delta * c, (float)n, level[0].m2[lane]);
        n = total;
    }
    *mean_out = mean;
    *variance_out = m2 / 512.0f;
}

/* ((x - mean) * rstd) * w + b, rstd = 1/sqrtf(var + eps); width 512 uses
 * moments_512, other widths a double two-pass variance
 * (src/phonon_transformer.c:153-185). */
int oracle_layer_norm(const float *input, const float *weight, const float *bias, size_t width,
                      float epsilon, float *output) {
    if (!input || !weight || !bias || !output || !width || !(epsilon > 0.0f) ||
        !isfinite(epsilon))
        return 0;
    double sum = 0.0;
    for (size_t i = 0; i < width; i++) {
        if (!isfinite(input[i]) || !isfinite(weight[i]) || !isfinite(bias[i]))
            return 0;
        sum += input[i];
    }
    double mean = sum / (double)width;
    float variance;
    if (width == 512) {
        float m;
        moments_512(input, &m, &variance);
        mean = m;
    } else {
        double squares = 0.0;
        for (size_t i = 0; i < width; i++) {
            double centered = (double)input[i] - mean;
            squares += centered * centered;
        }
        variance = (float)(squares / (double)width);
    }
    float scale = 1.0f / sqrtf(variance + epsilon);
    for (size_t i = 0; i < width; i++) {
        output[i] = ((float)((double)input[i] - mean) * scale) * weight[i] + bias[i];
        if (!isfinite(output[i]))
            return 0;
    }
    return 1;
}

/* x * w / sqrt(mean(x^2) + eps) with a double sum of squares
 * (src/phonon_transformer.c:66-85). */
int oracle_rms_norm(const float *input, const float *weight, size_t width, float epsilon,
                    float *output) {
    if (!input || !weight || !output || !width || !(epsilon > 0.0f) || !isfinite(epsilon))
        return 0;
    double squares = 0.0;
    for (size_t i = 0; i < width; i++) {
        if (!isfinite(input[i]) || !isfinite(weight[i]))
            return 0;
        squares += (double)input[i] * input[i];
    }
    float scale = 1.0f / sqrtf((float)(squares / (double)width) + epsilon);
    if (!isfinite(scale))
        return 0;
    for (size_t i = 0; i < width; i++) {
        output[i] = input[i] * scale * weight[i];
        if (!isfinite(output[i]))
            return 0;
    }
    return 1;
}

/* ------------------------------------------------------------------ GELU */

/* Abramowitz & Stegun 7.1.26 erf with explicit FMAs and libm expf, the form
 * PyTorch's NEON vectorized erf uses (src/phonon_transformer.c:190-200). */
static float erf_as7126(float x) {
    float t = 1.0f / fmaf(0.3275911f, fabsf(x), 1.0f);
    float r = fmaf(1.061405429f, t, -1.453152027f);
    r = fmaf(r, t, 1.421413741f);
    r = fmaf(r, t, -0.284496736f);
    r = fmaf(r, t, 0.254829592f);
    float negative_exp = -expf(-(x * x));
    return copysignf(fmaf(t * negative_exp, r, 1.0f), x);
}

/* 0.5*x*(1+erf(x/sqrt2)); full groups of four use the polynomial erf, the
 * count%4 tail uses libm erff (src/phonon_transformer.c:202-216). */
int oracle_erf_gelu(float *values, size_t count) {
    if (!values && count)
        return 0;
    size_t vector_end = count - count % 4;
    for (size_t i = 0; i < count; i++) {
        if (!isfinite(values[i]))
            return 0;
        float scaled = values[i] * 0.7071067811865475244f;
        float e = i < vector_end ? erf_as7126(scaled) : erff(scaled);
        values[i] = 0.5f * values[i] * (1.0f + e);
        if (!isfinite(values[i]))
            return 0;
    }
    return 1;
}

/* ------------------------------------------------------------------ RoPE */

/* Interleaved RoPE: pair (2i, 2i+1) of every head rotates by
 * position * theta^(-2i/head_width), frequencies and phases in fp32,
 * SLEEF u10 sincos on groups of four frequencies and libm on the tail
 * (src/phonon_transformer.c:218-251, src/phonon_math.c:30-40). */
int oracle_rope_interleaved(float *values, size_t width, size_t heads, size_t position,
                            float theta) {
    if (!values || !width || !heads || width % heads || (width / heads) % 2 || !(theta > 0.0f) ||
        !isfinite(theta))
        return 0;
    size_t head_width = width / heads, pairs = head_width / 2;
    for (size_t group = 0; group < pairs; group += 4) {
        size_t n = pairs - group < 4 ? pairs - group : 4;
        float phase[4] = {0}, c[4], s[4];
        for (size_t i = 0; i < n; i++) {
            float exponent = (float)(2 * (group + i)) / (float)head_width;
            float freq = 1.0f / powf(theta, exponent);
            phase[i] = (float)position * freq;
        }
        if (n == 4) {
            oracle_sleef_sincosf4(phase, c, s);
        } else {
            for (size_t i = 0; i < n; i++) {
                c[i] = cosf(phase[i]);
                s[i] = sinf(phase[i]);
            }
        }
        for (size_t h = 0; h < heads; h++) {
            float *head = values + h * head_width;
            for (size_t i = 0; i < n; i++) {
                size_t k = 2 * (group + i);
                float a = head[k], b = head[k + 1];
                if (!isfinite(a) || !isfinite(b) || !isfinite(c[i]) || !isfinite(s[i]))
                    return 0;
                head[k] = a * c[i] - b * s[i];
                head[k + 1] = a * s[i] + b * c[i];
                if (!isfinite(head[k]) || !isfinite(head[k + 1]))
                    return 0;
            }
        }
    }
    return 1;
}

/* ------------------------------------------------------------- attention */

/* q.k over one head in the [even | odd] component order the reference's
 * scratch permutation gives its GEMM (src/phonon_transformer.c:327-336). */
static float head_dot(const float *q, const float *k) {
    float acc = 0.0f;
    for (int parity = 0; parity < 2; parity++)
        for (int i = 0; i < 32; i++)
            acc += q[2 * i + parity] * k[2 * i + parity];
    return acc;
}

/* Single-query attention over `count` cached rows, online softmax in blocks
 * of 512 keys, scale 0.125, SLEEF exp on groups of four with lane sums
 * combined as (0+2)+(1+3), libm exp on the tail and for the rescale, and
 * normalisation after accumulating E@V (src/phonon_transformer.c:338-404).
 * Reductions the reference hands to SGEMM are sequential here. */
int oracle_attention(const float query[64], const float *keys, const float *values, size_t count,
                     size_t stride, float output[64]) {
    if (!count || count > ORACLE_MAX_POSITIONS || stride < 64)
        return 0;
    float maximum = -INFINITY, total = 0.0f, dest[64] = {0}, scores[512];
    for (size_t start = 0; start < count; start += 512) {
        size_t length = count - start < 512 ? count - start : 512;
        float next_max = maximum;
        for (size_t i = 0; i < length; i++) {
            scores[i] = head_dot(query, keys + (start + i) * stride) * 0.125f;
            if (!isfinite(scores[i]))
                return 0;
            if (scores[i] > next_max)
                next_max = scores[i];
        }
        float lanes[4] = {0};
        size_t vector_end = length - length % 4;
        for (size_t i = 0; i < vector_end; i += 4) {
            for (int l = 0; l < 4; l++)
                scores[i + l] -= next_max;
            oracle_sleef_expf4(scores + i);
            for (int l = 0; l < 4; l++)
                lanes[l] += scores[i + l];
        }
        float block_sum = (lanes[0] + lanes[2]) + (lanes[1] + lanes[3]);
        for (size_t i = vector_end; i < length; i++) {
            scores[i] = expf(scores[i] - next_max);
            block_sum += scores[i];
        }
        float rescale = expf(maximum - next_max);
        total = fmaf(rescale, total, block_sum);
        maximum = next_max;
        if (start)
            for (int d = 0; d < 64; d++)
                dest[d] *= rescale;
        for (int d = 0; d < 64; d++) {
            float acc = 0.0f;
            for (size_t j = 0; j < length; j++)
                acc += scores[j] * values[(start + j) * stride + d];
            dest[d] = start ? dest[d] + acc : acc;
        }
    }
    if (!(total > 0.0f) || !isfinite(total))
        return 0;
    float inverse = 1.0f / total;
    for (int d = 0; d < 64; d++) {
        output[d] = dest[d] * inverse;
        if (!isfinite(output[d]))
            return 0;
    }
    return 1;
}

/* --------------------------------------------------------------- caching */

/* Contiguous request cache [layer][capacity][512] for K and V, as the
 * reference lays out PhononKvCache (src/phonon_transformer.c:16-64), with a
 * runtime layer count. */
int oracle_cache_init(OracleCache *cache, size_t n_layers, size_t capacity) {
    if (!cache || !n_layers || !capacity)
        return 0;
    memset(cache, 0, sizeof(*cache));
    size_t count = n_layers * capacity * ORACLE_WIDTH;
    cache->keys = calloc(count, sizeof(float));
    cache->values = calloc(count, sizeof(float));
    if (!cache->keys || !cache->values) {
        oracle_cache_destroy(cache);
        return 0;
    }
    cache->n_layers = n_layers;
    cache->capacity = capacity;
    return 1;
}

void oracle_cache_destroy(OracleCache *cache) {
    if (!cache)
        return;
    free(cache->keys);
    free(cache->values);
    memset(cache, 0, sizeof(*cache));
}

/* ------------------------------------------------------------ layer step */

/* Pre-LN block: LN1 -> QKV -> RoPE(q,k) -> append -> 8-head attention over
 * position+1 keys -> out proj -> +x -> LN2 -> up -> GELU -> down -> +residual
 * (src/phonon_transformer.c:406-453). */
static int layer_step(const OracleLayer *w, OracleCache *cache, size_t layer, size_t position,
                      const float *input, float theta, float *output, int keep_row, float *k_out,
                      float *v_out) {
    if (!w || !cache || !input || !output || layer >= cache->n_layers ||
        position >= cache->capacity || position >= ORACLE_MAX_POSITIONS ||
        cache->length != position)
        return 0;
    float n1w[512], n1b[512], n2w[512], n2b[512], normalized[512], residual[512];
    float projected[1536], attended[512], attention[512], mlp[2048];
    if (!bf16_vector(w->norm1_w, n1w, 512) || !bf16_vector(w->norm1_b, n1b, 512) ||
        !bf16_vector(w->norm2_w, n2w, 512) || !bf16_vector(w->norm2_b, n2b, 512) ||
        !oracle_layer_norm(input, n1w, n1b, 512, 1e-5f, normalized) ||
        !oracle_linear_batch(&w->qkv, normalized, 1, NULL, projected))
        return 0;
    float *q = projected, *k = projected + 512, *v = projected + 1024;
    if (!oracle_rope_interleaved(q, 512, 8, position, theta) ||
        !oracle_rope_interleaved(k, 512, 8, position, theta))
        return 0;
    for (size_t i = 0; i < 512; i++)
        if (!isfinite(k[i]) || !isfinite(v[i]))
            return 0;
    if (cache->kv_bf16) /* bf16 KV pages (benchmark configs[3]): one rounding on append */
        for (size_t i = 0; i < 512; i++) {
            k[i] = round_bf16(k[i]);
            v[i] = round_bf16(v[i]);
        }
    if (k_out)
        memcpy(k_out, k, 512 * sizeof(float));
    if (v_out)
        memcpy(v_out, v, 512 * sizeof(float));
    size_t base = layer * cache->capacity * 512;
    if (!keep_row) {
        memcpy(cache->keys + base + position * 512, k, 512 * sizeof(float));
        memcpy(cache->values + base + position * 512, v, 512 * sizeof(float));
    }
    for (size_t h = 0; h < 8; h++)
        if (!oracle_attention(q + h * 64, cache->keys + base + h * 64,
                              cache->values + base + h * 64, position + 1, 512,
                              attended + h * 64))
            return 0;
    if (!oracle_linear_batch(&w->out, attended, 1, NULL, attention))
        return 0;
    for (size_t i = 0; i < 512; i++)
        residual[i] = input[i] + attention[i];
    if (!oracle_layer_norm(residual, n2w, n2b, 512, 1e-5f, normalized) ||
        !oracle_linear_batch(&w->up, normalized, 1, NULL, mlp) || !oracle_erf_gelu(mlp, 2048) ||
        !oracle_linear_batch(&w->down, mlp, 1, NULL, output))
        return 0;
    for (size_t i = 0; i < 512; i++) {
        output[i] += residual[i];
        if (!isfinite(output[i]))
            return 0;
    }
    return 1;
}

int oracle_layer_step(const OracleLayer *w, OracleCache *cache, size_t layer, size_t position,
                      const float *input, float theta, float *output) {
    return layer_step(w, cache, layer, position, input, theta, output, 0, NULL, NULL);
}

/* Test hook (teacher forcing of the K/V append): the same layer step, but
 * the row at `position` is the one the caller left in the cache (a device's
 * appended row) instead of the row this step computes; the computed rows
 * (bf16-rounded in a bf16 cache) go to k_out / v_out. */
int oracle_layer_step_forced(const OracleLayer *w, OracleCache *cache, size_t layer,
                             size_t position, const float *input, float theta, float *output,
                             float *k_out, float *v_out) {
    return layer_step(w, cache, layer, position, input, theta, output, 1, k_out, v_out);
}

/* All layers in order, then one commit of the position
 * (src/phonon_transformer.c:455-489). The output is written only on success. */
int oracle_stack_step(const OracleLayer *layers, size_t n_layers, OracleCache *cache,
                      size_t position, const float *input, float theta, float *output,
                      float *layer_outputs) {
    if (!layers || !cache || !input || !output || n_layers != cache->n_layers ||
        position != cache->length || position >= cache->capacity)
        return 0;
    float a[512], b[512];
    memcpy(a, input, sizeof(a));
    for (size_t l = 0; l < n_layers; l++) {
        if (!oracle_layer_step(&layers[l], cache, l, position, a, theta, b))
            return 0;
        if (layer_outputs)
            memcpy(layer_outputs + l * 512, b, sizeof(b));
        memcpy(a, b, sizeof(a));
    }
    cache->length++;
    memcpy(output, a, sizeof(a));
    return 1;
}
