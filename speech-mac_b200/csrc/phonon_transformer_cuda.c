/* libphonon_transformer_cuda: C17 drop-in for speech-mac's
 * src/phonon_transformer.c (Flow-LM step, KV cache, primitives, conditioning
 * and embedding helpers) and src/phonon_q8.c, running every numerical call
 * on a B200 through libphonon_cuda (include/phonon_cuda.h). An engine links
 * it in place of those two files; its pack reader (src/phonon_pack.c) stays.
 *
 * Contracts kept from the reference (src/phonon_transformer.h:7-9, :33-81):
 *  - 1 on success, 0 on failure; argument checks in the reference's order;
 *  - outputs of step/prefill are written only on success, a cancelled call
 *    resets the cache, and the cancel callback is polled on the reference's
 *    schedule (before each layer and once after, for steps);
 *  - PhononKvCache keeps host keys/values mirrors in the reference layout
 *    [layer][capacity][512]; device steps copy the rows they append back into
 *    the mirror so readers of cache->keys see what the reference would.
 *
 * Device state: one libphonon_cuda context per process (9 layers, one shared
 * KV page pool); each cache owns a device stream, found through its keys
 * pointer. Weights stay resident when all four linear views of a layer carry
 * linear_data (a prepared pack, immutable per src/phonon_pack.h:153-156);
 * otherwise the layer is uploaded again on every call, matching the
 * reference, which re-expands unprepared views per call
 * (src/phonon_transformer.c:288-294).
 */
#include "phonon_cuda.h"
#include "phonon_q8.h"
#include "phonon_transformer.h"

#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define DROPIN_MAX_STREAMS 1024
#define DROPIN_POOL_PAGES 4096
#define DROPIN_MAX_BATCH 1

typedef struct {
    const void *data[8];
    int dtype[8];
    uint64_t shape0[8], shape1[8];
    size_t bytes[8];
    int immutable;
    int valid;
} LayerKey;

typedef struct CacheEntry {
    const float *keys; /* identity of the PhononKvCache */
    uint32_t stream;
    size_t written; /* highest appended position + 1 (mirror rows to upload) */
    int on_device;
    struct CacheEntry *next;
} CacheEntry;

static pthread_mutex_t g_mu = PTHREAD_MUTEX_INITIALIZER;
static int g_device = 0;
static PhononCuda *g_ctx = NULL;
static LayerKey g_loaded[PHONON_FLOW_LAYERS];
static CacheEntry *g_caches = NULL;

int phonon_transformer_cuda_set_device(int device) {
    if (device < 0)
        return 0;
    pthread_mutex_lock(&g_mu);
    int ok = g_ctx == NULL;
    if (ok)
        g_device = device;
    pthread_mutex_unlock(&g_mu);
    return ok;
}

/* ------------------------------------------------------------------ views */

static int linear_view_ok(const PhononTensorView *v, uint64_t rows, uint64_t cols) {
    if (!v || !v->data || v->rank != 2 || v->shape[0] != rows || v->shape[1] != cols)
        return 0;
    if (v->dtype == PHONON_PACK_Q8_0)
        return cols % 32 == 0 && v->byte_count == rows * cols / 32 * sizeof(PhononQ8Block);
    return v->dtype == PHONON_PACK_BF16 && v->byte_count == rows * cols * 2;
}

static int norm_view_ok(const PhononTensorView *v) {
    return v && v->data && v->rank == 1 && v->shape[0] == PHONON_FLOW_WIDTH &&
           v->dtype == PHONON_PACK_BF16 && v->byte_count == PHONON_FLOW_WIDTH * 2;
}

/* Views of one layer -> upload descriptor. The four linears must share one
 * dtype (a layer is stored as all-Q8_0 or all-bf16 on the device). */
static int layer_to_cuda(const PhononFlowLayerWeights *w, PhononCudaLayer *out, LayerKey *key) {
    if (!w || !linear_view_ok(w->qkv, 1536, 512) || !linear_view_ok(w->attention_out, 512, 512) ||
        !linear_view_ok(w->mlp_in, 2048, 512) || !linear_view_ok(w->mlp_out, 512, 2048) ||
        !norm_view_ok(w->norm1_weight) || !norm_view_ok(w->norm1_bias) ||
        !norm_view_ok(w->norm2_weight) || !norm_view_ok(w->norm2_bias))
        return 0;
    const PhononTensorView *v[8] = {w->qkv,          w->attention_out, w->mlp_in,
                                    w->mlp_out,      w->norm1_weight,  w->norm1_bias,
                                    w->norm2_weight, w->norm2_bias};
    if (v[1]->dtype != v[0]->dtype || v[2]->dtype != v[0]->dtype || v[3]->dtype != v[0]->dtype)
        return 0;
    memset(key, 0, sizeof(*key));
    key->immutable = 1;
    for (int i = 0; i < 8; i++) {
        key->data[i] = v[i]->data;
        key->dtype[i] = v[i]->dtype;
        key->shape0[i] = v[i]->shape[0];
        key->shape1[i] = v[i]->rank > 1 ? v[i]->shape[1] : 0;
        key->bytes[i] = v[i]->byte_count;
        if (i < 4 && !v[i]->linear_data)
            key->immutable = 0;
    }
    key->valid = 1;
    out->qkv = v[0]->data;
    out->attention_out = v[1]->data;
    out->mlp_in = v[2]->data;
    out->mlp_out = v[3]->data;
    out->norm1_weight = v[4]->data;
    out->norm1_bias = v[5]->data;
    out->norm2_weight = v[6]->data;
    out->norm2_bias = v[7]->data;
    out->linear_kind =
        v[0]->dtype == PHONON_PACK_Q8_0 ? PHONON_CUDA_LINEAR_Q8_0 : PHONON_CUDA_LINEAR_BF16;
    return 1;
}

static int same_key(const LayerKey *a, const LayerKey *b) {
    return a->valid && b->valid && !memcmp(a->data, b->data, sizeof(a->data)) &&
           !memcmp(a->dtype, b->dtype, sizeof(a->dtype)) &&
           !memcmp(a->shape0, b->shape0, sizeof(a->shape0)) &&
           !memcmp(a->shape1, b->shape1, sizeof(a->shape1)) &&
           !memcmp(a->bytes, b->bytes, sizeof(a->bytes));
}

/* Make device layer `slot` hold `w` (caller holds g_mu). */
static int bind_layer(size_t slot, const PhononFlowLayerWeights *w) {
    PhononCudaLayer desc;
    LayerKey key;
    if (!layer_to_cuda(w, &desc, &key))
        return 0;
    if (!g_ctx) {
        PhononCudaConfig cfg = {g_device,          PHONON_FLOW_LAYERS, DROPIN_MAX_STREAMS,
                                DROPIN_MAX_BATCH,  DROPIN_POOL_PAGES,  PHONON_CUDA_KV_F32,
                                10000.0f};
        PhononCudaLayer all[PHONON_FLOW_LAYERS];
        for (size_t l = 0; l < PHONON_FLOW_LAYERS; l++)
            all[l] = desc;
        if (phonon_cuda_create(&cfg, all, &g_ctx) != PHONON_CUDA_OK) {
            g_ctx = NULL;
            return 0;
        }
        for (size_t l = 0; l < PHONON_FLOW_LAYERS; l++)
            g_loaded[l] = key;
        return 1;
    }
    if (key.immutable && g_loaded[slot].immutable && same_key(&key, &g_loaded[slot]))
        return 1;
    g_loaded[slot].valid = 0;
    if (phonon_cuda_set_layer(g_ctx, (uint32_t)slot, &desc) != PHONON_CUDA_OK)
        return 0;
    g_loaded[slot] = key;
    return 1;
}

/* ----------------------------------------------------------------- caches */

static CacheEntry *find_cache(const PhononKvCache *cache) {
    for (CacheEntry *e = g_caches; e; e = e->next)
        if (e->keys == cache->keys)
            return e;
    return NULL;
}

static CacheEntry *track_cache(const PhononKvCache *cache) {
    CacheEntry *e = find_cache(cache);
    if (e)
        return e;
    e = calloc(1, sizeof(*e));
    if (!e)
        return NULL;
    e->keys = cache->keys;
    e->next = g_caches;
    g_caches = e;
    return e;
}

static void forget_cache(const PhononKvCache *cache) {
    for (CacheEntry **p = &g_caches; *p; p = &(*p)->next)
        if ((*p)->keys == cache->keys) {
            CacheEntry *e = *p;
            *p = e->next;
            if (e->on_device && g_ctx)
                phonon_cuda_stream_free(g_ctx, e->stream);
            free(e);
            return;
        }
}

/* Give `cache` a device stream holding its mirror rows and committed length
 * (caller holds g_mu and has bound the weights, so g_ctx exists). */
static CacheEntry *device_cache(PhononKvCache *cache) {
    CacheEntry *e = track_cache(cache);
    if (!e || !g_ctx)
        return NULL;
    if (e->on_device)
        return e;
    if (cache->capacity > PHONON_CUDA_MAX_POSITIONS ||
        phonon_cuda_stream_alloc(g_ctx, (uint32_t)cache->capacity, &e->stream) != PHONON_CUDA_OK)
        return NULL;
    e->on_device = 1;
    size_t rows = e->written > cache->length ? e->written : cache->length;
    for (size_t l = 0; l < PHONON_FLOW_LAYERS && rows; l++)
        if (phonon_cuda_kv_write(g_ctx, e->stream, (uint32_t)l, 1, 0, (uint32_t)rows,
                                 cache->keys + l * cache->capacity * PHONON_FLOW_WIDTH,
                                 cache->values + l * cache->capacity * PHONON_FLOW_WIDTH) !=
            PHONON_CUDA_OK) {
            phonon_cuda_stream_free(g_ctx, e->stream);
            e->on_device = 0;
            return NULL;
        }
    for (size_t p = 0; p < cache->length; p++)
        phonon_cuda_commit(g_ctx, e->stream, (uint32_t)p);
    return e;
}

/* Copy device rows [position, position+count) of layers [first, first+n)
 * into the host mirror. */
static int mirror_rows(PhononKvCache *cache, const CacheEntry *e, size_t first, size_t n,
                       size_t position, size_t count) {
    const size_t row = PHONON_FLOW_WIDTH;
    float *k = malloc(n * count * row * sizeof(float)), *v = malloc(n * count * row * sizeof(float));
    int ok = k && v &&
             phonon_cuda_kv_read(g_ctx, e->stream, (uint32_t)first, (uint32_t)n,
                                 (uint32_t)position, (uint32_t)count, k, v) == PHONON_CUDA_OK;
    for (size_t l = 0; ok && l < n; l++) {
        size_t dst = ((first + l) * cache->capacity + position) * row;
        memcpy(cache->keys + dst, k + l * count * row, count * row * sizeof(float));
        memcpy(cache->values + dst, v + l * count * row, count * row * sizeof(float));
    }
    free(k);
    free(v);
    return ok;
}

int phonon_kv_cache_init(PhononKvCache *cache, size_t capacity) {
    if (!cache || !capacity ||
        capacity > SIZE_MAX / (PHONON_FLOW_WIDTH * PHONON_FLOW_LAYERS * sizeof(float)))
        return 0;
    memset(cache, 0, sizeof(*cache));
    size_t count = capacity * PHONON_FLOW_WIDTH * PHONON_FLOW_LAYERS;
    cache->keys = calloc(count, sizeof(float));
    cache->values = calloc(count, sizeof(float));
    if (!cache->keys || !cache->values) {
        free(cache->keys);
        free(cache->values);
        memset(cache, 0, sizeof(*cache));
        return 0;
    }
    cache->capacity = capacity;
    return 1;
}

void phonon_kv_cache_reset(PhononKvCache *cache) {
    if (!cache)
        return;
    cache->length = 0;
    pthread_mutex_lock(&g_mu);
    CacheEntry *e = cache->keys ? find_cache(cache) : NULL;
    if (e && e->on_device && g_ctx)
        phonon_cuda_stream_reset(g_ctx, e->stream);
    pthread_mutex_unlock(&g_mu);
}

void phonon_kv_cache_destroy(PhononKvCache *cache) {
    if (!cache)
        return;
    if (cache->keys) {
        pthread_mutex_lock(&g_mu);
        forget_cache(cache);
        pthread_mutex_unlock(&g_mu);
    }
    free(cache->keys);
    free(cache->values);
    memset(cache, 0, sizeof(*cache));
}

int phonon_kv_cache_append(PhononKvCache *cache, size_t layer, size_t position, const float *key,
                           const float *value, size_t width) {
    if (!cache || !cache->keys || !cache->values || !key || !value || width != PHONON_FLOW_WIDTH ||
        layer >= PHONON_FLOW_LAYERS || position >= cache->capacity)
        return 0;
    for (size_t i = 0; i < width; ++i)
        if (!isfinite(key[i]) || !isfinite(value[i]))
            return 0;
    pthread_mutex_lock(&g_mu);
    CacheEntry *e = track_cache(cache);
    int ok = e != NULL;
    if (ok && e->on_device)
        ok = phonon_cuda_kv_write(g_ctx, e->stream, (uint32_t)layer, 1, (uint32_t)position, 1, key,
                                  value) == PHONON_CUDA_OK;
    if (ok) {
        size_t offset = (layer * cache->capacity + position) * width;
        memcpy(cache->keys + offset, key, width * sizeof(float));
        memcpy(cache->values + offset, value, width * sizeof(float));
        if (position + 1 > e->written)
            e->written = position + 1;
    }
    pthread_mutex_unlock(&g_mu);
    return ok;
}

int phonon_kv_cache_commit_position(PhononKvCache *cache, size_t position) {
    if (!cache || !cache->keys || position != cache->length || position >= cache->capacity)
        return 0;
    pthread_mutex_lock(&g_mu);
    CacheEntry *e = find_cache(cache);
    int ok = 1;
    if (e && e->on_device)
        ok = phonon_cuda_commit(g_ctx, e->stream, (uint32_t)position) == PHONON_CUDA_OK;
    pthread_mutex_unlock(&g_mu);
    if (ok)
        cache->length++;
    return ok;
}

/* -------------------------------------------------------------- primitives */

int phonon_rms_norm(const float *input, const float *weight, size_t width, float epsilon,
                    float *output) {
    if (!input || !weight || !output || !width || !(epsilon > 0.0f) || !isfinite(epsilon))
        return 0;
    return phonon_cuda_rms_norm(g_device, input, weight, width, epsilon, output) == PHONON_CUDA_OK;
}

int phonon_layer_norm(const float *input, const float *weight, const float *bias, size_t width,
                      float epsilon, float *output) {
    if (!input || !weight || !bias || !output || !width || !(epsilon > 0.0f) || !isfinite(epsilon))
        return 0;
    return phonon_cuda_layer_norm(g_device, input, weight, bias, width, epsilon, output) ==
           PHONON_CUDA_OK;
}

int phonon_erf_gelu(float *values, size_t count) {
    if (!values && count)
        return 0;
    if (!count)
        return 1;
    return phonon_cuda_erf_gelu(g_device, values, count) == PHONON_CUDA_OK;
}

int phonon_rope_interleaved(float *values, size_t width, size_t heads, size_t position,
                            float theta) {
    if (!values || !width || !heads || width % heads || (width / heads) % 2 || !(theta > 0.0f) ||
        !isfinite(theta))
        return 0;
    return phonon_cuda_rope_interleaved(g_device, values, width, heads, position, theta) ==
           PHONON_CUDA_OK;
}

/* ----------------------------------------------------------------- linears */

static int ranges_overlap(uintptr_t a, size_t a_bytes, uintptr_t b, size_t b_bytes) {
    return a < b + b_bytes && b < a + a_bytes;
}

/* Upload (per call) and apply one matrix; rows x cols Q8_0 or bf16. */
static int apply_matrix(int kind, const void *data, size_t rows, size_t cols, const float *input,
                        size_t batch, const float *bias, float *output) {
    PhononCudaLinear *lin = NULL;
    if (phonon_cuda_linear_create(g_device, kind, data, rows, cols, &lin) != PHONON_CUDA_OK)
        return 0;
    int ok = 1;
    for (size_t b0 = 0; ok && b0 < batch; b0 += 4096) {
        size_t nb = batch - b0 < 4096 ? batch - b0 : 4096;
        ok = phonon_cuda_linear_apply(lin, input + b0 * cols, nb, bias, output + b0 * rows) ==
             PHONON_CUDA_OK;
    }
    phonon_cuda_linear_destroy(lin);
    return ok;
}

int phonon_linear_batch(const PhononTensorView *weight, const float *input, size_t rows,
                        size_t columns, const float *bias, float *output, size_t batch) {
    /* Argument checks of src/phonon_transformer.c:255-281. */
    if (!weight || !weight->data || !input || !output || !rows || !columns || !batch ||
        batch > INT32_MAX || batch > SIZE_MAX / rows || batch > SIZE_MAX / columns ||
        rows > SIZE_MAX / columns || weight->rank != 2 || weight->shape[0] != rows ||
        weight->shape[1] != columns || weight->byte_count == 0)
        return 0;
    size_t elements = rows * columns;
    if (rows > INT32_MAX || columns > INT32_MAX)
        return 0;
    for (size_t i = 0; i < batch * columns; ++i)
        if (!isfinite(input[i]))
            return 0;
    int kind;
    if (weight->dtype == PHONON_PACK_Q8_0) {
        if (columns % 32 || weight->byte_count != elements / 32 * sizeof(PhononQ8Block))
            return 0;
        size_t in_bytes = batch * columns * sizeof(float), out_bytes = batch * rows * sizeof(float);
        if (ranges_overlap((uintptr_t)input, in_bytes, (uintptr_t)output, out_bytes) ||
            ranges_overlap((uintptr_t)weight->data, weight->byte_count, (uintptr_t)output,
                           out_bytes))
            return 0;
        kind = PHONON_CUDA_LINEAR_Q8_0;
    } else if (weight->dtype == PHONON_PACK_BF16 && weight->byte_count == elements * 2) {
        kind = PHONON_CUDA_LINEAR_BF16;
    } else {
        return 0;
    }
    if (bias)
        for (size_t r = 0; r < rows; ++r)
            if (!isfinite(bias[r]))
                return 0;
    return apply_matrix(kind, weight->data, rows, columns, input, batch, bias, output);
}

int phonon_linear(const PhononTensorView *weight, const float *input, size_t rows, size_t columns,
                  const float *bias, float *output) {
    return phonon_linear_batch(weight, input, rows, columns, bias, output, 1);
}

int phonon_q8_dot(const PhononQ8Block *blocks, const float *input, size_t elements, float *result) {
    if (!blocks || !input || !result || !elements || elements % 32 ||
        elements / 32 > SIZE_MAX / sizeof(*blocks) || elements > SIZE_MAX / sizeof(*input))
        return 0;
    for (size_t i = 0; i < elements; i++)
        if (!isfinite(input[i]))
            return 0;
    float out;
    if (!apply_matrix(PHONON_CUDA_LINEAR_Q8_0, blocks, 1, elements, input, 1, NULL, &out))
        return 0;
    *result = out;
    return 1;
}

int phonon_q8_matvec(const PhononQ8Block *weights, const float *input, size_t rows, size_t columns,
                     float *output) {
    /* Checks of src/phonon_q8.c:66-86. */
    if (!weights || !input || !output || !rows || !columns || columns % 32 ||
        rows > SIZE_MAX / (columns / 32) || columns > SIZE_MAX / sizeof(*input) ||
        rows > SIZE_MAX / sizeof(*output))
        return 0;
    size_t in_bytes = columns * sizeof(float), out_bytes = rows * sizeof(float);
    size_t weight_bytes = rows * (columns / 32) * sizeof(*weights);
    if (ranges_overlap((uintptr_t)input, in_bytes, (uintptr_t)output, out_bytes) ||
        ranges_overlap((uintptr_t)weights, weight_bytes, (uintptr_t)output, out_bytes))
        return 0;
    for (size_t i = 0; i < columns; i++)
        if (!isfinite(input[i]))
            return 0;
    return apply_matrix(PHONON_CUDA_LINEAR_Q8_0, weights, rows, columns, input, 1, NULL, output);
}

/* -------------------------------------------------------------- Flow stack */

int phonon_flow_layer_step(const PhononFlowLayerWeights *weights, PhononKvCache *cache,
                           size_t layer, size_t position, const float input[PHONON_FLOW_WIDTH],
                           float theta, float output[PHONON_FLOW_WIDTH]) {
    if (!weights || !cache || !cache->keys || !input || !output || layer >= PHONON_FLOW_LAYERS ||
        position >= cache->capacity || position >= 8192 || cache->length != position ||
        !(theta > 0.0f) || !isfinite(theta))
        return 0;
    pthread_mutex_lock(&g_mu);
    int ok = bind_layer(layer, weights) &&
             phonon_cuda_set_theta(g_ctx, theta) == PHONON_CUDA_OK;
    CacheEntry *e = ok ? device_cache(cache) : NULL;
    float out[PHONON_FLOW_WIDTH];
    ok = e && phonon_cuda_layer_step(g_ctx, e->stream, (uint32_t)layer, (uint32_t)position, input,
                                     out) == PHONON_CUDA_OK;
    if (e && ok) {
        if (position + 1 > e->written)
            e->written = position + 1;
        ok = mirror_rows(cache, e, layer, 1, position, 1);
    }
    pthread_mutex_unlock(&g_mu);
    if (ok)
        memcpy(output, out, sizeof(out));
    return ok;
}

int phonon_flow_stack_step_cancel(const PhononFlowLayerWeights weights[PHONON_FLOW_LAYERS],
                                  PhononKvCache *cache, size_t position,
                                  const float input[PHONON_FLOW_WIDTH], float theta,
                                  float output[PHONON_FLOW_WIDTH], PhononCancelPoll cancel,
                                  void *context) {
    if (!weights || !cache || !cache->keys || !input || !output || position != cache->length ||
        position >= cache->capacity || !(theta > 0.0f) || !isfinite(theta))
        return 0;
    pthread_mutex_lock(&g_mu);
    int ok = 1;
    for (size_t l = 0; ok && l < PHONON_FLOW_LAYERS; l++)
        ok = bind_layer(l, &weights[l]);
    ok = ok && phonon_cuda_set_theta(g_ctx, theta) == PHONON_CUDA_OK;
    CacheEntry *e = ok ? device_cache(cache) : NULL;
    float out[PHONON_FLOW_WIDTH];
    int32_t status = 0;
    uint32_t stream = e ? e->stream : 0, pos = (uint32_t)position;
    int st = e ? phonon_cuda_step(g_ctx, 1, &stream, &pos, input, out, &status,
                                  (PhononCudaCancelPoll)cancel, context)
               : PHONON_CUDA_INVALID_ARGUMENT;
    ok = st == PHONON_CUDA_OK && status == PHONON_CUDA_OK;
    if (e && st == PHONON_CUDA_CANCELLED)
        cache->length = 0;
    if (e && (ok || st == PHONON_CUDA_OK)) {
        if (position + 1 > e->written)
            e->written = position + 1;
        mirror_rows(cache, e, 0, PHONON_FLOW_LAYERS, position, 1);
    }
    pthread_mutex_unlock(&g_mu);
    if (!ok)
        return 0;
    cache->length++;
    memcpy(output, out, sizeof(out));
    return 1;
}

int phonon_flow_stack_step(const PhononFlowLayerWeights weights[PHONON_FLOW_LAYERS],
                           PhononKvCache *cache, size_t position, const float input[512],
                           float theta, float output[512]) {
    return phonon_flow_stack_step_cancel(weights, cache, position, input, theta, output, NULL,
                                         NULL);
}

int phonon_flow_stack_prefill_cancel(const PhononFlowLayerWeights weights[PHONON_FLOW_LAYERS],
                                     PhononKvCache *cache, const float *input, size_t length,
                                     float theta, float output[512], PhononCancelPoll cancel,
                                     void *context) {
    if (!weights || !cache || !cache->keys || !cache->values || !input || !output || !length ||
        length > 8192 || length > cache->capacity || cache->length || !isfinite(theta) ||
        theta <= 0.0f)
        return 0;
    for (size_t i = 0; i < length * PHONON_FLOW_WIDTH; i++)
        if (!isfinite(input[i])) {
            phonon_kv_cache_reset(cache);
            return 0;
        }
    pthread_mutex_lock(&g_mu);
    int ok = 1;
    for (size_t l = 0; ok && l < PHONON_FLOW_LAYERS; l++)
        ok = bind_layer(l, &weights[l]);
    ok = ok && phonon_cuda_set_theta(g_ctx, theta) == PHONON_CUDA_OK;
    CacheEntry *e = ok ? device_cache(cache) : NULL;
    float out[PHONON_FLOW_WIDTH];
    ok = e && phonon_cuda_append(g_ctx, e->stream, input, (uint32_t)length, out,
                                 (PhononCudaCancelPoll)cancel, context) == PHONON_CUDA_OK;
    if (ok) {
        if (length > e->written)
            e->written = length;
        ok = mirror_rows(cache, e, 0, PHONON_FLOW_LAYERS, 0, length);
    } else if (e) {
        phonon_cuda_stream_reset(g_ctx, e->stream);
    }
    pthread_mutex_unlock(&g_mu);
    if (!ok) {
        cache->length = 0;
        return 0;
    }
    cache->length = length;
    memcpy(output, out, sizeof(out));
    return 1;
}

int phonon_flow_stack_prefill(const PhononFlowLayerWeights weights[PHONON_FLOW_LAYERS],
                              PhononKvCache *cache, const float *input, size_t length, float theta,
                              float output[512]) {
    return phonon_flow_stack_prefill_cancel(weights, cache, input, length, theta, output, NULL,
                                            NULL);
}

/* ---------------------------------------------- conditioning and embeddings
 * The helpers around the stack (src/phonon_transformer.c:711-914): speaker
 * and duration conditioning, voice projection, prefix assembly, and the
 * pack-backed embeddings and output norm. They run once per request or once
 * per frame on a few hundred values, so the glue stays on the host; their
 * matrix products go through phonon_linear / phonon_linear_batch and the
 * output norm through phonon_layer_norm, i.e. onto the device. Argument
 * checks come in the reference's order; tensor names are the pack's. */

/* The engine's pack reader (src/phonon_pack.c) owns the pack; it is
 * referenced weakly so that this library also loads where no pack reader is
 * linked (every pack-backed helper then returns 0). */
#pragma weak phonon_pack_tensor

static int pack_lookup(const PhononPack *pack, const char *name, PhononTensorView *view) {
    return phonon_pack_tensor != NULL && phonon_pack_tensor(pack, name, view);
}

/* bf16 bits -> fp32; 0 if any value is non-finite (phonon_bf16_to_float,
 * src/phonon_pack.c:321-340, without the overlap check: callers here never
 * alias). */
static int widen_bf16(const uint16_t *bits, size_t count, float *out) {
    for (size_t i = 0; i < count; i++) {
        uint32_t u = (uint32_t)bits[i] << 16;
        memcpy(&out[i], &u, sizeof(float));
        if (!isfinite(out[i]))
            return 0;
    }
    return 1;
}

/* A rank-1 bf16 vector of `count` values, exactly sized. */
static int bf16_vector_view(const PhononTensorView *v, size_t count, float *out) {
    return v && v->data && v->rank == 1 && v->shape[0] == count && v->dtype == PHONON_PACK_BF16 &&
           v->byte_count == count * sizeof(uint16_t) && widen_bf16(v->data, count, out);
}

int phonon_voice_project(const float *voice_latents, size_t frames,
                         const PhononTensorView *projection, float *projected) {
    if (!voice_latents || !projection || !projected || frames == 0 || frames > 8192)
        return 0;
    return phonon_linear_batch(projection, voice_latents, PHONON_FLOW_WIDTH, PHONON_FLOW_WIDTH,
                               NULL, projected, frames);
}

int phonon_flow_condition(const PhononTensorView *speaker_embeddings,
                          const PhononTensorView *speaker_projection,
                          const PhononTensorView *duration_projection, size_t speaker_count,
                          float duration_delta, float output[PHONON_FLOW_WIDTH]) {
    enum { SPEAKER_DIM = 16, DURATION_DIM = 128 };
    const PhononTensorView *table = speaker_embeddings;
    if (!table || !table->data || !speaker_projection || !duration_projection || !output ||
        table->rank != 2 || table->shape[1] != SPEAKER_DIM || speaker_count >= table->shape[0] ||
        !isfinite(duration_delta))
        return 0;
    if (table->dtype != PHONON_PACK_BF16 ||
        table->byte_count != table->shape[0] * SPEAKER_DIM * sizeof(uint16_t))
        return 0;
    /* speaker row (bf16 widened; a non-finite entry fails in the projection) */
    float speaker_row[SPEAKER_DIM], speaker[PHONON_FLOW_WIDTH];
    const uint16_t *row = (const uint16_t *)table->data + speaker_count * SPEAKER_DIM;
    for (size_t i = 0; i < SPEAKER_DIM; i++) {
        uint32_t u = (uint32_t)row[i] << 16;
        memcpy(&speaker_row[i], &u, sizeof(float));
    }
    if (!phonon_linear(speaker_projection, speaker_row, PHONON_FLOW_WIDTH, SPEAKER_DIM, NULL,
                       speaker))
        return 0;
    /* duration: 64 cosines then 64 sines of 1000*delta / 10000^(i/63), in double */
    float duration[DURATION_DIM], duration_out[PHONON_FLOW_WIDTH];
    const double amplitude = 1000.0 * (double)duration_delta;
    for (size_t i = 0; i < DURATION_DIM / 2; i++) {
        const double angle = amplitude / pow(10000.0, (double)i / 63.0);
        duration[i] = (float)cos(angle);
        duration[DURATION_DIM / 2 + i] = (float)sin(angle);
    }
    if (!phonon_linear(duration_projection, duration, PHONON_FLOW_WIDTH, DURATION_DIM, NULL,
                       duration_out))
        return 0;
    for (size_t i = 0; i < PHONON_FLOW_WIDTH; i++) {
        output[i] = speaker[i] + duration_out[i];
        if (!isfinite(output[i]))
            return 0;
    }
    return 1;
}

int phonon_flow_prepare_prefix(const int32_t *ids, size_t tokens, const float *token_embeddings,
                               size_t prompt_id, size_t bos_id, const float *projected_voice,
                               size_t voice_frames, const float *bos_latent_projection,
                               float *prefix_embeddings) {
    if (!ids || !tokens || !token_embeddings || !projected_voice || !voice_frames ||
        !bos_latent_projection || !prefix_embeddings || tokens > 8192 || voice_frames > tokens ||
        prompt_id > INT32_MAX || bos_id > INT32_MAX)
        return 0;
    const int32_t prompt = (int32_t)prompt_id, bos = (int32_t)bos_id;
    size_t n_prompt = 0, n_bos = 0;
    for (size_t i = 0; i < tokens; i++) {
        n_prompt += ids[i] == prompt;
        n_bos += ids[i] == bos;
    }
    if (n_prompt != voice_frames || n_bos != 1)
        return 0;
    /* prompt slots take the voice frames in order, the BOS slot its latent
     * projection, every other slot its own token embedding */
    const float *next_voice = projected_voice;
    for (size_t i = 0; i < tokens; i++) {
        const float *src;
        if (ids[i] == prompt) {
            src = next_voice;
            next_voice += PHONON_FLOW_WIDTH;
        } else if (ids[i] == bos) {
            src = bos_latent_projection;
        } else {
            src = token_embeddings + i * PHONON_FLOW_WIDTH;
        }
        float *dst = prefix_embeddings + i * PHONON_FLOW_WIDTH;
        memcpy(dst, src, PHONON_FLOW_WIDTH * sizeof(float));
        for (size_t j = 0; j < PHONON_FLOW_WIDTH; j++)
            if (!isfinite(dst[j]))
                return 0;
    }
    return 1;
}

int phonon_flow_load_layers(const PhononPack *pack, PhononTensorView storage[PHONON_FLOW_LAYERS][8],
                            PhononFlowLayerWeights weights[PHONON_FLOW_LAYERS]) {
    /* Per layer, the pack's eight tensors in the order of PhononFlowLayerWeights. */
    static const char *const suffix[8] = {"self_attn.in_proj.weight", "self_attn.out_proj.weight",
                                          "linear1.weight",           "linear2.weight",
                                          "norm1.weight",             "norm1.bias",
                                          "norm2.weight",             "norm2.bias"};
    if (!pack || !storage || !weights)
        return 0;
    for (size_t layer = 0; layer < PHONON_FLOW_LAYERS; layer++) {
        const PhononTensorView **field[8] = {
            &weights[layer].qkv,          &weights[layer].attention_out, &weights[layer].mlp_in,
            &weights[layer].mlp_out,      &weights[layer].norm1_weight,  &weights[layer].norm1_bias,
            &weights[layer].norm2_weight, &weights[layer].norm2_bias};
        for (size_t k = 0; k < 8; k++) {
            char name[160];
            (void)snprintf(name, sizeof(name), "flow_lm.transformer.layers.%zu.%s", layer, suffix[k]);
            if (!pack_lookup(pack, name, &storage[layer][k]))
                return 0;
            *field[k] = &storage[layer][k];
        }
    }
    return 1;
}

int phonon_flow_embed_tokens(const PhononPack *pack, const int32_t *ids, size_t count,
                             float *embeddings) {
    PhononTensorView table;
    if (!pack || !ids || !count || !embeddings || count > 8192 ||
        !pack_lookup(pack,
                     "flow_lm.condition_provider.conditioners.transcript_in_segment.embed.weight",
                     &table) ||
        table.rank != 2 || table.shape[1] != PHONON_FLOW_WIDTH || table.dtype != PHONON_PACK_BF16 ||
        table.byte_count != table.shape[0] * PHONON_FLOW_WIDTH * sizeof(uint16_t))
        return 0;
    for (size_t i = 0; i < count; i++) {
        if (ids[i] < 0 || (uint64_t)ids[i] >= table.shape[0] ||
            !widen_bf16((const uint16_t *)table.data + (size_t)ids[i] * PHONON_FLOW_WIDTH,
                        PHONON_FLOW_WIDTH, embeddings + i * PHONON_FLOW_WIDTH))
            return 0;
    }
    return 1;
}

/* output = input_linear(latent[32]) + condition, finite. */
static int project_latent(const PhononPack *pack, const float latent[32],
                          const float condition[PHONON_FLOW_WIDTH],
                          float output[PHONON_FLOW_WIDTH]) {
    PhononTensorView projection;
    if (!pack_lookup(pack, "flow_lm.input_linear.weight", &projection) ||
        !phonon_linear(&projection, latent, PHONON_FLOW_WIDTH, 32, NULL, output))
        return 0;
    for (size_t i = 0; i < PHONON_FLOW_WIDTH; i++) {
        output[i] += condition[i];
        if (!isfinite(output[i]))
            return 0;
    }
    return 1;
}

int phonon_flow_embed_bos(const PhononPack *pack, const float condition[PHONON_FLOW_WIDTH],
                          float output[PHONON_FLOW_WIDTH]) {
    PhononTensorView bos;
    float latent[32];
    if (!pack || !condition || !output || !pack_lookup(pack, "flow_lm.bos_emb", &bos) ||
        bos.rank != 1 || bos.shape[0] != 32 || bos.dtype != PHONON_PACK_BF16 || !bos.data ||
        !widen_bf16((const uint16_t *)bos.data, 32, latent))
        return 0;
    return project_latent(pack, latent, condition, output);
}

int phonon_flow_embed_latent(const PhononPack *pack, const float latent[32],
                             const float condition[PHONON_FLOW_WIDTH],
                             float output[PHONON_FLOW_WIDTH]) {
    if (!pack || !latent || !condition || !output)
        return 0;
    return project_latent(pack, latent, condition, output);
}

int phonon_flow_normalize_latent(const PhononPack *pack, const float denormalized[32],
                                 float normalized[32]) {
    PhononTensorView mean_view, std_view;
    float mean[32], std_dev[32];
    if (!pack || !denormalized || !normalized ||
        !pack_lookup(pack, "flow_lm.emb_mean", &mean_view) ||
        !pack_lookup(pack, "flow_lm.emb_std", &std_view) ||
        !bf16_vector_view(&mean_view, 32, mean) || !bf16_vector_view(&std_view, 32, std_dev))
        return 0;
    for (size_t i = 0; i < 32; i++) {
        if (!isfinite(denormalized[i]) || !(std_dev[i] > 0.0f))
            return 0;
        normalized[i] = (denormalized[i] - mean[i]) / std_dev[i];
        if (!isfinite(normalized[i]))
            return 0;
    }
    return 1;
}

int phonon_flow_output_norm(const PhononPack *pack, float values[PHONON_FLOW_WIDTH]) {
    PhononTensorView weight_view, bias_view;
    float weight[PHONON_FLOW_WIDTH], bias[PHONON_FLOW_WIDTH], result[PHONON_FLOW_WIDTH];
    if (!pack || !values || !pack_lookup(pack, "flow_lm.out_norm.weight", &weight_view) ||
        !pack_lookup(pack, "flow_lm.out_norm.bias", &bias_view) ||
        !bf16_vector_view(&weight_view, PHONON_FLOW_WIDTH, weight) ||
        !bf16_vector_view(&bias_view, PHONON_FLOW_WIDTH, bias) ||
        !phonon_layer_norm(values, weight, bias, PHONON_FLOW_WIDTH, 1e-5f, result))
        return 0;
    memcpy(values, result, sizeof(result));
    return 1;
}
