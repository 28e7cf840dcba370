/* Driver around the UNMODIFIED speech-mac reference (oracle/_ref build).
 *
 * TEST INFRASTRUCTURE ONLY: tests, smoke() and bench.py's reference /
 * cpu_baseline arm call this through ctypes. It is linked with
 * src/phonon_transformer.c, src/phonon_q8.c and src/phonon_pack.c compiled
 * from the reference tree plus the shims in oracle/shim.
 *
 * The reference fixes PHONON_FLOW_LAYERS at 9 (src/phonon_transformer.h:11).
 * An L-layer model is run with the reference's own phonon_flow_layer_step
 * (src/phonon_transformer.c:406) over ceil(L/9) request caches: layer l uses
 * cache l/9 at layer index l%9, and every cache commits the position once all
 * layers have appended (src/phonon_transformer.c:59,478). For L == 9 this is
 * exactly phonon_flow_stack_step. */
#include "phonon_pack.h"
#include "phonon_q8.h"
#include "phonon_transformer.h"
#include "phonon_transformer_test.h"

#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define REF_MAX_LAYERS 64
#define REF_MAX_CACHES ((REF_MAX_LAYERS + PHONON_FLOW_LAYERS - 1) / PHONON_FLOW_LAYERS)

void scipy_openblas_set_num_threads64_(int);

typedef struct {
    size_t n_layers;
    PhononTensorView views[REF_MAX_LAYERS][8];
    PhononFlowLayerWeights layers[REF_MAX_LAYERS];
} RefModel;

typedef struct {
    size_t n_caches;
    PhononKvCache caches[REF_MAX_CACHES];
} RefStream;

void ref_set_blas_threads(int threads) {
    scipy_openblas_set_num_threads64_(threads);
}

static void set_linear(PhononTensorView *v, int dtype, const void *data, size_t rows, size_t cols) {
    memset(v, 0, sizeof(*v));
    v->dtype = dtype == 2 ? PHONON_PACK_BF16 : PHONON_PACK_Q8_0;
    v->rank = 2;
    v->shape[0] = rows;
    v->shape[1] = cols;
    v->data = data;
    v->byte_count = dtype == 2 ? rows * cols * 2 : rows * cols / 32 * sizeof(PhononQ8Block);
}

static void set_norm(PhononTensorView *v, const uint16_t *data) {
    memset(v, 0, sizeof(*v));
    v->dtype = PHONON_PACK_BF16;
    v->rank = 1;
    v->shape[0] = PHONON_FLOW_WIDTH;
    v->data = data;
    v->byte_count = PHONON_FLOW_WIDTH * 2;
}

/* linears: 4*L pointers (qkv, out, mlp_in, mlp_out per layer); norms: 4*L
 * bf16 vectors (norm1 w, norm1 b, norm2 w, norm2 b). dtype 1 = Q8_0, 2 = BF16. */
RefModel *ref_model_create(size_t n_layers, int dtype, const void *const *linears,
                           const uint16_t *const *norms) {
    if (!n_layers || n_layers > REF_MAX_LAYERS || !linears || !norms)
        return NULL;
    RefModel *m = calloc(1, sizeof(*m));
    if (!m)
        return NULL;
    m->n_layers = n_layers;
    static const size_t shapes[4][2] = {{1536, 512}, {512, 512}, {2048, 512}, {512, 2048}};
    for (size_t l = 0; l < n_layers; l++) {
        for (size_t i = 0; i < 4; i++)
            set_linear(&m->views[l][i], dtype, linears[4 * l + i], shapes[i][0], shapes[i][1]);
        for (size_t i = 0; i < 4; i++)
            set_norm(&m->views[l][4 + i], norms[4 * l + i]);
        PhononFlowLayerWeights *w = &m->layers[l];
        w->qkv = &m->views[l][0];
        w->attention_out = &m->views[l][1];
        w->mlp_in = &m->views[l][2];
        w->mlp_out = &m->views[l][3];
        w->norm1_weight = &m->views[l][4];
        w->norm1_bias = &m->views[l][5];
        w->norm2_weight = &m->views[l][6];
        w->norm2_bias = &m->views[l][7];
    }
    return m;
}

/* Materialise every linear to fp32 once, as phonon_pack_prepare_linears does
 * for an engine (src/phonon_pack.c:413-448, called from src/speech.c:30-61),
 * so that timed steps do not re-expand Q8 weights per call. */
int ref_model_prepare(RefModel *m) {
    if (!m)
        return 0;
    for (size_t l = 0; l < m->n_layers; l++)
        for (size_t i = 0; i < 4; i++) {
            PhononTensorView *v = &m->views[l][i];
            if (v->linear_data)
                continue;
            float *expanded = NULL;
            if (!phonon_tensor_expand_linear(v, &expanded))
                return 0;
            v->linear_data = expanded;
        }
    return 1;
}

void ref_model_destroy(RefModel *m) {
    if (!m)
        return;
    for (size_t l = 0; l < m->n_layers; l++)
        for (size_t i = 0; i < 4; i++)
            free((void *)m->views[l][i].linear_data);
    free(m);
}

RefStream *ref_stream_create(const RefModel *m, size_t capacity) {
    if (!m)
        return NULL;
    RefStream *s = calloc(1, sizeof(*s));
    if (!s)
        return NULL;
    s->n_caches = (m->n_layers + PHONON_FLOW_LAYERS - 1) / PHONON_FLOW_LAYERS;
    for (size_t c = 0; c < s->n_caches; c++)
        if (!phonon_kv_cache_init(&s->caches[c], capacity)) {
            for (size_t j = 0; j < c; j++)
                phonon_kv_cache_destroy(&s->caches[j]);
            free(s);
            return NULL;
        }
    return s;
}

void ref_stream_destroy(RefStream *s) {
    if (!s)
        return;
    for (size_t c = 0; c < s->n_caches; c++)
        phonon_kv_cache_destroy(&s->caches[c]);
    free(s);
}

size_t ref_stream_length(const RefStream *s) {
    return s ? s->caches[0].length : 0;
}

/* One layer of the reference step; does not commit. */
int ref_layer_step(const RefModel *m, RefStream *s, size_t layer, size_t position,
                   const float *input, float theta, float *output) {
    if (!m || !s || layer >= m->n_layers)
        return 0;
    return phonon_flow_layer_step(&m->layers[layer], &s->caches[layer / PHONON_FLOW_LAYERS],
                                  layer % PHONON_FLOW_LAYERS, position, input, theta, output);
}

int ref_stream_commit(RefStream *s, size_t position) {
    if (!s)
        return 0;
    for (size_t c = 0; c < s->n_caches; c++)
        if (!phonon_kv_cache_commit_position(&s->caches[c], position))
            return 0;
    return 1;
}

/* Whole L-layer step. layer_outputs (optional) receives [L][512]. */
int ref_stream_step(const RefModel *m, RefStream *s, size_t position, const float *input,
                    float theta, float *output, float *layer_outputs) {
    if (!m || !s || !input || !output)
        return 0;
    if (m->n_layers == PHONON_FLOW_LAYERS && !layer_outputs)
        return phonon_flow_stack_step(m->layers, &s->caches[0], position, input, theta, output);
    float a[PHONON_FLOW_WIDTH], b[PHONON_FLOW_WIDTH];
    memcpy(a, input, sizeof(a));
    for (size_t l = 0; l < m->n_layers; l++) {
        if (!ref_layer_step(m, s, l, position, a, theta, b))
            return 0;
        if (layer_outputs)
            memcpy(layer_outputs + l * PHONON_FLOW_WIDTH, b, sizeof(b));
        memcpy(a, b, sizeof(a));
    }
    if (!ref_stream_commit(s, position))
        return 0;
    memcpy(output, a, sizeof(a));
    return 1;
}

/* The reference's batched prefill; only for 9-layer models (one cache). */
int ref_stream_prefill(const RefModel *m, RefStream *s, const float *input, size_t length,
                       float theta, float *output) {
    if (!m || !s || m->n_layers != PHONON_FLOW_LAYERS)
        return 0;
    return phonon_flow_stack_prefill(m->layers, &s->caches[0], input, length, theta, output);
}

/* Copy K and V of (layer, position) out of the contiguous reference cache. */
int ref_stream_kv(const RefStream *s, size_t layer, size_t position, float *key, float *value) {
    if (!s || layer / PHONON_FLOW_LAYERS >= s->n_caches)
        return 0;
    const PhononKvCache *c = &s->caches[layer / PHONON_FLOW_LAYERS];
    if (position >= c->capacity)
        return 0;
    size_t offset = ((layer % PHONON_FLOW_LAYERS) * c->capacity + position) * PHONON_FLOW_WIDTH;
    memcpy(key, c->keys + offset, PHONON_FLOW_WIDTH * sizeof(float));
    memcpy(value, c->values + offset, PHONON_FLOW_WIDTH * sizeof(float));
    return 1;
}

/* Fill positions [0, length) of every layer with caller-provided K/V rows and
 * mark them committed. keys/values are [L][length][512]. Used only to give the
 * CPU baseline a long context without timing a prefill. */
int ref_stream_fill(RefStream *s, size_t n_layers, size_t length, const float *keys,
                    const float *values) {
    if (!s || !keys || !values)
        return 0;
    for (size_t l = 0; l < n_layers; l++) {
        PhononKvCache *c = &s->caches[l / PHONON_FLOW_LAYERS];
        if (length > c->capacity)
            return 0;
        size_t offset = (l % PHONON_FLOW_LAYERS) * c->capacity * PHONON_FLOW_WIDTH;
        memcpy(c->keys + offset, keys + l * length * PHONON_FLOW_WIDTH,
               length * PHONON_FLOW_WIDTH * sizeof(float));
        memcpy(c->values + offset, values + l * length * PHONON_FLOW_WIDTH,
               length * PHONON_FLOW_WIDTH * sizeof(float));
    }
    for (size_t c = 0; c < s->n_caches; c++)
        s->caches[c].length = length;
    return 1;
}

/* ---- flow head (src/phonon_sampler.c) ----
 * The head's bf16 arrays arrive in the oracle's OracleFlowHead layout and are
 * wrapped in the reference's PhononTensorView contract (bf16 rank-2 linears,
 * rank-1 vectors), then run through the reference's own functions. */
#include "phonon_oracle.h"
#include "phonon_sampler.h"

static void set_vector(PhononTensorView *v, const uint16_t *data, size_t count) {
    memset(v, 0, sizeof(*v));
    v->dtype = PHONON_PACK_BF16;
    v->rank = 1;
    v->shape[0] = count;
    v->data = data;
    v->byte_count = count * 2;
}

static void set_affine(PhononTensorView *w, PhononTensorView *b, const OracleAffine *a) {
    set_linear(w, 2, a->w.data, a->w.rows, a->w.cols);
    set_vector(b, a->b, a->w.rows);
}

static void build_head(const OracleFlowHead *in, PhononFlowHead *h) {
    memset(h, 0, sizeof(*h));
    set_affine(&h->input_weight, &h->input_bias, &in->input);
    set_affine(&h->cond_weight, &h->cond_bias, &in->cond);
    for (size_t i = 0; i < 2; i++) {
        for (size_t j = 0; j < 2; j++)
            set_affine(&h->time_weight[i][j], &h->time_bias[i][j], &in->time[i][j]);
        set_vector(&h->time_freqs[i], in->time_freqs[i], 128);
        set_vector(&h->time_alpha[i], in->time_alpha[i], 512);
    }
    for (size_t b = 0; b < PHONON_FLOW_HEAD_BLOCKS; b++) {
        set_affine(&h->block_ada_weight[b], &h->block_ada_bias[b], &in->block_ada[b]);
        set_vector(&h->block_norm_weight[b], in->block_norm_w[b], 512);
        set_vector(&h->block_norm_bias[b], in->block_norm_b[b], 512);
        for (size_t j = 0; j < 2; j++)
            set_affine(&h->block_mlp_weight[b][j], &h->block_mlp_bias[b][j], &in->block_mlp[b][j]);
    }
    set_affine(&h->final_ada_weight, &h->final_ada_bias, &in->final_ada);
    set_affine(&h->final_weight, &h->final_bias, &in->final_out);
}

int ref_flow_head_forward(const OracleFlowHead *in, const float condition[512], const float state[32],
                          float s, float t, float velocity[32]) {
    PhononFlowHead h;
    build_head(in, &h);
    return phonon_flow_head_forward(&h, condition, state, s, t, velocity);
}

int ref_flow_lsd_one_step(const OracleFlowHead *in, const float condition[512], const float raw_noise[32],
                          float temperature, float output[32]) {
    PhononFlowHead h;
    build_head(in, &h);
    return phonon_flow_lsd_one_step(&h, condition, raw_noise, temperature, output);
}
