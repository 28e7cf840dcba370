/* CPU oracle for the Flow-transformer decode step: a plain-C restatement of
 * the speech-mac reference algorithm (src/phonon_transformer.c, src/phonon_q8.c,
 * src/phonon_pack.c) for any number of layers.
 *
 * TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference arm of bench.py may load this library, and only as
 * the checker. The CUDA product path never links or calls it.
 *
 * All entry points return 1 on success and 0 on failure, like the reference.
 * Linear layers use a sequential fp32 dot product where the reference calls
 * cblas_sgemm; every other routine follows the reference's operation order.
 */
#ifndef PHONON_ORACLE_H
#define PHONON_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#define ORACLE_WIDTH 512
#define ORACLE_HEADS 8
#define ORACLE_HEAD_WIDTH 64
#define ORACLE_FFN 2048
#define ORACLE_MAX_POSITIONS 8192

/* Linear storage kinds (reference PhononPackDType values). */
#define ORACLE_Q8_0 1
#define ORACLE_BF16 2

typedef struct {
    int dtype;
    size_t rows, cols;
    const void *data; /* Q8_0: rows*cols/32 34-byte blocks; BF16: rows*cols u16 */
} OracleLinear;

typedef struct {
    OracleLinear qkv, out, up, down;
    const uint16_t *norm1_w, *norm1_b, *norm2_w, *norm2_b; /* bf16 [512] */
} OracleLayer;

typedef struct {
    size_t n_layers, capacity, length;
    float *keys, *values; /* [layer][capacity][512], interleaved-RoPE order */
    int kv_bf16;          /* 1: K/V rows are rounded to bf16 (nearest-even) on append */
} OracleCache;

float oracle_half_to_float(uint16_t bits);
int oracle_q8_dot(const void *blocks, const float *input, size_t elements, float *result);
int oracle_q8_matvec(const void *weights, const float *input, size_t rows, size_t columns,
                     float *output);
int oracle_linear_batch(const OracleLinear *w, const float *input, size_t batch, const float *bias,
                        float *output);
int oracle_layer_norm(const float *input, const float *weight, const float *bias, size_t width,
                      float epsilon, float *output);
int oracle_rms_norm(const float *input, const float *weight, size_t width, float epsilon,
                    float *output);
int oracle_erf_gelu(float *values, size_t count);
int oracle_rope_interleaved(float *values, size_t width, size_t heads, size_t position,
                            float theta);
int oracle_attention(const float query[64], const float *keys, const float *values, size_t count,
                     size_t stride, float output[64]);

int oracle_cache_init(OracleCache *cache, size_t n_layers, size_t capacity);
void oracle_cache_destroy(OracleCache *cache);
int oracle_layer_step(const OracleLayer *w, OracleCache *cache, size_t layer, size_t position,
                      const float *input, float theta, float *output);
/* The layer step with the K/V row at `position` taken from the cache as the
 * caller left it; the rows the step computes go to k_out / v_out (test hook). */
int oracle_layer_step_forced(const OracleLayer *w, OracleCache *cache, size_t layer,
                             size_t position, const float *input, float theta, float *output,
                             float *k_out, float *v_out);
/* Full step over n_layers; layer_outputs (optional) receives [n_layers][512]. */
int oracle_stack_step(const OracleLayer *layers, size_t n_layers, OracleCache *cache,
                      size_t position, const float *input, float theta, float *output,
                      float *layer_outputs);

/* ---- flow head (src/phonon_sampler.h:48-75): bf16 linears with bf16 biases ---- */
#define ORACLE_HEAD_BLOCKS 6

typedef struct {
    OracleLinear w;     /* ORACLE_BF16 [rows, cols] */
    const uint16_t *b;  /* bf16 [rows] */
} OracleAffine;

typedef struct {
    OracleAffine input;                   /* [512, 32] latent state in */
    OracleAffine cond;                    /* [512, 512] condition in */
    OracleAffine time[2][2];              /* per flow time: [512, 256], [512, 512] */
    const uint16_t *time_freqs[2];        /* bf16 [128] */
    const uint16_t *time_alpha[2];        /* bf16 [512] */
    OracleAffine block_ada[ORACLE_HEAD_BLOCKS];      /* [1536, 512]: shift, scale, gate */
    const uint16_t *block_norm_w[ORACLE_HEAD_BLOCKS];  /* bf16 [512] */
    const uint16_t *block_norm_b[ORACLE_HEAD_BLOCKS];
    OracleAffine block_mlp[ORACLE_HEAD_BLOCKS][2];   /* [512, 512] x 2 */
    OracleAffine final_ada;               /* [1024, 512]: shift, scale */
    OracleAffine final_out;               /* [32, 512] velocity out */
} OracleFlowHead;

/* phonon_flow_head_forward (src/phonon_sampler.c:307-364): velocity of the
 * flow at state for times s, t, conditioned on a transformer output row. */
int oracle_flow_head_forward(const OracleFlowHead *head, const float condition[512],
                             const float state[32], float s, float t, float velocity[32]);
/* phonon_flow_lsd_one_step (src/phonon_sampler.c:366-393). */
int oracle_flow_lsd_one_step(const OracleFlowHead *head, const float condition[512],
                             const float raw_noise[32], float temperature, float output[32]);

/* ---- Mimi latent transformer (src/phonon_mimi.c): bf16 weights, no biases ---- */
typedef struct {
    OracleLinear projection;                 /* [512, 32] mimi.quantizer.output_proj */
    const uint16_t *upsample;                /* [512][32] depthwise transposed-conv kernel */
    OracleLinear in_proj[2], out_proj[2];    /* [1536, 512], [512, 512] */
    OracleLinear linear1[2], linear2[2];     /* [2048, 512], [512, 2048] */
    const uint16_t *norm1_w[2], *norm1_b[2], *norm2_w[2], *norm2_b[2];  /* bf16 [512] */
    const uint16_t *scale1[2], *scale2[2];   /* layer scales, bf16 [512] */
    float rope_theta;
} OracleMimi;

typedef struct {
    size_t position;
    int failed;
    float previous[512];
    float *keys, *values; /* [2][250][512] ring */
} OracleMimiState;

int oracle_mimi_state_init(OracleMimiState *state);
void oracle_mimi_state_free(OracleMimiState *state);
void oracle_mimi_state_reset(OracleMimiState *state);
int oracle_mimi_upsample_frame(const uint16_t *weight, const float *input, const float *previous,
                               size_t channels, size_t stride, float *output);
/* latents [frames][32] -> features [frames * 16][512] (src/phonon_mimi.c:246-283). */
int oracle_mimi_process(const OracleMimi *model, OracleMimiState *state, const float *latents,
                        size_t frames, float *features);

#endif
