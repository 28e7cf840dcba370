/* libphonon_cuda: B200 (sm_100a) Flow-transformer decode step behind a C ABI.
 *
 * This is the only boundary between host code and the GPU. It replaces the
 * compute of speech-mac's src/phonon_transformer.c / src/phonon_q8.c; the C17
 * drop-in (libphonon_transformer_cuda, include/phonon_transformer.h) keeps the
 * reference prototypes and calls these entry points. Plain pointers and sizes
 * only; every call returns a PhononCudaStatus and never throws.
 *
 * Model: d_model 512, 8 heads x 64, FFN 2048 (src/phonon_transformer.h:11-14),
 * pre-LayerNorm blocks with interleaved RoPE (src/phonon_transformer.c:406-453),
 * a runtime layer count (the reference fixes 9).
 *
 * KV cache: a device pool of fixed 16-position pages. A page holds the K and
 * V rows of 16 consecutive positions for every layer; each stream owns a page
 * table (position p lives in page table[p / 16], slot p % 16). Reading a
 * stream's K/V back (phonon_cuda_kv_read) returns exactly the rows the
 * reference would hold in its contiguous PhononKvCache.
 *
 * Threading: a context may be shared by threads; calls on one context are
 * serialised internally. Contexts on different devices run independently.
 */
#ifndef PHONON_CUDA_H
#define PHONON_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    PHONON_CUDA_OK = 0,
    PHONON_CUDA_INVALID_ARGUMENT = 1, /* bad pointer, size, stream id or shape */
    PHONON_CUDA_NON_FINITE = 2,       /* a non-finite input, weight or result */
    PHONON_CUDA_OUT_OF_MEMORY = 3,    /* device or pinned host allocation failed */
    PHONON_CUDA_POOL_EXHAUSTED = 4,   /* no free KV page */
    PHONON_CUDA_CAPACITY = 5,         /* position >= stream capacity or 8192 */
    PHONON_CUDA_BAD_POSITION = 6,     /* position != committed stream length */
    PHONON_CUDA_CANCELLED = 7,        /* cancel poll returned nonzero */
    PHONON_CUDA_DEVICE_ERROR = 8      /* CUDA runtime/driver error */
} PhononCudaStatus;

typedef enum { PHONON_CUDA_LINEAR_Q8_0 = 1, PHONON_CUDA_LINEAR_BF16 = 2 } PhononCudaLinearKind;
typedef enum { PHONON_CUDA_KV_F32 = 0, PHONON_CUDA_KV_BF16 = 1 } PhononCudaKvType;

#define PHONON_CUDA_WIDTH 512
#define PHONON_CUDA_PAGE_POSITIONS 16
#define PHONON_CUDA_MAX_POSITIONS 8192

typedef struct {
    int device;            /* CUDA ordinal */
    uint32_t n_layers;     /* 1..64 */
    uint32_t max_streams;  /* resident stream slots */
    uint32_t max_batch;    /* streams per step call */
    uint32_t pool_pages;   /* KV pool size in 16-position pages */
    uint32_t kv_type;      /* PhononCudaKvType */
    float theta;           /* RoPE base, 10000 in the reference */
} PhononCudaConfig;

/* One Flow layer, host memory, borrowed only while a call uploads it.
 * Linears are Q8_0 blocks (34-byte PhononQ8Block, row-major) or bf16 per
 * linear_kind: qkv [1536,512] (rows 0-511 Q, 512-1023 K, 1024-1535 V, RoPE
 * interleaved), attention_out [512,512], mlp_in [2048,512], mlp_out [512,2048]
 * (src/phonon_transformer.h:24-31). Norm vectors are bf16 [512]. */
typedef struct {
    const void *qkv, *attention_out, *mlp_in, *mlp_out;
    const uint16_t *norm1_weight, *norm1_bias, *norm2_weight, *norm2_bias;
    uint32_t linear_kind; /* PhononCudaLinearKind of the four projections */
} PhononCudaLayer;

typedef struct PhononCuda PhononCuda;
typedef int (*PhononCudaCancelPoll)(void *context);

/* Upload weights (repacked for the GEMV kernels) and allocate the KV pool and
 * step scratch. Rejects non-finite scales or norm values (the reference
 * rejects them on first use, src/phonon_pack.c:389-397, :320-325). */
int phonon_cuda_create(const PhononCudaConfig *config, const PhononCudaLayer *layers,
                       PhononCuda **out);
void phonon_cuda_destroy(PhononCuda *ctx);
/* Replace the weights of one layer in place (streams and KV are kept). */
int phonon_cuda_set_layer(PhononCuda *ctx, uint32_t layer, const PhononCudaLayer *weights);
/* Change the RoPE base for subsequent calls (the reference passes theta per call). */
int phonon_cuda_set_theta(PhononCuda *ctx, float theta);

/* Streams replace the reference's request-owned PhononKvCache
 * (src/phonon_transformer.c:16-43): alloc ~ kv_cache_init, reset ~
 * kv_cache_reset (pages return to the pool), free ~ kv_cache_destroy. */
int phonon_cuda_stream_alloc(PhononCuda *ctx, uint32_t capacity, uint32_t *stream);
int phonon_cuda_stream_reset(PhononCuda *ctx, uint32_t stream);
int phonon_cuda_stream_free(PhononCuda *ctx, uint32_t stream);
int phonon_cuda_stream_length(PhononCuda *ctx, uint32_t stream, uint32_t *length);
/* Page ids backing positions [0, n_pages*16): the KV page table of a stream. */
int phonon_cuda_stream_pages(PhononCuda *ctx, uint32_t stream, int32_t *pages, uint32_t max_pages,
                             uint32_t *n_pages);
uint32_t phonon_cuda_free_pages(PhononCuda *ctx);

/* Batched decode step (phonon_flow_stack_step_cancel, src/phonon_transformer.c:455-482,
 * for n streams at once). Host buffers x[n][512] in, y[n][512] out. Each
 * streams[i] must be at positions[i] == its committed length. status[i] gets
 * a PhononCudaStatus; a stream commits its position and has y[i] written only
 * when status[i] == OK. cancel (optional) is polled before every layer and
 * once after the last one; a nonzero poll resets every stream of the call and
 * returns PHONON_CUDA_CANCELLED without writing y. x in page-locked memory
 * (cudaHostAlloc / cudaHostRegister) is copied to the device directly, and so
 * are the rows of y (for the streams that succeeded) when y is page-locked;
 * other host memory is staged through the context's page-locked buffers. */
int phonon_cuda_step(PhononCuda *ctx, uint32_t n, const uint32_t *streams,
                     const uint32_t *positions, const float *x, float *y, int32_t *status,
                     PhononCudaCancelPoll cancel, void *cancel_context);

/* Same step with device-resident activations x_dev/y_dev ([n][512] fp32),
 * enqueued on the context's CUDA stream without waiting; commit happens at
 * phonon_cuda_sync, which also returns per-stream status. Between the two
 * calls no other call may use the context. */
int phonon_cuda_step_device(PhononCuda *ctx, uint32_t n, const uint32_t *streams,
                            const uint32_t *positions, const float *x_dev, float *y_dev);
int phonon_cuda_sync(PhononCuda *ctx, int32_t *status);
/* The context's CUDA stream (a cudaStream_t) for event timing. */
void *phonon_cuda_cuda_stream(PhononCuda *ctx);

/* One layer of one stream (phonon_flow_layer_step, src/phonon_transformer.c:406-453):
 * appends K/V at `position`, attends over position+1 keys, does not commit. */
int phonon_cuda_layer_step(PhononCuda *ctx, uint32_t stream, uint32_t layer, uint32_t position,
                           const float *x, float *y);
/* Commit `position` (phonon_kv_cache_commit_position, src/phonon_transformer.c:59-64). */
int phonon_cuda_commit(PhononCuda *ctx, uint32_t stream, uint32_t position);

/* Prefill (phonon_flow_stack_prefill_cancel, src/phonon_transformer.c:619-702):
 * run `length` rows [length][512] through the stack as consecutive positions
 * of an empty stream and commit them; last_output gets the last row's output.
 * On failure or cancel the stream is reset and last_output is untouched. */
int phonon_cuda_append(PhononCuda *ctx, uint32_t stream, const float *rows, uint32_t length,
                       float *last_output, PhononCudaCancelPoll cancel, void *cancel_context);

/* K/V rows of layers [layer_begin, layer_begin+layer_count) at positions
 * [position, position+count), as [layer_count][count][512] fp32 in the
 * reference's interleaved-RoPE order (phonon_kv_cache_append,
 * src/phonon_transformer.c:45-57). Positions in pages the stream never
 * allocated read as zeros; positions of an allocated page that were never
 * written hold unspecified values (pages are not cleared on allocation).
 * kv_write accepts only finite rows and allocates pages on first touch; it
 * does not change the length. */
int phonon_cuda_kv_read(PhononCuda *ctx, uint32_t stream, uint32_t layer_begin, uint32_t layer_count,
                        uint32_t position, uint32_t count, float *keys, float *values);
int phonon_cuda_kv_write(PhononCuda *ctx, uint32_t stream, uint32_t layer_begin,
                         uint32_t layer_count, uint32_t position, uint32_t count,
                         const float *keys, const float *values);
/* Fill positions [0, length) of every layer with seeded pseudo-random K/V on
 * the device and commit them: a synthetic context for decode benchmarks. */
int phonon_cuda_stream_fill_synthetic(PhononCuda *ctx, uint32_t stream, uint32_t length,
                                      uint64_t seed);

/* ---- standalone linear (phonon_linear_batch / phonon_q8_matvec) ---- */
typedef struct PhononCudaLinear PhononCudaLinear;
/* Upload a [rows, cols] Q8_0 or bf16 matrix (cols % 32 == 0) to `device`. */
int phonon_cuda_linear_create(int device, int kind, const void *data, size_t rows, size_t cols,
                              PhononCudaLinear **out);
void phonon_cuda_linear_destroy(PhononCudaLinear *linear);
/* y[batch][rows] = x[batch][cols] W^T (+ bias), host buffers
 * (src/phonon_transformer.c:253-313, src/phonon_q8.c:64-92). */
int phonon_cuda_linear_apply(PhononCudaLinear *linear, const float *x, size_t batch,
                             const float *bias, float *y);
/* Same on device buffers, enqueued on `cuda_stream` (a cudaStream_t, may be 0).
 * x_dev must be 16-byte aligned (rows are read four floats at a time; cudaMalloc
 * memory and whole-row offsets of it are), else PHONON_CUDA_INVALID_ARGUMENT. */
int phonon_cuda_linear_apply_device(PhononCudaLinear *linear, const float *x_dev, size_t batch,
                                    const float *bias_dev, float *y_dev, int32_t *status_dev,
                                    void *cuda_stream);
/* Allocation-free variant of phonon_cuda_linear_apply_device, for callers
 * that may not allocate device memory once they are running: a host thread
 * inside a real-time audio callback (cudaMalloc can block for milliseconds
 * and take driver locks an audio deadline cannot wait for), or an engine
 * whose device memory budget was fixed at start-up and must not grow. It has
 * no counterpart in the reference (the reference's linears are host SGEMMs,
 * src/phonon_transformer.c:253-313).
 *
 * It runs the tensor-core path: the batch is digit-sliced into a scratch
 * array that the library owns as a file-scope device array (sized for
 * PHONON_CUDA_NOALLOC_MAX_BATCH streams of up to 2048 columns, about 513 KB,
 * held by every device that loads the library until exit), then contracted
 * by the int8 tcgen05 kernel. No cudaMalloc, cudaFree or other allocating
 * routine is called. Requirements: the linear has Q8_0 weights whose
 * 32-blocks share one scale per row and 512 or 2048 columns; batch <=
 * PHONON_CUDA_NOALLOC_MAX_BATCH (else PHONON_CUDA_CAPACITY); x_dev 16-byte
 * aligned, as for phonon_cuda_linear_apply_device. The first call
 * on a device looks up the scratch address on that device; make that first
 * call before any stream capture. Every call shares the one scratch array:
 * calls that overlap on the GPU (different streams or threads without
 * ordering) race and corrupt each other's results. When a bounded wait inside
 * the tensor-core kernel expires (about two seconds; see
 * phonon_cuda_wait_expiry_probe), the rows of y_dev are not written and every
 * status_dev[b], b < batch, is set to PHONON_CUDA_DEVICE_ERROR (pass
 * status_dev to learn of it: the call itself returns before the GPU runs). */
#define PHONON_CUDA_NOALLOC_MAX_BATCH 64
int phonon_cuda_linear_apply_device_noalloc(PhononCudaLinear *linear, const float *x_dev,
                                            size_t batch, const float *bias_dev, float *y_dev,
                                            int32_t *status_dev, void *cuda_stream);
/* Bytes of the device copy (int8 plane + fp16 scales, or bf16). */
size_t phonon_cuda_linear_bytes(const PhononCudaLinear *linear);

/* ---- primitives on host buffers (src/phonon_transformer.c:66-251) ---- */
int phonon_cuda_layer_norm(int device, const float *x, const float *w, const float *b,
                           size_t width, float epsilon, float *out);
int phonon_cuda_rms_norm(int device, const float *x, const float *w, size_t width, float epsilon,
                         float *out);
int phonon_cuda_erf_gelu(int device, float *values, size_t count);
int phonon_cuda_rope_interleaved(int device, float *values, size_t width, size_t heads,
                                 size_t position, float theta);

/* ---- tensor-core contraction (diagnostic) ----
 * D[m][n] = sum_k A[m][k] * B[n][k] in exact int32 on the tcgen05 kernel the
 * batched step uses for its projections (A = int8 weight rows, B = int8 digit
 * rows). Host buffers; K must be a multiple of 128. Has no counterpart in the
 * reference, which never accumulates integers (src/phonon_q8.c:46-57 sums
 * fp32 partials); it exists so the integer accumulation can be checked
 * bit-exactly against a CPU integer product. */
int phonon_cuda_i8_gemm(int device, const int8_t *a, const int8_t *b, size_t m, size_t n, size_t k,
                        int32_t *d);

/* ---- bounded device waits (diagnostic) ----
 * Every spin-wait in the library's kernels (mbarrier waits of the tensor-core
 * and attention kernels, grid barriers of the persistent step) gives up after
 * a budget of about two seconds, raises the context's error flag and lets
 * the kernel finish; the call then returns PHONON_CUDA_DEVICE_ERROR and the
 * context stays usable. This entry point runs those wait routines with a
 * budget of budget_us microseconds on something nothing completes: kind 0,
 * an mbarrier; kind 1, a grid barrier that one CTA never reaches; kind 2,
 * an mbarrier whose expiry is reported through the error flag of the
 * allocation-free entry point's scratch, which must then reach all four
 * status words of a call as PHONON_CUDA_DEVICE_ERROR. It returns
 * PHONON_CUDA_DEVICE_ERROR when the wait expired and reported it (the
 * expected outcome), and the wall time of the wait kernel in *elapsed_ns. */
int phonon_cuda_wait_expiry_probe(int device, int kind, uint32_t budget_us, uint64_t *elapsed_ns);

/* ---- live kernel profiling (CUDA events on the context's stream) ---- */
typedef enum {
    PHONON_CUDA_K_QKV = 0,       /* LN1 + QKV GEMV + RoPE + KV append */
    PHONON_CUDA_K_ATTENTION = 1, /* split-K paged flash-decode */
    PHONON_CUDA_K_COMBINE = 2,   /* split merge */
    PHONON_CUDA_K_OUT = 3,       /* out projection + residual */
    PHONON_CUDA_K_UP = 4,        /* LN2 + FFN up + GELU */
    PHONON_CUDA_K_DOWN = 5,      /* FFN down + residual */
    PHONON_CUDA_K_OTHER = 6,     /* page-table updates, KV fills */
    PHONON_CUDA_K_FUSED = 7,     /* whole step in one persistent launch (small batches) */
    PHONON_CUDA_K_HEAD = 8,      /* frame loop: flow head, EOS, embedding, output norm */
    PHONON_CUDA_K_COUNT = 9
} PhononCudaKernelClass;
/* Enable (1) or disable (0) per-launch event timing; enabling clears the
 * totals. While enabled, every step accumulates per class: device time (ms),
 * algorithmic bytes (weights + K/V rows + activations each launch must move)
 * and launch counts. Arrays have PHONON_CUDA_K_COUNT entries. */
int phonon_cuda_profile_enable(PhononCuda *ctx, int enable);
int phonon_cuda_profile_read(PhononCuda *ctx, double *ms, double *bytes, uint64_t *launches);
/* Kernels this context has launched since creation. */
uint64_t phonon_cuda_launch_count(PhononCuda *ctx);

/* ---- step paths by batch size ----
 * A decode step (phonon_cuda_step / phonon_cuda_step_device without a cancel
 * poll) of fused_min_batch..fused_max_batch streams runs as ONE persistent
 * launch that keeps a CTA on every SM for all layers; other batches run one
 * launch per stage, with the projections on the tensor cores from
 * tensor_min_batch streams up, and from split_min_batch streams up as two
 * half batches on two CUDA streams, so that one half's attention overlaps
 * the other half's projections. Defaults: 2, 3, 4, 96 (measured on B200:
 * one stream is fastest on the per-stage GEMVs, two and three in the
 * persistent step, from four on the tensor-core projections win; halves gain
 * from about a hundred streams; the second lane exists when max_batch >= 96). A step
 * on two lanes gives the results of one lane up to rounding: each half
 * plans its attention splits on its own, so partial sums merge in another
 * order. fused_min_batch > fused_max_batch disables the
 * persistent step; fused_min_batch = 0, fused_max_batch >
 * PHONON_CUDA_FUSED_MAX_BATCH, tensor_min_batch = 0 or split_min_batch < 2
 * are PHONON_CUDA_INVALID_ARGUMENT. The persistent and per-stage GEMV paths
 * give the same results bit for bit (the tensor-core path within the
 * tolerances of the reference's tests). The persistent step needs Q8_0
 * weights, cooperative launch and enough shared memory for the batch;
 * otherwise the per-stage path runs. */
#define PHONON_CUDA_FUSED_MAX_BATCH 64
int phonon_cuda_set_batch_paths(PhononCuda *ctx, uint32_t fused_min_batch, uint32_t fused_max_batch,
                                uint32_t tensor_min_batch, uint32_t split_min_batch);

/* ---- single-stream step on one thread-block cluster ----
 * A decode step of ONE stream (phonon_cuda_step / phonon_cuda_step_device
 * without a cancel poll) at a position below max_position runs as one launch
 * of a 16-CTA cluster: the CTAs pass activations through distributed shared
 * memory and meet at hardware cluster barriers, with no kernel boundary or
 * grid-wide barrier between the ~60 dependent stages of the step. Replaces
 * phonon_flow_stack_step_cancel (src/phonon_transformer.c:455-482) for the
 * reference engine's one-request-per-thread decode loop (src/speech.c:170).
 * max_position 0 sends every batch through the paths of
 * phonon_cuda_set_batch_paths; the default is 1152 with fp32 K/V and 1248
 * with bf16 K/V: the cluster reads the stream's K/V on its 16 SMs, and past
 * those positions the per-stage path, whose attention runs on every SM, is
 * faster (measured on B200).
 * *available (optional) receives 0 when the context cannot run the path, 1
 * when it runs it with every projection on the CUDA cores (Q8_0 weights, TMA
 * K/V staging, a 16-CTA cluster resident on the device), 2 when it runs the
 * four projections on the tensor cores (every layer's weights carry one scale
 * per row). Projections and appended K/V rows equal those of the per-stage
 * path with the same arithmetic bit for bit: the GEMV path's in form 1, the
 * tensor-core path's (digit-sliced activations) in form 2. The attention
 * merges its partial sums in another order (within rounding). */
int phonon_cuda_set_cluster_step(PhononCuda *ctx, uint32_t max_position, int *available);

/* ---- per-layer output trace (test instrumentation) ----
 * trace_dev: device memory of [n_layers][max_rows][512] fp32, or NULL to
 * switch the trace off. While it is set, every decode step
 * (phonon_cuda_step, phonon_cuda_step_device) also writes each layer's output
 * rows there: row i of the batch after layer l at
 * trace_dev[(l * max_rows + i) * 512]. A step takes the same path as without
 * the trace (the per-stage path launches its kernels directly instead of
 * replaying a graph and adds one device copy per layer; the persistent and
 * cluster kernels store the rows themselves). A step of more than max_rows
 * streams is PHONON_CUDA_INVALID_ARGUMENT; max_rows must be 1..max_batch.
 * No counterpart in the reference: it lets tests compare every layer of a
 * batched step with a CPU layer step given the same input and K/V rows. */
int phonon_cuda_set_layer_trace(PhononCuda *ctx, float *trace_dev, uint32_t max_rows);

/* ---- the frame loop around the step: flow head, EOS logit, embedding,
 * output norm (src/phonon_sampler.c:280-402, src/phonon_transformer.c:860-914) ----
 * Weights are bf16 bits, host memory, borrowed only during
 * phonon_cuda_head_create. Matrices are row-major [rows][cols], biases
 * [rows]; the names are the pack tensors phonon_flow_head_load
 * (src/phonon_sampler.c:160-212) and the frame loop read. */
typedef struct {
    const uint16_t *weight, *bias;
} PhononCudaAffine;

#define PHONON_CUDA_HEAD_BLOCKS 6 /* PHONON_FLOW_HEAD_BLOCKS */
#define PHONON_CUDA_LATENT 32     /* PHONON_LATENT_WIDTH */

typedef struct {
    PhononCudaAffine input;                 /* flow_net.input_proj [512][32] */
    PhononCudaAffine cond;                  /* flow_net.cond_embed [512][512] */
    PhononCudaAffine time[2][2];            /* time_embed.{0,1}.mlp.{0,2}: [512][256], [512][512] */
    const uint16_t *time_freqs[2];          /* time_embed.{0,1}.freqs [128] */
    const uint16_t *time_alpha[2];          /* time_embed.{0,1}.mlp.3.alpha [512] */
    PhononCudaAffine block_ada[PHONON_CUDA_HEAD_BLOCKS];     /* res_blocks.i.adaLN_modulation.1 [1536][512] */
    const uint16_t *block_norm_w[PHONON_CUDA_HEAD_BLOCKS];   /* res_blocks.i.in_ln.weight [512] */
    const uint16_t *block_norm_b[PHONON_CUDA_HEAD_BLOCKS];   /* res_blocks.i.in_ln.bias [512] */
    PhononCudaAffine block_mlp[PHONON_CUDA_HEAD_BLOCKS][2];  /* res_blocks.i.mlp.{0,2} [512][512] */
    PhononCudaAffine final_ada;             /* final_layer.adaLN_modulation.1 [1024][512] */
    PhononCudaAffine final_out;             /* final_layer.linear [32][512] */
    /* The frame loop's neighbours (flow_lm.*); NULL pointers leave the head
     * usable on its own but phonon_cuda_frame_step / _output_norm refuse. */
    PhononCudaAffine eos;                   /* out_eos [1][512] */
    const uint16_t *embed;                  /* input_linear.weight [512][32], no bias */
    const uint16_t *out_norm_w, *out_norm_b;  /* out_norm.{weight,bias} [512] */
} PhononCudaHeadWeights;

typedef struct PhononCudaHead PhononCudaHead;
/* Upload a head for batches of up to the context's max_batch rows; calls
 * run on the context's stream under its lock. A non-finite weight is
 * PHONON_CUDA_NON_FINITE. Free before the context. */
int phonon_cuda_head_create(PhononCuda *ctx, const PhononCudaHeadWeights *weights, PhononCudaHead **out);
void phonon_cuda_head_free(PhononCudaHead *head);
/* Batches of at least min_batch rows (default 32) run the head's linears on
 * the tensor cores (bf16 weights times three bf16 slices of the fp32
 * activations, fp32 accumulation); smaller ones on the GEMV. *available: 1
 * when the tensor-core path could be set up. */
int phonon_cuda_head_set_tensor_min(PhononCudaHead *head, uint32_t min_batch, int *available);
/* phonon_flow_head_forward for `batch` rows (host buffers: condition
 * [batch][512], state [batch][32], velocity [batch][32]); s and t are shared.
 * PHONON_CUDA_NON_FINITE when any row fails the reference's checks (no row
 * is then written). */
int phonon_cuda_head_forward(PhononCudaHead *head, uint32_t batch, const float *condition, const float *state,
                             float s, float t, float *velocity);
/* phonon_flow_lsd_one_step for `batch` rows: output = noise*sqrt(T) +
 * head(condition, noise*sqrt(T), 0, 1), raw_noise [batch][32]. */
int phonon_cuda_lsd_one_step(PhononCudaHead *head, uint32_t batch, const float *condition, const float *raw_noise,
                             float temperature, float *output);
/* phonon_flow_eos_logit for `batch` rows of state [batch][512]. */
int phonon_cuda_eos_logit(PhononCudaHead *head, uint32_t batch, const float *state, float *logit);
/* phonon_flow_output_norm of `batch` device rows (in place allowed). */
int phonon_cuda_output_norm_device(PhononCudaHead *head, uint32_t batch, const float *x_dev, float *out_dev);
/* One frame of src/speech.c:127-172 for `batch` streams, all on the device:
 *   logit = eos(state), latent = lsd_one_step(state, raw_noise, temperature),
 *   x = input_linear(latent) + condition          (phonon_flow_embed_latent)
 *   y = decode step of x at positions[i]          (phonon_cuda_step)
 *   state = output_norm(y)                        (phonon_flow_output_norm)
 * state_dev [batch][512] (read, then overwritten with the new state) and
 * condition_dev [batch][512] are device rows; raw_noise [batch][32] is host
 * memory; eos_logit [batch] and latent [batch][32] are host outputs (the
 * frame's logit and normalized latent). status[i] as phonon_cuda_step; a row
 * whose head or embedding is non-finite gets PHONON_CUDA_NON_FINITE and its
 * stream does not advance. */
int phonon_cuda_frame_step(PhononCudaHead *head, uint32_t batch, const uint32_t *streams, const uint32_t *positions,
                           float *state_dev, const float *condition_dev, const float *raw_noise, float temperature,
                           float *eos_logit, float *latent, int32_t *status);

/* ---- Mimi latent transformer (src/phonon_mimi.c:108-283) ----
 * Each latent frame [32] of a request becomes 16 feature rows [512]: the
 * projection, the depthwise transposed-convolution upsample and two
 * transformer layers whose queries attend over at most 250 earlier rows.
 * Weights are bf16 bits, host memory, borrowed only during create; matrices
 * row-major: in_proj [1536][512], out_proj [512][512], linear1 [2048][512],
 * linear2 [512][2048], vectors [512]; the pack tensors
 * mimi.quantizer.output_proj.weight [512][32][1], mimi.upsample.convtr.convtr.weight
 * [512][1][32] and mimi.decoder_transformer.transformer.layers.{0,1}.* that
 * phonon_mimi_model_load reads. */
#define PHONON_CUDA_MIMI_MAX_FRAMES 8192 /* PHONON_MIMI_MAX_FRAMES */
typedef struct {
    const uint16_t *projection, *upsample;
    const uint16_t *in_proj[2], *out_proj[2], *linear1[2], *linear2[2];
    const uint16_t *norm1_w[2], *norm1_b[2], *norm2_w[2], *norm2_b[2];
    const uint16_t *scale1[2], *scale2[2]; /* layer_scale_1, layer_scale_2 */
} PhononCudaMimiWeights;

typedef struct PhononCudaMimi PhononCudaMimi;
/* max_states request states resident on `device`; steps of up to max_batch states. */
int phonon_cuda_mimi_create(int device, const PhononCudaMimiWeights *weights, uint32_t max_states,
                            uint32_t max_batch, PhononCudaMimi **out);
void phonon_cuda_mimi_destroy(PhononCudaMimi *mimi);
/* A request state (phonon_mimi_state_create / _reset / _destroy / _positions). */
int phonon_cuda_mimi_state_alloc(PhononCudaMimi *mimi, uint32_t *state);
int phonon_cuda_mimi_state_reset(PhononCudaMimi *mimi, uint32_t state);
int phonon_cuda_mimi_state_free(PhononCudaMimi *mimi, uint32_t state);
int phonon_cuda_mimi_positions(PhononCudaMimi *mimi, uint32_t state, uint64_t *positions);
/* One frame of each of n distinct states at once: latents [n][32] (host) ->
 * features [n][16][512] (host). status[i] is OK, or NON_FINITE when the
 * state's frame produced a non-finite value: that state is then unusable
 * until reset (calls with it return INVALID_ARGUMENT), as in the reference.
 * A non-finite latent rejects the whole call before any work. */
int phonon_cuda_mimi_step(PhononCudaMimi *mimi, uint32_t n, const uint32_t *states, const float *latents,
                          float *features, int32_t *status);
/* Steps of at least min_states states (default 4) run the four linears on
 * the tensor cores (bf16 weights times three bf16 slices of the fp32
 * activations); *available: 1 when that path could be set up. */
int phonon_cuda_mimi_set_tensor_min(PhononCudaMimi *mimi, uint32_t min_states, int *available);
/* phonon_mimi_process for one state: frames latents [frames][32] ->
 * features [frames * 16][512], capacity in feature rows. */
int phonon_cuda_mimi_process(PhononCudaMimi *mimi, uint32_t state, const float *latents, size_t frames,
                             float *features, size_t capacity);

const char *phonon_cuda_status_string(int status);

#ifdef __cplusplus
}
#endif
#endif
