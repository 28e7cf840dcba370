// Device code of libphonon_cuda (sm_100a).
//
// Kernels of one Flow layer step, in launch order:
//   gemv_kernel<LN, EPI_QKV>   LN1 -> [q|k|v] = xn Wqkv^T -> RoPE(q,k) -> q to scratch,
//                              k/v appended to the stream's KV page
//   attn_tma_kernel            split-K flash-decode over 16-position pages
//   gemv_kernel<MERGE, RESID>  merge the splits of each (stream, head), then
//                              h = x + attn Wout^T
//   gemv_kernel<LN, EPI_GELU>  g = GELU(LN2(h) Wup^T)
//   gemv_kernel<-, EPI_RESID>  x' = h + g Wdown^T
//
// Numerics follow speech-mac src/phonon_transformer.c. LayerNorm reproduces
// the reference's Welford cascade bit for bit; RoPE uses the reference's fp32
// frequencies and phases; GELU uses the same A&S erf polynomial. Linear and
// attention reductions run in a GPU order (fp32 accumulate).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

namespace phonon {

constexpr int kWidth = 512;
constexpr int kHeads = 8;
constexpr int kHeadDim = 64;
constexpr int kFfn = 2048;
constexpr int kPage = 16;
constexpr int kGemvWarps = 8;      // warps per GEMV CTA
constexpr int kRowsPerWarp = 2;    // a RoPE pair (2i, 2i+1) stays in one warp
constexpr int kAttnWarps = 4;      // warps per attention CTA
constexpr unsigned kFull = 0xffffffffu;
constexpr int kStatusNonFinite = 2;  // PHONON_CUDA_NON_FINITE

// EPI_SILU: y = silu(acc + bias); EPI_GATE: y = res + gate * (acc + bias)
// (the flow head's MLP, src/phonon_sampler.c:333-345).
enum Epilogue : int { EPI_STORE = 0, EPI_RESID = 1, EPI_GELU = 2, EPI_QKV = 3, EPI_SILU = 4, EPI_GATE = 5 };
// Where a GEMV's activation rows come from: x as is, LayerNorm(x), or the
// merge of the step's attention split partials (the attention output).
// SRC_HEADLN: the flow head's block LayerNorm with its modulation
// (head_ln_modulate) of each x row, in place of a head_block_kernel launch.
enum GemvSource : int { SRC_X = 0, SRC_LN = 1, SRC_MERGE = 2, SRC_HEADLN = 3 };

// Programmatic dependent launch: kernels of a step are launched so that the
// next one may start while this one drains. pdl_wait() blocks until the
// previous kernel of the stream has completed and its writes are visible
// (call it before touching anything it produced); pdl_trigger() lets the
// next kernel begin launching. Both are no-ops without the launch attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float bf16_to_f32(uint16_t b) {
    return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return static_cast<uint16_t>(u >> 16);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}

// x / (1 + e^-x) (src/phonon_math.c:18-28; CUDA's expf where the reference
// calls SLEEF's u10 exp: both within ~1 ulp of e^-x).
__device__ __forceinline__ float silu_f(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x))); }

__device__ __forceinline__ void flag_nonfinite(int32_t* status, int b) {
    if (status) atomicOr(status + b, kStatusNonFinite);
}

// ------------------------------------------------------------------ LayerNorm
// Merge a block (a_mean, a_m2) into (mean, m2) holding n samples, in the
// reference's unfused order: mean += c*delta; m2 += a_m2 + delta*delta*c*n
// with c = added / (n + added) (src/phonon_transformer.c:90-98). The cascade
// below only ever merges equal halves or into an empty level, so c is 1, 1/2
// or 0 (nothing into nothing) and exact.
__device__ __forceinline__ void ln_merge(float a_mean, float a_m2, float& mean, float& m2, float c, float n) {
    const float delta = __fsub_rn(a_mean, mean);
    mean = __fadd_rn(mean, __fmul_rn(c, delta));
    m2 = __fadd_rn(m2, __fadd_rn(a_m2, __fmul_rn(__fmul_rn(__fmul_rn(delta, delta), c), n)));
}

// One level of the chunk tree: lanes whose chunk index differs in the bit
// `mask` (a lane bit: chunk = lane >> 2) merge their blocks; the lower
// chunk is the accumulator holding n samples, the higher one is added with
// c = 1/2 (equal halves), i.e. ln_merge(higher, lower, 1/2, n). Both lanes
// of a pair compute the same operation on the same operands.
__device__ __forceinline__ void ln_tree_level(float& mean, float& m2, int mask, float n) {
    const int lane = threadIdx.x & 31;
    const float om = __shfl_xor_sync(kFull, mean, mask), oq = __shfl_xor_sync(kFull, m2, mask);
    const bool low = (lane & mask) == 0;
    float lm = low ? mean : om, lq = low ? m2 : oq;
    ln_merge(low ? om : mean, low ? oq : m2, lm, lq, 0.5f, n);
    mean = lm;
    m2 = lq;
}

// Moments of one 512-wide row held by a warp, lane (chunk*4 + l) holding
// elements chunk*64 + j*4 + l (j = 0..15), as the reference's moments_512
// (src/phonon_transformer.c:99-151): a 16-step Welford per lane; then, for
// each l, the reference folds the 8 chunk results (16 samples each) through
// the three levels of a binary counter (after chunk ch, level 0 carries into
// level 1 when bit 0 of ch + 1 is clear, level 1 into level 2 when bits 0-1
// are; a block carried onto an empty level is copied exactly, and the final
// folds of the empty levels 0 and 1 are exact too), which is a balanced
// tree: ((c0 c1)(c2 c3))((c4 c5)(c6 c7)), every node the merge of two equal
// halves with the earlier one as accumulator. Here the tree runs across
// lanes, one shuffle level per tree level, with the reference's operations
// at every node; then the four lanes l are merged in order. Returns the
// mean and 1/sqrt(var + eps).
__device__ __forceinline__ void ln_moments512(const float (&v)[16], float eps, float& mu_out, float& scale_out) {
    constexpr float kRecip[16] = {1.0f / 1,  1.0f / 2,  1.0f / 3,  1.0f / 4,  1.0f / 5,  1.0f / 6,
                                  1.0f / 7,  1.0f / 8,  1.0f / 9,  1.0f / 10, 1.0f / 11, 1.0f / 12,
                                  1.0f / 13, 1.0f / 14, 1.0f / 15, 1.0f / 16};
    float mean = 0.0f, m2 = 0.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const float delta = __fsub_rn(v[j], mean);
        mean = __fadd_rn(mean, __fmul_rn(delta, kRecip[j]));
        m2 = __fadd_rn(m2, __fmul_rn(delta, __fsub_rn(v[j], mean)));
    }
    ln_tree_level(mean, m2, 4, 16.0f);   // chunk pairs (16 + 16)
    ln_tree_level(mean, m2, 8, 32.0f);   // pairs of pairs (32 + 32)
    ln_tree_level(mean, m2, 16, 64.0f);  // halves (64 + 64)
    // four-lane merge, 128 samples each: c = 1, 1/2, 1/3, 1/4
    float mu = 0.0f, q = 0.0f;
    constexpr float kC[4] = {128.0f / 128.0f, 128.0f / 256.0f, 128.0f / 384.0f, 128.0f / 512.0f};
    constexpr float kN[4] = {0.0f, 128.0f, 256.0f, 384.0f};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float lm = __shfl_sync(kFull, mean, k), lq = __shfl_sync(kFull, m2, k);
        const float delta = __fsub_rn(lm, mu);
        mu = __fmaf_rn(kC[k], delta, mu);
        q = __fadd_rn(q, __fmaf_rn(__fmul_rn(__fmul_rn(delta, delta), kC[k]), kN[k], lq));
    }
    const float var = __fmul_rn(q, 1.0f / 512.0f);  // == q / 512 exactly (power of two)
    mu_out = mu;
    scale_out = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
}

// One warp normalises one 512-wide row: out = ((x - mean) * rstd) * w + b with
// the moments of ln_moments512 and the reference's affine step
// (src/phonon_transformer.c:178-183). x is read once; each lane applies the
// affine step to the elements it holds. Returns false (on every lane) if an
// input, weight, bias or output is non-finite. kL2: read x through L2 only
// (rows that other CTAs of a running kernel wrote). kChunk: floats from one
// 64-element chunk of x, w, b and out to the next (64: plain rows; 68: the
// padded shared-memory rows of the cluster step, where the lanes' strided
// accesses fall into 32 different banks).
template <bool kL2 = false>
__device__ __forceinline__ float ln_load(const float* p) {
    if constexpr (kL2) return __ldcg(p);
    return *p;
}

template <bool kL2 = false, int kChunk = 64>
__device__ __forceinline__ bool warp_layernorm512(const float* __restrict__ x,
                                                  const float* __restrict__ w,
                                                  const float* __restrict__ b,
                                                  float* __restrict__ out,
                                                  float eps = 1e-5f) {
    const int lane = threadIdx.x & 31;
    const int base = (lane >> 2) * kChunk + (lane & 3);
    float v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = ln_load<kL2>(x + base + j * 4);
    bool ok = true;
#pragma unroll
    for (int j = 0; j < 16; ++j) ok &= isfinite(v[j]);
    float mu, scale;
    ln_moments512(v, eps, mu, scale);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int i = base + j * 4;
        const float wi = w[i], bi = b[i];
        ok &= isfinite(wi) && isfinite(bi);
        // The reference centres in double and rounds once to float; for fp32
        // operands that equals the fp32 subtraction bit for bit (binary64 has
        // 53 >= 2*24 + 2 bits, so rounding twice is innocuous for +, -).
        const float centered = __fsub_rn(v[j], mu);
        float y = __fadd_rn(__fmul_rn(__fmul_rn(centered, scale), wi), bi);
        ok &= isfinite(y);
        out[i] = y;
    }
    return __all_sync(kFull, ok);
}

// ----------------------------------------------------------------------- GELU
// 0.5*x*(1+erf(x/sqrt2)) with the A&S 7.1.26 erf in the reference's fused
// order (src/phonon_transformer.c:190-200, :209-211). exp(-x^2) is evaluated
// in double and rounded once, which is the correctly rounded fp32 exp.
__device__ __forceinline__ float gelu_erf(float v) {
    const float x = __fmul_rn(v, 0.7071067811865475244f);
    const float t = __fdiv_rn(1.0f, __fmaf_rn(0.3275911f, fabsf(x), 1.0f));
    float r = __fmaf_rn(1.061405429f, t, -1.453152027f);
    r = __fmaf_rn(r, t, 1.421413741f);
    r = __fmaf_rn(r, t, -0.284496736f);
    r = __fmaf_rn(r, t, 0.254829592f);
    const float sq = __fmul_rn(x, x);
    const float neg_exp = -__double2float_rn(exp(-static_cast<double>(sq)));
    const float e = copysignf(__fmaf_rn(__fmul_rn(t, neg_exp), r, 1.0f), x);
    return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, e));
}

// ---------------------------------------------------------------------- RoPE
// Rotate pair (a, b) = (x[2i], x[2i+1]) by position * freq[i]; phases in
// fp32 like the reference (src/phonon_transformer.c:229-244), cos/sin
// evaluated in double and rounded once.
__device__ __forceinline__ void rope_pair(float& a, float& b, int position, float freq) {
    const float phase = __fmul_rn(static_cast<float>(position), freq);
    double sd, cd;
    sincos(static_cast<double>(phase), &sd, &cd);
    const float c = __double2float_rn(cd), s = __double2float_rn(sd);
    const float ra = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    const float rb = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
    a = ra;
    b = rb;
}

// Rotate with a precomputed (cos, sin) of the pair's phase.
__device__ __forceinline__ void rope_apply(float& a, float& b, float2 cs) {
    const float ra = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
    const float rb = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
    a = ra;
    b = rb;
}

// Start of a step: apply the page-table updates ((slot, index, page)
// triples) and build the step's RoPE table, cs[e][i] = (cos, sin) of
// pos[e] * freq[i] for the 32 frequencies of a 64-wide head (every layer of
// the step reuses it).
__global__ void step_prep_kernel(const int32_t* pos, const float* freq, int R, float2* cs, int32_t* table,
                                 int max_pages, const int32_t* updates, int U, int32_t* counters, int n_counters) {
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t < n_counters) counters[t] = 0;
    if (t < U) table[static_cast<size_t>(updates[3 * t]) * max_pages + updates[3 * t + 1]] = updates[3 * t + 2];
    if (t >= R * 32) return;
    const float phase = __fmul_rn(static_cast<float>(pos[t >> 5]), freq[t & 31]);
    double sd, cd;
    sincos(static_cast<double>(phase), &sd, &cd);
    cs[t] = make_float2(__double2float_rn(cd), __double2float_rn(sd));
}

// ----------------------------------------------------------------- KV pages
// A page holds 16 positions of every layer. The pool is layer-major:
// [layer][page][k|v][head][slot][dim], so the K/V blocks one layer's
// attention reads are the pool's pages in a contiguous range of memory (a
// page-major pool, [page][layer][...], spaces them n_layers blocks apart,
// and a bare TMA page ring measured ~7 % less DRAM bandwidth on that stride).
struct KvView {
    void* pool;
    int pool_pages;         // pages per layer
    int bf16;               // 1: bf16 elements, 0: fp32
    const int32_t* table;   // [stream slot][max_pages]
    int max_pages;
};

__device__ __forceinline__ long long kv_offset(const KvView& kv, int page, int layer, int which,
                                               int head, int slot) {
    return ((static_cast<long long>(layer) * kv.pool_pages + page) * 2 + which) * (kHeads * kPage * kHeadDim) +
           (head * kPage + slot) * kHeadDim;
}

__device__ __forceinline__ void kv_store2(const KvView& kv, long long off, float a, float b) {
    if (kv.bf16) {
        uint32_t packed = static_cast<uint32_t>(f32_to_bf16(a)) |
                          (static_cast<uint32_t>(f32_to_bf16(b)) << 16);
        *reinterpret_cast<uint32_t*>(static_cast<uint16_t*>(kv.pool) + off) = packed;
    } else {
        *reinterpret_cast<float2*>(static_cast<float*>(kv.pool) + off) = make_float2(a, b);
    }
}

// Attention split partials: per (split, head) the running max, the sum of
// exponentials and the 64 accumulated output dims.
constexpr int kPartStride = 2 + kHeadDim;

// Split merge, one step: fold the partial (pm, pl, pa) of the next split (in
// page order) into the running (M, S, A): M' = max(M, pm), S' = S e^(M-M') +
// pl e^(pm-M'), A' = A e^(M-M') + pa e^(pm-M'); the merged head output is
// A / S. All merge paths (per-stage, tensor-core and persistent) use it.
struct MergeWeights {
    float alpha, beta;
};

__device__ __forceinline__ MergeWeights merge_weights(float& M, float pm) {
    const float M2 = fmaxf(M, pm);
    MergeWeights w;
    w.alpha = M == -INFINITY ? 0.0f : expf(M - M2);
    w.beta = pm == -INFINITY ? 0.0f : expf(pm - M2);
    M = M2;
    return w;
}

__device__ __forceinline__ float merge_fold(float acc, MergeWeights w, float v) { return fmaf(acc, w.alpha, w.beta * v); }

// --------------------------------------------------------------------- GEMV
// Device weight layout ("lane-interleaved", cols a multiple of 512): in row r,
// the 16 bytes at r*cols + c*512 + lane*16 hold the int8 weights of logical
// columns c*512 + j*128 + lane*4 + e (byte j*4 + e), so one 16-byte load per
// lane feeds four float4 reads of x from shared memory without bank
// conflicts. Q8_0 scales: r*(cols/32) + c*16 + g*4 + j holds the binary16
// scale of block c*16 + j*4 + g, so lane l reads its four scales
// (g = l/8) as one 8-byte load. bf16 weights use the same column order.
// Mean of a 512-wide row in the order of src/phonon_sampler.c:229-248 (the
// reference's restatement of PyTorch's SumKernel): element
// e = chunk*256 + group*16 + v*4 + l; each (chunk, v, l) sums its 16 groups
// from zero in order, the two chunks are added into a zeroed accumulator,
// the vectors v = 1..3 are added to v = 0 in order, and the four lanes are
// summed from zero. Lane (chunk*16 + v*4 + l) owns one chain; every lane
// returns the mean. `row` may be shared or global memory.
__device__ __forceinline__ float head_mean512(const float* row) {
    const int lane = threadIdx.x & 31;
    float p = 0.0f;
#pragma unroll
    for (int g = 0; g < 16; ++g) p = __fadd_rn(p, row[(lane >> 4) * 256 + g * 16 + (lane & 15)]);
    const float p1 = __shfl_down_sync(kFull, p, 16);          // chunk 1 of the same (v, l)
    const float s = __fadd_rn(__fadd_rn(0.0f, p), p1);        // sums[v][l], lanes 0..15
    const int l = lane & 3;
    const float s1 = __shfl_sync(kFull, s, 4 + l), s2 = __shfl_sync(kFull, s, 8 + l),
                s3 = __shfl_sync(kFull, s, 12 + l);
    const float f = __fadd_rn(__fadd_rn(__fadd_rn(s, s1), s2), s3);  // sums[0][l], lanes 0..3
    float sum = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) sum = __fadd_rn(sum, __shfl_sync(kFull, f, k));
    return __fmul_rn(sum, 1.0f / 512.0f);  // == sum / 512 (power of two)
}

// The head's LayerNorm (src/phonon_sampler.c:250-278) of a 512-wide row in
// shared memory, by one warp: float mean (head_mean512), variance from the
// double sum of centred squares rounded once to float, eps 1e-6, optional
// affine, then the adaLN modulation out = h * (1 + scale) + shift. Lane i
// writes elements i + 32k. Returns false on every lane if an input, weight,
// bias or result is non-finite.
__device__ __forceinline__ bool head_ln_modulate(const float* x, const float* w, const float* b, const float* shift,
                                                 const float* scale, float* out) {
    const int lane = threadIdx.x & 31;
    // every operand loaded up front (independent loads, no load behind a
    // branch on an earlier one)
    float xv[16], wv[16], bv[16], sc[16], sh[16];
    const bool hw = w != nullptr, hb = b != nullptr;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const int i = lane + 32 * k;
        xv[k] = x[i];
        wv[k] = hw ? w[i] : 1.0f;
        bv[k] = hb ? b[i] : 0.0f;
        sc[k] = scale[i];
        sh[k] = shift[i];
    }
    bool ok = true;
#pragma unroll
    for (int k = 0; k < 16; ++k) ok &= isfinite(xv[k]) & isfinite(wv[k]) & isfinite(bv[k]);
    ok = __all_sync(kFull, ok);
    const float mean = head_mean512(x);
    double sq = 0.0;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const double c = __dsub_rn(static_cast<double>(xv[k]), static_cast<double>(mean));
        sq = __dadd_rn(sq, __dmul_rn(c, c));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(kFull, sq, o);
    const float variance = static_cast<float>(sq / 512.0);
    const float inverse = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(variance, 1e-6f)));
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        float n = __fmul_rn(__fsub_rn(xv[k], mean), inverse);
        if (hw) n = __fmul_rn(n, wv[k]);
        if (hb) n = __fadd_rn(n, bv[k]);
        ok &= isfinite(n);
        out[lane + 32 * k] = __fadd_rn(__fmul_rn(n, __fadd_rn(1.0f, sc[k])), sh[k]);
    }
    return __all_sync(kFull, ok);
}

struct GemvParams {
    const void* w;            // int8 plane (Q8_0) or bf16 plane
    const __half* scales;     // Q8_0 only
    int rows, cols;
    const float* x;           // [B][ldx]
    int ldx, B;
    const float* ln_w;        // SRC_LN, SRC_HEADLN: LayerNorm weight and bias (fp32 [512])
    const float* ln_b;
    const float* mod;         // SRC_HEADLN: row b's shift at mod + b * ldmod, its scale 512 floats on
    int ldmod;
    const float* part;        // SRC_MERGE: split partials [S][8][66] ...
    const int32_t* first;     // ... and each stream's first split and split count
    const int32_t* count;
    const float* bias;        // EPI_STORE (optional), EPI_SILU, EPI_GATE
    const float* gate;        // EPI_GATE: [B][ldgate]
    int ldgate;
    float* y;                 // output [B][ldy]
    int ldy;
    const float* res;         // EPI_RESID residual [B][ldres]
    int ldres;
    // EPI_QKV
    float* q;                 // [B][512]
    const int32_t* slot;      // [B] stream slot
    const int32_t* pos;       // [B] position
    const float2* rope;       // [B][32] per-step (cos, sin)
    KvView kv;
    int layer;
    int32_t* status;          // [B]
    int b_per_cta;            // streams per CTA along grid.y (a multiple of the tile), 0: all
};

template <bool kQ8, int kChunks, int kBT, int kSrc, int kEpi>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_kernel(GemvParams p) {
    constexpr bool kLN = kSrc == SRC_LN;
    extern __shared__ __align__(16) float xs[];  // [kBT][kChunks * 512]
    __shared__ int ln_bad[kBT];
    constexpr int cols = kChunks * 512;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = (blockIdx.x * kGemvWarps + warp) * kRowsPerWarp;
    const bool active = row0 < p.rows;

    // Weights for this warp's two rows live in registers for the whole call.
    uint4 wq[kRowsPerWarp][kChunks][kQ8 ? 1 : 2];
    float sc[kRowsPerWarp][kChunks][4];
    if (active) {
#pragma unroll
        for (int rr = 0; rr < kRowsPerWarp; ++rr) {
            const int r = min(row0 + rr, p.rows - 1);
#pragma unroll
            for (int c = 0; c < kChunks; ++c) {
                if constexpr (kQ8) {
                    const uint8_t* base = static_cast<const uint8_t*>(p.w) +
                                          static_cast<size_t>(r) * cols + c * 512 + lane * 16;
                    wq[rr][c][0] = __ldg(reinterpret_cast<const uint4*>(base));
                    const __half* sb = p.scales + static_cast<size_t>(r) * (cols / 32) + c * 16 +
                                       (lane >> 3) * 4;
                    uint2 raw = __ldg(reinterpret_cast<const uint2*>(sb));
                    __half2 h01 = *reinterpret_cast<__half2*>(&raw.x);
                    __half2 h23 = *reinterpret_cast<__half2*>(&raw.y);
                    sc[rr][c][0] = __low2float(h01);
                    sc[rr][c][1] = __high2float(h01);
                    sc[rr][c][2] = __low2float(h23);
                    sc[rr][c][3] = __high2float(h23);
                } else {
                    const uint16_t* base = static_cast<const uint16_t*>(p.w) +
                                           static_cast<size_t>(r) * cols + c * 512 + lane * 16;
                    wq[rr][c][0] = __ldg(reinterpret_cast<const uint4*>(base));
                    wq[rr][c][1] = __ldg(reinterpret_cast<const uint4*>(base + 8));
#pragma unroll
                    for (int j = 0; j < 4; ++j) sc[rr][c][j] = 1.0f;
                }
            }
        }
    }

    pdl_wait();  // weights above are independent of the previous kernel
    // Streams [b_begin, b_end) of this CTA: blockIdx.y picks a slice of the
    // batch when the launch splits it (p.b_per_cta > 0) so that a matrix of
    // few rows still spreads over the SMs at large batches.
    const int b_begin = p.b_per_cta > 0 ? static_cast<int>(blockIdx.y) * p.b_per_cta : 0;
    const int b_end = p.b_per_cta > 0 ? min(p.B, b_begin + p.b_per_cta) : p.B;
    for (int b0 = b_begin; b0 < b_end; b0 += kBT) {
        const int nb = min(kBT, b_end - b0);
        __syncthreads();
        if constexpr (kLN) {
            for (int r = warp; r < nb; r += kGemvWarps) {
                bool ok = warp_layernorm512(p.x + static_cast<size_t>(b0 + r) * p.ldx, p.ln_w,
                                            p.ln_b, xs + r * cols);
                if (lane == 0) ln_bad[r] = ok ? 0 : 1;
            }
        } else if constexpr (kSrc == SRC_HEADLN) {
            for (int r = warp; r < nb; r += kGemvWarps) {
                const float* shift = p.mod + static_cast<size_t>(b0 + r) * p.ldmod;
                const bool ok = head_ln_modulate(p.x + static_cast<size_t>(b0 + r) * p.ldx, p.ln_w, p.ln_b, shift,
                                                 shift + kWidth, xs + r * cols);
                if (lane == 0) ln_bad[r] = ok ? 0 : 1;
            }
        } else if constexpr (kSrc == SRC_MERGE) {
            // Warp h merges head h of every stream of the tile (the
            // arithmetic of attn_combine_kernel).
            const int head = warp, lane_ = threadIdx.x & 31;
            for (int r = 0; r < nb; ++r) {
                const int b = b0 + r, first = p.first[b], n = p.count[b];
                float M = -INFINITY, total = 0.0f, a0 = 0.0f, a1 = 0.0f;
                for (int s = 0; s < n; ++s) {
                    const float* pp = p.part + (static_cast<size_t>(first + s) * kHeads + head) * kPartStride;
                    const MergeWeights w = merge_weights(M, pp[0]);
                    total = merge_fold(total, w, pp[1]);
                    const float2 av = *reinterpret_cast<const float2*>(pp + 2 + 2 * lane_);
                    a0 = merge_fold(a0, w, av.x);
                    a1 = merge_fold(a1, w, av.y);
                }
                bool ok = total > 0.0f && isfinite(total);
                const float inv = __fdiv_rn(1.0f, total);
                const float o0 = __fmul_rn(a0, inv), o1 = __fmul_rn(a1, inv);
                ok &= isfinite(o0) && isfinite(o1);
                *reinterpret_cast<float2*>(xs + r * cols + head * kHeadDim + 2 * lane_) = make_float2(o0, o1);
                if (!__all_sync(kFull, ok) && lane_ == 0 && blockIdx.x == 0) flag_nonfinite(p.status, b);
            }
        } else {
            const int n4 = nb * cols / 4;
            for (int i = threadIdx.x; i < n4; i += blockDim.x) {
                const int e = i * 4, r = e / cols, cc = e % cols;
                *reinterpret_cast<float4*>(xs + e) =
                    *reinterpret_cast<const float4*>(p.x + static_cast<size_t>(b0 + r) * p.ldx + cc);
            }
        }
        __syncthreads();
        if constexpr (kLN || kSrc == SRC_HEADLN) {
            if (blockIdx.x == 0 && threadIdx.x < nb && ln_bad[threadIdx.x])
                flag_nonfinite(p.status, b0 + threadIdx.x);
        }
        if (!active) continue;

        float acc[kRowsPerWarp][kBT];
#pragma unroll
        for (int rr = 0; rr < kRowsPerWarp; ++rr)
#pragma unroll
            for (int bb = 0; bb < kBT; ++bb) acc[rr][bb] = 0.0f;

#pragma unroll
        for (int c = 0; c < kChunks; ++c) {
            float wf[kRowsPerWarp][16];
#pragma unroll
            for (int rr = 0; rr < kRowsPerWarp; ++rr) {
                if constexpr (kQ8) {
                    const uint32_t words[4] = {wq[rr][c][0].x, wq[rr][c][0].y, wq[rr][c][0].z,
                                               wq[rr][c][0].w};
#pragma unroll
                    for (int j = 0; j < 4; ++j)
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            wf[rr][j * 4 + e] = static_cast<float>(
                                static_cast<int8_t>((words[j] >> (8 * e)) & 0xffu));
                } else {
                    const uint32_t words[8] = {wq[rr][c][0].x, wq[rr][c][0].y, wq[rr][c][0].z,
                                               wq[rr][c][0].w, wq[rr][c][1].x, wq[rr][c][1].y,
                                               wq[rr][c][1].z, wq[rr][c][1].w};
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        wf[rr][2 * k] = __uint_as_float(words[k] << 16);
                        wf[rr][2 * k + 1] = __uint_as_float(words[k] & 0xffff0000u);
                    }
                }
            }
#pragma unroll
            for (int bb = 0; bb < kBT; ++bb) {
                if (bb < nb) {
                    const float* xr = xs + bb * cols + c * 512 + lane * 4;
                    float4 xv[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) xv[j] = *reinterpret_cast<const float4*>(xr + j * 128);
#pragma unroll
                    for (int rr = 0; rr < kRowsPerWarp; ++rr) {
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            float part = wf[rr][j * 4 + 0] * xv[j].x;
                            part = fmaf(wf[rr][j * 4 + 1], xv[j].y, part);
                            part = fmaf(wf[rr][j * 4 + 2], xv[j].z, part);
                            part = fmaf(wf[rr][j * 4 + 3], xv[j].w, part);
                            acc[rr][bb] = fmaf(sc[rr][c][j], part, acc[rr][bb]);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int rr = 0; rr < kRowsPerWarp; ++rr)
#pragma unroll
            for (int bb = 0; bb < kBT; ++bb) acc[rr][bb] = warp_sum(acc[rr][bb]);

        if (b0 + kBT >= b_end) pdl_trigger();
        // Lane bb finishes stream b0+bb for both rows of the pair.
#pragma unroll
        for (int bb = 0; bb < kBT; ++bb) {
            if (lane != bb || bb >= nb) continue;
            const int b = b0 + bb;
            float v0 = acc[0][bb], v1 = acc[1][bb];
            const int r0 = row0, r1 = row0 + 1;
            const bool has1 = r1 < p.rows;
            if constexpr (kEpi == EPI_QKV) {
                const int region = r0 >> 9;          // 0 = q, 1 = k, 2 = v
                const int within = r0 & 511;
                const int pos = p.pos[b];
                if (region < 2) rope_apply(v0, v1, p.rope[b * 32 + ((within & 63) >> 1)]);
                if (!isfinite(v0) || !isfinite(v1)) flag_nonfinite(p.status, b);
                if (region == 0) {
                    *reinterpret_cast<float2*>(p.q + static_cast<size_t>(b) * kWidth + within) =
                        make_float2(v0, v1);
                } else {
                    const int page = p.kv.table[static_cast<size_t>(p.slot[b]) * p.kv.max_pages + pos / kPage];
                    const long long off = kv_offset(p.kv, page, p.layer, region - 1, within >> 6,
                                                    pos % kPage) + (within & 63);
                    kv_store2(p.kv, off, v0, v1);
                }
            } else {
                float out[2] = {v0, v1};
#pragma unroll
                for (int rr = 0; rr < 2; ++rr) {
                    if (rr == 1 && !has1) break;
                    const int r = row0 + rr;
                    float v = out[rr];
                    if constexpr (kEpi == EPI_RESID) v = __fadd_rn(p.res[static_cast<size_t>(b) * p.ldres + r], v);
                    if constexpr (kEpi == EPI_GELU) {
                        if (!isfinite(v)) flag_nonfinite(p.status, b);
                        v = gelu_erf(v);
                    }
                    if constexpr (kEpi == EPI_STORE) {
                        if (p.bias) v = __fadd_rn(v, p.bias[r]);
                    }
                    if constexpr (kEpi == EPI_SILU) v = silu_f(__fadd_rn(v, p.bias[r]));
                    if constexpr (kEpi == EPI_GATE)
                        v = __fadd_rn(p.res[static_cast<size_t>(b) * p.ldres + r],
                                      __fmul_rn(p.gate[static_cast<size_t>(b) * p.ldgate + r], __fadd_rn(v, p.bias[r])));
                    if (!isfinite(v)) flag_nonfinite(p.status, b);
                    p.y[static_cast<size_t>(b) * p.ldy + r] = v;
                }
            }
        }
    }
}

// Any-shape linear (cols % 32 == 0 for Q8_0, any cols for bf16), natural
// row-major layout: one warp per (stream, row). Used for shapes outside the
// four Flow projections (e.g. the reference's small test matrices).
template <bool kQ8>
__global__ void linear_generic_kernel(const void* __restrict__ w, const __half* __restrict__ scales,
                                      int rows, int cols, const float* __restrict__ x, int B,
                                      const float* __restrict__ bias, float* __restrict__ y,
                                      int32_t* status) {
    const long long gw = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw >= static_cast<long long>(rows) * B) return;
    const int b = static_cast<int>(gw / rows), r = static_cast<int>(gw % rows);
    const float* xr = x + static_cast<size_t>(b) * cols;
    float acc = 0.0f;
    for (int c = lane; c < cols; c += 32) {
        float wv;
        if constexpr (kQ8) {
            const int8_t q = static_cast<const int8_t*>(w)[static_cast<size_t>(r) * cols + c];
            wv = __fmul_rn(__half2float(scales[static_cast<size_t>(r) * (cols / 32) + c / 32]),
                           static_cast<float>(q));
        } else {
            wv = bf16_to_f32(static_cast<const uint16_t*>(w)[static_cast<size_t>(r) * cols + c]);
        }
        acc = fmaf(xr[c], wv, acc);
    }
    // Lane sums combine in an adjacent-pair tree (lanes 2i and 2i+1 first,
    // then pairs of pairs), i.e. columns in a balanced tree over their
    // natural order. On the reference's pinned cancellation row
    // ([1e8, 1, -1e8, 1] x 8 against unit weights,
    // tests/test_phonon_transformer.c:617-652) that order gives its SGEMM's
    // 0 (+bias); the reverse butterfly would give 16.
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) acc += __shfl_xor_sync(kFull, acc, o);
    if (lane == 0) {
        if (bias) acc = __fadd_rn(acc, bias[r]);
        if (!isfinite(acc)) flag_nonfinite(status, b);
        y[static_cast<size_t>(b) * rows + r] = acc;
    }
}

// ---------------------------------------------------------------- attention
// Split descriptor: stream index b in the batch, first page, page count and
// the number of valid keys of that stream (position + 1).
struct Split {
    int b, page_begin, page_count, n_keys;
};

struct AttnParams {
    const float* q;        // [B][512] RoPE'd queries
    const int32_t* slot;   // [B]
    const Split* splits;   // [S]
    // TMA kernel: the step's plan header, [0] splits, [1] chunks C, then the
    // offsets (in ints, from the header) of [2] cta_split and [3] cta_page
    // (first split and first page of each chunk, at least C + 1 entries) and
    // [4] the page ids of all splits in split order (a stream's last page,
    // which the step appends to, stored as ~id)
    const int32_t* plan;
    int32_t* chunk_ctr;    // TMA kernel: chunk tickets of this launch (zeroed at step start)
    int n_splits;
    KvView kv;
    int layer;
    float* part;           // [S][8][66]: max, sum, acc[64]
    int32_t* status;
};


// One warp per (split, head). Lane l scores key (l & 15) of the current page
// over dims (l >> 4)*32 .. +31, so the two halves of a 64-dim dot meet with a
// single shuffle; for P.V lane l owns output dims 2l, 2l+1. Online softmax:
// running max m, sum s, accumulator a; exp(-inf) = 0 for masked keys.
template <bool kBf16>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_partial_kernel(AttnParams p) {
    const int lane = threadIdx.x & 31;
    pdl_wait();
    const long long item = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (item >= static_cast<long long>(p.n_splits) * kHeads) return;
    const int s_idx = static_cast<int>(item >> 3), head = static_cast<int>(item & 7);
    const Split sp = p.splits[s_idx];
    const int half = lane >> 4, key_lane = lane & 15;
    const int slot = p.slot[sp.b];
    float qh[32];
    {
        const float4* qs = reinterpret_cast<const float4*>(p.q + static_cast<size_t>(sp.b) * kWidth +
                                                           head * kHeadDim + half * 32);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float4 v = qs[i];
            qh[4 * i] = v.x;
            qh[4 * i + 1] = v.y;
            qh[4 * i + 2] = v.z;
            qh[4 * i + 3] = v.w;
        }
    }
    float m = -INFINITY, l = 0.0f, a0 = 0.0f, a1 = 0.0f;
    bool finite_ok = true;
    const int32_t* table = p.kv.table + static_cast<size_t>(slot) * p.kv.max_pages;
    for (int pg = sp.page_begin; pg < sp.page_begin + sp.page_count; ++pg) {
        const int page = table[pg];
        const long long kbase = kv_offset(p.kv, page, p.layer, 0, head, 0);
        const long long vbase = kv_offset(p.kv, page, p.layer, 1, head, 0);
        const int key = pg * kPage + key_lane;
        const bool valid = key < sp.n_keys;
        float dot = 0.0f;
        if constexpr (kBf16) {
            const uint4* kr = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.kv.pool) +
                                                             kbase + key_lane * kHeadDim + half * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                uint4 v = kr[i];
                const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    dot = fmaf(qh[8 * i + 2 * k], __uint_as_float(words[k] << 16), dot);
                    dot = fmaf(qh[8 * i + 2 * k + 1], __uint_as_float(words[k] & 0xffff0000u), dot);
                }
            }
        } else {
            const float4* kr = reinterpret_cast<const float4*>(static_cast<const float*>(p.kv.pool) +
                                                               kbase + key_lane * kHeadDim + half * 32);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                float4 v = kr[i];
                dot = fmaf(qh[4 * i], v.x, dot);
                dot = fmaf(qh[4 * i + 1], v.y, dot);
                dot = fmaf(qh[4 * i + 2], v.z, dot);
                dot = fmaf(qh[4 * i + 3], v.w, dot);
            }
        }
        dot += __shfl_xor_sync(kFull, dot, 16);
        float score = dot * 0.125f;
        if (valid) finite_ok &= isfinite(score);
        score = valid ? score : -INFINITY;
        float pm = score;
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) pm = fmaxf(pm, __shfl_xor_sync(kFull, pm, o));
        const float m_new = fmaxf(m, pm);
        const float alpha = m == -INFINITY ? 0.0f : expf(m - m_new);
        const float pr = valid ? expf(score - m_new) : 0.0f;
        float ps = pr;
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) ps += __shfl_xor_sync(kFull, ps, o);
        l = fmaf(l, alpha, ps);
        a0 *= alpha;
        a1 *= alpha;
        const int n_valid = min(kPage, sp.n_keys - pg * kPage);
#pragma unroll
        for (int j = 0; j < kPage; ++j) {
            const float pj = __shfl_sync(kFull, pr, j);
            if (j < n_valid) {
                float v0, v1;
                if constexpr (kBf16) {
                    uint32_t w2 = *reinterpret_cast<const uint32_t*>(
                        static_cast<const uint16_t*>(p.kv.pool) + vbase + j * kHeadDim + 2 * lane);
                    v0 = __uint_as_float(w2 << 16);
                    v1 = __uint_as_float(w2 & 0xffff0000u);
                } else {
                    float2 w2 = *reinterpret_cast<const float2*>(static_cast<const float*>(p.kv.pool) +
                                                                 vbase + j * kHeadDim + 2 * lane);
                    v0 = w2.x;
                    v1 = w2.y;
                }
                a0 = fmaf(pj, v0, a0);
                a1 = fmaf(pj, v1, a1);
            }
        }
        m = m_new;
    }
    float* out = p.part + (static_cast<size_t>(s_idx) * kHeads + head) * kPartStride;
    *reinterpret_cast<float2*>(out + 2 + 2 * lane) = make_float2(a0, a1);
    if (lane == 0) {
        out[0] = m;
        out[1] = l;
    }
    if (!__all_sync(kFull, finite_ok) && lane == 0) flag_nonfinite(p.status, sp.b);
}

struct CombineParams {
    const float* part;        // [S][8][66]
    const int32_t* first;     // [B] first split of stream b
    const int32_t* count;     // [B] splits of stream b
    int B;
    float* out;               // [B][512]
    int32_t* status;
};

// One warp per (stream, head): merge the stream's splits in page order.
__global__ void __launch_bounds__(kAttnWarps * 32) attn_combine_kernel(CombineParams p) {
    const int lane = threadIdx.x & 31;
    pdl_wait();
    pdl_trigger();
    const long long item = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (item >= static_cast<long long>(p.B) * kHeads) return;
    const int b = static_cast<int>(item >> 3), head = static_cast<int>(item & 7);
    const int first = p.first[b], n = p.count[b];
    float M = -INFINITY, total = 0.0f, a0 = 0.0f, a1 = 0.0f;
    for (int s = 0; s < n; ++s) {
        const float* pp = p.part + (static_cast<size_t>(first + s) * kHeads + head) * kPartStride;
        const MergeWeights w = merge_weights(M, pp[0]);
        total = merge_fold(total, w, pp[1]);
        const float2 av = *reinterpret_cast<const float2*>(pp + 2 + 2 * lane);
        a0 = merge_fold(a0, w, av.x);
        a1 = merge_fold(a1, w, av.y);
    }
    bool ok = total > 0.0f && isfinite(total);
    const float inv = __fdiv_rn(1.0f, total);
    const float o0 = __fmul_rn(a0, inv), o1 = __fmul_rn(a1, inv);
    ok &= isfinite(o0) && isfinite(o1);
    *reinterpret_cast<float2*>(p.out + static_cast<size_t>(b) * kWidth + head * kHeadDim + 2 * lane) =
        make_float2(o0, o1);
    if (!__all_sync(kFull, ok) && lane == 0) flag_nonfinite(p.status, b);
}

// ------------------------------------------------------------- small kernels
// Copy K/V rows between a staging buffer and the pages of one stream.
// Staging layout: keys [layer_count][count][512] then values, fp32.
// dir 0: pages -> staging, 1: staging -> pages.
__global__ void kv_rows_kernel(KvView kv, int slot, int layer_begin, int layer_count, int position, int count,
                               float* stage, int dir) {
    const long long n = static_cast<long long>(layer_count) * count * kWidth;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < 2 * n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int which = static_cast<int>(i / n);
        const long long r = i % n;
        const int l = static_cast<int>(r / (static_cast<long long>(count) * kWidth));
        const int p = position + static_cast<int>((r / kWidth) % count);
        const int d = static_cast<int>(r % kWidth);
        const int page = kv.table[static_cast<size_t>(slot) * kv.max_pages + p / kPage];
        const long long off = kv_offset(kv, page, layer_begin + l, which, d >> 6, p % kPage) + (d & 63);
        if (dir == 0) {
            stage[i] = kv.bf16 ? bf16_to_f32(static_cast<const uint16_t*>(kv.pool)[off])
                               : static_cast<const float*>(kv.pool)[off];
        } else {
            const float v = stage[i];
            if (kv.bf16) static_cast<uint16_t*>(kv.pool)[off] = f32_to_bf16(v);
            else static_cast<float*>(kv.pool)[off] = v;
        }
    }
}

// Seeded pseudo-random K/V (roughly N(0,1): sum of four uniforms, centred and
// scaled) for positions [0, length) of every layer of one stream.
__device__ __forceinline__ uint32_t hash32(uint64_t x) {
    x ^= x >> 33;
    x *= 0xff51afd7ed558ccdull;
    x ^= x >> 33;
    x *= 0xc4ceb9fe1a85ec53ull;
    x ^= x >> 33;
    return static_cast<uint32_t>(x);
}

__global__ void kv_fill_kernel(KvView kv, int slot, int n_layers, int length, uint64_t seed) {
    const long long per_pos = static_cast<long long>(n_layers) * 2 * kWidth;
    const long long total = per_pos * length;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int position = static_cast<int>(i / per_pos);
        const long long r = i % per_pos;
        const int layer = static_cast<int>(r / (2 * kWidth));
        const int which = static_cast<int>((r / kWidth) & 1);
        const int d = static_cast<int>(r % kWidth);
        const uint32_t h = hash32(seed * 0x9E3779B97F4A7C15ull + static_cast<uint64_t>(i));
        const float u = (static_cast<float>(h & 0xffff) + static_cast<float>(h >> 16)) * (1.0f / 65536.0f);
        const float v = (u - 1.0f) * 2.449f;  // ~unit variance
        const int page = kv.table[static_cast<size_t>(slot) * kv.max_pages + position / kPage];
        const long long off = kv_offset(kv, page, layer, which, d >> 6, position % kPage) + (d & 63);
        if (kv.bf16) static_cast<uint16_t*>(kv.pool)[off] = f32_to_bf16(v);
        else static_cast<float*>(kv.pool)[off] = v;
    }
}

// ------------------------------------------------ standalone primitive kernels
__global__ void layernorm_rows_kernel(const float* x, const float* w, const float* b, float* out,
                                      int rows, int32_t* status) {
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;
    if (!warp_layernorm512(x + static_cast<size_t>(row) * kWidth, w, b, out + static_cast<size_t>(row) * kWidth) &&
        (threadIdx.x & 31) == 0)
        flag_nonfinite(status, 0);
}

}  // namespace phonon
