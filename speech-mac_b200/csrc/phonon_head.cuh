// The frame loop around the decode step, on the device: the flow head (the
// MLP that turns a transformer output row into the next 32-wide latent,
// speech-mac src/phonon_sampler.c:280-393), the EOS logit
// (src/phonon_sampler.c:395-402), phonon_flow_embed_latent and
// phonon_flow_output_norm (src/phonon_transformer.c:860-914).
//
// The head's linears are bf16 matrices applied with gemv_kernel (fp32
// arithmetic, bias added after the sum); everything between them runs here,
// one warp or one CTA per stream row:
//
//   head_time_kernel     time embedding of one flow time (sin/cos, MLP, RMS
//                        normalisation with a learned gain), stream-independent
//   head_in_kernel       x = input_proj(noise), silu(cond_embed(c) + time terms)
//   head_block_kernel    LayerNorm(x) modulated by the block's shift/scale,
//                        written as bf16 slices for the tensor-core linears
//                        (below 32 streams the same head_ln_modulate runs in
//                        the first MLP GEMV's prologue, SRC_HEADLN)
//   (gemv EPI_SILU)      silu(mlp.0(h))
//   (gemv EPI_GATE)      x += gate * mlp.2(...)
//   head_final_kernel    final LayerNorm + modulation, final linear, the Euler
//                        step noise + velocity, and the embedding of that
//                        latent as the next step's input row
//
// Sums that the reference evaluates in a fixed order outside BLAS (the
// 512-element means, the double variance) follow that order; the linears
// sum in the GEMV's order, as the reference's SGEMM calls do in theirs.
#pragma once

#include "phonon_head_gemm.cuh"

namespace phonon {

constexpr int kHeadBlocks = 6;                          // PHONON_FLOW_HEAD_BLOCKS
constexpr int kLatent = 32;                             // PHONON_LATENT_WIDTH
constexpr int kAdaBlockRows = 3 * kWidth;               // shift, scale, gate
constexpr int kAdaRows = kHeadBlocks * kAdaBlockRows + 2 * kWidth;  // every modulation row, final layer last
constexpr int kHeadCondLd = 520;                        // cond_embed rows, then the EOS row, padded


// bf16 pair of a 32-bit word -> two floats (element 2i in the low half).
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Rows r0 .. r0+3 of a natural row-major bf16 matrix [rows][cols] times v
// (shared memory), summed by one warp (cols a multiple of 256, rows 16-byte
// aligned): lane l takes columns [8l + 256s, +8); every 16-byte load of the
// four rows is issued before the arithmetic; then the warp tree.
__device__ __forceinline__ float4 head_rows4_dot(const uint16_t* __restrict__ w, int cols, int r0, const float* v) {
    const int lane = threadIdx.x & 31;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int c0 = lane * 8; c0 < cols; c0 += 256) {
        uint4 u[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
            u[q] = __ldg(reinterpret_cast<const uint4*>(w + static_cast<size_t>(r0 + q) * cols + c0));
        const float4 va = *reinterpret_cast<const float4*>(v + c0);
        const float4 vb = *reinterpret_cast<const float4*>(v + c0 + 4);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            float a = acc[q];
            a = fmaf(bf16_lo(u[q].x), va.x, a);
            a = fmaf(bf16_hi(u[q].x), va.y, a);
            a = fmaf(bf16_lo(u[q].y), va.z, a);
            a = fmaf(bf16_hi(u[q].y), va.w, a);
            a = fmaf(bf16_lo(u[q].z), vb.x, a);
            a = fmaf(bf16_hi(u[q].z), vb.y, a);
            a = fmaf(bf16_lo(u[q].w), vb.z, a);
            a = fmaf(bf16_hi(u[q].w), vb.w, a);
            acc[q] = a;
        }
    }
    return make_float4(warp_sum(acc[0]), warp_sum(acc[1]), warp_sum(acc[2]), warp_sum(acc[3]));
}

// Row i of a natural row-major bf16 [rows][32] matrix times lat[32]
// (shared memory), one thread: four 16-byte loads, then the products.
__device__ __forceinline__ float head_row32_dot(const uint16_t* __restrict__ w, int i, const float* lat) {
    const uint4* row = reinterpret_cast<const uint4*>(w + static_cast<size_t>(i) * kLatent);
    uint4 u[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) u[q] = __ldg(row + q);
    float acc = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const uint32_t wd[4] = {u[q].x, u[q].y, u[q].z, u[q].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            acc = fmaf(bf16_lo(wd[e]), lat[8 * q + 2 * e], acc);
            acc = fmaf(bf16_hi(wd[e]), lat[8 * q + 2 * e + 1], acc);
        }
    }
    return acc;
}

// Time embedding of one flow time (src/phonon_sampler.c:280-305), one CTA
// of 512 threads: phase_i = t * freq_i, [cos | sin] of the 128 phases,
// hidden = silu(W0 e + b0) (512 x 256), o = W1 hidden + b1 (512 x 512),
// out_i = (alpha_i * o_i) / sqrt(mean(o^2) + 1e-5). W0 and W1 are natural
// row-major bf16; bias, freqs and alpha are fp32 copies of bf16 vectors.
__global__ void __launch_bounds__(512) head_time_kernel(float value, const float* __restrict__ freqs,
                                                        const uint16_t* __restrict__ w0, const float* __restrict__ b0,
                                                        const uint16_t* __restrict__ w1, const float* __restrict__ b1,
                                                        const float* __restrict__ alpha, float* __restrict__ out,
                                                        int32_t* status) {
    __shared__ __align__(16) float e[256];
    __shared__ __align__(16) float hidden[kWidth];
    __shared__ __align__(16) float o[kWidth];
    __shared__ __align__(16) float sq[kWidth];
    __shared__ float inverse;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    if (t < 128) {
        float s, c;
        sincosf(__fmul_rn(value, freqs[t]), &s, &c);
        e[t] = c;
        e[128 + t] = s;
    }
    __syncthreads();
    for (int r = 4 * warp; r < kWidth; r += 64) {
        const float4 d = head_rows4_dot(w0, 256, r, e);
        if (lane < 4) hidden[r + lane] = silu_f(__fadd_rn(lane == 0 ? d.x : lane == 1 ? d.y : lane == 2 ? d.z : d.w,
                                                          b0[r + lane]));
    }
    __syncthreads();
    for (int r = 4 * warp; r < kWidth; r += 64) {
        const float4 d = head_rows4_dot(w1, kWidth, r, hidden);
        if (lane < 4) o[r + lane] = __fadd_rn(lane == 0 ? d.x : lane == 1 ? d.y : lane == 2 ? d.z : d.w, b1[r + lane]);
    }
    __syncthreads();
    sq[t] = __fmul_rn(o[t], o[t]);
    __syncthreads();
    if (warp == 0) {
        const float m = head_mean512(sq);
        if (lane == 0) inverse = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(m, 1e-5f)));
    }
    __syncthreads();
    const float v = __fmul_rn(__fmul_rn(alpha[t], o[t]), inverse);
    if (!isfinite(v)) flag_nonfinite(status, 0);
    out[t] = v;
}

struct HeadInParams {
    const float* noise;      // [B][32] raw noise (lsd) or the latent state (forward)
    float noise_scale;       // sqrt(temperature) (lsd) or 1 with scaled = false
    int scaled;
    const uint16_t* in_w;    // input_proj [512][32] bf16
    const float* in_b;       // [512]
    const float* cond;       // cond_embed(condition) + bias, [B][ldc]
    int ldc;
    const float* temb;       // [2][512] time embeddings of s and t
    float* x;                // [B][512]
    float* silu_y;           // [B][512]
    uint16_t* sy_slices;     // optional: silu(y) as bf16 slice rows (tensor-core path)
    int B;
    int32_t* status;
};

// Streams [8 * blockIdx.x, +8) per CTA of 512 threads, thread t = output
// row t with its input_proj row in registers (src/phonon_sampler.c:310-318):
// x = input_proj(noise) + b, y = cond + 0.5 * (time_s + time_t), silu(y)
// (the same silu(y) feeds every block's and the final modulation).
constexpr int kHeadInStreams = 8;
__global__ void __launch_bounds__(512) head_in_kernel(HeadInParams p) {
    __shared__ float nz[kHeadInStreams][kLatent];
    const int t = threadIdx.x;
    const int b_first = blockIdx.x * kHeadInStreams;
    float wr[kLatent];
    {
        const uint4* row = reinterpret_cast<const uint4*>(p.in_w + static_cast<size_t>(t) * kLatent);
#pragma unroll
        for (int q = 0; q < kLatent / 8; ++q) {
            const uint4 u = __ldg(row + q);
            const uint32_t wd[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                wr[8 * q + 2 * e] = __uint_as_float(wd[e] << 16);
                wr[8 * q + 2 * e + 1] = __uint_as_float(wd[e] & 0xffff0000u);
            }
        }
    }
    const float in_b = p.in_b[t];
    pdl_wait();  // the time embeddings, conditions and noise come from earlier work
    pdl_trigger();
    const float half_t = __fmul_rn(0.5f, __fadd_rn(p.temb[t], p.temb[kWidth + t]));
    if (t < kHeadInStreams * kLatent) {
        const int bb = t / kLatent, k = t % kLatent, b = b_first + bb;
        float r = 0.0f;
        if (b < p.B) {
            r = p.noise[static_cast<size_t>(b) * kLatent + k];
            if (!isfinite(r)) flag_nonfinite(p.status, b);
        }
        nz[bb][k] = p.scaled ? __fmul_rn(r, p.noise_scale) : r;
    }
    __syncthreads();
    for (int bb = 0; bb < kHeadInStreams; ++bb) {
        const int b = b_first + bb;
        if (b >= p.B) break;
        float acc = 0.0f;
#pragma unroll
        for (int k = 0; k < kLatent; ++k) acc = fmaf(wr[k], nz[bb][k], acc);
        const float x = __fadd_rn(acc, in_b);
        const float y = __fadd_rn(p.cond[static_cast<size_t>(b) * p.ldc + t], half_t);
        const float sy = silu_f(y);
        if (!isfinite(x) || !isfinite(sy)) flag_nonfinite(p.status, b);
        p.x[static_cast<size_t>(b) * kWidth + t] = x;
        if (p.sy_slices) {
            uint16_t s0, s1, s2;
            bf16x3_split(sy, s0, s1, s2);
            uint16_t* row = p.sy_slices + static_cast<size_t>(3 * b) * kWidth + t;
            row[0] = s0;
            row[kWidth] = s1;
            row[2 * kWidth] = s2;
        } else {
            p.silu_y[static_cast<size_t>(b) * kWidth + t] = sy;
        }
    }
}

// Residual block LayerNorm (src/phonon_sampler.c:319-332): h = LN(x; w, b)
// * (1 + scale) + shift, shift/scale the block's first two modulation
// thirds. One warp per stream, the row staged in shared memory.
__global__ void __launch_bounds__(256) head_block_kernel(const float* __restrict__ x, const float* __restrict__ mod,
                                                         int block, const float* __restrict__ norm_w,
                                                         const float* __restrict__ norm_b, float* __restrict__ h, int B,
                                                         int32_t* status, uint16_t* __restrict__ h_slices) {
    __shared__ float row[8][kWidth];
    __shared__ float hr[8][kWidth];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.x * 8 + warp;
    pdl_wait();
    pdl_trigger();
    if (b >= B) return;
    for (int k = 0; k < 16; ++k) row[warp][lane + 32 * k] = x[static_cast<size_t>(b) * kWidth + lane + 32 * k];
    __syncwarp();
    const float* m = mod + static_cast<size_t>(b) * kAdaRows + block * kAdaBlockRows;
    float* out = h_slices ? hr[warp] : h + static_cast<size_t>(b) * kWidth;
    if (!head_ln_modulate(row[warp], norm_w, norm_b, m, m + kWidth, out) && lane == 0) flag_nonfinite(status, b);
    if (h_slices) {  // the next linear's operand: three bf16 slice rows
        __syncwarp();
        for (int k = 0; k < 16; ++k) {
            const int i = lane + 32 * k;
            uint16_t s0, s1, s2;
            bf16x3_split(hr[warp][i], s0, s1, s2);
            uint16_t* dst = h_slices + static_cast<size_t>(3 * b) * kWidth + i;
            dst[0] = s0;
            dst[kWidth] = s1;
            dst[2 * kWidth] = s2;
        }
    }
}

struct HeadFinalParams {
    const float* x;          // [B][512]
    const float* mod;        // [B][kAdaRows]: the final shift/scale are its last 1024
    const uint16_t* fin_w;   // final_layer.linear [32][512] bf16
    const float* fin_b;      // [32]
    const float* noise;      // as HeadInParams
    float noise_scale;
    int scaled;              // 1: out = noise * scale + velocity (lsd); 0: out = velocity
    float* out;              // [B][32]
    const uint16_t* embed_w; // optional: input_linear [512][32] bf16 ...
    const float* condition;  // ... [B][512] ...
    float* embed_out;        // ... -> [B][512] = input_linear(out) + condition
    int B;
    int32_t* status;
};

// Final layer and Euler step (src/phonon_sampler.c:349-393), then the
// embedding of the new latent (phonon_flow_embed_latent,
// src/phonon_transformer.c:860-875) when the frame loop asks for it: one
// CTA of 256 threads per stream.
__global__ void __launch_bounds__(256) head_final_kernel(HeadFinalParams p) {
    __shared__ __align__(16) float xr[kWidth];
    __shared__ __align__(16) float h[kWidth];
    __shared__ __align__(16) float lat[kLatent];
    __shared__ int bad;
    const int b = blockIdx.x, t = threadIdx.x, warp = t >> 5, lane = t & 31;
    pdl_wait();
    pdl_trigger();
    if (t == 0) bad = 0;
    for (int i = t; i < kWidth; i += 256) xr[i] = p.x[static_cast<size_t>(b) * kWidth + i];
    __syncthreads();
    if (warp == 0) {
        const float* m = p.mod + static_cast<size_t>(b) * kAdaRows + kHeadBlocks * kAdaBlockRows;
        if (!head_ln_modulate(xr, nullptr, nullptr, m, m + kWidth, h) && lane == 0) bad = 1;
    }
    __syncthreads();
    {  // warp w: final rows 4w .. 4w+3
        const int j0 = 4 * warp;
        const float4 d = head_rows4_dot(p.fin_w, kWidth, j0, h);
        if (lane < 4) {
            const int j = j0 + lane;
            const float v = __fadd_rn(lane == 0 ? d.x : lane == 1 ? d.y : lane == 2 ? d.z : d.w, p.fin_b[j]);
            float o = v;
            if (p.scaled) o = __fadd_rn(__fmul_rn(p.noise[static_cast<size_t>(b) * kLatent + j], p.noise_scale), v);
            if (!isfinite(o)) bad = 1;
            lat[j] = o;
            p.out[static_cast<size_t>(b) * kLatent + j] = o;
        }
    }
    __syncthreads();
    if (p.embed_out) {
        const float c0 = p.condition[static_cast<size_t>(b) * kWidth + t];
        const float c1 = p.condition[static_cast<size_t>(b) * kWidth + t + 256];
        const float v0 = __fadd_rn(head_row32_dot(p.embed_w, t, lat), c0);
        const float v1 = __fadd_rn(head_row32_dot(p.embed_w, t + 256, lat), c1);
        if (!isfinite(v0) || !isfinite(v1)) bad = 1;
        p.embed_out[static_cast<size_t>(b) * kWidth + t] = v0;
        p.embed_out[static_cast<size_t>(b) * kWidth + t + 256] = v1;
        __syncthreads();
    }
    if (t == 0 && bad) flag_nonfinite(p.status, b);
}

// phonon_flow_output_norm of B rows (src/phonon_transformer.c:904-914): the
// transformer's LayerNorm (eps 1e-5) with the out_norm weight and bias, one
// warp per row; non-finite rows are flagged per stream.
__global__ void __launch_bounds__(256) output_norm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                          const float* __restrict__ b, float* __restrict__ out, int B,
                                                          int32_t* status) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = blockIdx.x * 8 + warp;
    pdl_wait();
    pdl_trigger();
    if (r >= B) return;
    if (!warp_layernorm512(x + static_cast<size_t>(r) * kWidth, w, b, out + static_cast<size_t>(r) * kWidth) &&
        lane == 0)
        flag_nonfinite(status, r);
}

}  // namespace phonon
