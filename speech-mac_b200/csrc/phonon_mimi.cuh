// The Mimi latent transformer on the device (speech-mac src/phonon_mimi.c:
// 108-283): every latent frame of a request becomes 16 feature rows of 512
// through a linear projection (512 x 32), a depthwise transposed-convolution
// upsample, and two pre-LayerNorm transformer layers whose 16 queries per
// frame attend causally over at most 250 keys.
//
// A step runs one frame of each of B request states at once (16 B rows):
//
//   mimi_in_kernel       projection + upsample -> hidden rows, keeps the
//                        projection as the next frame's `previous`
//   per layer (the linears on gemv_kernel, or from 4 states on the tensor
//   cores: head_gemm_kernel, bf16 weights x three bf16 slices of the
//   activations, whose producers then write slice rows):
//     mimi_ln_kernel     LayerNorm 1 (the transformer's LayerNorm, eps 1e-5)
//     linear             in_proj -> q | k | v
//     mimi_rope_kv_kernel RoPE of q and k at each row's position; k and v
//                        of all 16 rows into the state's ring
//     mimi_attn_kernel   softmax(q k / 8) v over each row's window, one CTA
//                        per (state, head) with the window staged once
//     linear, gated     hidden += layer_scale_1 * out_proj(att)
//     mimi_ln_kernel     LayerNorm 2
//     linear, GELU       erf-GELU(linear1)
//     linear, gated     hidden += layer_scale_2 * linear2(.)
//
// The ring: the reference keeps 250 slots and inserts a frame's keys query by
// query, so that a later row's write never evicts a key an earlier row still
// reads. Here the 16 rows' keys are written first and then every row attends,
// so the ring holds kMimiRing = 272 >= 250 + 15 slots: position p lives in
// slot p % 272, and each query still sees exactly the positions
// [max(0, p - 249), p] of the reference.
#pragma once

#include "phonon_head_gemm.cuh"

namespace phonon {

constexpr int kMimiRows = 16;      // feature rows per latent frame (PHONON_MIMI_STRIDE)
constexpr int kMimiContext = 250;  // keys a query attends to at most (PHONON_MIMI_CONTEXT)
constexpr int kMimiRing = 272;     // ring slots per layer
constexpr int kMimiLayers = 2;

// Ring of one state: [layer][k | v][slot][512] fp32.
__device__ __forceinline__ float* mimi_ring(float* rings, int slot, int layer, int which) {
    return rings + ((static_cast<size_t>(slot) * kMimiLayers + layer) * 2 + which) * kMimiRing * kWidth;
}

// One CTA of 512 threads per state (src/phonon_mimi.c:270-279, :108-131):
// channel c: projected = W[c] . latent (bias-free linear), then for tap o
// hidden[o][c] = previous[c] * k[c][16 + o] + projected[c] * k[c][o] (two
// products, one sum, no contraction), previous[c] = projected.
__global__ void __launch_bounds__(512) mimi_in_kernel(const float* __restrict__ latents, const int32_t* __restrict__ slots,
                                                      const uint16_t* __restrict__ proj_w,
                                                      const uint16_t* __restrict__ up_w, float* __restrict__ previous,
                                                      float* __restrict__ hidden, int32_t* status) {
    __shared__ float lat[32];
    const int b = blockIdx.x, c = threadIdx.x;
    const uint4* wrow = reinterpret_cast<const uint4*>(proj_w + static_cast<size_t>(c) * 32);
    const uint4* krow = reinterpret_cast<const uint4*>(up_w + static_cast<size_t>(c) * 32);
    uint4 wq[4], kq[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        wq[q] = __ldg(wrow + q);
        kq[q] = __ldg(krow + q);
    }
    pdl_wait();
    pdl_trigger();
    if (c < 32) lat[c] = latents[static_cast<size_t>(b) * 32 + c];
    __syncthreads();
    float acc = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const uint32_t wd[4] = {wq[q].x, wq[q].y, wq[q].z, wq[q].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            acc = fmaf(__uint_as_float(wd[e] << 16), lat[8 * q + 2 * e], acc);
            acc = fmaf(__uint_as_float(wd[e] & 0xffff0000u), lat[8 * q + 2 * e + 1], acc);
        }
    }
    float k[32];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const uint32_t kd[4] = {kq[q].x, kq[q].y, kq[q].z, kq[q].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            k[8 * q + 2 * e] = __uint_as_float(kd[e] << 16);
            k[8 * q + 2 * e + 1] = __uint_as_float(kd[e] & 0xffff0000u);
        }
    }
    float* prev = previous + static_cast<size_t>(slots[b]) * kWidth + c;
    const float old_in = *prev;
    bool ok = isfinite(acc) && isfinite(old_in);
#pragma unroll
    for (int o = 0; o < kMimiRows; ++o) {
        const float v = __fadd_rn(__fmul_rn(old_in, k[kMimiRows + o]), __fmul_rn(acc, k[o]));
        ok &= isfinite(v);
        hidden[(static_cast<size_t>(b) * kMimiRows + o) * kWidth + c] = v;
    }
    *prev = acc;
    if (!ok) flag_nonfinite(status, b * kMimiRows);
}

// LayerNorm of rows (eps 1e-5, the reference's Welford cascade), one warp per
// row; a non-finite row flags its status word. With `slices`, the row also
// goes out as its three bf16 slice rows (the tensor-core linears' operand).
__global__ void __launch_bounds__(256) mimi_ln_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                      const float* __restrict__ b, float* __restrict__ out, int rows,
                                                      int32_t* status, uint16_t* __restrict__ slices) {
    const int r = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    pdl_wait();
    pdl_trigger();
    if (r >= rows) return;
    float* o = out + static_cast<size_t>(r) * kWidth;
    if (!warp_layernorm512(x + static_cast<size_t>(r) * kWidth, w, b, o) && lane == 0) flag_nonfinite(status, r);
    if (slices) {
        __syncwarp();
        for (int k = 0; k < kWidth / 32; ++k) {
            const int i = lane + 32 * k;
            uint16_t s0, s1, s2;
            bf16x3_split(o[i], s0, s1, s2);
            uint16_t* dst = slices + static_cast<size_t>(3 * r) * kWidth + i;
            dst[0] = s0;
            dst[kWidth] = s1;
            dst[2 * kWidth] = s2;
        }
    }
}

// One CTA of 256 threads per row: RoPE of q and k (interleaved pairs, eight
// 64-wide heads, the phase of pair i of a head at position p is p * freq[i]
// in fp32, cos and sin rounded from double; src/phonon_transformer.c:222-251),
// q rotated in place, k and v of the row written into ring slot p % 272.
__global__ void __launch_bounds__(256) mimi_rope_kv_kernel(float* __restrict__ qkv, const int32_t* __restrict__ slots,
                                                           const int32_t* __restrict__ pos0, const float* __restrict__ freq,
                                                           float* __restrict__ rings, int layer) {
    const int row = blockIdx.x, t = threadIdx.x;
    const int b = row / kMimiRows;
    pdl_wait();
    pdl_trigger();
    const int position = pos0[b] + row % kMimiRows;
    const int ring_slot = position % kMimiRing;
    float* q = qkv + static_cast<size_t>(row) * 3 * kWidth;
    float2 cs;
    {
        const float phase = __fmul_rn(static_cast<float>(position), freq[t & 31]);
        double sd, cd;
        sincos(static_cast<double>(phase), &sd, &cd);
        cs = make_float2(__double2float_rn(cd), __double2float_rn(sd));
    }
    // pair t of q (dims 2t, 2t+1), pair t of k
    float2 qp = *reinterpret_cast<float2*>(q + 2 * t);
    float2 kp = *reinterpret_cast<float2*>(q + kWidth + 2 * t);
    rope_apply(qp.x, qp.y, cs);
    rope_apply(kp.x, kp.y, cs);
    *reinterpret_cast<float2*>(q + 2 * t) = qp;
    const int slot = slots[b];
    float* kr = mimi_ring(rings, slot, layer, 0) + static_cast<size_t>(ring_slot) * kWidth;
    float* vr = mimi_ring(rings, slot, layer, 1) + static_cast<size_t>(ring_slot) * kWidth;
    *reinterpret_cast<float2*>(kr + 2 * t) = kp;
    *reinterpret_cast<float2*>(vr + 2 * t) = *reinterpret_cast<const float2*>(q + 2 * kWidth + 2 * t);
}

// Keys of a frame's window staged per (state, head): at most 250 + 15
// positions, rows padded to 68 floats (lanes reading different rows at the
// same column fall into different banks).
constexpr int kMimiWin = kMimiContext + kMimiRows - 1;
constexpr int kMimiKvStride = kHeadDim + 4;
constexpr int kMimiAttnSmem = (2 * kMimiWin * kMimiKvStride + kMimiRows * (kMimiContext + 2)) * 4;

// One CTA per (state, head), warp r = the frame's query row r
// (src/phonon_mimi.c:136-193): the head's K and V rows of every position the
// frame's 16 queries see are staged in shared memory once; then each warp
// scores its query against the keys of its window [first, p] (lane j takes
// keys j, j + 32, ...; each dot over the head's [even | odd] component order,
// as the reference's permuted GEMM operands), scale 1/8, max, e^(s - max) and
// their sum over the warp, then P.V with lane l owning dims 2l, 2l+1, and the
// output scaled by 1 / sum.
__global__ void __launch_bounds__(512, 1) mimi_attn_kernel(const float* __restrict__ qkv, const int32_t* __restrict__ slots,
                                                           const int32_t* __restrict__ pos0, const float* __restrict__ rings,
                                                           int layer, float* __restrict__ att, int32_t* status,
                                                           uint16_t* __restrict__ slices) {
    extern __shared__ __align__(16) float mimi_smem[];
    float* ks = mimi_smem;                                   // [kMimiWin][68]
    float* vs = ks + kMimiWin * kMimiKvStride;                // [kMimiWin][68]
    float* ps_all = vs + kMimiWin * kMimiKvStride;            // [16][252]
    __shared__ __align__(16) float qs[kMimiRows][kHeadDim];
    const int b = blockIdx.x / kHeads, head = blockIdx.x % kHeads;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_wait();
    pdl_trigger();
    const int p0 = pos0[b];
    const int win_first = p0 > kMimiContext - 1 ? p0 - (kMimiContext - 1) : 0;  // the first row's first key
    const int win_count = p0 + kMimiRows - win_first;                              // through the last row's key
    const float* kg = mimi_ring(const_cast<float*>(rings), slots[b], layer, 0) + head * kHeadDim;
    const float* vg = mimi_ring(const_cast<float*>(rings), slots[b], layer, 1) + head * kHeadDim;
    for (int i = threadIdx.x; i < win_count * (kHeadDim / 4); i += blockDim.x) {
        const int key = i / (kHeadDim / 4), c4 = i % (kHeadDim / 4);
        const size_t src = static_cast<size_t>((win_first + key) % kMimiRing) * kWidth + 4 * c4;
        *reinterpret_cast<float4*>(ks + key * kMimiKvStride + 4 * c4) = *reinterpret_cast<const float4*>(kg + src);
        *reinterpret_cast<float4*>(vs + key * kMimiKvStride + 4 * c4) = *reinterpret_cast<const float4*>(vg + src);
    }
    const int row = b * kMimiRows + warp;
    const float* q = qkv + static_cast<size_t>(row) * 3 * kWidth + head * kHeadDim;
    qs[warp][lane] = q[lane];
    qs[warp][lane + 32] = q[lane + 32];
    __syncthreads();
    const int position = p0 + warp;
    const int count = position < kMimiContext - 1 ? position + 1 : kMimiContext;
    const int first = position + 1 - count - win_first;  // the row's first key in the staged window
    float* ps = ps_all + warp * (kMimiContext + 2);
    float mx = -INFINITY;
    bool ok = true;
    for (int j = lane; j < count; j += 32) {
        const float* kr = ks + (first + j) * kMimiKvStride;
        float kv[kHeadDim];
#pragma unroll
        for (int i = 0; i < kHeadDim / 4; ++i) {
            const float4 f = *reinterpret_cast<const float4*>(kr + 4 * i);
            kv[4 * i] = f.x;
            kv[4 * i + 1] = f.y;
            kv[4 * i + 2] = f.z;
            kv[4 * i + 3] = f.w;
        }
        float dot = 0.0f;
#pragma unroll
        for (int parity = 0; parity < 2; ++parity)
#pragma unroll
            for (int i = 0; i < 32; ++i) dot = fmaf(qs[warp][2 * i + parity], kv[2 * i + parity], dot);
        const float s = __fmul_rn(dot, 0.125f);
        ok &= isfinite(s);
        ps[j] = s;
        mx = fmaxf(mx, s);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
    __syncwarp();
    float total = 0.0f;
    for (int j = lane; j < count; j += 32) {
        const float e = expf(__fsub_rn(ps[j], mx));
        ps[j] = e;
        total = __fadd_rn(total, e);
    }
    total = warp_sum(total);
    __syncwarp();
    float a0 = 0.0f, a1 = 0.0f;
#pragma unroll 4
    for (int j = 0; j < count; ++j) {
        const float2 v = *reinterpret_cast<const float2*>(vs + (first + j) * kMimiKvStride + 2 * lane);
        const float p = ps[j];
        a0 = fmaf(p, v.x, a0);
        a1 = fmaf(p, v.y, a1);
    }
    const float inv = __fdiv_rn(1.0f, total);
    const float o0 = __fmul_rn(a0, inv), o1 = __fmul_rn(a1, inv);
    ok &= total > 0.0f && isfinite(total) && isfinite(o0) && isfinite(o1);
    const int col = head * kHeadDim + 2 * lane;
    if (slices) {  // operand of the tensor-core out projection
        uint16_t a0s, a1s, a2s, b0s, b1s, b2s;
        bf16x3_split(o0, a0s, a1s, a2s);
        bf16x3_split(o1, b0s, b1s, b2s);
        uint16_t* dst = slices + static_cast<size_t>(3 * row) * kWidth + col;
        *reinterpret_cast<uint32_t*>(dst) = a0s | (static_cast<uint32_t>(b0s) << 16);
        *reinterpret_cast<uint32_t*>(dst + kWidth) = a1s | (static_cast<uint32_t>(b1s) << 16);
        *reinterpret_cast<uint32_t*>(dst + 2 * kWidth) = a2s | (static_cast<uint32_t>(b2s) << 16);
    } else {
        *reinterpret_cast<float2*>(att + static_cast<size_t>(row) * kWidth + col) = make_float2(o0, o1);
    }
    if (!__all_sync(kFull, ok) && lane == 0) flag_nonfinite(status, row);
}

}  // namespace phonon
