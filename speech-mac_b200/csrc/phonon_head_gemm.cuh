// The flow head's linears at large batches on the tcgen05 tensor cores.
//
// y[b][r] = sum_k W[r][k] x[b][k] + bias[r], K = 512, with bf16 weights W
// (exact MMA operands) and fp32 activations x split into three bf16 slices:
// s0 = bf16(x), s1 = bf16(x - s0), s2 = bf16(x - s0 - s1). Both differences
// are exact in fp32, and s0 + s1 + s2 holds x to its 24 bits (up to the last
// rounding of s2). Slice row 3b + j is operand B; one kind::f16 MMA chain
// (bf16 x bf16 products, exact, accumulated in fp32) gives
// D[r][3b + j] = sum_k W[r][k] s_j[b][k], and the epilogue adds the three
// columns, smallest slice first, then the bias.
//
// Tile: M = 128 weight rows x N = 96 slice rows (32 streams); K in 64-element
// (128-byte) SWIZZLE_128B tiles through a 3-deep TMA/mbarrier ring. Warp 0
// issues the TMA loads (no multicast), warp 1 allocates 128 TMEM columns and
// issues the MMAs, warps 2-9 drain TMEM (two per 32-lane quarter, 16 streams
// each). Every wait is bounded as in i8_gemm_kernel: on expiry the CTA
// raises the error flag, skips its stores and still frees its TMEM.
//
// Epilogues: HG_STORE y = acc + bias (fp32 rows); HG_GATE y = res + gate *
// (acc + bias) in place (the residual update of a head block, or a layer
// scale with a gate stride of 0); HG_SILU silu(acc + bias) and HG_GELU
// erf-GELU(acc + bias) written as the three slice rows of the next linear's
// operand B. K is 512 or 2048 (kK).
#pragma once

#include "phonon_gemm.cuh"

namespace phonon {

constexpr int kHgM = 128;
constexpr int kHgN = 96;           // slice rows per tile = 32 streams x 3
constexpr int kHgStreams = kHgN / 3;
constexpr int kHgK = 512;
constexpr int kHgKTile = 64;       // bf16 elements per stage row (128 bytes)
constexpr int kHgStages = 3;
constexpr int kHgThreads = 320;
constexpr int kHgTmemCols = 128;
constexpr int kHgStageBytes = (kHgM + kHgN) * kHgKTile * 2;
constexpr int kHgSmem = 1024 + kHgStages * kHgStageBytes + 256;

enum HeadGemmEpilogue : int { HG_STORE = 0, HG_GATE = 1, HG_SILU = 2, HG_GELU = 3 };

struct HeadGemmParams {
    int rows;               // weight rows (M)
    int B;                  // streams
    const float* bias;      // [rows]
    float* y;               // HG_STORE / HG_GATE: [B][ldy] (HG_GATE: also the residual)
    int ldy;
    const float* gate;      // HG_GATE: [B][ldgate]
    int ldgate;
    uint16_t* slices;       // HG_SILU, HG_GELU: [3 * Bpad][slice_ld] bf16 (the next linear's operand B)
    int slice_ld;
    int32_t* status;        // [B]
    int32_t* error;         // set when a bounded wait expires
};

// The three bf16 slices of x (see the header comment).
__device__ __forceinline__ void bf16x3_split(float x, uint16_t& s0, uint16_t& s1, uint16_t& s2) {
    s0 = f32_to_bf16(x);
    const float r1 = __fsub_rn(x, bf16_to_f32(s0));
    s1 = f32_to_bf16(r1);
    s2 = f32_to_bf16(__fsub_rn(r1, bf16_to_f32(s1)));
}

// kind::f16 instruction descriptor: f32 accumulator, bf16 A and B, both
// K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int m, int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
        : "memory");
}

// Eight consecutive accumulator columns of the warp's 32 lanes into r[o..o+7];
// complete after tmem_wait_ld().
template <int N>
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[N], int o) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[o]), "=r"(r[o + 1]), "=r"(r[o + 2]), "=r"(r[o + 3]), "=r"(r[o + 4]), "=r"(r[o + 5]),
                   "=r"(r[o + 6]), "=r"(r[o + 7])
                 : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

template <int kEpi, int kK = kHgK>
__global__ void __launch_bounds__(kHgThreads, 2)
    head_gemm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                     HeadGemmParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;                                        // [stages][128 rows][128 B]
    uint8_t* sB = smem + kHgStages * kHgM * kHgKTile * 2;      // [stages][96 rows][128 B]
    uint64_t* bars = reinterpret_cast<uint64_t*>(sB + kHgStages * kHgN * kHgKTile * 2);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kHgStages + 1);
    volatile int* failed = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const uint32_t full0 = smem_addr(bars), empty0 = full0 + 8 * kHgStages, accum = full0 + 16 * kHgStages;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m_tile = blockIdx.x, n_tile = blockIdx.y;
    constexpr int nk = kK / kHgKTile;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kHgStages; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        mbar_init(accum, 1);
        *failed = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(kHgTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // Weight tiles of the first stages do not depend on the previous
        // kernel: issue them before waiting for it.
        constexpr int pre = nk < kHgStages ? nk : kHgStages;
        for (int kt = 0; kt < pre; ++kt) {
            mbar_expect_tx(full0 + 8 * kt, kHgStageBytes);
            tma_load_2d(smem_addr(sA + kt * kHgM * kHgKTile * 2), &tm_w, kt * kHgKTile, m_tile * kHgM, full0 + 8 * kt);
        }
        pdl_wait();
        for (int kt = 0; kt < nk; ++kt) {
            const int s = kt % kHgStages;
            if (kt >= pre) {
                if (!mbar_wait(empty0 + 8 * s, ((kt / kHgStages) - 1) & 1, p.error, failed)) break;
                mbar_expect_tx(full0 + 8 * s, kHgStageBytes);
                tma_load_2d(smem_addr(sA + s * kHgM * kHgKTile * 2), &tm_w, kt * kHgKTile, m_tile * kHgM,
                            full0 + 8 * s);
            }
            tma_load_2d(smem_addr(sB + s * kHgN * kHgKTile * 2), &tm_x, kt * kHgKTile, n_tile * kHgN, full0 + 8 * s);
        }
    } else if (warp == 1 && lane == 0) {
        // four K = 16 steps (32 bytes) per 128-byte stage row
        constexpr uint32_t idesc = umma_idesc_bf16(kHgM, kHgN);
        bool ok = true;
        for (int kt = 0; kt < nk; ++kt) {
            const int s = kt % kHgStages;
            if (!mbar_wait(full0 + 8 * s, (kt / kHgStages) & 1, p.error, failed)) {
                ok = false;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t a0 = smem_addr(sA + s * kHgM * kHgKTile * 2);
            const uint32_t b0 = smem_addr(sB + s * kHgN * kHgKTile * 2);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
                umma_bf16(tmem, umma_desc_sw128(a0 + kk * 32), umma_desc_sw128(b0 + kk * 32), idesc, (kt | kk) != 0);
            umma_commit(empty0 + 8 * s);
        }
        if (ok) umma_commit(accum);
    } else if (warp >= 2) {
        // warp w drains TMEM lanes 32*(w%4) .. +31 (weight rows); warps 2-5
        // streams 0-15 of the tile (columns 0-47), warps 6-9 streams 16-31.
        constexpr int kHalf = kHgStreams / 2;
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;
        const int r = m_tile * kHgM + quarter * 32 + lane;
        const bool row_ok = r < p.rows;
        const int b0 = n_tile * kHgStreams + half * kHalf;
        pdl_wait();  // residuals and gates come from earlier kernels
        const float bias = row_ok ? p.bias[r] : 0.0f;
        float res[kHalf], gate[kHalf];
        if constexpr (kEpi == HG_GATE) {
#pragma unroll
            for (int t = 0; t < kHalf; ++t) {
                const int b = b0 + t;
                const bool live = row_ok && b < p.B;
                res[t] = live ? p.y[static_cast<size_t>(b) * p.ldy + r] : 0.0f;
                gate[t] = live ? p.gate[static_cast<size_t>(b) * p.ldgate + r] : 0.0f;
            }
        }
        const bool have = __all_sync(kFull, mbar_wait(accum, 0, p.error, failed));
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        pdl_trigger();
        if (have) {
            const uint32_t base = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + half * 48;
#pragma unroll
            for (int g = 0; g < 2; ++g) {  // 8 streams (24 columns) at a time keeps the registers in bounds
                uint32_t d[24];
                tmem_ld8(base + g * 24, d, 0);
                tmem_ld8(base + g * 24 + 8, d, 8);
                tmem_ld8(base + g * 24 + 16, d, 16);
                tmem_wait_ld();
#pragma unroll
                for (int t8 = 0; t8 < 8; ++t8) {
                    const int t = g * 8 + t8;
                    const int b = b0 + t;
                    float v = __fadd_rn(__fadd_rn(__uint_as_float(d[3 * t8 + 2]), __uint_as_float(d[3 * t8 + 1])),
                                        __uint_as_float(d[3 * t8]));
                    v = __fadd_rn(v, bias);
                    if constexpr (kEpi == HG_GATE) v = __fadd_rn(res[t], __fmul_rn(gate[t], v));
                    if constexpr (kEpi == HG_SILU) v = silu_f(v);
                    if constexpr (kEpi == HG_GELU) v = gelu_erf(v);
                    if (!row_ok || b >= p.B) continue;
                    if (!isfinite(v)) flag_nonfinite(p.status, b);
                    if constexpr (kEpi == HG_SILU || kEpi == HG_GELU) {
                        uint16_t s0, s1, s2;
                        bf16x3_split(v, s0, s1, s2);
                        uint16_t* row = p.slices + static_cast<size_t>(3 * b) * p.slice_ld + r;
                        row[0] = s0;
                        row[p.slice_ld] = s1;
                        row[2 * p.slice_ld] = s2;
                    } else {
                        p.y[static_cast<size_t>(b) * p.ldy + r] = v;
                    }
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kHgTmemCols) : "memory");
    }
}

// fp32 rows [B][ldx] (512 wide) -> slice rows 3b + j of `slices`, 128
// threads per row, 4 columns each.
__global__ void __launch_bounds__(128) slice_rows_kernel(const float* __restrict__ x, int ldx, int B,
                                                         uint16_t* __restrict__ slices) {
    const int b = blockIdx.x, t = threadIdx.x;
    pdl_wait();
    pdl_trigger();
    if (b >= B) return;
    const float4 v = *reinterpret_cast<const float4*>(x + static_cast<size_t>(b) * ldx + 4 * t);
    const float e[4] = {v.x, v.y, v.z, v.w};
    uint16_t s[3][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) bf16x3_split(e[i], s[0][i], s[1][i], s[2][i]);
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        uint2 w;
        w.x = static_cast<uint32_t>(s[j][0]) | (static_cast<uint32_t>(s[j][1]) << 16);
        w.y = static_cast<uint32_t>(s[j][2]) | (static_cast<uint32_t>(s[j][3]) << 16);
        *reinterpret_cast<uint2*>(slices + static_cast<size_t>(3 * b + j) * kHgK + 4 * t) = w;
    }
}

}  // namespace phonon
