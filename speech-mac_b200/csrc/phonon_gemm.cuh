// Batched projections on the 5th-generation tensor cores (sm_100a tcgen05).
//
// y[b][r] = s_r * sum_k x[b][k] * q[r][k] for B streams at once, with the
// weight rows r as the MMA M dimension and the streams as N.
//
// Activations become exact int8 data by digit slicing: each stream row x_b
// gets an exponent e_b (max|x_b| < 2^(e_b-1)) and four signed base-128
// digits d_j in [-64, 64] with x_b ~= 2^e_b * sum_j d_j * 2^(-7(j+1)); the
// residual is below 2^(e_b-29). Digit row 4b+j is operand B. One int8 MMA
// chain then yields D[r][4b+j] = sum_k q[r][k] * d_j[b][k] exactly in int32
// (|D| <= 2048 * 64 * 127 < 2^24, so it is also exact in fp32), and the
// epilogue recombines y = s_r * sum_j D[r][4b+j] * 2^(e_b - 7(j+1)).
//
// Per-block-scale Q8_0 (one fp16 scale per 32 weights, as real packs carry):
// with d_b = M_b 2^E_b (M_b the 11-bit integer significand) and E the row's
// largest E_b, the weights become integers W = q M_b 2^(E_b - E + 2) (exact
// for blocks within a factor 4 of the row's largest scale exponent, rounded
// to the nearest integer below that: an error below 2^-21 of the row's
// largest weight), |W| < 2^20, and the row scale is 2^(E - 2). W is split into
// three balanced base-128 digit planes w_0..w_2 (W = w_0 2^14 + w_1 2^7 + w_2,
// |w_i| <= 64), stacked as rows [i * rows, (i + 1) * rows) of operand A; the
// CTA runs one MMA chain per plane into its own 128 accumulator columns
// (kWD = 3, 512 TMEM columns), and the epilogue forms
// T_j = D_0j 2^14 + D_1j 2^7 + D_2j exactly in 64-bit integers before the
// recombination with the activation digits.
//
// Kernel shape: one CTA per 128-row x 32-stream tile (M = 128, N = 128 digit
// rows), 10 warps: warp 0 issues TMA tile loads (no multicast), warp 1 owns
// the TMEM accumulator and issues tcgen05.mma, warps 2-9 drain TMEM in the
// epilogue (two warps per 32-lane quarter, each half of the columns). K is
// staged in 128-byte tiles (SWIZZLE_128B) through a 3-deep mbarrier ring. Every mbarrier wait is bounded: on expiry the CTA raises the
// context's error flag, skips its remaining work and still frees its TMEM.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "phonon_kernels.cuh"

namespace phonon {

constexpr int kGemmM = 128;       // weight rows per tile (MMA M)
constexpr int kGemmN = 128;       // digit rows per tile (MMA N) = 32 streams x 4 slices
constexpr int kGemmKTile = 128;   // bytes of K per stage
constexpr int kGemmStages = 3;
constexpr int kGemmThreads = 320;  // producer, MMA issuer, 8 epilogue warps
constexpr int kGemmEpiThreads = kGemmThreads - 64;
constexpr int kGemmStreamsPerTile = kGemmN / 4;
constexpr int kDigits = 4;
// Per-tile stream data staged by the epilogue warps (exponents, pages, RoPE).
struct GemmTileMeta {
    int32_t exp[kGemmN / 4];
    int32_t pos[kGemmN / 4];
    int32_t page[kGemmN / 4];
    float2 cs[kGemmN / 4][32];
};
// Shared memory of a launch with kWD weight digit planes per tile (see below).
__host__ __device__ constexpr int gemm_smem(int wd) {
    return 1024 + kGemmStages * (wd * kGemmM + kGemmN) * kGemmKTile + 256 + static_cast<int>(sizeof(GemmTileMeta));
}
constexpr int kGemmSmem = gemm_smem(1);
constexpr long long kWaitBudgetCycles = 4ll << 30;  // ~2 s at 1.9 GHz

enum GemmEpilogue : int { GEPI_RAW = 0, GEPI_RESID = 1, GEPI_GELU = 2, GEPI_QKV = 3, GEPI_STORE = 4 };

// Phase timestamps for profiling builds (-DPHONON_GEMM_TRACE): one thread per
// role writes %globaltimer into g_gemm_trace[(cta * 8) + slot] for launches
// whose epilogue kind equals g_gemm_trace_kind (the last such launch wins;
// CTAs past kGemmTraceCtas write nothing). Empty otherwise.
#ifdef PHONON_GEMM_TRACE
constexpr unsigned kGemmTraceCtas = 4096;
__device__ unsigned long long* g_gemm_trace;
__device__ int g_gemm_trace_kind;
#define GEMM_MARK(slot)                                                                  \
    do {                                                                                \
        const unsigned cta_ = blockIdx.y * gridDim.x + blockIdx.x;                      \
        if (g_gemm_trace && g_gemm_trace_kind == kEpi && cta_ < kGemmTraceCtas) {       \
            unsigned long long t_;                                                      \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                      \
            g_gemm_trace[static_cast<size_t>(cta_) * 8 + (slot)] = t_;                  \
        }                                                                               \
    } while (0)
#else
#define GEMM_MARK(slot) \
    do {                \
    } while (0)
#endif

struct GemmParams {
    int rows;              // weight rows (M)
    int K;                 // bytes per row
    int B;                 // streams
    const float* row_scale;  // [rows] weight row scales
    const int32_t* exps;   // [B] e_b of the digit rows
    // outputs, as in GemvParams
    float* y;
    int ldy;
    const float* res;
    int ldres;
    float* q;
    const int32_t* slot;
    const int32_t* pos;
    const float2* rope;    // [B][32] per-step (cos, sin)
    KvView kv;
    int layer;
    int32_t* status;
    int32_t* raw;          // GEPI_RAW: D as [rows][n_total] int32
    int n_total;
    int32_t* error;        // set when a bounded wait expires
    const float* bias;     // GEPI_STORE: optional [rows]
};

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait: returns false (and raises *error) when `budget` clock cycles
// run out or another role of this CTA already failed.
__device__ __forceinline__ bool mbar_wait_for(uint32_t bar, uint32_t parity, int32_t* error,
                                              volatile int* cta_failed, long long budget) {
    if (mbar_try_wait(bar, parity)) return true;  // the common case: no clock read
    const long long start = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (*cta_failed) return false;
        if (clock64() - start > budget) {
            *cta_failed = 1;
            if (error) atomicExch(error, 1);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int32_t* error,
                                          volatile int* cta_failed) {
    return mbar_wait_for(bar, parity, error, cta_failed, kWaitBudgetCycles);
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

// L2 policy for data read once per step (K/V pages): evict first, so that
// the stream does not push weights, metadata and activations out of L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}

__device__ __forceinline__ void tma_load_2d_hint(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar,
                                                 uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4}], [%2], %5;"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "l"(policy)
        : "memory");
}

// K-major operand tile in SWIZZLE_128B form: 8-row atoms of 8 x 16 bytes,
// atoms 1024 bytes apart (stride byte offset 64 x 16), descriptor version 1.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t addr) {
    uint64_t d = (static_cast<uint64_t>(addr) >> 4) & 0x3FFFull;
    d |= static_cast<uint64_t>(1) << 16;                 // leading byte offset (unused when swizzled)
    d |= static_cast<uint64_t>(1024 >> 4) << 32;         // stride byte offset
    d |= static_cast<uint64_t>(1) << 46;                 // descriptor version (sm_100)
    d |= static_cast<uint64_t>(2) << 61;                 // SWIZZLE_128B
    return d;
}

// kind::i8 instruction descriptor: s32 accumulator, signed A and B, both
// K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t umma_idesc_i8(int m, int n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tmem_load32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ float pow2f(int e) {  // exact 2^e for normal exponents
    return __int_as_float((127 + e) << 23);
}

template <int kEpi, int kWD = 1>
__global__ void __launch_bounds__(kGemmThreads, kWD == 1 ? 2 : 1)
    i8_gemm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                   GemmParams p) {
    static_assert(kWD == 1 || kWD == 3, "one or three weight digit planes");
    constexpr int kStageA = kWD * kGemmM * kGemmKTile;            // bytes of the A planes of one stage
    constexpr uint32_t kTmemCols = kWD == 1 ? kGemmN : 512;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;                                           // [stages][kWD planes][128 rows][128 B]
    uint8_t* sB = smem + kGemmStages * kStageA;                   // [stages][128 rows][128 B]
    uint64_t* bars = reinterpret_cast<uint64_t*>(sB + kGemmStages * kGemmN * kGemmKTile);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kGemmStages + 1);
    volatile int* failed = reinterpret_cast<volatile int*>(tmem_slot + 1);
    GemmTileMeta* meta =
        reinterpret_cast<GemmTileMeta*>(smem + kGemmStages * (kStageA + kGemmN * kGemmKTile) + 256);
    const uint32_t full0 = smem_addr(bars), empty0 = full0 + 8 * kGemmStages, accum = full0 + 16 * kGemmStages;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m_tile = blockIdx.x, n_tile = blockIdx.y;
    const int nk = p.K / kGemmKTile;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kGemmStages; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        mbar_init(accum, 1);
        *failed = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    if (threadIdx.x == 0) GEMM_MARK(0);  // set up (barriers, TMEM)

    if (warp == 0 && lane == 0) {
        // TMA producer: weight tile rows [m_tile*128, +128), digit rows [n_tile*128, +128).
        // Weight tiles of the first stages do not depend on the previous
        // kernel: issue them before waiting for it.
        // Plane i of the weights is rows [i * p.rows, (i + 1) * p.rows) of tm_w.
        const int pre = nk < kGemmStages ? nk : kGemmStages;
        for (int kt = 0; kt < pre; ++kt) {
            mbar_expect_tx(full0 + 8 * kt, kStageA + kGemmN * kGemmKTile);
            for (int i = 0; i < kWD; ++i)
                tma_load_2d(smem_addr(sA + kt * kStageA + i * kGemmM * kGemmKTile), &tm_w, kt * kGemmKTile,
                            i * p.rows + m_tile * kGemmM, full0 + 8 * kt);
        }
        pdl_wait();
        GEMM_MARK(1);  // previous launch complete
        for (int kt = 0; kt < nk; ++kt) {
            const int s = kt % kGemmStages;
            if (kt >= pre) {
                if (!mbar_wait(empty0 + 8 * s, ((kt / kGemmStages) - 1) & 1, p.error, failed)) break;
                mbar_expect_tx(full0 + 8 * s, kStageA + kGemmN * kGemmKTile);
                for (int i = 0; i < kWD; ++i)
                    tma_load_2d(smem_addr(sA + s * kStageA + i * kGemmM * kGemmKTile), &tm_w, kt * kGemmKTile,
                                i * p.rows + m_tile * kGemmM, full0 + 8 * s);
            }
            tma_load_2d(smem_addr(sB + s * kGemmN * kGemmKTile), &tm_x, kt * kGemmKTile, n_tile * kGemmN,
                        full0 + 8 * s);
        }
    } else if (warp == 1 && lane == 0) {
        // MMA issuer: four K=32 steps per 128-byte stage.
        constexpr uint32_t idesc = umma_idesc_i8(kGemmM, kGemmN);
        bool ok = true;
        for (int kt = 0; kt < nk; ++kt) {
            const int s = kt % kGemmStages;
            if (!mbar_wait(full0 + 8 * s, (kt / kGemmStages) & 1, p.error, failed)) {
                ok = false;
                break;
            }
            if (kt == 0) GEMM_MARK(2);  // first stage landed
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t a0 = smem_addr(sA + s * kStageA);
            const uint32_t b0 = smem_addr(sB + s * kGemmN * kGemmKTile);
#pragma unroll
            for (int i = 0; i < kWD; ++i)
#pragma unroll
                for (int kk = 0; kk < kGemmKTile / 32; ++kk)
                    umma_i8(tmem + i * kGemmN, umma_desc_sw128(a0 + i * kGemmM * kGemmKTile + kk * 32),
                            umma_desc_sw128(b0 + kk * 32), idesc, (kt | kk) != 0);
            umma_commit(empty0 + 8 * s);
        }
        if (ok) umma_commit(accum);
        GEMM_MARK(3);  // all MMAs issued
    } else if (warp >= 2) {
        // Epilogue: warp w reads TMEM lanes 32*(w%4) .. +31 = weight rows;
        // warps 2-5 drain accumulator columns 0-63 (streams 0-15 of the
        // tile), warps 6-9 columns 64-127 (streams 16-31). While the MMAs
        // run, stage this tile's per-stream data in shared memory and
        // prefetch the residual, so that draining the accumulator issues no
        // dependent global loads.
        constexpr int kHalf = kGemmStreamsPerTile / 2;
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;
        const int r = m_tile * kGemmM + quarter * 32 + lane;
        const int et = threadIdx.x - 64;  // 0..255 over the epilogue warps
        const int b0 = n_tile * kGemmStreamsPerTile;
        pdl_wait();  // exponents, residuals and positions come from earlier kernels
        if constexpr (kEpi != GEPI_RAW) {
            if (et < kGemmStreamsPerTile) {
                const int b = b0 + et;
                const bool live = b < p.B;
                meta->exp[et] = live ? p.exps[b] : 0;
                if constexpr (kEpi == GEPI_QKV) {
                    const int position = live ? p.pos[b] : 0;
                    meta->pos[et] = position;
                    meta->page[et] = live ? p.kv.table[static_cast<size_t>(p.slot[b]) * p.kv.max_pages + position / kPage] : 0;
                }
            }
            if constexpr (kEpi == GEPI_QKV) {
                constexpr int kPer = kGemmStreamsPerTile * 32 / kGemmEpiThreads;
                float2 cs[kPer];
#pragma unroll
                for (int k = 0; k < kPer; ++k) {  // independent loads, then the stores
                    const int i = et + k * kGemmEpiThreads;
                    const int b = b0 + i / 32;
                    cs[k] = b < p.B ? p.rope[b * 32 + (i % 32)] : make_float2(1.0f, 0.0f);
                }
#pragma unroll
                for (int k = 0; k < kPer; ++k) {
                    const int i = et + k * kGemmEpiThreads;
                    meta->cs[i / 32][i % 32] = cs[k];
                }
            }
            asm volatile("bar.sync 1, %0;" ::"n"(kGemmEpiThreads) : "memory");
        }
        float res[kHalf];
        if constexpr (kEpi == GEPI_RESID) {
#pragma unroll
            for (int t = 0; t < kHalf; ++t) {
                const int b = b0 + half * kHalf + t;
                res[t] = (b < p.B && r < p.rows) ? p.res[static_cast<size_t>(b) * p.ldres + r] : 0.0f;
            }
        }
        const float scale = (kEpi == GEPI_RAW || r >= p.rows) ? 1.0f : p.row_scale[r];
        if (et == 0) GEMM_MARK(4);  // epilogue staged, waiting for the accumulator
        const bool have = __all_sync(kFull, mbar_wait(accum, 0, p.error, failed));
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (et == 0) GEMM_MARK(5);  // accumulator ready
        pdl_trigger();
        if (have) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int c0 = half * (kGemmN / 2) + h * 32;
                uint32_t d[32];
                tmem_load32(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + c0, d);
                uint32_t d1[kWD == 3 ? 32 : 1], d2[kWD == 3 ? 32 : 1];
                if constexpr (kWD == 3) {
                    tmem_load32(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + kGemmN + c0, d1);
                    tmem_load32(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + 2 * kGemmN + c0, d2);
                }
                if constexpr (kEpi == GEPI_RAW) {
                    if (r < p.rows)
                        for (int i = 0; i < 32; ++i) {
                            const int n = n_tile * kGemmN + c0 + i;
                            if (n < p.n_total) p.raw[static_cast<size_t>(r) * p.n_total + n] = static_cast<int32_t>(d[i]);
                        }
                } else {
                    // 8 streams per 32 columns: recombine the four digit slices.
                    // Values of padded streams and rows are computed (from zero
                    // digits) and not stored, keeping the 8 chains branch-free.
                    float v[8];
#pragma unroll
                    for (int t = 0; t < 8; ++t) {
                        const int e = meta->exp[(c0 >> 2) + t];
                        float acc = 0.0f;
#pragma unroll
                        for (int j = 0; j < kDigits; ++j) {
                            float dj;
                            if constexpr (kWD == 3) {
                                const long long T = (static_cast<long long>(static_cast<int32_t>(d[4 * t + j])) << 14) +
                                                    (static_cast<long long>(static_cast<int32_t>(d1[4 * t + j])) << 7) +
                                                    static_cast<long long>(static_cast<int32_t>(d2[4 * t + j]));
                                dj = __ll2float_rn(T);
                            } else {
                                dj = static_cast<float>(static_cast<int32_t>(d[4 * t + j]));
                            }
                            acc = fmaf(dj, pow2f(e - 7 * (j + 1)), acc);
                        }
                        v[t] = acc * scale;
                    }
                    if constexpr (kEpi == GEPI_QKV) {
                        const int region = r >> 9, within = r & 511;
#pragma unroll
                        for (int t = 0; t < 8; ++t) {
                            // rows r (even lane) and r+1 (odd lane) form a RoPE pair
                            const int tt = (c0 >> 2) + t;
                            const float other = __shfl_xor_sync(kFull, v[t], 1);
                            float a = (lane & 1) ? other : v[t], bb = (lane & 1) ? v[t] : other;
                            if (region < 2) rope_apply(a, bb, meta->cs[tt][(within & 63) >> 1]);
                            v[t] = (lane & 1) ? bb : a;
                        }
                        if (r < p.rows) {
#pragma unroll
                            for (int t = 0; t < 8; ++t) {
                                const int tt = (c0 >> 2) + t;
                                const int b = b0 + tt;
                                if (b >= p.B) break;
                                if (!isfinite(v[t])) flag_nonfinite(p.status, b);
                                if (region == 0) {
                                    p.q[static_cast<size_t>(b) * kWidth + within] = v[t];
                                } else {
                                    const long long off = kv_offset(p.kv, meta->page[tt], p.layer, region - 1, within >> 6,
                                                                    meta->pos[tt] % kPage) + (within & 63);
                                    if (p.kv.bf16) static_cast<uint16_t*>(p.kv.pool)[off] = f32_to_bf16(v[t]);
                                    else static_cast<float*>(p.kv.pool)[off] = v[t];
                                }
                            }
                        }
                    } else {
#pragma unroll
                        for (int t = 0; t < 8; ++t) {
                            if constexpr (kEpi == GEPI_RESID) v[t] = __fadd_rn(res[h * 8 + t], v[t]);
                            if constexpr (kEpi == GEPI_STORE) {
                                if (p.bias && r < p.rows) v[t] = __fadd_rn(v[t], p.bias[r]);
                            }
                            if constexpr (kEpi == GEPI_GELU) v[t] = gelu_erf(v[t]);
                        }
                        if (r < p.rows) {
#pragma unroll
                            for (int t = 0; t < 8; ++t) {
                                const int b = b0 + (c0 >> 2) + t;
                                if (b >= p.B) break;
                                // GELU keeps non-finite inputs non-finite, so the check after it also covers them
                                if (!isfinite(v[t])) flag_nonfinite(p.status, b);
                                p.y[static_cast<size_t>(b) * p.ldy + r] = v[t];
                            }
                        }
                    }
                }
            }
        }
    }
    if (threadIdx.x == 64) GEMM_MARK(6);  // first epilogue warp done
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
    if (threadIdx.x == 0) GEMM_MARK(7);  // CTA end
}

// Exponent e of a row whose largest magnitude is mx: |x| * 2^-e < 1/2.
// Rows below 2^-91 get e = 0 and all-zero digits (keeps every 2^(e-28) a
// normal float).
__device__ __forceinline__ int digit_exponent(float mx, bool& zero) {
    int e = 0;
    frexpf(mx, &e);
    e += 1;
    zero = !(mx > 0.0f) || e < -90;
    return zero ? 0 : e;
}

// Four base-128 digits of r = x * 2^-e (|r| < 1/2), packed little-endian.
__device__ __forceinline__ uint32_t slice_digits(float r) {
    uint32_t packed = 0;
#pragma unroll
    for (int j = 0; j < kDigits; ++j) {
        r *= 128.0f;
        const float dj = rintf(r);
        r -= dj;  // exact: the fractional part of r
        packed |= (static_cast<uint32_t>(static_cast<int32_t>(dj)) & 0xffu) << (8 * j);
    }
    return packed;
}

// One head's share of the split merge of a stream (warp = head): the
// stream's splits folded in page order like attn_combine_kernel; lane l holds
// output dims 2l, 2l+1. ok: finite, with a positive sum. Loads go to L2 (the
// partials may have been written by other SMs).
struct HeadMerge {
    float o0, o1;
    bool ok;
};

__device__ __forceinline__ HeadMerge merge_head(const float* part, int first, int n, int head, int lane) {
    constexpr int kBatch = 8;  // splits whose loads are in flight together
    float M = -INFINITY, total = 0.0f, a0 = 0.0f, a1 = 0.0f;
    for (int s0 = 0; s0 < n; s0 += kBatch) {
        float pm[kBatch], pl[kBatch];
        float2 av[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            if (s0 + j < n) {
                const float* pp = part + (static_cast<size_t>(first + s0 + j) * kHeads + head) * kPartStride;
                pm[j] = __ldcg(pp);
                pl[j] = __ldcg(pp + 1);
                av[j] = __ldcg(reinterpret_cast<const float2*>(pp + 2 + 2 * lane));
            }
        }
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            if (s0 + j < n) {
                const MergeWeights w = merge_weights(M, pm[j]);
                total = merge_fold(total, w, pl[j]);
                a0 = merge_fold(a0, w, av[j].x);
                a1 = merge_fold(a1, w, av[j].y);
            }
        }
    }
    HeadMerge h;
    h.ok = total > 0.0f && isfinite(total);
    const float inv = __fdiv_rn(1.0f, total);
    h.o0 = __fmul_rn(a0, inv);
    h.o1 = __fmul_rn(a1, inv);
    h.ok &= isfinite(h.o0) && isfinite(h.o1);
    return h;
}

// Largest output magnitude of the head over the warp (0 for lanes not ok).
__device__ __forceinline__ float head_abs_max(const HeadMerge& h) {
    float m = h.ok ? fmaxf(fabsf(h.o0), fabsf(h.o1)) : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, o));
    return m;
}

// The head's two dims per lane of the stream's four digit rows (drow points
// at row 4b, dim head*64 + 2*lane), for a row whose largest magnitude is
// row_max; returns the row exponent e_b.
__device__ __forceinline__ int write_head_digits(const HeadMerge& h, float row_max, int8_t* drow) {
    bool zero;
    const int e = digit_exponent(row_max, zero);
    const float down = pow2f(-e);
    const uint32_t d0 = (zero || !h.ok) ? 0u : slice_digits(h.o0 * down);
    const uint32_t d1 = (zero || !h.ok) ? 0u : slice_digits(h.o1 * down);
#pragma unroll
    for (int j = 0; j < kDigits; ++j)
        *reinterpret_cast<uint16_t*>(drow + j * kWidth) =
            static_cast<uint16_t>(((d0 >> (8 * j)) & 0xffu) | (((d1 >> (8 * j)) & 0xffu) << 8));
    return e;
}

// Attention combine fused with digit slicing (tensor-core path when attention
// runs without the TMA page ring): one CTA per stream (8 warps = 8 heads)
// merges the head's splits like attn_combine_kernel, then the CTA takes the
// row maximum over all 512 outputs and writes the stream's four digit rows
// and exponent. CTAs for padded streams write zeros.
__global__ void __launch_bounds__(256) attn_combine_digits_kernel(CombineParams p, int Bpad, int8_t* __restrict__ digits,
                                                                  int32_t* __restrict__ exps) {
    __shared__ float head_max[kHeads];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.x, head = warp;
    pdl_wait();
    pdl_trigger();
    int8_t* drow = digits + static_cast<size_t>(4 * b) * kWidth + head * kHeadDim + 2 * lane;
    if (b >= p.B) {
#pragma unroll
        for (int j = 0; j < kDigits; ++j) *reinterpret_cast<uint16_t*>(drow + j * kWidth) = 0;
        if (threadIdx.x == 0) exps[b] = 0;
        return;
    }
    const HeadMerge h = merge_head(p.part, p.first[b], p.count[b], head, lane);
    if (!__all_sync(kFull, h.ok) && lane == 0) flag_nonfinite(p.status, b);
    const float m = head_abs_max(h);
    if (lane == 0) head_max[head] = m;
    __syncthreads();
    float row_max = 0.0f;
#pragma unroll
    for (int hh = 0; hh < kHeads; ++hh) row_max = fmaxf(row_max, head_max[hh]);
    const int e = write_head_digits(h, row_max, drow);
    if (threadIdx.x == 0) exps[b] = e;
}

// LayerNorm then digit slicing (see the header comment), one warp per stream
// row of 512: the row is layer-normalised exactly as in warp_layernorm512,
// then sliced. Writes digit rows 4b..4b+3 and e_b; rows of streams B..Bpad-1
// are zeroed so that padded tiles multiply zeros.
__global__ void __launch_bounds__(256) ln_digits_kernel(const float* __restrict__ x, int ldx, const float* ln_w,
                                                        const float* ln_b, int B, int Bpad, int8_t* __restrict__ digits,
                                                        int32_t* __restrict__ exps, int32_t* status) {
    constexpr int kCols = kWidth;
    __shared__ __align__(16) float row[8][kCols];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.x * 8 + warp;
    if (b >= Bpad) return;
    constexpr int per_lane = kCols / 32;
    if (b >= B) {
        for (int j = 0; j < kDigits; ++j)
            for (int i = lane * 16; i < kCols; i += 32 * 16)
                *reinterpret_cast<int4*>(digits + (static_cast<size_t>(4 * b + j)) * kCols + i) = make_int4(0, 0, 0, 0);
        if (lane == 0) exps[b] = 0;
        return;
    }
    const bool ok = warp_layernorm512(x + static_cast<size_t>(b) * ldx, ln_w, ln_b, row[warp]);
    if (!ok && lane == 0) flag_nonfinite(status, b);
    __syncwarp();
    const float* src = row[warp];
    // lane owns columns lane*4 + 128*i .. +3 (i < per_lane/4): float4 reads
    float v[per_lane];
#pragma unroll
    for (int i = 0; i < per_lane / 4; ++i) {
        const float4 f = *reinterpret_cast<const float4*>(src + i * 128 + lane * 4);
        v[4 * i] = f.x;
        v[4 * i + 1] = f.y;
        v[4 * i + 2] = f.z;
        v[4 * i + 3] = f.w;
    }
    float mx = 0.0f;
    bool finite_ok = true;
#pragma unroll
    for (int i = 0; i < per_lane; ++i) {
        finite_ok &= isfinite(v[i]);
        mx = fmaxf(mx, fabsf(v[i]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
    if (!__all_sync(kFull, finite_ok)) {
        if (lane == 0) flag_nonfinite(status, b);
        mx = 0.0f;
    }
    bool zero;
    const int e = digit_exponent(mx, zero);
    const float down = pow2f(-e);
    uint32_t packed[kDigits][per_lane / 4];
#pragma unroll
    for (int i = 0; i < per_lane / 4; ++i)
#pragma unroll
        for (int j = 0; j < kDigits; ++j) packed[j][i] = 0;
#pragma unroll
    for (int i = 0; i < per_lane; ++i) {
        // exact scaling by a power of two, then the four digits
        const uint32_t d = (finite_ok && !zero) ? slice_digits(v[i] * down) : 0u;
#pragma unroll
        for (int j = 0; j < kDigits; ++j) packed[j][i / 4] |= ((d >> (8 * j)) & 0xffu) << (8 * (i % 4));
    }
#pragma unroll
    for (int j = 0; j < kDigits; ++j)
#pragma unroll
        for (int i = 0; i < per_lane / 4; ++i)
            *reinterpret_cast<uint32_t*>(digits + static_cast<size_t>(4 * b + j) * kCols + i * 128 + lane * 4) =
                packed[j][i];
    if (lane == 0) exps[b] = e;
}

// Digit slicing of rows of width kCols (no LayerNorm): kCols/8 threads per
// stream row, 8 consecutive columns each, the row maximum reduced across the
// row's warps through shared memory. A row holding a non-finite value is
// flagged and gets all-zero digits and e_b = 0, as do the padded rows
// B..Bpad-1.
template <int kCols>
__global__ void __launch_bounds__(256) digits_kernel(const float* __restrict__ x, int ldx, int B, int Bpad,
                                                     int8_t* __restrict__ digits, int32_t* __restrict__ exps,
                                                     int32_t* status) {
    constexpr int kRowThreads = kCols / 8;
    constexpr int kRows = 256 / kRowThreads;  // stream rows per CTA
    constexpr int kRowWarps = kRowThreads / 32;
    static_assert(kRowWarps >= 1 && kRows * kRowThreads == 256, "kCols must be 256..2048");
    __shared__ float warp_max[8];
    __shared__ int warp_bad[8];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rt = threadIdx.x % kRowThreads;
    const int b = blockIdx.x * kRows + threadIdx.x / kRowThreads;
    pdl_wait();
    pdl_trigger();
    float v[8];
    if (b < B) {
        const float4* src = reinterpret_cast<const float4*>(x + static_cast<size_t>(b) * ldx + rt * 8);
        const float4 f0 = src[0], f1 = src[1];
        v[0] = f0.x, v[1] = f0.y, v[2] = f0.z, v[3] = f0.w;
        v[4] = f1.x, v[5] = f1.y, v[6] = f1.z, v[7] = f1.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.0f;
    }
    float mx = 0.0f;
    bool finite_ok = true;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        finite_ok &= isfinite(v[i]);
        mx = fmaxf(mx, fabsf(v[i]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
    finite_ok = __all_sync(kFull, finite_ok);
    if (lane == 0) {
        warp_max[warp] = mx;
        warp_bad[warp] = !finite_ok;
    }
    __syncthreads();
    const int w0 = (threadIdx.x / kRowThreads) * kRowWarps;
    bool bad = false;
#pragma unroll
    for (int w = 0; w < kRowWarps; ++w) {
        mx = fmaxf(mx, warp_max[w0 + w]);
        bad |= warp_bad[w0 + w] != 0;
    }
    if (b >= Bpad) return;
    if (bad) {
        if (rt == 0) flag_nonfinite(status, b);
        mx = 0.0f;
    }
    bool zero;
    const int e = digit_exponent(mx, zero);
    const float down = pow2f(-e);
    uint32_t lo[kDigits], hi[kDigits];
#pragma unroll
    for (int j = 0; j < kDigits; ++j) lo[j] = hi[j] = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        // exact scaling by a power of two, then the four digits
        const uint32_t d = zero ? 0u : slice_digits(v[i] * down);
#pragma unroll
        for (int j = 0; j < kDigits; ++j) {
            const uint32_t byte = ((d >> (8 * j)) & 0xffu) << (8 * (i % 4));
            if (i < 4) lo[j] |= byte;
            else hi[j] |= byte;
        }
    }
#pragma unroll
    for (int j = 0; j < kDigits; ++j)
        *reinterpret_cast<uint2*>(digits + static_cast<size_t>(4 * b + j) * kCols + rt * 8) = make_uint2(lo[j], hi[j]);
    if (rt == 0) exps[b] = e;
}

}  // namespace phonon
