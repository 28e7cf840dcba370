// Whole-step persistent kernel for small batches (sm_100a).
//
// A decode step of a few streams is a chain of dependent, latency-bound
// stages: at one launch per stage the step costs several launch latencies
// per layer. Here one cooperative launch runs every layer of the step (the
// loop of phonon_flow_stack_step, speech-mac src/phonon_transformer.c:455-489).
// One CTA per SM stays resident; CTAs meet at grid barriers between the
// stages of a layer:
//
//   A  LN1 + QKV + RoPE + KV append   (src/phonon_transformer.c:414-431)
//   B  paged attention over balanced page chunks, one chunk per CTA, TMA
//      page staging as in attn_tma_kernel; writes per-split partials
//      (flow_attention, :340-404)
//   C  split merge + out projection + residual (:432-443)
//   D  LN2 + FFN up + GELU             (:444-447)
//   E  FFN down + residual             (:448-452)
//
// Work split: CTAs form ceil(R/8) groups. A group owns 8 streams (one per
// compute warp for the LayerNorms, which each CTA of the group computes for
// itself) and divides the rows of every projection, in RoPE pairs, among
// its CTAs. Warp 8 is a copy warp: it stages the CTA's weight rows (and the
// LayerNorm vectors) of the next projections in shared memory with bulk
// async copies (two buffers: QKV and up share one, out and down the other;
// QKV rows are staged during stage E, out and up rows at the start of stage
// C, down rows at the start of stage D), stages the GELU rows for stage E,
// and in stage B it is the TMA producer of the page ring, which then spans
// the activation region and both weight buffers. Row dot products and their epilogues use gemv_kernel's
// per-lane arithmetic and summation order; the attention partials use
// attn_tma_kernel's.
//
// Every wait (grid barrier, mbarrier) is bounded: on expiry it raises the
// context's error flag; once raised, every wait in the grid returns at once,
// the kernel runs to its end without issuing new copies, and the copy warp
// waits (bounded) for the copies it has in flight before the CTA exits.
#pragma once

#include "phonon_attention.cuh"

namespace phonon {

// Stage timestamps for profiling builds (-DPHONON_PERSIST_TRACE): thread 0
// of every CTA writes %globaltimer at marked points into
// g_persist_trace[(cta * 65 + layer) * 16 + slot]. Empty otherwise.
#ifdef PHONON_PERSIST_TRACE
__device__ unsigned long long* g_persist_trace;
#define PERSIST_MARK(layer, slot)                                                                   \
    do {                                                                                             \
        if (threadIdx.x == 0 && g_persist_trace) {                                                   \
            unsigned long long t_;                                                                   \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                   \
            g_persist_trace[(static_cast<size_t>(blockIdx.x) * 65 + (layer)) * 16 + (slot)] = t_;    \
        }                                                                                            \
    } while (0)
#else
#define PERSIST_MARK(layer, slot) \
    do {                          \
    } while (0)
#endif

constexpr int kPersistWarps = 8;                          // compute warps
constexpr int kPersistThreads = 32 * (kPersistWarps + 1);  // + copy warp
constexpr int kPersistGroup = 8;                          // streams per CTA group
constexpr int kPersistMaxBatch = 64;
constexpr int kPersistMinChunk = 4;                       // pages per attention chunk, at least
constexpr int kPersistNormBytes = 2 * kWidth * 4;         // LayerNorm weight + bias, fp32
constexpr long long kDrainBudgetCycles = 1ll << 28;       // ~0.14 s

// Page ring of stage B: one stage = the K and V blocks of one page; the
// number of stages (2..kPersistMaxRing) is what shared memory leaves after
// the weight buffers, chosen per launch.
constexpr int kPersistMaxRing = 6;
template <bool kBf16>
struct PersistAttn {
    static constexpr int kStageBytes = AttnTma<kBf16>::kStageBytes;
};

enum PersistMat : int { PM_QKV = 0, PM_OUT = 1, PM_UP = 2, PM_DOWN = 3 };

__host__ __device__ constexpr int persist_rows(int m) { return m == PM_QKV ? 1536 : (m == PM_UP ? 2048 : 512); }
__host__ __device__ constexpr int persist_cols(int m) { return m == PM_DOWN ? 2048 : 512; }
// Shared-memory bytes per weight row: int8 plane + binary16 block scales.
__host__ __device__ constexpr int persist_row_bytes(int m) { return persist_cols(m) + persist_cols(m) / 16; }
// Rows of matrix m held by one CTA of a group of nct CTAs (at most); rows go
// in quads (two RoPE pairs), the unit of one warp task.
__host__ __device__ constexpr int persist_cta_rows(int m, int nct) {
    return 4 * ((persist_rows(m) / 4 + nct - 1) / nct);
}

struct PersistLayer {
    const uint8_t* plane[4];   // qkv, out, up, down: lane-interleaved int8 rows
    const __half* scales[4];   // their Q8_0 block scales
    const float* norms;        // fp32 [4][512]: norm1 w, b, norm2 w, b
};

struct PersistParams {
    const PersistLayer* layers;
    int n_layers, R, S, U, n_groups;
    const float* in;           // [R][512]
    float* out;                // [R][512]
    float *xbuf0, *xbuf1, *h, *g, *q, *part;
    int32_t* status;           // [R]
    int32_t* error;            // context error flag
    unsigned* barrier;         // grid barrier counter (monotonic across launches)
    unsigned barrier_base;     // its value when this launch starts
    const int32_t *slot, *pos, *first, *count, *updates;
    const Split* splits;       // in (stream, page) order
    const int32_t* cta_split;  // [gridDim.x + 1]: CTA c runs splits [cta_split[c], cta_split[c+1])
    const float* freq;         // [32] RoPE inverse frequencies
    float2* rope;              // [R][32] (cos, sin), written in stage 0
    KvView kv;                 // kv.table is written in stage 0 (page updates)
    int off_x, off_w0, off_w1, off_norm, off_bar;  // shared-memory offsets from the 1024-aligned base
    int ring;                  // stage-B ring stages (2..kPersistMaxRing)
    float* trace;              // optional [n_layers][trace_rows][512]: every layer's output rows
    int trace_rows;
};

struct RowSlice {
    int row0, n_quads;
};

__device__ __forceinline__ RowSlice persist_slice(int m, int grank, int nct) {
    const int quads = persist_rows(m) / 4;
    const int per = (quads + nct - 1) / nct;
    const int q0 = grank * per;
    return RowSlice{4 * q0, max(0, min(per, quads - q0))};
}

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Drain wait of the copy warp: bounded, and independent of the failure flag.
__device__ __forceinline__ void mbar_drain(uint32_t bar, uint32_t parity) {
    const long long start = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - start > kDrainBudgetCycles) return;
}

// Grid barrier. Every CTA adds one to the counter (release); the k-th
// barrier of a launch completes when it reaches base + k * gridDim.x
// (wrap-safe compare, acquire). The failure flags are polled every 64 spins.
__device__ __forceinline__ void grid_sync_for(const PersistParams& p, unsigned& epoch, volatile int* failed,
                                              long long budget) {
    __syncthreads();
    epoch += gridDim.x;
    if (threadIdx.x == 0) {
        asm volatile("fence.acq_rel.gpu;" ::: "memory");
        atomicAdd(p.barrier, 1u);
        const unsigned target = p.barrier_base + epoch;
        const long long start = clock64();
        for (unsigned spin = 1; static_cast<int>(ld_acquire_gpu(p.barrier) - target) < 0; ++spin) {
            if ((spin & 63) != 0) continue;
            if (*failed || *reinterpret_cast<volatile int32_t*>(p.error)) {
                *failed = 1;
                break;
            }
            if (clock64() - start > budget) {
                *failed = 1;
                atomicExch(p.error, 1);
                break;
            }
        }
    }
    __syncthreads();
}

__device__ __forceinline__ void grid_sync(const PersistParams& p, unsigned& epoch, volatile int* failed) {
    grid_sync_for(p, epoch, failed, kWaitBudgetCycles);
}

// Expiry of the bounded waits, for tests: kind 0 waits on an mbarrier that
// nothing completes; kind 1 is a grid barrier that CTA 1 never reaches. Each
// wait gives up after `budget` cycles, raises *error and the kernel returns.
__global__ void wait_expiry_kernel(int kind, long long budget, int32_t* error, unsigned* counter) {
    __shared__ uint64_t bar;
    __shared__ int failed;
    if (threadIdx.x == 0) {
        mbar_init(smem_addr(&bar), 1);
        failed = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (kind == 0) {
        if (blockIdx.x == 0 && threadIdx.x == 0)
            mbar_wait_for(smem_addr(&bar), 0, error, reinterpret_cast<volatile int*>(&failed), budget);
        return;
    }
    if (blockIdx.x != 0) return;  // CTA 1 never arrives
    PersistParams p{};
    p.error = error;
    p.barrier = counter;
    p.barrier_base = 0;
    unsigned epoch = 0;
    grid_sync_for(p, epoch, reinterpret_cast<volatile int*>(&failed), budget);
}

// Stage rows rs of matrix m of layer L into `buf` (plane bytes, then
// scales); with norm_dst, also the LayerNorm vectors `norm` (w then b).
__device__ __forceinline__ void fill_weights(uint8_t* buf, uint32_t bar, const PersistLayer& L, int m, RowSlice rs,
                                             uint8_t* norm_dst, const float* norm) {
    const int cols = persist_cols(m);
    const uint32_t wbytes = static_cast<uint32_t>(rs.n_quads) * 4 * cols;
    const uint32_t sbytes = static_cast<uint32_t>(rs.n_quads) * 4 * (cols / 32) * 2;
    mbar_expect_tx(bar, wbytes + sbytes + (norm_dst ? kPersistNormBytes : 0));
    if (wbytes) {
        bulk_load(smem_addr(buf), L.plane[m] + static_cast<size_t>(rs.row0) * cols, wbytes, bar);
        bulk_load(smem_addr(buf + wbytes), L.scales[m] + static_cast<size_t>(rs.row0) * (cols / 32), sbytes, bar);
    }
    if (norm_dst) bulk_load(smem_addr(norm_dst), norm, kPersistNormBytes, bar);
}

// Sum over the warp of 32 per-lane values v[rr][bb] (rr < 4, bb < 8) by
// recursive halving: at each of the five levels (xor 16, 8, 4, 2, 1) a lane
// keeps half of its values and adds the partner's copy of them. The additions
// are those of a butterfly warp_sum of each value (same pairs, same levels),
// so the sums are the same to the bit; lane l ends with value (l >> 3, l & 7).
__device__ __forceinline__ float warp_reduce32(const float (&v)[4][kPersistGroup]) {
    const int lane = threadIdx.x & 31;
    float a[16], b[8], c[4], d[2];
    const bool u16 = lane & 16, u8 = lane & 8, u4 = lane & 4, u2 = lane & 2;
#pragma unroll
    for (int i = 0; i < 16; ++i) {  // value index i (+16): rr = i >> 3 (+2), bb = i & 7
        const float lo = v[i >> 3][i & 7], hi = v[2 + (i >> 3)][i & 7];
        a[i] = (u16 ? hi : lo) + __shfl_xor_sync(kFull, u16 ? lo : hi, 16);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) b[i] = (u8 ? a[i + 8] : a[i]) + __shfl_xor_sync(kFull, u8 ? a[i] : a[i + 8], 8);
#pragma unroll
    for (int i = 0; i < 4; ++i) c[i] = (u4 ? b[i + 4] : b[i]) + __shfl_xor_sync(kFull, u4 ? b[i] : b[i + 4], 4);
#pragma unroll
    for (int i = 0; i < 2; ++i) d[i] = (u2 ? c[i + 2] : c[i]) + __shfl_xor_sync(kFull, u2 ? c[i] : c[i + 2], 2);
    const bool u1 = lane & 1;
    return (u1 ? d[1] : d[0]) + __shfl_xor_sync(kFull, u1 ? d[0] : d[1], 1);
}

// Four signed int8 weights of a word as exact floats: each byte, offset by
// 128, is placed in the mantissa of 2^23 and the offset subtracted again.
__device__ __forceinline__ void i8x4_to_float(uint32_t word, float* f) {
    const uint32_t u = word ^ 0x80808080u;
#pragma unroll
    for (int e = 0; e < 4; ++e)
        f[e] = __uint_as_float(__byte_perm(u, 0x4B000000u, e | (4 << 4) | (5 << 8) | (7 << 12))) - 8388736.0f;
}

// The CTA's row quads of one projection against the group's streams: weights
// (rows rs.row0 ..) and activations xs[nb][cols] in shared memory. After the
// reduction lane l holds row r0 + (l >> 3) of stream b0 + (l & 7) and runs
// its epilogue (for RoPE the even row of a pair rotates both); the epilogue
// operands are loaded before the dot products so their latency overlaps them.
template <int kChunks, int kEpi>
__device__ __forceinline__ void persist_gemv(const PersistParams& p, int layer, const uint8_t* wb, RowSlice rs,
                                             const float* xs, int b0, int nb, const float* res, float* y, int ldy) {
    constexpr int cols = kChunks * 512;
    const __half* wsc = reinterpret_cast<const __half*>(wb + static_cast<size_t>(rs.n_quads) * 4 * cols);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int my_rr = lane >> 3, my_bb = lane & 7;
    const bool my_live = my_bb < nb;
    const int eb = b0 + min(my_bb, nb - 1);  // this lane's epilogue stream (clamped for idle lanes)
    for (int t = warp; t < rs.n_quads; t += kPersistWarps) {
        const int r0 = rs.row0 + 4 * t;
        const int my_r = r0 + my_rr;
        float pre = 0.0f;
        float2 cs = make_float2(1.0f, 0.0f);
        int page = 0;
        if constexpr (kEpi == EPI_RESID) pre = __ldcg(res + static_cast<size_t>(eb) * kWidth + my_r);
        if constexpr (kEpi == EPI_QKV) {
            const int region = r0 >> 9;
            if (region < 2) cs = __ldcg(p.rope + eb * 32 + ((my_r & 63) >> 1));
            if (region > 0)
                page = __ldcg(p.kv.table + static_cast<size_t>(p.slot[eb]) * p.kv.max_pages + p.pos[eb] / kPage);
        }
        float acc[4][kPersistGroup];
#pragma unroll
        for (int rr = 0; rr < 4; ++rr)
#pragma unroll
            for (int bb = 0; bb < kPersistGroup; ++bb) acc[rr][bb] = 0.0f;
#pragma unroll 1
        for (int c = 0; c < kChunks; ++c) {
            float wf[4][16], sc[4][4];
#pragma unroll
            for (int rr = 0; rr < 4; ++rr) {
                const int lr = 4 * t + rr;
                const uint4 wq = *reinterpret_cast<const uint4*>(wb + static_cast<size_t>(lr) * cols + c * 512 + lane * 16);
                const uint2 raw = *reinterpret_cast<const uint2*>(wsc + static_cast<size_t>(lr) * (cols / 32) + c * 16 +
                                                                  (lane >> 3) * 4);
                const __half2 h01 = *reinterpret_cast<const __half2*>(&raw.x);
                const __half2 h23 = *reinterpret_cast<const __half2*>(&raw.y);
                sc[rr][0] = __low2float(h01);
                sc[rr][1] = __high2float(h01);
                sc[rr][2] = __low2float(h23);
                sc[rr][3] = __high2float(h23);
                i8x4_to_float(wq.x, wf[rr] + 0);
                i8x4_to_float(wq.y, wf[rr] + 4);
                i8x4_to_float(wq.z, wf[rr] + 8);
                i8x4_to_float(wq.w, wf[rr] + 12);
            }
#pragma unroll
            for (int bb = 0; bb < kPersistGroup; ++bb) {
                if (bb < nb) {
                    const float* xr = xs + bb * cols + c * 512 + lane * 4;
                    float4 xv[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) xv[j] = *reinterpret_cast<const float4*>(xr + j * 128);
#pragma unroll
                    for (int rr = 0; rr < 4; ++rr) {
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            float part = wf[rr][j * 4 + 0] * xv[j].x;
                            part = fmaf(wf[rr][j * 4 + 1], xv[j].y, part);
                            part = fmaf(wf[rr][j * 4 + 2], xv[j].z, part);
                            part = fmaf(wf[rr][j * 4 + 3], xv[j].w, part);
                            acc[rr][bb] = fmaf(sc[rr][j], part, acc[rr][bb]);
                        }
                    }
                }
            }
        }
        float v = warp_reduce32(acc);  // (row r0 + my_rr, stream b0 + my_bb)
        const int b = b0 + my_bb;
        if constexpr (kEpi == EPI_QKV) {
            const float partner = __shfl_xor_sync(kFull, v, 8);  // the other row of this lane's RoPE pair
            if (!my_live || (my_rr & 1)) continue;
            const int region = r0 >> 9;  // 0 = q, 1 = k, 2 = v
            const int within = my_r & 511;
            float v0 = v, v1 = partner;
            if (region < 2) rope_apply(v0, v1, cs);
            if (!isfinite(v0) || !isfinite(v1)) flag_nonfinite(p.status, b);
            if (region == 0) {
                *reinterpret_cast<float2*>(p.q + static_cast<size_t>(b) * kWidth + within) = make_float2(v0, v1);
            } else {
                const int pos = p.pos[b];
                const long long off = kv_offset(p.kv, page, layer, region - 1, within >> 6, pos % kPage) + (within & 63);
                kv_store2(p.kv, off, v0, v1);
            }
        } else {
            if (!my_live) continue;
            if constexpr (kEpi == EPI_RESID) v = __fadd_rn(pre, v);
            if constexpr (kEpi == EPI_GELU) {
                if (!isfinite(v)) flag_nonfinite(p.status, b);
                v = gelu_erf(v);
            }
            if (!isfinite(v)) flag_nonfinite(p.status, b);
            y[static_cast<size_t>(b) * ldy + my_r] = v;
        }
    }
}

// Stage B: the CTA's chunk of pages, as splits [cta_split[c], cta_split[c+1])
// (one split per stream segment). The copy warp is the TMA producer of the
// page ring; warp h consumes head h and writes the split's partial
// (max, sum, acc[64]). The ring counter runs on across splits and layers
// (identical in all roles).
template <bool kBf16>
__device__ __forceinline__ void persist_attention(const CUtensorMap* tm, const PersistParams& p, int layer,
                                                  uint8_t* stages, uint32_t full0, uint32_t empty0, uint32_t& ring,
                                                  int* last_issue, volatile int* failed) {
    using A = PersistAttn<kBf16>;
    using T = AttnTma<kBf16>;
    const uint32_t kSt = static_cast<uint32_t>(p.ring);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int s_begin = p.cta_split[blockIdx.x], s_end = p.cta_split[blockIdx.x + 1];
    if (warp == kPersistWarps) {
        uint32_t n = ring;
        if (lane == 0) fence_proxy_async_global();  // KV appended in stage A
        for (int s = s_begin; s < s_end; ++s) {
            const Split sp = p.splits[s];
            const int32_t* table = p.kv.table + static_cast<size_t>(p.slot[sp.b]) * p.kv.max_pages;
            for (int i = 0; i < sp.page_count; ++i, ++n) {
                if (lane != 0 || *failed) continue;
                const int st = static_cast<int>(n % kSt);
                if (n >= kSt && !mbar_wait(empty0 + 8 * st, ((n / kSt) - 1) & 1, p.error, failed)) continue;
                const int page = __ldcg(table + sp.page_begin + i);
                const int row0 = (layer * p.kv.pool_pages + page) * 256;  // K block; V block follows
                uint8_t* stage = stages + st * A::kStageBytes;
                mbar_expect_tx(full0 + 8 * st, A::kStageBytes);
#pragma unroll
                for (int bx = 0; bx < T::kBoxes; ++bx) {
                    tma_load_2d(smem_addr(stage + bx * T::kBoxBytes), tm, bx * T::kBoxCols, row0, full0 + 8 * st);
                    tma_load_2d(smem_addr(stage + T::kBlockBytes + bx * T::kBoxBytes), tm, bx * T::kBoxCols, row0 + 128,
                                full0 + 8 * st);
                }
                last_issue[st] = static_cast<int>(n);
            }
        }
        __syncwarp();
        ring = n;
        return;
    }

    const int head = warp, half = lane >> 4;
    const AttnLane<kBf16> ad = attn_lane<kBf16>(head, lane);
    uint32_t n = ring;
    for (int s = s_begin; s < s_end; ++s) {
        const Split sp = p.splits[s];
        float qh[32];
        {
            const float4* qs = reinterpret_cast<const float4*>(p.q + static_cast<size_t>(sp.b) * kWidth +
                                                               head * kHeadDim + half * 32);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float4 v = __ldcg(qs + i);
                qh[4 * i] = v.x;
                qh[4 * i + 1] = v.y;
                qh[4 * i + 2] = v.z;
                qh[4 * i + 3] = v.w;
            }
        }
        float m = -INFINITY, l = 0.0f, a0 = 0.0f, a1 = 0.0f;
        bool finite_ok = true;
        for (int i = 0; i < sp.page_count; ++i, ++n) {
            const int st = static_cast<int>(n % kSt);
            const bool got = __all_sync(kFull, mbar_wait(full0 + 8 * st, (n / kSt) & 1, p.error, failed));
            if (got) {
                const uint8_t* sK = stages + st * A::kStageBytes;
                attn_page<kBf16>(sK, sK + T::kBlockBytes, ad, qh, (sp.page_begin + i) * kPage, sp.n_keys, m, l, a0,
                                 a1, finite_ok);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty0 + 8 * st);
        }
        float* out = p.part + (static_cast<size_t>(s) * kHeads + head) * kPartStride;
        *reinterpret_cast<float2*>(out + 2 + 2 * lane) = make_float2(a0, a1);
        if (lane == 0) {
            out[0] = m;
            out[1] = l;
        }
        if (!__all_sync(kFull, finite_ok) && lane == 0) flag_nonfinite(p.status, sp.b);
    }
    ring = n;
}

// Stage C prologue: merge the splits of every (stream, head) of the group
// into the attention output rows xs[nb][512] (merge_weights / merge_fold, in
// page order). Four threads per (stream, head), 16 dims each; partials are
// read four splits at a time.
__device__ __forceinline__ void persist_merge(const PersistParams& p, float* xs, int b0, int nb) {
    const int t = threadIdx.x, item = t >> 2, quarter = t & 3;
    if (item >= nb * kHeads) return;
    const int bb = item >> 3, head = item & 7, b = b0 + bb;
    const int first = p.first[b], cnt = p.count[b];
    float M = -INFINITY, S = 0.0f, acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = 0.0f;
    for (int k0 = 0; k0 < cnt; k0 += 4) {
        float pm[4], pl[4];
        float2 pa[4][8];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int k = min(k0 + u, cnt - 1);
            const float* pp = p.part + (static_cast<size_t>(first + k) * kHeads + head) * kPartStride;
            pm[u] = __ldcg(pp);
            pl[u] = __ldcg(pp + 1);
#pragma unroll
            for (int i = 0; i < 8; ++i) pa[u][i] = __ldcg(reinterpret_cast<const float2*>(pp + 2 + quarter * 16) + i);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            if (k0 + u >= cnt) break;
            const MergeWeights w = merge_weights(M, pm[u]);
            S = merge_fold(S, w, pl[u]);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                acc[2 * i] = merge_fold(acc[2 * i], w, pa[u][i].x);
                acc[2 * i + 1] = merge_fold(acc[2 * i + 1], w, pa[u][i].y);
            }
        }
    }
    bool ok = S > 0.0f && isfinite(S);
    const float inv = __fdiv_rn(1.0f, S);
    float* dst = xs + bb * kWidth + head * kHeadDim + quarter * 16;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const float o = __fmul_rn(acc[i], inv);
        ok &= isfinite(o);
        dst[i] = o;
    }
    if (!ok) flag_nonfinite(p.status, b);
}

template <bool kBf16>
__global__ void __launch_bounds__(kPersistThreads, 1)
    step_persist_kernel(const __grid_constant__ CUtensorMap tm_kv, const __grid_constant__ PersistParams p) {
    constexpr int kSt = kPersistMaxRing;  // mbarrier slots; p.ring of them are used
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* xs = reinterpret_cast<float*>(smem + p.off_x);
    uint8_t* stages = smem + p.off_x;  // stage B only; xs in the other stages
    uint8_t* wb[2] = {smem + p.off_w0, smem + p.off_w1};
    uint8_t* norm_s = smem + p.off_norm;
    const float* ln_w = reinterpret_cast<const float*>(norm_s);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.off_bar);
    const uint32_t full0 = smem_addr(bars), empty0 = full0 + 8 * kSt, wfull0 = full0 + 16 * kSt,
                   xfull = wfull0 + 16;
    volatile int* failed = reinterpret_cast<volatile int*>(bars + 2 * kSt + 3);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool copy_lane = warp == kPersistWarps && lane == 0;
    const int gi = blockIdx.x % p.n_groups, grank = blockIdx.x / p.n_groups;
    const int nct = (static_cast<int>(gridDim.x) - gi + p.n_groups - 1) / p.n_groups;
    const int b0 = gi * kPersistGroup, nb = min(kPersistGroup, p.R - b0);
    const RowSlice rs[4] = {persist_slice(PM_QKV, grank, nct), persist_slice(PM_OUT, grank, nct),
                            persist_slice(PM_UP, grank, nct), persist_slice(PM_DOWN, grank, nct)};

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.ring; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, kPersistWarps);
        }
        mbar_init(wfull0, 1);
        mbar_init(wfull0 + 8, 1);
        mbar_init(xfull, 1);
        *failed = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    uint32_t fills[2] = {0, 0};      // weight fills per buffer (same count in every thread)
    uint32_t issued[2] = {0, 0};     // fills the copy lane actually issued
    uint32_t xfills = 0, xissued = 0;
    int last_issue[kSt];             // copy lane: newest page-ring index per stage
#pragma unroll
    for (int s = 0; s < kSt; ++s) last_issue[s] = -1;
    uint32_t ring = 0;
    unsigned epoch = 0;
    // Buffer 0 holds QKV or up rows and the LayerNorm vectors in front of them.
    auto fill = [&](int k, int layer, int m) {
        if (warp == kPersistWarps) {
            if (lane == 0 && !*failed) {
                const PersistLayer L = p.layers[layer];
                const float* norm = m == PM_QKV ? L.norms : (m == PM_UP ? L.norms + 2 * kWidth : nullptr);
                fill_weights(wb[k], wfull0 + 8 * k, L, m, rs[m], norm ? norm_s : nullptr, norm);
                ++issued[k];
            }
            __syncwarp();
        }
        ++fills[k];
    };
    auto wait_fill = [&](int k) { mbar_wait(wfull0 + 8 * k, (fills[k] - 1) & 1, p.error, failed); };

    fill(0, 0, PM_QKV);

    // Stage 0: page-table updates and the step's RoPE table.
    {
        const int tid = blockIdx.x * blockDim.x + threadIdx.x, nt = gridDim.x * blockDim.x;
        if (blockIdx.x == 0)
            for (int i = threadIdx.x; i < p.U; i += blockDim.x)
                const_cast<int32_t*>(p.kv.table)[static_cast<size_t>(p.updates[3 * i]) * p.kv.max_pages +
                                                 p.updates[3 * i + 1]] = p.updates[3 * i + 2];
        for (int t = tid; t < p.R * 32; t += nt) {
            const float phase = __fmul_rn(static_cast<float>(p.pos[t >> 5]), p.freq[t & 31]);
            double sd, cd;
            sincos(static_cast<double>(phase), &sd, &cd);
            p.rope[t] = make_float2(__double2float_rn(cd), __double2float_rn(sd));
        }
    }
    grid_sync(p, epoch, failed);
    PERSIST_MARK(64, 0);

    for (int l = 0; l < p.n_layers; ++l) {
        const float* cur = l == 0 ? p.in : (((l - 1) & 1) ? p.xbuf1 : p.xbuf0);
        float* next = l == p.n_layers - 1 ? p.out : ((l & 1) ? p.xbuf1 : p.xbuf0);

        // A: LN1 -> QKV -> RoPE -> q, KV append
        if (warp < kPersistWarps) wait_fill(0);
        if (warp < nb) {
            const bool ok = warp_layernorm512<true>(cur + static_cast<size_t>(b0 + warp) * kWidth, ln_w, ln_w + kWidth,
                                                    xs + warp * kWidth);
            if (!ok && lane == 0 && grank == 0) flag_nonfinite(p.status, b0 + warp);
        }
        __syncthreads();
        PERSIST_MARK(l, 1);
        if (warp < kPersistWarps) persist_gemv<1, EPI_QKV>(p, l, wb[0], rs[PM_QKV], xs, b0, nb, nullptr, nullptr, 0);
        fence_proxy_async_global();  // KV stores before stage B's TMA reads
        PERSIST_MARK(l, 2);
        grid_sync(p, epoch, failed);
        PERSIST_MARK(l, 3);

        // B: attention partials. No weight copy is in flight now, so the
        // page ring may span both weight buffers as well.
        persist_attention<kBf16>(&tm_kv, p, l, stages, full0, empty0, ring, last_issue, failed);
        PERSIST_MARK(l, 4);
        grid_sync(p, epoch, failed);
        PERSIST_MARK(l, 5);

        // C: merge the splits, h = x + attn Wout^T (the out rows arrive while
        // the merge runs; the up rows are needed in D)
        fill(1, l, PM_OUT);
        fill(0, l, PM_UP);
        if (warp < kPersistWarps) persist_merge(p, xs, b0, nb);
        __syncthreads();
        PERSIST_MARK(l, 6);
        if (warp < kPersistWarps) {
            wait_fill(1);
            persist_gemv<1, EPI_RESID>(p, l, wb[1], rs[PM_OUT], xs, b0, nb, cur, p.h, kWidth);
        }
        PERSIST_MARK(l, 7);
        grid_sync(p, epoch, failed);
        PERSIST_MARK(l, 8);

        // D: g = GELU(LN2(h) Wup^T)
        fill(1, l, PM_DOWN);
        if (warp < kPersistWarps) wait_fill(0);
        if (warp < nb) {
            const bool ok = warp_layernorm512<true>(p.h + static_cast<size_t>(b0 + warp) * kWidth, ln_w, ln_w + kWidth,
                                                    xs + warp * kWidth);
            if (!ok && lane == 0 && grank == 0) flag_nonfinite(p.status, b0 + warp);
        }
        __syncthreads();
        PERSIST_MARK(l, 9);
        if (warp < kPersistWarps) persist_gemv<1, EPI_GELU>(p, l, wb[0], rs[PM_UP], xs, b0, nb, nullptr, p.g, kFfn);
        fence_proxy_async_global();  // GELU rows before stage E's bulk copy
        PERSIST_MARK(l, 10);
        grid_sync(p, epoch, failed);
        PERSIST_MARK(l, 11);

        // E: x' = h + g Wdown^T; the copy warp stages the group's GELU rows
        if (warp == kPersistWarps) {
            if (lane == 0 && !*failed) {
                fence_proxy_async_global();
                const uint32_t bytes = static_cast<uint32_t>(nb) * kFfn * 4;
                mbar_expect_tx(xfull, bytes);
                bulk_load(smem_addr(xs), p.g + static_cast<size_t>(b0) * kFfn, bytes, xfull);
                ++xissued;
            }
            __syncwarp();
        }
        ++xfills;
        if (l + 1 < p.n_layers) fill(0, l + 1, PM_QKV);
        if (warp < kPersistWarps) {
            mbar_wait(xfull, (xfills - 1) & 1, p.error, failed);
            wait_fill(1);
            PERSIST_MARK(l, 12);
            persist_gemv<4, EPI_RESID>(p, l, wb[1], rs[PM_DOWN], xs, b0, nb, p.h, next, kWidth);
        }
        PERSIST_MARK(l, 13);
        grid_sync(p, epoch, failed);
        PERSIST_MARK(l, 14);
        if (p.trace) {  // test instrumentation: this layer's output rows (written by other CTAs: via L2)
            float* dst = p.trace + static_cast<size_t>(l) * p.trace_rows * kWidth;
            for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < p.R * kWidth; i += gridDim.x * blockDim.x)
                dst[i] = __ldcg(next + i);
        }
    }

    // Copies still in flight (only after a failure) land before the CTA exits.
    if (copy_lane) {
        for (int s = 0; s < p.ring; ++s)
            if (last_issue[s] >= 0)
                mbar_drain(full0 + 8 * s, (static_cast<uint32_t>(last_issue[s]) / static_cast<uint32_t>(p.ring)) & 1);
        for (int k = 0; k < 2; ++k)
            if (issued[k] > 0) mbar_drain(wfull0 + 8 * k, (issued[k] - 1) & 1);
        if (xissued > 0) mbar_drain(xfull, (xissued - 1) & 1);
    }
}

}  // namespace phonon
