// Single-stream decode step on one thread-block cluster (sm_100a).
//
// A decode step of one stream is a chain of ~60 dependent stages whose work
// is small (a 512-wide LayerNorm, a few hundred GEMV rows, attention over a
// few hundred keys per head): its time is the latency of the chain, not the
// ~50 MB of traffic. Here one cluster of 16 CTAs (one per SM) runs every
// layer of the step (the loop of phonon_flow_stack_step, speech-mac
// src/phonon_transformer.c:455-489) without kernel boundaries, grid barriers
// or cluster barriers between stages. CTA `rank` serves head rank / 2,
// half rank % 2:
//
//   A  LN1 of x (each CTA) -> the head's 64 q rows and the k and v rows of
//      dims [32*half, +32); RoPE; k and v appended to the stream's KV page
//      (src/phonon_transformer.c:414-431)
//   B  attention of q over the keys of this CTA's half of the stream's
//      earlier pages (TMA page staging, the page math of the other paths);
//      the current position's key is not read back from the page: each CTA
//      contributes its half of q.k and its half of v, and the key joins the
//      softmax as one more term of the merge (flow_attention, :340-404)
//   C  every CTA merges, per head, the two CTA partials and the current key
//      into the attention row; out rows [32*rank, +32) + residual -> h
//      (:432-443)
//   D  LN2 (each CTA) -> up rows [128*rank, +128) + GELU -> g (:444-447)
//   E  down rows [32*rank, +32) + residual -> x' (:448-452)
//
// Exchanges: every stage output a CTA produces (its attention message, and
// its slices of h, g and x') is pushed into the same buffer of all 16 CTAs
// with st.async, which completes the bytes on that buffer's mbarrier in the
// receiving CTA; a CTA waits on its own mbarrier for exactly the bytes its
// next stage reads. One DSMEM hop per exchange, four per layer, and no
// release fences: the stores complete on the receiver's barrier. Every
// exchange buffer is single-buffered: a CTA can only produce layer l+1's data
// for a buffer after it received data that every other CTA sends after it
// has finished reading that buffer for layer l (the chain is A..E in order),
// and each buffer's barrier completes exactly one phase per layer.
//
// Warp 8 is the copy warp. It streams, in the order the compute
// warps consume them, the CTA's weight rows through a ring of 17 KB slots
// (32 rows of a 512-column matrix or 8 rows of the 2048-column one, with
// their Q8_0 scales), the LayerNorm vectors through a two-slot ring and its
// head's K/V blocks of the stream's earlier pages through an eight-slot page
// ring (TMA, 16-row SWIZZLE_128B boxes), each as soon as the slot it refills
// is released; the first eight pages of a layer go out right after the
// previous layer's out unit. No page read waits for this step's append. Most copies are
// issued several microseconds before their data is read; the two that are
// not (the next layer's v unit, whose slot frees at the end of a layer, and
// the last down unit, whose slot frees in stage D) are prefetched into L2 a
// layer ahead (cp.async.bulk.prefetch.L2). Prefetching more costs more than
// it saves: prefetches queue in the SM's bulk-copy unit ahead of the ring's
// copies (the whole step's weights prefetched at launch, ~3 MB per CTA, held
// the first layer back ~20 us; a layer ahead, the attention pages ~3 us).
//
// Code size: the LayerNorm, the row dot products and the attention page are
// each one non-inlined routine, so the ~60 stages of a step run through a
// small, hot instruction footprint.
//
// Numerics: the LayerNorm, the row dot products (gemv_kernel's per-lane fp32
// accumulation and butterfly sum), RoPE, GELU and residuals are those of the
// other step paths, so projections and appended K/V rows are bit-identical
// to them; the attention partials merge in another order (pages split
// between two CTAs and eight warps, the current key last), which changes
// sums within rounding.
//
// Every mbarrier wait is bounded: on expiry the CTA raises the context's
// error flag and skips the rest of its work (its waits return at once); it
// still takes the final cluster barrier, so no CTA exits while another could
// still store into its shared memory, and the copy warp waits (bounded) for
// its copies in flight first. No multicast.
#pragma once

#include "phonon_persist.cuh"

namespace phonon {

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Phase timestamps for profiling builds (-DPHONON_CLUSTER_TRACE): thread 0
// (CL_MARK_T: the given thread) of every CTA writes %globaltimer at marked points into
// g_cluster_trace[(rank * 64 + layer) * 32 + slot] (layer 63: set-up). Marks
// sit right after waits and named barriers, which order them against the
// work before them. Empty otherwise.
#ifdef PHONON_CLUSTER_TRACE
__device__ unsigned long long g_cluster_trace[16 * 64 * 32];
#define CL_MARK_T(thread, layer, slot)                                                             \
    do {                                                                                           \
        if (threadIdx.x == (thread)) {                                                             \
            unsigned long long t_;                                                                 \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_)::"memory");                      \
            g_cluster_trace[(static_cast<size_t>(cluster_ctarank()) * 64 + (layer)) * 32 + (slot)] = t_; \
        }                                                                                          \
    } while (0)
#define CL_MARK(layer, slot) CL_MARK_T(0, layer, slot)
#else
#define CL_MARK_T(thread, layer, slot) \
    do {                               \
    } while (0)
#define CL_MARK(layer, slot) CL_MARK_T(0, layer, slot)
#endif

constexpr int kClusterCtas = 16;
constexpr int kClWarps = 8;                       // compute warps
constexpr int kClThreads = 32 * (kClWarps + 1);   // + copy warp
constexpr int kClUnitPlane = 16384;               // int8 bytes of a weight unit
constexpr int kClUnitBytes = kClUnitPlane + 1024; // + binary16 block scales
// Weight units of a layer, in consumption order: q rows [0, 32) and [32, 64)
// of the head, k rows and v rows of the CTA's 32 dims, out, 4 x up, 4 x down.
constexpr int kClUnitsPerLayer = 13;
constexpr int kClUnitOut = 4, kClUnitUp = 5, kClUnitDown = 9;
constexpr int kClKvSlots = 8;                     // page ring
constexpr int kClPartStride = 68;                 // warp partials: max, sum, acc[64], pad
// A CTA's attention message: max, sum, its half of the current key's q.k,
// pad, acc[64], its half of the current key's v [32].
constexpr int kClMsgFloats = 100;
constexpr int kClNormBytes = 2 * kWidth * 4;      // one LayerNorm's weight + bias (fp32)
constexpr int kClMaxUpdates = 2;                  // page-table updates carried in the parameters
// Exchange buffers with one mbarrier each, completing once per layer.
// CLX_R (kTc): the down projection's int32 partial sums, reduced by the
// CTA that owns the rows.
enum ClExchange : int { CLX_PART = 0, CLX_H = 1, CLX_G = 2, CLX_X = 3, CLX_R = 4 };
constexpr int kClExchanges = 5;
constexpr uint32_t kClBytesPart = kClusterCtas * kClMsgFloats * 4;  // 16 messages
constexpr uint32_t kClBytesH = kWidth * 4;                          // 16 slices of 32 rows
constexpr uint32_t kClBytesG = kFfn * 4;                            // 16 slices of 128 rows
constexpr uint32_t kClBytesX = kWidth * 4;
constexpr uint32_t kClBytesR = 4 * 32 * 4 * 4;  // four senders x 32 rows x 4 digit sums
// kTc: with its slice of g every CTA pushes, per up epilogue warp, the largest
// |g| of the warp's 32 rows (+inf if any is not finite) to every CTA: the down
// projection's digit exponent without a pass over the 2048-wide row.
constexpr uint32_t kClBytesGmax = kClusterCtas * 4 * 16;  // 16 CTAs x 4 warps, one float4 each
// Activation rows in shared memory are padded: 4 floats after every 64, so
// that the LayerNorm lanes' stride-4 accesses (lane = chunk * 4 + l) fall into
// 32 banks; element e lives at cl_pad(e).
constexpr int kClChunk = 68;
constexpr int kClRowPad = kWidth / 64 * kClChunk;  // 544 floats
constexpr int kClFfnPad = kFfn / 64 * kClChunk;    // 2176 floats
__host__ __device__ constexpr int cl_pad(int e) { return e + 4 * (e >> 6); }
constexpr int kClNormPadBytes = 2 * kClRowPad * 4;  // a LayerNorm's padded weight + bias

// Tensor-core units (kTc): with one scale per weight row (every Q8_0 block of
// a row shares it), a CTA's 128 q/k/v rows and its 128 up rows are each one
// M = 128 tile of a tcgen05 int8 MMA. The out and down projections are split
// over K: CTA rank computes rows [128 (rank / 4), +128) over columns
// [128 (rank % 4), +128) (out) or [512 (rank % 4), +512) (down), and the four
// CTAs of a row group send their int32 partial sums of rows [32 r, +32) to
// CTA r, which adds them (exactly) and finishes those rows. The weight units
// of the four projections are K
// slices: unit k holds 128 columns of the 128 rows as a SWIZZLE_128B tile
// (16 KB) followed by the 128 fp32 row scales. Activations enter as four
// base-128 digit rows (operand B, N = 16: rows 4-15 stay zero), sliced with
// the exponent of the whole row exactly as the batched tensor path slices
// its rows (ln_digits_kernel, digits_kernel<2048>).
constexpr int kClTcDigRowBytes = 16 * 128;         // B tile of one K slice: 16 rows x 128 bytes
constexpr int kClTcDigBytes = 4 * kClTcDigRowBytes;  // K = 512
constexpr int kClTcUnits = kClUnitsPerLayer;       // per layer and CTA: 4 q/k/v, out, 4 up, 4 down slices

template <bool kBf16, bool kTc = false>
struct ClShape {
    static constexpr int kWSlots = kBf16 ? (kTc ? 8 : 9) : 7;        // weight ring slots
    static constexpr int kBox = kPage * 128;                          // 16 rows x 128 bytes
    static constexpr int kKvBlock = kPage * kHeadDim * (kBf16 ? 2 : 4);  // K (or V) of one head, one page
    static constexpr int kKvSlot = 2 * kKvBlock;
    // Offsets from the 1024-aligned base (SWIZZLE_128B boxes first).
    static constexpr int kOffKv = 0;
    static constexpr int kOffW = kOffKv + kClKvSlots * kKvSlot;
    static constexpr int kOffDig = kOffW + kWSlots * kClUnitBytes;   // digit rows (kTc), 1024-aligned
    static constexpr int kOffNorm = kOffDig + (kTc ? kClTcDigBytes : 0);
    static constexpr int kOffX = kOffNorm + kClNormPadBytes;        // layer input x [512], padded
    static constexpr int kOffXn = kOffX + kClRowPad * 4;            // LayerNorm output, padded
    static constexpr int kOffH = kOffXn + kClRowPad * 4;            // h = x + attn Wout, padded
    static constexpr int kOffA = kOffH + kClRowPad * 4;             // attention row, padded
    static constexpr int kOffG = kOffA + kClRowPad * 4;             // GELU row [2048], padded
    static constexpr int kOffQ = kOffG + kClFfnPad * 4;             // q of the head [64]
    static constexpr int kOffSelf = kOffQ + kHeadDim * 4;           // this CTA's k, v of the current key [2][32]
    static constexpr int kOffMsg = kOffSelf + 64 * 4;               // messages of the 16 CTAs [16][100]
    static constexpr int kOffMine = kOffMsg + kClusterCtas * kClMsgFloats * 4;  // this CTA's message [100]
    static constexpr int kOffWPart = kOffMine + kClMsgFloats * 4;   // warp partials [8][68]
    static constexpr int kOffRope = kOffWPart + kClWarps * kClPartStride * 4;  // (cos, sin) [32]
    static constexpr int kOffRed = kOffRope + 32 * 8;               // kTc: down partial sums [4][32][4] int32
    static constexpr int kOffGmax = kOffRed + (kTc ? static_cast<int>(kClBytesR) : 0);  // kTc: [64] float4
    static constexpr int kOffBar = kOffGmax + (kTc ? static_cast<int>(kClBytesGmax) : 0);
    // weight ring full/empty, LayerNorm vectors full/empty, page ring
    // full/empty, the exchanges, the MMA accumulator
    static constexpr int kBars = 2 * kWSlots + 2 + 2 * kClKvSlots + kClExchanges + 1;
    static constexpr int kOffFlag = kOffBar + kBars * 8;            // failed flag, TMEM base, digit exponent
    static constexpr int kSmem = kOffFlag + 16 + 1024;  // + alignment slack
    static_assert(kKvSlot % 1024 == 0 && kOffW % 1024 == 0 && kClUnitBytes % 1024 == 0 && kOffDig % 1024 == 0,
                  "slot alignment (SWIZZLE_128B operand tiles)");
    static_assert(kOffMsg % 16 == 0 && kOffH % 16 == 0 && kOffG % 16 == 0 && kOffX % 16 == 0 &&
                      kOffMine % 16 == 0 && kOffQ % 16 == 0 && kOffSelf % 16 == 0 && kOffRed % 16 == 0 &&
                      kOffBar % 8 == 0,
                  "vector and st.async alignment");
    static_assert(kSmem <= 232448, "shared memory of one CTA");
};

struct ClusterParams {
    const PersistLayer* layers;  // per layer: lane-interleaved Q8_0 planes, scales, fp32 norms
    const uint8_t* tc;           // kTc: [layer][16 CTAs][8 units][kClUnitBytes] tensor-core units
    int n_layers;
    const float* in;             // [512]
    float* out;                  // [512]
    int32_t* status;             // [1]
    int32_t* error;              // context error flag (bounded waits)
    int slot, pos;               // the stream's slot and the position decoded
    int last_page;               // page holding position pos
    int n_updates;               // page-table updates (slot, index, page), for later steps
    int updates[3 * kClMaxUpdates];
    const float* freq;           // [32] RoPE inverse frequencies
    KvView kv;
    float* trace;                // optional: layer l's output row at trace[l * trace_stride]
    int trace_stride;
};

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_map(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}

// 16 bytes into CTA `rank`'s shared memory at (its copy of) saddr; the bytes
// complete on its copy of the mbarrier bar.
__device__ __forceinline__ void st_async4(uint32_t saddr, uint32_t bar, uint32_t rank, float4 v) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];"
                 ::"r"(cluster_map(saddr, rank)), "r"(__float_as_uint(v.x)), "r"(__float_as_uint(v.y)),
                   "r"(__float_as_uint(v.z)), "r"(__float_as_uint(v.w)), "r"(cluster_map(bar, rank))
                 : "memory");
}

// Bounded wait on an exchange barrier (completions come from other CTAs:
// acquire at cluster scope).
__device__ __forceinline__ bool cl_try_wait_cluster(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

__device__ __noinline__ bool cl_exchange_wait(uint32_t bar, uint32_t parity, int32_t* error, volatile int* failed) {
    if (cl_try_wait_cluster(bar, parity)) return true;
    const long long start = clock64();
    while (!cl_try_wait_cluster(bar, parity)) {
        if (*failed) return false;
        if (clock64() - start > kWaitBudgetCycles) {
            *failed = 1;
            if (error) atomicExch(error, 1);
            return false;
        }
    }
    return true;
}

// The copy warp's bounded wait for a slot release. The copy warp is warp 8
// and shares a scheduler with compute warps 0 and 4 (warps are assigned to
// the SM's four schedulers by warp index mod 4); polling without a pause took
// issue slots from them (a LayerNorm on warp 0 ran ~4x longer than the same
// routine on warp 1), so it sleeps between polls.
__device__ __noinline__ bool cl_copy_wait(uint32_t bar, uint32_t parity, int32_t* error, volatile int* failed) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long start = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (*failed) return false;
        if (clock64() - start > kWaitBudgetCycles) {
            *failed = 1;
            if (error) atomicExch(error, 1);
            return false;
        }
        __nanosleep(64);
    }
    return true;
}

__device__ __forceinline__ void mbar_arrive_count(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// All threads of all CTAs of the cluster; release/acquire at cluster scope.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// The 256 compute threads (named barrier 1; the copy warp never takes it).
__device__ __forceinline__ void compute_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// A consumer lane's offsets into one head's K and V blocks of a page, each a
// 16-row SWIZZLE_128B box (fp32: two boxes of 32 dims, 2 KB apart): the
// offsets attn_lane gives for head 0 of a 128-row box, with 16-row boxes.
template <bool kBf16>
__device__ __forceinline__ AttnLane<kBf16> cl_attn_lane(int lane) {
    AttnLane<kBf16> a;
    const int half = lane >> 4, krow = lane & 15;
#pragma unroll
    for (int c = 0; c < (kBf16 ? 4 : 8); ++c) {
        if constexpr (kBf16) a.k_off[c] = krow * 128 + (((half * 4 + c) ^ (krow & 7)) << 4);
        else a.k_off[c] = half * ClShape<false>::kBox + krow * 128 + ((c ^ (krow & 7)) << 4);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        if constexpr (kBf16) a.v_off[j] = j * 128 + (((lane >> 2) ^ (j & 7)) << 4) + (lane & 3) * 4;
        else a.v_off[j] = (lane >> 4) * ClShape<false>::kBox + j * 128 + ((((lane & 15) >> 1) ^ (j & 7)) << 4) +
                          (lane & 1) * 8;
    }
    return a;
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic): each element is computed
// exactly as the scalar operation would, two rows per instruction.
__device__ __forceinline__ uint64_t cl_pk(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float2 cl_upk(uint64_t v) {
    float a, b;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
    return make_float2(a, b);
}
__device__ __forceinline__ uint64_t cl_fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t cl_mul2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t cl_sub2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

// Four rows (local rows 4q .. 4q+3 of a weight unit in shared memory) of a
// chunks*512-column matrix against one padded activation row xs: gemv_kernel's
// per-lane arithmetic (int8 widened exactly, fp32 dot per 4 columns, scaled
// fma per 32-block, in that order per row; two rows per packed f32x2
// instruction) and butterfly sum. Every lane returns the four row sums.
__device__ __noinline__ float4 cl_rows4(const uint8_t* unit, int q, const float* xs, int chunks) {
    const int cols = chunks * 512;
    const __half* wsc = reinterpret_cast<const __half*>(unit + kClUnitPlane);
    const int lane = threadIdx.x & 31;
    const uint64_t magic = cl_pk(8388736.0f, 8388736.0f);
    uint64_t acc[2] = {cl_pk(0.0f, 0.0f), cl_pk(0.0f, 0.0f)};  // row pairs (0, 1), (2, 3)
#pragma unroll 1
    for (int c = 0; c < chunks; ++c) {
        uint4 wq[4];
        float sc[4][4];
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
            const int lr = 4 * q + rr;
            wq[rr] = *reinterpret_cast<const uint4*>(unit + static_cast<size_t>(lr) * cols + c * 512 + lane * 16);
            const uint2 raw =
                *reinterpret_cast<const uint2*>(wsc + static_cast<size_t>(lr) * (cols / 32) + c * 16 + (lane >> 3) * 4);
            const __half2 h01 = *reinterpret_cast<const __half2*>(&raw.x);
            const __half2 h23 = *reinterpret_cast<const __half2*>(&raw.y);
            sc[rr][0] = __low2float(h01);
            sc[rr][1] = __high2float(h01);
            sc[rr][2] = __low2float(h23);
            sc[rr][3] = __high2float(h23);
        }
        // x[c*512 + lane*4 + j*128 .. +3] in the padded row
        const float* xr = xs + c * (512 / 64 * kClChunk) + lane * 4 + 4 * (lane >> 4);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float4 xv = *reinterpret_cast<const float4*>(xr + j * (2 * kClChunk));
            const uint64_t x2[4] = {cl_pk(xv.x, xv.x), cl_pk(xv.y, xv.y), cl_pk(xv.z, xv.z), cl_pk(xv.w, xv.w)};
#pragma unroll
            for (int pr = 0; pr < 2; ++pr) {
                const int r0 = 2 * pr, r1 = 2 * pr + 1;
                const uint32_t w0 = (j == 0 ? wq[r0].x : j == 1 ? wq[r0].y : j == 2 ? wq[r0].z : wq[r0].w) ^ 0x80808080u;
                const uint32_t w1 = (j == 0 ? wq[r1].x : j == 1 ? wq[r1].y : j == 2 ? wq[r1].z : wq[r1].w) ^ 0x80808080u;
                uint64_t wf[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const uint32_t sel = e | (4 << 4) | (5 << 8) | (7 << 12);
                    wf[e] = cl_sub2(cl_pk(__uint_as_float(__byte_perm(w0, 0x4B000000u, sel)),
                                          __uint_as_float(__byte_perm(w1, 0x4B000000u, sel))),
                                    magic);
                }
                uint64_t part = cl_mul2(wf[0], x2[0]);
                part = cl_fma2(wf[1], x2[1], part);
                part = cl_fma2(wf[2], x2[2], part);
                part = cl_fma2(wf[3], x2[3], part);
                acc[pr] = cl_fma2(cl_pk(sc[r0][j], sc[r1][j]), part, acc[pr]);
            }
        }
    }
    const float2 a01 = cl_upk(acc[0]), a23 = cl_upk(acc[1]);
    return make_float4(warp_sum(a01.x), warp_sum(a01.y), warp_sum(a23.x), warp_sum(a23.y));
}

struct ClRows8 {
    float4 a, b;  // rows 4qa .. 4qa+3 of unit ua, rows 4qb .. 4qb+3 of unit ub
};

// Eight rows against one padded 512-wide activation row: four rows of unit
// ua and four of unit ub, computed as four row pairs with packed fp32
// arithmetic. Per row, every operation and its order are cl_rows4's
// (gemv_kernel's per-lane arithmetic), so the sums are bit-identical; the
// pairs halve the instructions and the eight independent chains hide each
// other's latency.
__device__ __noinline__ ClRows8 cl_rows8(const uint8_t* ua, int qa, const uint8_t* ub, int qb, const float* xs) {
    const int lane = threadIdx.x & 31;
    const uint64_t magic = cl_pk(8388736.0f, 8388736.0f);
    uint4 wq[8];
    float sc[8][4];
#pragma unroll
    for (int rr = 0; rr < 8; ++rr) {
        const uint8_t* unit = rr < 4 ? ua : ub;
        const int lr = 4 * (rr < 4 ? qa : qb) + (rr & 3);
        wq[rr] = *reinterpret_cast<const uint4*>(unit + static_cast<size_t>(lr) * 512 + lane * 16);
        const uint2 raw = *reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(unit + kClUnitPlane) +
                                                          static_cast<size_t>(lr) * 16 + (lane >> 3) * 4);
        const __half2 h01 = *reinterpret_cast<const __half2*>(&raw.x);
        const __half2 h23 = *reinterpret_cast<const __half2*>(&raw.y);
        sc[rr][0] = __low2float(h01);
        sc[rr][1] = __high2float(h01);
        sc[rr][2] = __low2float(h23);
        sc[rr][3] = __high2float(h23);
    }
    const float* xr = xs + lane * 4 + 4 * (lane >> 4);
    float4 xv[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) xv[j] = *reinterpret_cast<const float4*>(xr + j * (2 * kClChunk));
    uint64_t acc[4];
#pragma unroll
    for (int pr = 0; pr < 4; ++pr) acc[pr] = cl_pk(0.0f, 0.0f);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float xe[4] = {xv[j].x, xv[j].y, xv[j].z, xv[j].w};
        uint64_t x2[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) x2[e] = cl_pk(xe[e], xe[e]);
#pragma unroll
        for (int pr = 0; pr < 4; ++pr) {
            const int r0 = 2 * pr, r1 = 2 * pr + 1;
            const uint32_t w0 = (j == 0 ? wq[r0].x : j == 1 ? wq[r0].y : j == 2 ? wq[r0].z : wq[r0].w) ^ 0x80808080u;
            const uint32_t w1 = (j == 0 ? wq[r1].x : j == 1 ? wq[r1].y : j == 2 ? wq[r1].z : wq[r1].w) ^ 0x80808080u;
            uint64_t wf[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const uint32_t sel = e | (4 << 4) | (5 << 8) | (7 << 12);
                wf[e] = cl_sub2(cl_pk(__uint_as_float(__byte_perm(w0, 0x4B000000u, sel)),
                                      __uint_as_float(__byte_perm(w1, 0x4B000000u, sel))),
                                magic);
            }
            uint64_t part = cl_mul2(wf[0], x2[0]);
            part = cl_fma2(wf[1], x2[1], part);
            part = cl_fma2(wf[2], x2[2], part);
            part = cl_fma2(wf[3], x2[3], part);
            acc[pr] = cl_fma2(cl_pk(sc[r0][j], sc[r1][j]), part, acc[pr]);
        }
    }
    float sum[8];
#pragma unroll
    for (int pr = 0; pr < 4; ++pr) {
        const float2 v = cl_upk(acc[pr]);
        sum[2 * pr] = warp_sum(v.x);
        sum[2 * pr + 1] = warp_sum(v.y);
    }
    return ClRows8{make_float4(sum[0], sum[1], sum[2], sum[3]), make_float4(sum[4], sum[5], sum[6], sum[7])};
}

// warp_layernorm512 on padded rows, as one routine (one copy of its code).
__device__ __noinline__ bool cl_layernorm(const float* src, const float* w, const float* b, float* dst) {
    return warp_layernorm512<false, kClChunk>(src, w, b, dst);
}

// Online-softmax state of a warp (max, sum, the lane's two accumulated
// dims) and its finite flag, passed by value so that it stays in registers.
struct ClAttnState {
    float m, l, a0, a1;
    int ok;
};

// One page of the warp's head into its online-softmax state.
template <bool kBf16>
__device__ __noinline__ ClAttnState cl_attn_page(const uint8_t* sK, const float* q, int key0, int n_keys,
                                                 ClAttnState st) {
    const int lane = threadIdx.x & 31;
    const AttnLane<kBf16> ad = cl_attn_lane<kBf16>(lane);
    float qh[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 v = reinterpret_cast<const float4*>(q + (lane >> 4) * 32)[i];
        qh[4 * i] = v.x;
        qh[4 * i + 1] = v.y;
        qh[4 * i + 2] = v.z;
        qh[4 * i + 3] = v.w;
    }
    bool ok = st.ok != 0;
    attn_page<kBf16>(sK, sK + ClShape<kBf16>::kKvBlock, ad, qh, key0, n_keys, st.m, st.l, st.a0, st.a1, ok);
    st.ok = ok;
    return st;
}

// Source rows of weight unit u (layer u / 13) for CTA `rank`. With kTc the
// q/k/v and up units are the K slices of the tensor-core pack.
template <bool kTc = false>
__device__ __forceinline__ void cl_unit_src(const ClusterParams& p, int u, int rank, const uint8_t*& plane,
                                            const uint8_t*& scales) {
    const int l = u / kClUnitsPerLayer, k = u % kClUnitsPerLayer;
    if (kTc) {
        plane = p.tc + (static_cast<size_t>(l * kClusterCtas + rank) * kClTcUnits + k) * kClUnitBytes;
        scales = plane + kClUnitPlane;
        return;
    }
    const int head = rank >> 1, half = rank & 1;
    int m, row0;
    if (k < 2) {
        m = PM_QKV;
        row0 = head * kHeadDim + 32 * k;
    } else if (k < kClUnitOut) {
        m = PM_QKV;
        row0 = (k - 1) * kWidth + head * kHeadDim + half * 32;
    } else if (k == kClUnitOut) {
        m = PM_OUT;
        row0 = 32 * rank;
    } else if (k < kClUnitDown) {
        m = PM_UP;
        row0 = 128 * rank + 32 * (k - kClUnitUp);
    } else {
        m = PM_DOWN;
        row0 = 32 * rank + 8 * (k - kClUnitDown);
    }
    const int cols = persist_cols(m);
    const PersistLayer& L = p.layers[l];
    plane = L.plane[m] + static_cast<size_t>(row0) * cols;
    scales = reinterpret_cast<const uint8_t*>(L.scales[m] + static_cast<size_t>(row0) * (cols / 32));
}

template <bool kBf16, bool kTc>
__global__ void __launch_bounds__(kClThreads, 1)
    step_cluster_kernel(const __grid_constant__ CUtensorMap tm_kv16, const __grid_constant__ ClusterParams p) {
    using Sh = ClShape<kBf16, kTc>;
    constexpr int kW = Sh::kWSlots;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* kv_ring = smem + Sh::kOffKv;
    uint8_t* w_ring = smem + Sh::kOffW;
    uint8_t* n_ring = smem + Sh::kOffNorm;
    float* x_s = reinterpret_cast<float*>(smem + Sh::kOffX);
    float* xn_s = reinterpret_cast<float*>(smem + Sh::kOffXn);
    float* h_s = reinterpret_cast<float*>(smem + Sh::kOffH);
    float* a_s = reinterpret_cast<float*>(smem + Sh::kOffA);
    float* g_s = reinterpret_cast<float*>(smem + Sh::kOffG);
    float* q_s = reinterpret_cast<float*>(smem + Sh::kOffQ);
    float* self_s = reinterpret_cast<float*>(smem + Sh::kOffSelf);
    float* msg_s = reinterpret_cast<float*>(smem + Sh::kOffMsg);
    float* mine_s = reinterpret_cast<float*>(smem + Sh::kOffMine);
    float* wpart_s = reinterpret_cast<float*>(smem + Sh::kOffWPart);
    float2* rope_s = reinterpret_cast<float2*>(smem + Sh::kOffRope);
    int32_t* red_s = reinterpret_cast<int32_t*>(smem + Sh::kOffRed);
    float4* gmax_s = reinterpret_cast<float4*>(smem + Sh::kOffGmax);
    const uint32_t bar0 = smem_addr(smem + Sh::kOffBar);
    const uint32_t wfull0 = bar0, wempty0 = bar0 + 8 * kW, nfull = bar0 + 16 * kW, nempty = nfull + 8,
                   kfull0 = nfull + 16, kempty0 = kfull0 + 8 * kClKvSlots, xbar0 = kempty0 + 8 * kClKvSlots,
                   accum = xbar0 + 8 * kClExchanges;
    volatile int* failed = reinterpret_cast<volatile int*>(smem + Sh::kOffFlag);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Sh::kOffFlag + 4);
    int* dig_e = reinterpret_cast<int*>(smem + Sh::kOffFlag + 8);
    uint8_t* dig = smem + Sh::kOffDig;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rank = static_cast<int>(cluster_ctarank());
    const int head = rank >> 1, half = rank & 1;
    const int L = p.n_layers;
    // Earlier keys [0, pos) live on pages [0, n_old); the head's two CTAs
    // take [0, n_first) and [n_first, n_old); this CTA's: [pg0, pg0 + npc).
    const int n_old = (p.pos + kPage - 1) / kPage;
    const int n_first = (n_old + 1) / 2;
    const int pg0 = half ? n_first : 0;
    const int npc = half ? n_old - n_first : n_first;
    const int32_t* table = p.kv.table + static_cast<size_t>(p.slot) * p.kv.max_pages;

    CL_MARK(63, 0);
    if (threadIdx.x == 0) {
        for (int s = 0; s < kW; ++s) {
            mbar_init(wfull0 + 8 * s, 1);
            mbar_init(wempty0 + 8 * s, kClWarps);
        }
        mbar_init(nfull, 1);
        mbar_init(nempty, kTc ? kClWarps : 1);  // kTc: every compute warp reads the LayerNorm vectors
        for (int s = 0; s < kClKvSlots; ++s) {
            mbar_init(kfull0 + 8 * s, 1);
            mbar_init(kempty0 + 8 * s, 1);
        }
        for (int x = 0; x < kClExchanges; ++x) mbar_init(xbar0 + 8 * x, 1);
        mbar_init(accum, kClWarps);  // kTc: the eight issuing warps' commits
        *failed = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (threadIdx.x < 32) {  // the step's RoPE (cos, sin), as step_prep_kernel computes them
        const float phase = __fmul_rn(static_cast<float>(p.pos), p.freq[threadIdx.x]);
        double sd, cd;
        sincos(static_cast<double>(phase), &sd, &cd);
        rope_s[threadIdx.x] = make_float2(__double2float_rn(cd), __double2float_rn(sd));
    }
    // scalar loads: the caller's row need only be float-aligned, as on the other step paths
    for (int i = threadIdx.x; i < kWidth; i += kClThreads) x_s[cl_pad(i)] = p.in[i];
    if (rank == 0 && threadIdx.x < p.n_updates) {  // for later steps; this one reads only earlier pages
        const int* u = p.updates + 3 * threadIdx.x;
        const_cast<int32_t*>(p.kv.table)[static_cast<size_t>(u[0]) * p.kv.max_pages + u[1]] = u[2];
    }
    if constexpr (kTc) {
        // digit rows 4-15 of the B tiles stay zero; eight 16-column TMEM accumulator blocks
        for (int i = threadIdx.x; i < kClTcDigBytes / 16; i += kClThreads)
            reinterpret_cast<uint4*>(dig)[i] = make_uint4(0u, 0u, 0u, 0u);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        if (warp == 1) {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 128;" ::"r"(smem_addr(tmem_slot))
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        }
    }
    cluster_sync();  // barriers initialised in every CTA before any st.async reaches them
    CL_MARK(63, 1);
    if constexpr (kTc) asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");

    if (warp == kClWarps) {
        // ------------------------------------------------------ copy warp
        if (lane == 0) {
            int w_last[kW], k_last[kClKvSlots], n_last = -1;
            for (int s = 0; s < kW; ++s) w_last[s] = -1;
            for (int s = 0; s < kClKvSlots; ++s) k_last[s] = -1;
            int w_next = 0, k_next = 0;
            // Each issue waits (bounded) until the slot it refills has been
            // released by every consumer of its previous contents.
            auto issue_unit = [&]() {
                const int u = w_next++, s = u % kW;
                if (*failed) return;
                if (u >= kW && !cl_copy_wait(wempty0 + 8 * s, ((u / kW) - 1) & 1, p.error, failed)) return;
                const uint8_t *plane, *scales;
                cl_unit_src<kTc>(p, u, rank, plane, scales);
                uint8_t* dst = w_ring + s * kClUnitBytes;
                mbar_expect_tx(wfull0 + 8 * s, kClUnitBytes);
                bulk_load(smem_addr(dst), plane, kClUnitPlane, wfull0 + 8 * s);
                bulk_load(smem_addr(dst + kClUnitPlane), scales, kClUnitBytes - kClUnitPlane, wfull0 + 8 * s);
                w_last[s] = u;
            };
            // norm n: layer n / 2, LN1 (even) or LN2 (odd), through one slot
            // (a layer's LN2 vectors are read ~5 us after its LN1 vectors)
            auto issue_norm = [&](int n) {
                if (*failed) return;
                if (n >= 1 && !cl_copy_wait(nempty, (n - 1) & 1, p.error, failed)) return;
                mbar_expect_tx(nfull, kClNormBytes);
                // weight and bias, each as 8 chunks of 64 floats into padded rows
                const float* src = p.layers[n >> 1].norms + (n & 1) * 2 * kWidth;
                for (int k = 0; k < 16; ++k)
                    bulk_load(smem_addr(n_ring + ((k >> 3) * kClRowPad + (k & 7) * kClChunk) * 4), src + 64 * k, 256,
                              nfull);
                n_last = n;
            };
            auto issue_page = [&](int layer, int i) {  // page ring index k_next = layer * npc + i
                const int n = k_next++, s = n % kClKvSlots;
                if (*failed) return;
                if (n >= kClKvSlots && !cl_copy_wait(kempty0 + 8 * s, ((n / kClKvSlots) - 1) & 1, p.error, failed))
                    return;
                const int page = __ldcg(table + pg0 + i);
                const int row = (layer * p.kv.pool_pages + page) * 256 + head * kPage;  // K rows; V 128 rows on
                uint8_t* dst = kv_ring + s * Sh::kKvSlot;
                const uint32_t bar = kfull0 + 8 * s;
                mbar_expect_tx(bar, Sh::kKvSlot);
#pragma unroll
                for (int bx = 0; bx < (kBf16 ? 1 : 2); ++bx) {
                    tma_load_2d(smem_addr(dst + bx * Sh::kBox), &tm_kv16, bx * 32, row, bar);
                    tma_load_2d(smem_addr(dst + Sh::kKvBlock + bx * Sh::kBox), &tm_kv16, bx * 32, row + 128, bar);
                }
                k_last[s] = n;
            };
            // The compute warps' consumption order, layer by layer.
            auto prefetch_unit = [&](int u) {
                const uint8_t *plane, *scales;
                cl_unit_src<kTc>(p, u, rank, plane, scales);
                prefetch_l2(plane, kClUnitPlane);
                prefetch_l2(scales, kClUnitBytes - kClUnitPlane);
            };
            // The first pages of layer l + 1 go out right after layer l's out
            // unit: their ring slots free as soon as layer l's attention has
            // read its pages, so they land while stages C-E run.
            const int early = npc < kClKvSlots ? npc : kClKvSlots;
            for (int l = 0; l < L; ++l) {
                issue_norm(2 * l);
                for (int k = 0; k < kClUnitOut; ++k) issue_unit();
                if (l == 0) prefetch_unit(kClUnitsPerLayer - 1);
                if (l + 1 < L) {
                    prefetch_unit(kClUnitsPerLayer * (l + 1) + kClUnitOut - 1);  // v
                    prefetch_unit(kClUnitsPerLayer * (l + 2) - 1);                // last down unit
                }
                for (int i = l == 0 ? 0 : early; i < npc; ++i) issue_page(l, i);
                issue_unit();  // out
                if (l + 1 < L)
                    for (int i = 0; i < early; ++i) issue_page(l + 1, i);
                issue_norm(2 * l + 1);
                for (int k = kClUnitUp; k < kClUnitsPerLayer; ++k) issue_unit();
            }
            // Copies still in flight (only after a failure) land before the CTA exits.
            for (int s = 0; s < kW; ++s)
                if (w_last[s] >= 0) mbar_drain(wfull0 + 8 * s, (w_last[s] / kW) & 1);
            for (int s = 0; s < kClKvSlots; ++s)
                if (k_last[s] >= 0) mbar_drain(kfull0 + 8 * s, (k_last[s] / kClKvSlots) & 1);
            if (n_last >= 0) mbar_drain(nfull, n_last & 1);
        }
        __syncwarp();
    } else {
        // ---------------------------------------------------- compute warps
        const uint32_t msg_addr = smem_addr(msg_s), h_addr = smem_addr(h_s), g_addr = smem_addr(g_s),
                       x_addr = smem_addr(x_s);
        // Every wait of a compute warp ends warp-uniform (__all_sync): the
        // lanes leave a spin loop at different iterations, and a warp that
        // enters the row dot products or the LayerNorm split into groups of
        // lanes runs them several times over.
        auto wait_unit = [&](int u) {
            return __all_sync(kFull, mbar_wait(wfull0 + 8 * (u % kW), (u / kW) & 1, p.error, failed));
        };
        auto release_unit = [&](int u) {
            __syncwarp();
            if (lane == 0) mbar_arrive(wempty0 + 8 * (u % kW));
        };
        auto unit_ptr = [&](int u) { return w_ring + (u % kW) * kClUnitBytes; };
        // Exchange x of layer `use`: arm its barrier with the bytes it
        // expects (before or after they arrive), then wait for the phase.
        auto exchange_wait = [&](int x, uint32_t bytes, int use) {
            if (threadIdx.x == 0) mbar_expect_tx(xbar0 + 8 * x, bytes);
            return __all_sync(kFull, cl_exchange_wait(xbar0 + 8 * x, use & 1, p.error, failed));
        };
        // LayerNorm of a 512-wide row (norm n of the ring) into xn_s, by warp
        // 1, which shares its scheduler with no copy-warp polling (measured on
        // B200: LN2 on warp 0 took 3.9 us per layer, LN1 on warp 1 1.0 us).
        auto layer_norm = [&](int n, const float* src) {
            if (warp != 1) return;
            if (__all_sync(kFull, mbar_wait(nfull, n & 1, p.error, failed))) {
                const float* nw = reinterpret_cast<const float*>(n_ring);
                if (!cl_layernorm(src, nw, nw + kClRowPad, xn_s) && lane == 0 && rank == 0) flag_nonfinite(p.status, 0);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(nempty);
        };
        int cur_l = 0;  // the layer, for trace marks
        // kTc, all compute warps: columns [k0, k0 + ncs) of the padded row as
        // digit rows in the B tiles, given the row maximum mx and whether the
        // row is finite (else zero digits). Warp w, lane l: columns
        // k0 + 64 w + 2 l and the next. Ends with the proxy fence that makes
        // the digits visible to the MMA; a compute_sync follows.
        auto tc_slice_cols = [&](const float* row, int k0, int ncs, float mx, bool ok) {
            bool zero;
            const int e = digit_exponent(ok ? mx : 0.0f, zero);
            const int c = 64 * warp + 2 * lane;  // column within [k0, k0 + ncs)
            if (c < ncs) {
                const float2 f = *reinterpret_cast<const float2*>(row + cl_pad(k0 + c));
                const float down = pow2f(-e);
                const uint32_t d0 = (ok && !zero) ? slice_digits(f.x * down) : 0u;
                const uint32_t d1 = (ok && !zero) ? slice_digits(f.y * down) : 0u;
                uint8_t* tile = dig + (c >> 7) * kClTcDigRowBytes + (c & 15);
                const int chunk = (c & 127) >> 4;
#pragma unroll
                for (int j = 0; j < kDigits; ++j)  // SWIZZLE_128B: chunk q of row j at q ^ j
                    *reinterpret_cast<uint16_t*>(tile + j * 128 + ((chunk ^ j) << 4)) =
                        static_cast<uint16_t>(((d0 >> (8 * j)) & 0xffu) | (((d1 >> (8 * j)) & 0xffu) << 8));
            }
            if (threadIdx.x == 0) *dig_e = e;
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        };
        // kTc, all compute warps: columns [k0, k0 + ncs) of the padded row
        // `row` (ncols wide) as four base-128 digit rows into the B tiles,
        // with the exponent of the whole row (a row holding a non-finite value
        // gives zero digits), as the batched tensor path slices its rows. The
        // row maximum of a 512-wide row: every warp over the whole row; of the
        // 2048-wide row: warp w over columns [256 w, +256), combined through
        // the warp-partial buffer (free outside the attention stage) -- one
        // named barrier more, which costs a 512-wide row more than it saves.
        // The slicing: warp w, lane l, columns k0 + 64 w + 2 l and the next.
        // Ends with the proxy fence that makes the digits visible to the MMA;
        // a compute_sync follows.
        auto tc_slice = [&](const float* row, int ncols, int k0, int ncs, const float4* maxima = nullptr) {
            if (maxima) {  // the row maximum from the 64 pushed per-warp maxima
                float mx = fmaxf(maxima[lane].x, maxima[32 + lane].x);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
                tc_slice_cols(row, k0, ncs, mx, isfinite(mx));
                return;
            }
            const bool split = ncols > kWidth;
            const int span = split ? ncols / kClWarps : ncols;  // columns of this warp's maximum
            const int c0 = split ? span * warp : 0;
            float mx = 0.0f;
            bool fin = true;
            for (int i = 0; i < span / 128; ++i) {  // columns c0 + 128 i + 4 lane .. +3
                const float4 f = *reinterpret_cast<const float4*>(row + cl_pad(c0 + 128 * i + 4 * lane));
                fin &= isfinite(f.x) && isfinite(f.y) && isfinite(f.z) && isfinite(f.w);
                mx = fmaxf(mx, fmaxf(fmaxf(fabsf(f.x), fabsf(f.y)), fmaxf(fabsf(f.z), fabsf(f.w))));
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
            bool ok = __all_sync(kFull, fin);
            if (split) {
                if (lane == 0) {
                    wpart_s[warp * kClPartStride] = mx;
                    wpart_s[warp * kClPartStride + 1] = ok ? 1.0f : 0.0f;
                }
                compute_sync();
#pragma unroll
                for (int w = 0; w < kClWarps; ++w) {
                    mx = fmaxf(mx, wpart_s[w * kClPartStride]);
                    ok &= wpart_s[w * kClPartStride + 1] != 0.0f;
                }
            }
            tc_slice_cols(row, k0, ncs, mx, ok);
        };
        // kTc, all compute warps: LayerNorm n of the padded row src and its
        // digit rows in one pass, without a shared-memory row in between.
        // Every warp computes the row's moments (ln_moments512, the cascade of
        // warp_layernorm512) and the affine outputs of its lanes' 16 elements
        // for the row maximum; then it recomputes the outputs of its columns
        // 64 w + 2 l and the next with the same operations and slices them
        // into the B tiles as tc_slice does. Every warp releases the vectors.
        auto tc_ln_slice = [&](int n, const float* src) {
            const bool got = __all_sync(kFull, mbar_wait(nfull, n & 1, p.error, failed));
            const float* nw = reinterpret_cast<const float*>(n_ring);
            const float* nb = nw + kClRowPad;
            const int base = (lane >> 2) * kClChunk + (lane & 3);
            float v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = src[base + j * 4];
            bool ok = got;
#pragma unroll
            for (int j = 0; j < 16; ++j) ok &= isfinite(v[j]);
            float mu, scale;
            ln_moments512(v, 1e-5f, mu, scale);
            float mx = 0.0f;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int i = base + j * 4;
                const float wi = nw[i], bi = nb[i];
                ok &= isfinite(wi) && isfinite(bi);
                const float y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[j], mu), scale), wi), bi);
                ok &= isfinite(y);
                mx = fmaxf(mx, fabsf(y));
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
            ok = __all_sync(kFull, ok);
            if (got && !ok && warp == 1 && lane == 0 && rank == 0) flag_nonfinite(p.status, 0);
            bool zero;
            const int e = digit_exponent(ok ? mx : 0.0f, zero);
            const int c = 64 * warp + 2 * lane;  // this lane's two columns
            const float down = pow2f(-e);
            uint32_t d[2];
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                const int i = cl_pad(c + t);
                const float y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(src[i], mu), scale), nw[i]), nb[i]);
                d[t] = (ok && !zero) ? slice_digits(y * down) : 0u;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(nempty);
            uint8_t* tile = dig + (c >> 7) * kClTcDigRowBytes + (c & 15);
            const int chunk = (c & 127) >> 4;
#pragma unroll
            for (int j = 0; j < kDigits; ++j)  // SWIZZLE_128B: chunk q of row j at q ^ j
                *reinterpret_cast<uint16_t*>(tile + j * 128 + ((chunk ^ j) << 4)) =
                    static_cast<uint16_t>(((d[0] >> (8 * j)) & 0xffu) | (((d[1] >> (8 * j)) & 0xffu) << 8));
            if (threadIdx.x == 0) *dig_e = e;
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        };
        // kTc, all compute warps: the MMAs of one projection (weights A,
        // M = 128; digits B, N = 16), issued in parallel into accumulator
        // block w (TMEM columns [16 w, +16)) of warp w, each warp committing
        // to `accum` (eight arrivals a phase). With n = 4 units warps 2k and
        // 2k+1 issue unit k's K = 32 steps {0, 1} and {2, 3}; with n = 1 (out)
        // warp w < 4 issues step w of the one unit. Issuing four MMAs and a
        // commit takes a warp ~0.4 us: one warp issuing a projection's 16
        // took 1.5 us. Every unit but the last (whose tail holds the row
        // scales the epilogue reads) is released by its two warps' commits
        // plus six arrivals, so its slot refills as soon as the tensor core
        // has read it; the last is released by all eight warps.
        auto tc_mma = [&](int u_first, int n, int mark) {
            const uint32_t tmem = *tmem_slot + 16 * warp;
            constexpr uint32_t idesc = umma_idesc_i8(kGemmM, 16);
            const int k = n == 4 ? warp >> 1 : 0;  // the unit (K slice) of this warp
            const int u = u_first + k;
            if ((n == 4 || warp < 4) && wait_unit(u)) {
                if (warp == 1) CL_MARK_T(32, cur_l, mark);
                if (lane == 0) {
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t a0 = smem_addr(unit_ptr(u)), b0 = smem_addr(dig + k * kClTcDigRowBytes);
                    if (n == 4) {
#pragma unroll
                        for (int kk = 0; kk < 2; ++kk) {  // K = 32 bytes per MMA
                            const uint32_t off = 32 * (2 * (warp & 1) + kk);
                            umma_i8(tmem, umma_desc_sw128(a0 + off), umma_desc_sw128(b0 + off), idesc, kk);
                        }
                        if (k < 3) {
                            umma_commit(wempty0 + 8 * (u % kW));
                            mbar_arrive_count(wempty0 + 8 * (u % kW), kClWarps / 2 - 1);
                        }
                    } else {
                        umma_i8(tmem, umma_desc_sw128(a0 + 32 * warp), umma_desc_sw128(b0 + 32 * warp), idesc, 0u);
                    }
                }
            }
            if (lane == 0) umma_commit(accum);
            __syncwarp();
            if (warp == 1) CL_MARK_T(32, cur_l, mark + 1);
        };
        // kTc, warps 0-3: the four digit sums of row 32 warp + lane of the
        // projection's 128 rows (TMEM lane quarter `warp`): the accumulator
        // blocks the projection wrote (8, or 4 for out) added, exact in int32,
        // once `accum` completes the phase of this parity.
        auto tc_sums = [&](int parity, uint32_t (&d)[4], int mark, int blocks) {
            if (!__all_sync(kFull, mbar_wait(accum, parity, p.error, failed))) return false;
            CL_MARK_T(0, cur_l, mark);
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t t0 = *tmem_slot + (static_cast<uint32_t>(32 * warp) << 16);
            uint32_t r[8][4];
#pragma unroll
            for (int b = 0; b < 8; ++b)
                asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                             : "=r"(r[b][0]), "=r"(r[b][1]), "=r"(r[b][2]), "=r"(r[b][3])
                             : "r"(t0 + 16 * b));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                d[j] = r[0][j] + r[1][j] + r[2][j] + r[3][j];
                if (blocks == 8) d[j] += r[4][j] + r[5][j] + r[6][j] + r[7][j];
            }
            return true;
        };
        // Digit sums recombined as i8_gemm_kernel's epilogue does, times the
        // row scale: row i of the 128 rows of unit u's tail.
        auto tc_finish = [&](const uint32_t (&d)[4], int u, int i) {
            const int e = *dig_e;
            float acc = 0.0f;
#pragma unroll
            for (int j = 0; j < kDigits; ++j)
                acc = fmaf(static_cast<float>(static_cast<int32_t>(d[j])), pow2f(e - 7 * (j + 1)), acc);
            return acc * reinterpret_cast<const float*>(unit_ptr(u) + kClUnitPlane)[i];
        };
        // kTc, split over K (out, down): warps 0-3 send the digit sums of rows
        // [32 w, +32) of the row group to CTA (rank & ~3) + w; warp 0 of the
        // owner adds the four senders' sums (exact in int32) and returns its
        // row 32 rank + lane, scaled with the holder unit u's row scales.
        auto tc_reduce = [&](int parity, int use, int u, float& y, int mark, int blocks) {
            uint32_t d[4];
            if (warp < 4 && tc_sums(parity, d, mark, blocks) && !*failed) {
                const uint32_t dst = smem_addr(red_s) + (((rank & 3) * 32 + lane) * 4) * 4;
                st_async4(dst, xbar0 + 8 * CLX_R, (rank & ~3) + warp,
                          make_float4(__uint_as_float(d[0]), __uint_as_float(d[1]), __uint_as_float(d[2]),
                                      __uint_as_float(d[3])));
            }
            if (warp != 0 || !exchange_wait(CLX_R, kClBytesR, use)) return false;
            CL_MARK(cur_l, mark + 1);
            uint32_t t[4];
#pragma unroll
            for (int j = 0; j < kDigits; ++j) {
                int32_t sum = 0;
#pragma unroll
                for (int q = 0; q < 4; ++q) sum += red_s[(q * 32 + lane) * 4 + j];
                t[j] = static_cast<uint32_t>(sum);
            }
            y = tc_finish(t, u, 32 * (rank & 3) + lane);
            return true;
        };
        // One row per lane (rows r0 + lane) of a warp into exchange x of every
        // CTA: rows 4m .. 4m+3 (m = lane % 8) gathered from lanes 4m .. 4m+3
        // and pushed by lane l to CTAs l / 8 + 4i.
        auto push_rows = [&](uint32_t buf, int x, int r0, float v) {
            const int m = lane & 7;
            const float4 v4 = make_float4(__shfl_sync(kFull, v, 4 * m), __shfl_sync(kFull, v, 4 * m + 1),
                                          __shfl_sync(kFull, v, 4 * m + 2), __shfl_sync(kFull, v, 4 * m + 3));
            if (*failed) return;
#pragma unroll
            for (int i = 0; i < 4; ++i) st_async4(buf + cl_pad(r0 + 4 * m) * 4, xbar0 + 8 * x, (lane >> 3) + 4 * i, v4);
        };

        for (int l = 0; l < L; ++l) {
            const int u0 = kClUnitsPerLayer * l;
            const bool last_layer = l == L - 1;
            cur_l = l;
            (void)cur_l;

            // ---- A: LN1 -> q (64), k, v (the CTA's 32 dims) of the head
            if (l > 0) exchange_wait(CLX_X, kClBytesX, l - 1);
            CL_MARK(l, 0);
            if constexpr (kTc) {
                tc_ln_slice(2 * l, x_s);
                compute_sync();
                CL_MARK_T(32, l, 13);
                tc_mma(u0, 4, 14);
                CL_MARK(l, 1);
                uint32_t d[4];
                if (warp < 4 && tc_sums(0, d, 11, 8)) {
                    float y = tc_finish(d, u0 + 3, 32 * warp + lane);
                    // warps 0, 1: q dims [32 warp, +32); 2: k, 3: v, dims [32 half, +32)
                    const int d = (warp < 2 ? 32 * warp : 32 * half) + lane;
                    if (warp < 3) {  // RoPE pairs (2i, 2i+1) in adjacent lanes
                        const float other = __shfl_xor_sync(kFull, y, 1);
                        float a = (lane & 1) ? other : y, b = (lane & 1) ? y : other;
                        rope_apply(a, b, rope_s[d >> 1]);
                        y = (lane & 1) ? b : a;
                    }
                    if (!__all_sync(kFull, isfinite(y)) && lane == 0) flag_nonfinite(p.status, 0);
                    if (warp < 2) {
                        q_s[d] = y;
                    } else {
                        const int which = warp - 2;
                        const long long off = kv_offset(p.kv, p.last_page, l, which, head, p.pos % kPage) + d;
                        if (kBf16) {  // the current key joins the softmax as the cache holds it
                            const uint16_t hb = f32_to_bf16(y);
                            static_cast<uint16_t*>(p.kv.pool)[off] = hb;
                            y = bf16_to_f32(hb);
                        } else {
                            static_cast<float*>(p.kv.pool)[off] = y;
                        }
                        self_s[32 * which + lane] = y;
                    }
                }
                release_unit(u0 + 3);  // the scale holder: warps 0-3 after their reads
            } else {
            layer_norm(2 * l, x_s);
            compute_sync();
            CL_MARK(l, 1);
            for (int k0 = 0; k0 < kClUnitOut; k0 += 2) {
                const bool got = wait_unit(u0 + k0) & wait_unit(u0 + k0 + 1);
                if (got) {
                    const ClRows8 s8 = cl_rows8(unit_ptr(u0 + k0), warp, unit_ptr(u0 + k0 + 1), warp, xn_s);
                    if (lane == 0) {
#pragma unroll
                        for (int kk = 0; kk < 2; ++kk) {
                            const int k = k0 + kk;
                            const float4 s = kk ? s8.b : s8.a;
                            // rows 4w .. 4w+3 of unit k: two RoPE pairs (q, k) or plain (v)
                            float v[4] = {s.x, s.y, s.z, s.w};
                            const int d = (k < 2 ? 32 * k : 32 * half) + 4 * warp;  // dim within the head
                            if (k < 3) {
                                rope_apply(v[0], v[1], rope_s[d >> 1]);
                                rope_apply(v[2], v[3], rope_s[(d >> 1) + 1]);
                            }
                            bool ok = true;
#pragma unroll
                            for (int e = 0; e < 4; ++e) ok &= isfinite(v[e]);
                            if (!ok) flag_nonfinite(p.status, 0);
                            if (k < 2) {
                                *reinterpret_cast<float4*>(q_s + d) = make_float4(v[0], v[1], v[2], v[3]);
                            } else {
                                const long long off = kv_offset(p.kv, p.last_page, l, k - 2, head, p.pos % kPage) + d;
                                kv_store2(p.kv, off, v[0], v[1]);
                                kv_store2(p.kv, off + 2, v[2], v[3]);
                                if (kBf16) {  // the current key joins the softmax as the cache holds it
#pragma unroll
                                    for (int e = 0; e < 4; ++e) v[e] = bf16_to_f32(f32_to_bf16(v[e]));
                                }
                                *reinterpret_cast<float4*>(self_s + 32 * (k - 2) + (d - 32 * half)) =
                                    make_float4(v[0], v[1], v[2], v[3]);
                            }
                        }
                    }
                }
                release_unit(u0 + k0);
                release_unit(u0 + k0 + 1);
            }
            }
            compute_sync();
            CL_MARK(l, 2);

            // ---- B: attention of the head over this CTA's earlier pages
            {
                ClAttnState st{-INFINITY, 0.0f, 0.0f, 0.0f, 1};
                for (int i = warp; i < npc; i += kClWarps) {
                    const int n = l * npc + i, s = n % kClKvSlots;
                    if (__all_sync(kFull, mbar_wait(kfull0 + 8 * s, (n / kClKvSlots) & 1, p.error, failed)))
                        st = cl_attn_page<kBf16>(kv_ring + s * Sh::kKvSlot, q_s, (pg0 + i) * kPage, p.pos, st);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(kempty0 + 8 * s);
                }
                if (!__all_sync(kFull, st.ok != 0) && lane == 0) flag_nonfinite(p.status, 0);
                float* wp = wpart_s + warp * kClPartStride;
                *reinterpret_cast<float2*>(wp + 2 + 2 * lane) = make_float2(st.a0, st.a1);
                if (lane == 0) {
                    wp[0] = st.m;
                    wp[1] = st.l;
                }
            }
            compute_sync();
            if (warp == 1) {  // the CTA's message: warps merged in page order, the current key's halves
                float M = -INFINITY, S = 0.0f, A0 = 0.0f, A1 = 0.0f;
                for (int w = 0; w < kClWarps && w < npc; ++w) {
                    const float* wp = wpart_s + w * kClPartStride;
                    const MergeWeights mw = merge_weights(M, wp[0]);
                    S = merge_fold(S, mw, wp[1]);
                    const float2 pa = *reinterpret_cast<const float2*>(wp + 2 + 2 * lane);
                    A0 = merge_fold(A0, mw, pa.x);
                    A1 = merge_fold(A1, mw, pa.y);
                }
                // this CTA's half of q.k of the current key (dims [32*half, +32))
                const float qk = warp_sum(q_s[32 * half + lane] * self_s[lane]);
                *reinterpret_cast<float2*>(mine_s + 4 + 2 * lane) = make_float2(A0, A1);
                mine_s[68 + lane] = self_s[32 + lane];
                if (lane == 0) *reinterpret_cast<float4*>(mine_s) = make_float4(M, S, qk, 0.0f);
            }
            compute_sync();
            // to every CTA: warp w sends the 25 16-byte pieces to CTAs 2w, 2w+1
            if (lane < kClMsgFloats / 4 && !*failed) {
                const float4 v = reinterpret_cast<const float4*>(mine_s)[lane];
                const uint32_t dst = msg_addr + (rank * kClMsgFloats + 4 * lane) * 4;
                st_async4(dst, xbar0 + 8 * CLX_PART, 2 * warp, v);
                st_async4(dst, xbar0 + 8 * CLX_PART, 2 * warp + 1, v);
            }
            CL_MARK(l, 3);

            // ---- C: merge each head's two CTA partials and the current key;
            //      h = x + attn Wout^T, slices to every CTA
            exchange_wait(CLX_PART, kClBytesPart, l);
            CL_MARK(l, 4);
            {
                const int hh = warp;  // warp w merges head w; lane j owns dims 2j, 2j+1
                float M = -INFINITY, S = 0.0f, A0 = 0.0f, A1 = 0.0f;
#pragma unroll
                for (int k = 0; k < 2; ++k) {
                    const float* pp = msg_s + (2 * hh + k) * kClMsgFloats;
                    const MergeWeights mw = merge_weights(M, pp[0]);
                    S = merge_fold(S, mw, pp[1]);
                    const float2 pa = *reinterpret_cast<const float2*>(pp + 4 + 2 * lane);
                    A0 = merge_fold(A0, mw, pa.x);
                    A1 = merge_fold(A1, mw, pa.y);
                }
                // the current key: q.k from both halves, v dims 2j, 2j+1 from half j / 16
                const float* m0 = msg_s + (2 * hh) * kClMsgFloats;
                const float* m1 = m0 + kClMsgFloats;
                const float score = __fmul_rn(__fadd_rn(m0[2], m1[2]), 0.125f);
                const float2 vs = *reinterpret_cast<const float2*>((lane < 16 ? m0 : m1) + 68 + 2 * (lane & 15));
                bool ok = isfinite(score);
                const MergeWeights mw = merge_weights(M, score);
                S = merge_fold(S, mw, 1.0f);
                A0 = merge_fold(A0, mw, vs.x);
                A1 = merge_fold(A1, mw, vs.y);
                ok &= S > 0.0f && isfinite(S);
                const float inv = __fdiv_rn(1.0f, S);
                const float o0 = __fmul_rn(A0, inv), o1 = __fmul_rn(A1, inv);
                ok &= isfinite(o0) && isfinite(o1);
                *reinterpret_cast<float2*>(a_s + hh * kClChunk + 2 * lane) = make_float2(o0, o1);  // head hh = chunk hh
                if (!__all_sync(kFull, ok) && lane == 0 && rank == 0) flag_nonfinite(p.status, 0);
            }
            compute_sync();
            if constexpr (kTc) {
                // rows [128 (rank / 4), +128) over columns [128 (rank % 4), +128)
                tc_slice(a_s, kWidth, 128 * (rank & 3), 128);
                compute_sync();
                tc_mma(u0 + kClUnitOut, 1, 27);
                float y;
                if (tc_reduce(1, 2 * l, u0 + kClUnitOut, y, 29, 4)) {
                    const int r = 32 * rank + lane;
                    const float h = __fadd_rn(x_s[cl_pad(r)], y);
                    if (!__all_sync(kFull, isfinite(h)) && lane == 0) flag_nonfinite(p.status, 0);
                    push_rows(h_addr, CLX_H, 32 * rank, h);
                }
                release_unit(u0 + kClUnitOut);
            } else {
                const int u = u0 + kClUnitOut;
                if (wait_unit(u)) {
                    const float4 s = cl_rows4(unit_ptr(u), warp, a_s, 1);
                    const int r = 32 * rank + 4 * warp;
                    const float4 xr = *reinterpret_cast<const float4*>(x_s + cl_pad(r));
                    const float4 h = make_float4(__fadd_rn(xr.x, s.x), __fadd_rn(xr.y, s.y), __fadd_rn(xr.z, s.z),
                                                 __fadd_rn(xr.w, s.w));
                    if (lane == 0 && !(isfinite(h.x) && isfinite(h.y) && isfinite(h.z) && isfinite(h.w)))
                        flag_nonfinite(p.status, 0);
                    if (lane < kClusterCtas) st_async4(h_addr + cl_pad(r) * 4, xbar0 + 8 * CLX_H, lane, h);
                }
                release_unit(u);
            }
            CL_MARK(l, 5);

            // ---- D: g = GELU(LN2(h) Wup^T), slices to every CTA
            exchange_wait(CLX_H, kClBytesH, l);
            CL_MARK(l, 6);
            if constexpr (kTc) {
                tc_ln_slice(2 * l + 1, h_s);
                compute_sync();
                CL_MARK_T(32, l, 17);
                tc_mma(u0 + kClUnitUp, 4, 18);
                CL_MARK(l, 7);
                uint32_t d[4];
                if (warp < 4 && tc_sums(0, d, 22, 8)) {
                    const float y = tc_finish(d, u0 + kClUnitUp + 3, 32 * warp + lane);
                    const float gm = gelu_erf(y);
                    if (!__all_sync(kFull, isfinite(y) && isfinite(gm)) && lane == 0) flag_nonfinite(p.status, 0);
                    push_rows(g_addr, CLX_G, 128 * rank + 32 * warp, gm);
                    float m = isfinite(y) && isfinite(gm) ? fabsf(gm) : INFINITY;
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, o));
                    if (lane < kClusterCtas && !*failed)
                        st_async4(smem_addr(gmax_s + rank * 4 + warp), xbar0 + 8 * CLX_G, lane, make_float4(m, 0.0f, 0.0f, 0.0f));
                }
                release_unit(u0 + kClUnitUp + 3);
            } else {
            layer_norm(2 * l + 1, h_s);
            compute_sync();
            CL_MARK(l, 7);
            for (int k0 = 0; k0 < 4; k0 += 2) {
                const int ua = u0 + kClUnitUp + k0;
                const bool got = wait_unit(ua) & wait_unit(ua + 1);
                if (got) {
                    const ClRows8 s8 = cl_rows8(unit_ptr(ua), warp, unit_ptr(ua + 1), warp, xn_s);
                    // lane i < 8 takes the GELU of row sum i (one erf chain per lane
                    // instead of eight), then every lane gathers the eight
                    const float sv[8] = {s8.a.x, s8.a.y, s8.a.z, s8.a.w, s8.b.x, s8.b.y, s8.b.z, s8.b.w};
                    float mine = sv[0];
#pragma unroll
                    for (int i = 1; i < 8; ++i) mine = (lane & 7) == i ? sv[i] : mine;
                    const float gm = gelu_erf(mine);
                    if (lane < 8 && !(isfinite(mine) && isfinite(gm))) flag_nonfinite(p.status, 0);
                    float gv[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) gv[i] = __shfl_sync(kFull, gm, i);
#pragma unroll
                    for (int kk = 0; kk < 2; ++kk) {
                        const int r = 128 * rank + 32 * (k0 + kk) + 4 * warp;
                        const float4 g = make_float4(gv[4 * kk], gv[4 * kk + 1], gv[4 * kk + 2], gv[4 * kk + 3]);
                        if (lane < kClusterCtas) st_async4(g_addr + cl_pad(r) * 4, xbar0 + 8 * CLX_G, lane, g);
                    }
                }
                release_unit(ua);
                release_unit(ua + 1);
            }
            }
            CL_MARK(l, 8);

            // ---- E: x' = h + g Wdown^T, slices to every CTA (the last layer: to `out`)
            exchange_wait(CLX_G, kTc ? kClBytesG + kClBytesGmax : kClBytesG, l);
            CL_MARK(l, 9);
            if constexpr (kTc) {
                // rows [128 (rank / 4), +128) over columns [512 (rank % 4), +512)
                tc_slice(g_s, kFfn, 512 * (rank & 3), 512, gmax_s);
                compute_sync();
                CL_MARK_T(32, l, 20);
                tc_mma(u0 + kClUnitDown, 4, 23);
                float y;
                if (tc_reduce(1, 2 * l + 1, u0 + kClUnitDown + 3, y, 25, 8)) {
                    const int r = 32 * rank + lane;
                    const float x = __fadd_rn(h_s[cl_pad(r)], y);
                    if (!__all_sync(kFull, isfinite(x)) && lane == 0) flag_nonfinite(p.status, 0);
                    if (p.trace) p.trace[static_cast<size_t>(l) * p.trace_stride + r] = x;
                    if (last_layer) p.out[r] = x;
                    else push_rows(x_addr, CLX_X, 32 * rank, x);
                }
                release_unit(u0 + kClUnitDown + 3);
            } else {
                const int u = u0 + kClUnitDown + (warp >> 1);
                if (wait_unit(u)) {
                    const float4 s = cl_rows4(unit_ptr(u), warp & 1, g_s, 4);
                    const int r = 32 * rank + 8 * (warp >> 1) + 4 * (warp & 1);
                    const float4 hr = *reinterpret_cast<const float4*>(h_s + cl_pad(r));
                    const float4 x = make_float4(__fadd_rn(hr.x, s.x), __fadd_rn(hr.y, s.y), __fadd_rn(hr.z, s.z),
                                                 __fadd_rn(hr.w, s.w));
                    if (lane == 0 && !(isfinite(x.x) && isfinite(x.y) && isfinite(x.z) && isfinite(x.w)))
                        flag_nonfinite(p.status, 0);
                    if (p.trace && lane == 0)
                        *reinterpret_cast<float4*>(p.trace + static_cast<size_t>(l) * p.trace_stride + r) = x;
                    if (last_layer) {
                        if (lane == 0) {  // float-aligned caller rows: scalar stores
                            p.out[r] = x.x;
                            p.out[r + 1] = x.y;
                            p.out[r + 2] = x.z;
                            p.out[r + 3] = x.w;
                        }
                    } else if (lane < kClusterCtas) {
                        st_async4(x_addr + cl_pad(r) * 4, xbar0 + 8 * CLX_X, lane, x);
                    }
                }
                // a down unit is read by two warps: each counts for four of
                // the slot's eight arrivals, so the slot refills (the next
                // layer's q/k/v/out/up units) while the other warps still work
                __syncwarp();
                if (lane == 0) mbar_arrive_count(wempty0 + 8 * (u % kW), kClWarps / 2);
            }
            CL_MARK(l, 10);
        }
    }
    // No CTA exits while another may still store into its shared memory.
    if constexpr (kTc) asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    cluster_sync();
    if constexpr (kTc) {
        if (warp == 1) {
            // the last accumulator phase before the columns are
            // freed; bounded, for MMAs left running after a failure
            if (lane == 0) mbar_drain(accum, 1);  // 4 L commits: the last phase is odd
            __syncwarp();
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 128;" ::"r"(*tmem_slot) : "memory");
        }
    }
}

// Tensor-core units of one layer for step_cluster_kernel<kBf16, true>, in the
// order the step consumes them (unit k of CTA rank at (rank * 13 + k) *
// kClUnitBytes): k < 4: K slice k of the CTA's 128 q/k/v rows (q rows
// [64 head, +64), k and v rows of dims [32 half, +32) of the head); k = 4:
// columns [128 (rank % 4), +128) of out rows [128 (rank / 4), +128);
// 5 <= k < 9: K slice k - 5 of up rows [128 rank, +128); k >= 9: columns
// [512 (rank % 4) + 128 (k - 9), +128) of down rows [128 (rank / 4), +128).
// Each unit: a 128-row x 128-byte SWIZZLE_128B tile (row i at
// (i / 8) * 1024 + (i % 8) * 128, 16-byte chunk c at position c ^ (i % 8))
// from the natural int8 planes, then the 128 fp32 row scales, then zeros to
// kClUnitBytes. One CTA per unit, 256 threads.
struct ClTcSource {
    const int8_t* w[4];     // natural int8 planes: qkv, out, up, down
    const float* scale[4];  // their row scales
};

__global__ void cluster_tc_pack_kernel(const ClTcSource src, uint8_t* __restrict__ dst) {
    const int rank = blockIdx.x / kClTcUnits, k = blockIdx.x % kClTcUnits;
    const int head = rank >> 1, half = rank & 1, group = rank >> 2, quarter = rank & 3;
    uint8_t* out = dst + static_cast<size_t>(blockIdx.x) * kClUnitBytes;
    const int m = k < kClUnitOut ? PM_QKV : k == kClUnitOut ? PM_OUT : k < kClUnitDown ? PM_UP : PM_DOWN;
    const int cols = m == PM_DOWN ? kFfn : kWidth;
    const int col0 = m == PM_QKV ? 128 * k
                   : m == PM_OUT ? 128 * quarter
                   : m == PM_UP  ? 128 * (k - kClUnitUp)
                                 : 512 * quarter + 128 * (k - kClUnitDown);
    auto src_row = [&](int i) {
        if (m == PM_OUT || m == PM_DOWN) return 128 * group + i;
        if (m == PM_UP) return 128 * rank + i;
        if (i < 64) return head * kHeadDim + i;
        return (i < 96 ? kWidth : 2 * kWidth) + head * kHeadDim + half * 32 + (i & 31);
    };
    for (int q = threadIdx.x; q < 128 * 8; q += blockDim.x) {
        const int i = q >> 3, c = q & 7;
        const uint4 v = *reinterpret_cast<const uint4*>(src.w[m] + static_cast<size_t>(src_row(i)) * cols + col0 + 16 * c);
        *reinterpret_cast<uint4*>(out + (i >> 3) * 1024 + (i & 7) * 128 + ((c ^ (i & 7)) << 4)) = v;
    }
    for (int i = threadIdx.x; i < (kClUnitBytes - kClUnitPlane) / 4; i += blockDim.x)
        reinterpret_cast<float*>(out + kClUnitPlane)[i] = i < 128 ? src.scale[m][src_row(i)] : 0.0f;
}

}  // namespace phonon
