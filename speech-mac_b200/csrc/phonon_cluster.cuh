// Single-stream decode step on one thread-block cluster (sm_100a).
//
// A decode step of one stream is a chain of ~60 dependent stages whose work
// is small (a 512-wide LayerNorm, a few hundred GEMV rows, attention over a
// few hundred keys per head): its time is the latency of the chain, not the
// ~50 MB of traffic. Kernel boundaries and grid-wide barriers each cost
// microseconds per stage. Here one cluster of 16 CTAs (one per SM) runs
// every layer of the step (the loop of phonon_flow_stack_step, speech-mac
// src/phonon_transformer.c:455-489). CTAs exchange activations through
// distributed shared memory and meet at hardware cluster barriers; every CTA
// keeps the full rows it reads. CTA `rank` serves head rank / 2, half
// rank % 2:
//
//   A  LN1 of x (each CTA) -> QKV rows of dims [32*half, +32) of its head;
//      RoPE; q to both CTAs of the head, k and v appended to the stream's
//      KV page (src/phonon_transformer.c:414-431)
//   B  attention of its head over its half of the stream's pages, one page
//      per warp at a time (TMA page staging, the page math of the other
//      paths); the CTA's partial goes to every CTA (flow_attention, :340-404)
//   C  every CTA merges the two partials of each head into the attention
//      row; out rows [32*rank, +32) + residual -> h to every CTA (:432-443)
//   D  LN2 (each CTA) -> up rows [128*rank, +128) + GELU -> to every CTA
//      (:444-447)
//   E  down rows [32*rank, +32) + residual -> x' to every CTA (:448-452)
//
// Warp 8 is the copy warp. It streams the CTA's weight rows through a ring
// of shared-memory slots (bulk copies; a unit is 17 KB: 32 rows of a
// 512-column matrix or 8 rows of the 2048-column one, with their Q8_0
// scales), the LayerNorm vectors through a two-slot ring, and its head's
// K/V blocks of the stream's pages through a third ring (TMA, 16-row
// SWIZZLE_128B boxes), each unit as soon as its slot is released. Only the
// page this step appends to waits for phase A.
//
// Numerics: the LayerNorm, the row dot products (gemv_kernel's per-lane
// fp32 accumulation and butterfly sum), RoPE, GELU, residuals and the page
// math of the attention are those of the other step paths, so projections
// and appended K/V rows are bit-identical to them; the attention partials
// are merged in another order (pages are split between two CTAs and eight
// warps), which changes sums within rounding.
//
// Every mbarrier wait is bounded: on expiry the CTA raises the context's
// error flag and skips the rest of its work, but every thread still takes
// every cluster barrier, so the launch ends; the copy warp waits (bounded)
// for its copies in flight before the CTA exits. No multicast.
#pragma once

#include "phonon_persist.cuh"

namespace phonon {

// Phase timestamps for profiling builds (-DPHONON_CLUSTER_TRACE): thread 0
// of every CTA writes %globaltimer at marked points into
// g_cluster_trace[(rank * 64 + layer) * 32 + slot] (layer 63: set-up).
// Empty otherwise.
#ifdef PHONON_CLUSTER_TRACE
__device__ unsigned long long g_cluster_trace[16 * 64 * 32];
#define CL_MARK(layer, slot)                                                                       \
    do {                                                                                           \
        if (threadIdx.x == 0) {                                                                    \
            unsigned long long t_;                                                                 \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                 \
            g_cluster_trace[(static_cast<size_t>(cluster_ctarank()) * 64 + (layer)) * 32 + (slot)] = t_; \
        }                                                                                          \
    } while (0)
#else
#define CL_MARK(layer, slot) \
    do {                     \
    } while (0)
#endif

constexpr int kClusterCtas = 16;
constexpr int kClWarps = 8;                       // compute warps
constexpr int kClThreads = 32 * (kClWarps + 1);   // + copy warp
constexpr int kClUnitPlane = 16384;               // int8 bytes of a weight unit
constexpr int kClUnitBytes = kClUnitPlane + 1024; // + binary16 block scales
constexpr int kClUnitsPerLayer = 12;              // q, k, v, out, 4 x up, 4 x down
constexpr int kClKvSlots = 8;                     // page ring: one page per compute warp
constexpr int kClPartStride = 68;                 // floats: max, sum, acc[64], pad
constexpr int kClNormBytes = 2 * kWidth * 4;      // one LayerNorm's weight + bias (fp32)
constexpr int kClMaxUpdates = 2;                  // page-table updates carried in the parameters

template <bool kBf16>
struct ClShape {
    static constexpr int kWSlots = kBf16 ? 9 : 7;                    // weight ring slots
    static constexpr int kBox = kPage * 128;                          // 16 rows x 128 bytes
    static constexpr int kKvBlock = kPage * kHeadDim * (kBf16 ? 2 : 4);  // K (or V) of one head, one page
    static constexpr int kKvSlot = 2 * kKvBlock;
    // Offsets from the 1024-aligned base (SWIZZLE_128B boxes first).
    static constexpr int kOffKv = 0;
    static constexpr int kOffW = kOffKv + kClKvSlots * kKvSlot;
    static constexpr int kOffNorm = kOffW + kWSlots * kClUnitBytes;
    static constexpr int kOffX = kOffNorm + 2 * kClNormBytes;      // layer input x [512]
    static constexpr int kOffXn = kOffX + kWidth * 4;               // LayerNorm output [512]
    static constexpr int kOffH = kOffXn + kWidth * 4;               // h = x + attn Wout [512]
    static constexpr int kOffA = kOffH + kWidth * 4;                // attention row [512]
    static constexpr int kOffG = kOffA + kWidth * 4;                // GELU row [2048]
    static constexpr int kOffQ = kOffG + kFfn * 4;                  // q of the head [64]
    static constexpr int kOffPart = kOffQ + kHeadDim * 4;           // CTA partials [16][68]
    static constexpr int kOffWPart = kOffPart + kClusterCtas * kClPartStride * 4;  // warp partials [8][68]
    static constexpr int kOffRope = kOffWPart + kClWarps * kClPartStride * 4;      // (cos, sin) [32]
    static constexpr int kOffBar = kOffRope + 32 * 8;
    static constexpr int kBars = 2 * kWSlots + 4 + 2 * kClKvSlots;
    static constexpr int kOffFlag = kOffBar + kBars * 8;
    static constexpr int kSmem = kOffFlag + 16 + 1024;  // + alignment slack
    static_assert(kKvSlot % 1024 == 0 && kOffW % 16 == 0 && kClUnitBytes % 16 == 0, "slot alignment");
    static_assert(kSmem <= 232448, "shared memory of one CTA");
};

struct ClusterParams {
    const PersistLayer* layers;  // per layer: lane-interleaved Q8_0 planes, scales, fp32 norms
    int n_layers;
    const float* in;             // [512]
    float* out;                  // [512]
    int32_t* status;             // [1]
    int32_t* error;              // context error flag (bounded waits)
    int slot, pos;               // the stream's slot and the position decoded
    int n_updates;               // page-table updates (slot, index, page), applied first
    int updates[3 * kClMaxUpdates];
    const float* freq;           // [32] RoPE inverse frequencies
    KvView kv;
    float* trace;                // optional: layer l's output row at trace[l * trace_stride]
    int trace_stride;
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_map(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}

__device__ __forceinline__ void st_cluster(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

__device__ __forceinline__ void st_cluster2(uint32_t addr, float a, float b) {
    asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(a), "f"(b) : "memory");
}

// All threads of all CTAs of the cluster; release/acquire at cluster scope
// (shared memory of every CTA and global memory).
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// The 256 compute threads (named barrier 1; the copy warp never takes it).
__device__ __forceinline__ void compute_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

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

// Four rows (local rows 4q .. 4q+3 of a weight unit in shared memory)
// against one activation row xs[kChunks * 512]: gemv_kernel's per-lane
// arithmetic (int8 widened exactly, fp32 dot per 4 columns, scaled fma per
// 32-block) and butterfly sum. Every lane returns the four row sums.
template <int kChunks>
__device__ __forceinline__ void cl_rows4(const uint8_t* unit, int q, const float* xs, float (&sum)[4]) {
    constexpr int cols = kChunks * 512;
    const __half* wsc = reinterpret_cast<const __half*>(unit + kClUnitPlane);
    const int lane = threadIdx.x & 31;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 1
    for (int c = 0; c < kChunks; ++c) {
        float wf[4][16], sc[4][4];
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
            const int lr = 4 * q + rr;
            const uint4 wq = *reinterpret_cast<const uint4*>(unit + static_cast<size_t>(lr) * cols + c * 512 + lane * 16);
            const uint2 raw =
                *reinterpret_cast<const uint2*>(wsc + static_cast<size_t>(lr) * (cols / 32) + c * 16 + (lane >> 3) * 4);
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
        const float* xr = xs + c * 512 + lane * 4;
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
                acc[rr] = fmaf(sc[rr][j], part, acc[rr]);
            }
        }
    }
#pragma unroll
    for (int rr = 0; rr < 4; ++rr) sum[rr] = warp_sum(acc[rr]);
}

__device__ __forceinline__ float pick4(const float (&v)[4], int i) {
    return i == 0 ? v[0] : (i == 1 ? v[1] : (i == 2 ? v[2] : v[3]));
}

// Source rows of weight unit u (layer u / 12) for CTA `rank`.
__device__ __forceinline__ void cl_unit_src(const ClusterParams& p, int u, int rank, const uint8_t*& plane,
                                            const uint8_t*& scales) {
    const int l = u / kClUnitsPerLayer, k = u % kClUnitsPerLayer;
    const int head = rank >> 1, half = rank & 1;
    int m, row0;
    if (k < 3) {
        m = PM_QKV;
        row0 = k * kWidth + head * kHeadDim + half * 32;
    } else if (k == 3) {
        m = PM_OUT;
        row0 = 32 * rank;
    } else if (k < 8) {
        m = PM_UP;
        row0 = 128 * rank + 32 * (k - 4);
    } else {
        m = PM_DOWN;
        row0 = 32 * rank + 8 * (k - 8);
    }
    const int cols = persist_cols(m);
    const PersistLayer& L = p.layers[l];
    plane = L.plane[m] + static_cast<size_t>(row0) * cols;
    scales = reinterpret_cast<const uint8_t*>(L.scales[m] + static_cast<size_t>(row0) * (cols / 32));
}

template <bool kBf16>
__global__ void __launch_bounds__(kClThreads, 1)
    step_cluster_kernel(const __grid_constant__ CUtensorMap tm_kv16, const __grid_constant__ ClusterParams p) {
    using Sh = ClShape<kBf16>;
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
    float* part_s = reinterpret_cast<float*>(smem + Sh::kOffPart);
    float* wpart_s = reinterpret_cast<float*>(smem + Sh::kOffWPart);
    float2* rope_s = reinterpret_cast<float2*>(smem + Sh::kOffRope);
    const uint32_t bar0 = smem_addr(smem + Sh::kOffBar);
    const uint32_t wfull0 = bar0, wempty0 = bar0 + 8 * kW, nfull0 = bar0 + 16 * kW, nempty0 = nfull0 + 16,
                   kfull0 = nfull0 + 32, kempty0 = kfull0 + 8 * kClKvSlots;
    volatile int* failed = reinterpret_cast<volatile int*>(smem + Sh::kOffFlag);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rank = static_cast<int>(cluster_ctarank());
    const int head = rank >> 1, half = rank & 1;
    const int L = p.n_layers;
    const int n_units = kClUnitsPerLayer * L;
    const int n_keys = p.pos + 1;
    const int n_pages = p.pos / kPage + 1;
    // Pages of the stream split between the head's two CTAs: [pg0, pg0 + npc).
    const int n_first = (n_pages + 1) / 2;
    const int pg0 = half ? n_first : 0;
    const int npc = half ? n_pages - n_first : n_first;
    const bool holds_last = npc > 0 && pg0 + npc == n_pages;  // the page this step appends to
    const int32_t* table = p.kv.table + static_cast<size_t>(p.slot) * p.kv.max_pages;

    CL_MARK(63, 0);
    if (threadIdx.x == 0) {
        for (int s = 0; s < kW; ++s) {
            mbar_init(wfull0 + 8 * s, 1);
            mbar_init(wempty0 + 8 * s, kClWarps);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(nfull0 + 8 * s, 1);
            mbar_init(nempty0 + 8 * s, 1);
        }
        for (int s = 0; s < kClKvSlots; ++s) {
            mbar_init(kfull0 + 8 * s, 1);
            mbar_init(kempty0 + 8 * s, 1);
        }
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
    for (int i = threadIdx.x; i < kWidth; i += kClThreads) x_s[i] = p.in[i];
    if (rank == 0 && threadIdx.x < p.n_updates) {
        const int* u = p.updates + 3 * threadIdx.x;
        const_cast<int32_t*>(p.kv.table)[static_cast<size_t>(u[0]) * p.kv.max_pages + u[1]] = u[2];
    }
    cluster_sync();  // barriers initialised, page table updated, every CTA running
    CL_MARK(63, 1);
    const int last_page = __ldcg(table + (n_pages - 1));

    if (warp == kClWarps) {
        // ------------------------------------------------------ copy warp
        const bool issuer = lane == 0;
        int w_last[kW], k_last[kClKvSlots], n_last[2];
#pragma unroll
        for (int s = 0; s < kW; ++s) w_last[s] = -1;
#pragma unroll
        for (int s = 0; s < kClKvSlots; ++s) k_last[s] = -1;
        n_last[0] = n_last[1] = -1;
        int kv_next = 0, kv_last_ok = -1;  // next page-ring index; layer whose appended page may be read

        auto issue_unit = [&](int u) {
            const int s = u % kW;
            const uint32_t bar = wfull0 + 8 * s;
            const uint8_t *plane, *scales;
            cl_unit_src(p, u, rank, plane, scales);
            uint8_t* dst = w_ring + s * kClUnitBytes;
            mbar_expect_tx(bar, kClUnitBytes);
            bulk_load(smem_addr(dst), plane, kClUnitPlane, bar);
            bulk_load(smem_addr(dst + kClUnitPlane), scales, kClUnitBytes - kClUnitPlane, bar);
            w_last[s] = u;
        };
        // Unit u has been consumed: refill its slot with unit u + kW.
        auto refill_after = [&](int u) {
            if (!issuer || *failed || u + kW >= n_units) return;
            if (!mbar_wait(wempty0 + 8 * (u % kW), (u / kW) & 1, p.error, failed)) return;
            issue_unit(u + kW);
        };
        auto issue_norm = [&](int n) {  // norm n: layer n / 2, LN1 (even) or LN2 (odd)
            const int s = n & 1;
            const uint32_t bar = nfull0 + 8 * s;
            mbar_expect_tx(bar, kClNormBytes);
            bulk_load(smem_addr(n_ring + s * kClNormBytes), p.layers[n >> 1].norms + (n & 1) * 2 * kWidth,
                      kClNormBytes, bar);
            n_last[s] = n;
        };
        auto renorm_after = [&](int n) {
            if (!issuer || *failed || n + 2 >= 2 * L) return;
            if (!mbar_wait(nempty0 + 8 * (n & 1), (n >> 1) & 1, p.error, failed)) return;
            issue_norm(n + 2);
        };
        // K/V blocks of this CTA's pages, ring index n = layer * npc + i,
        // up to `limit`; the appended page of a layer waits for its phase A.
        auto issue_kv = [&](int limit) {
            if (!issuer) return;
            for (; kv_next < limit && !*failed; ++kv_next) {
                const int layer = kv_next / npc, i = kv_next % npc;
                if (holds_last && i == npc - 1 && layer > kv_last_ok) break;
                const int s = kv_next % kClKvSlots;
                if (kv_next >= kClKvSlots &&
                    !mbar_wait(kempty0 + 8 * s, ((kv_next / kClKvSlots) - 1) & 1, p.error, failed))
                    break;
                const int page = i == npc - 1 && holds_last ? last_page : __ldcg(table + pg0 + i);
                const int row = (layer * p.kv.pool_pages + page) * 256 + head * kPage;  // K rows; V 128 rows on
                uint8_t* dst = kv_ring + s * Sh::kKvSlot;
                const uint32_t bar = kfull0 + 8 * s;
                mbar_expect_tx(bar, Sh::kKvSlot);
#pragma unroll
                for (int bx = 0; bx < (kBf16 ? 1 : 2); ++bx) {
                    tma_load_2d(smem_addr(dst + bx * Sh::kBox), &tm_kv16, bx * 32, row, bar);
                    tma_load_2d(smem_addr(dst + Sh::kKvBlock + bx * Sh::kBox), &tm_kv16, bx * 32, row + 128, bar);
                }
                k_last[s] = kv_next;
            }
        };

        if (issuer) {
            for (int u = 0; u < kW && u < n_units; ++u) issue_unit(u);
            for (int n = 0; n < 2 && n < 2 * L; ++n) issue_norm(n);
        }
        issue_kv(min(npc, kClKvSlots));
        __syncwarp();
        for (int l = 0; l < L; ++l) {
            const int u0 = kClUnitsPerLayer * l;
            // A
            for (int k = 0; k < 3; ++k) refill_after(u0 + k);
            renorm_after(2 * l);
            __syncwarp();
            cluster_sync();
            // B: the appended page is in global memory now
            if (issuer) fence_proxy_async_global();
            kv_last_ok = l;
            issue_kv(min(min((l + 1) * npc + kClKvSlots, (l + 2) * npc), L * npc));
            __syncwarp();
            cluster_sync();
            // C
            refill_after(u0 + 3);
            __syncwarp();
            cluster_sync();
            // D
            for (int k = 4; k < 8; ++k) refill_after(u0 + k);
            renorm_after(2 * l + 1);
            __syncwarp();
            cluster_sync();
            // E
            for (int k = 8; k < 12; ++k) refill_after(u0 + k);
            __syncwarp();
            cluster_sync();
        }
        // Copies still in flight (only after a failure) land before the CTA exits.
        if (issuer) {
            for (int s = 0; s < kW; ++s)
                if (w_last[s] >= 0) mbar_drain(wfull0 + 8 * s, (w_last[s] / kW) & 1);
            for (int s = 0; s < kClKvSlots; ++s)
                if (k_last[s] >= 0) mbar_drain(kfull0 + 8 * s, (k_last[s] / kClKvSlots) & 1);
            for (int s = 0; s < 2; ++s)
                if (n_last[s] >= 0) mbar_drain(nfull0 + 8 * s, (n_last[s] >> 1) & 1);
        }
        return;
    }

    // ---------------------------------------------------------- compute warps
    const AttnLane<kBf16> ad = cl_attn_lane<kBf16>(lane);
    const uint32_t q_addr = smem_addr(q_s), part_addr = smem_addr(part_s), h_addr = smem_addr(h_s),
                   g_addr = smem_addr(g_s), x_addr = smem_addr(x_s);
    auto wait_unit = [&](int u) { return mbar_wait(wfull0 + 8 * (u % kW), (u / kW) & 1, p.error, failed); };
    auto release_unit = [&](int u) {
        __syncwarp();
        if (lane == 0) mbar_arrive(wempty0 + 8 * (u % kW));
    };
    auto unit_ptr = [&](int u) { return w_ring + (u % kW) * kClUnitBytes; };
    // LayerNorm of a 512-wide row (norm n of the ring) into xn_s, by warp 0.
    auto layer_norm = [&](int n, const float* src) {
        if (warp != 0) return;
        const int s = n & 1;
        const bool got = mbar_wait(nfull0 + 8 * s, (n >> 1) & 1, p.error, failed);
        CL_MARK(n >> 1, 28 + 2 * (n & 1));
        if (got) {
            const float* nw = reinterpret_cast<const float*>(n_ring + s * kClNormBytes);
            const bool ok = warp_layernorm512(src, nw, nw + kWidth, xn_s);
            if (!ok && lane == 0 && rank == 0) flag_nonfinite(p.status, 0);
        }
        CL_MARK(n >> 1, 29 + 2 * (n & 1));
        __syncwarp();
        if (lane == 0) mbar_arrive(nempty0 + 8 * s);
    };

    for (int l = 0; l < L; ++l) {
        const int u0 = kClUnitsPerLayer * l;
        const bool last_layer = l == L - 1;

        // ---- A: LN1 -> q, k, v dims [32*half, +32) of the head
        CL_MARK(l, 0);
        layer_norm(2 * l, x_s);
        compute_sync();
        CL_MARK(l, 1);
        for (int region = 0; region < 3; ++region) {
            const int u = u0 + region;
            const bool got_u = wait_unit(u);
            CL_MARK(l, 16 + region);
            if (got_u) {
                float s[4];
                cl_rows4<1>(unit_ptr(u), warp, xn_s, s);
                if (lane < 2) {
                    const int d = half * 32 + 4 * warp + 2 * lane;  // dim within the head (even)
                    float v0 = lane ? s[2] : s[0], v1 = lane ? s[3] : s[1];
                    if (region < 2) rope_apply(v0, v1, rope_s[d >> 1]);
                    if (!isfinite(v0) || !isfinite(v1)) flag_nonfinite(p.status, 0);
                    if (region == 0) {
                        const uint32_t a = q_addr + d * 4;
                        st_cluster2(cluster_map(a, rank), v0, v1);
                        st_cluster2(cluster_map(a, rank ^ 1), v0, v1);
                    } else {
                        const long long off =
                            kv_offset(p.kv, last_page, l, region - 1, head, p.pos % kPage) + d;
                        kv_store2(p.kv, off, v0, v1);
                    }
                }
            }
            release_unit(u);
        }
        fence_proxy_async_global();  // K/V appends before phase B's TMA reads
        CL_MARK(l, 2);
        cluster_sync();
        CL_MARK(l, 3);

        // ---- B: attention of the head over this CTA's pages
        {
            float qh[32];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float4 v = reinterpret_cast<const float4*>(q_s + (lane >> 4) * 32)[i];
                qh[4 * i] = v.x;
                qh[4 * i + 1] = v.y;
                qh[4 * i + 2] = v.z;
                qh[4 * i + 3] = v.w;
            }
            float m = -INFINITY, lsum = 0.0f, a0 = 0.0f, a1 = 0.0f;
            bool finite_ok = true;
            for (int i = warp; i < npc; i += kClWarps) {
                const int n = l * npc + i, s = n % kClKvSlots;
                const bool got =
                    __all_sync(kFull, mbar_wait(kfull0 + 8 * s, (n / kClKvSlots) & 1, p.error, failed));
                if (got) {
                    const uint8_t* sK = kv_ring + s * Sh::kKvSlot;
                    attn_page<kBf16>(sK, sK + Sh::kKvBlock, ad, qh, (pg0 + i) * kPage, n_keys, m, lsum, a0, a1,
                                     finite_ok);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(kempty0 + 8 * s);
            }
            if (!__all_sync(kFull, finite_ok) && lane == 0) flag_nonfinite(p.status, 0);
            float* wp = wpart_s + warp * kClPartStride;
            *reinterpret_cast<float2*>(wp + 2 + 2 * lane) = make_float2(a0, a1);
            if (lane == 0) {
                wp[0] = m;
                wp[1] = lsum;
            }
        }
        CL_MARK(l, 4);
        compute_sync();
        CL_MARK(l, 5);
        if (warp == 0) {  // the CTA's partial: warps in page order, then to every CTA
            float M = -INFINITY, S = 0.0f, A0 = 0.0f, A1 = 0.0f;
            for (int w = 0; w < kClWarps && w < npc; ++w) {
                const float* wp = wpart_s + w * kClPartStride;
                const MergeWeights mw = merge_weights(M, wp[0]);
                S = merge_fold(S, mw, wp[1]);
                const float2 pa = *reinterpret_cast<const float2*>(wp + 2 + 2 * lane);
                A0 = merge_fold(A0, mw, pa.x);
                A1 = merge_fold(A1, mw, pa.y);
            }
            const uint32_t dst = part_addr + rank * kClPartStride * 4;
#pragma unroll 4
            for (int r = 0; r < kClusterCtas; ++r) {
                const uint32_t a = cluster_map(dst, r);
                st_cluster2(a + 8 + 8 * lane, A0, A1);
                if (lane == 0) st_cluster2(a, M, S);
            }
        }
        CL_MARK(l, 6);
        cluster_sync();
        CL_MARK(l, 7);

        // ---- C: merge the heads' partials; h = x + attn Wout^T, to every CTA
        {
            const int hh = warp;  // warp w merges head w; lane j owns dims 2j, 2j+1
            float M = -INFINITY, S = 0.0f, A0 = 0.0f, A1 = 0.0f;
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const float* pp = part_s + (2 * hh + k) * kClPartStride;
                const MergeWeights mw = merge_weights(M, pp[0]);
                S = merge_fold(S, mw, pp[1]);
                const float2 pa = *reinterpret_cast<const float2*>(pp + 2 + 2 * lane);
                A0 = merge_fold(A0, mw, pa.x);
                A1 = merge_fold(A1, mw, pa.y);
            }
            bool ok = S > 0.0f && isfinite(S);
            const float inv = __fdiv_rn(1.0f, S);
            const float o0 = __fmul_rn(A0, inv), o1 = __fmul_rn(A1, inv);
            ok &= isfinite(o0) && isfinite(o1);
            *reinterpret_cast<float2*>(a_s + hh * kHeadDim + 2 * lane) = make_float2(o0, o1);
            if (!__all_sync(kFull, ok) && lane == 0 && rank == 0) flag_nonfinite(p.status, 0);
        }
        compute_sync();
        {
            const int u = u0 + 3;
            const bool got_u = wait_unit(u);
            CL_MARK(l, 19);
            if (got_u) {
                float s[4];
                cl_rows4<1>(unit_ptr(u), warp, a_s, s);
                const int rr = lane & 3, r = 32 * rank + 4 * warp + rr;
                const float v = __fadd_rn(x_s[r], pick4(s, rr));
                if (lane < 4 && !isfinite(v)) flag_nonfinite(p.status, 0);
                st_cluster(cluster_map(h_addr + r * 4, lane >> 2), v);
                st_cluster(cluster_map(h_addr + r * 4, (lane >> 2) + 8), v);
            }
            release_unit(u);
        }
        CL_MARK(l, 8);
        cluster_sync();
        CL_MARK(l, 9);

        // ---- D: g = GELU(LN2(h) Wup^T), to every CTA
        layer_norm(2 * l + 1, h_s);
        compute_sync();
        CL_MARK(l, 10);
        for (int k = 0; k < 4; ++k) {
            const int u = u0 + 4 + k;
            const bool got_u = wait_unit(u);
            CL_MARK(l, 20 + k);
            if (got_u) {
                float s[4];
                cl_rows4<1>(unit_ptr(u), warp, xn_s, s);
                const int rr = lane & 3, r = 128 * rank + 32 * k + 4 * warp + rr;
                float v = pick4(s, rr);
                bool ok = isfinite(v);
                v = gelu_erf(v);
                ok &= isfinite(v);
                if (lane < 4 && !ok) flag_nonfinite(p.status, 0);
                st_cluster(cluster_map(g_addr + r * 4, lane >> 2), v);
                st_cluster(cluster_map(g_addr + r * 4, (lane >> 2) + 8), v);
            }
            release_unit(u);
        }
        CL_MARK(l, 11);
        cluster_sync();
        CL_MARK(l, 12);

        // ---- E: x' = h + g Wdown^T, to every CTA (the last layer: to `out`)
        for (int k = 0; k < 4; ++k) {
            const int u = u0 + 8 + k;
            const bool got = wait_unit(u);
            CL_MARK(l, 24 + k);
            if (got && (warp >> 1) == k) {
                float s[4];
                cl_rows4<4>(unit_ptr(u), warp & 1, g_s, s);
                const int rr = lane & 3, r = 32 * rank + 4 * warp + rr;
                const float v = __fadd_rn(h_s[r], pick4(s, rr));
                if (lane < 4 && !isfinite(v)) flag_nonfinite(p.status, 0);
                if (p.trace && lane < 4) p.trace[static_cast<size_t>(l) * p.trace_stride + r] = v;
                if (last_layer) {
                    if (lane < 4) p.out[r] = v;
                } else {
                    st_cluster(cluster_map(x_addr + r * 4, lane >> 2), v);
                    st_cluster(cluster_map(x_addr + r * 4, (lane >> 2) + 8), v);
                }
            }
            release_unit(u);
        }
        CL_MARK(l, 13);
        cluster_sync();
        CL_MARK(l, 14);
    }
}

}  // namespace phonon
