// Split-K paged flash-decode with TMA page staging (sm_100a).
//
// The step's pages, in (stream, page) order, are cut into chunks (large
// first, small last: guided self-scheduling) and each chunk into one split
// per stream segment it covers. A CTA runs its own chunk c = blockIdx.x
// first, then takes chunks by ticket from an atomic counter until they run
// out, so that CTAs whose memory traffic is slower (or that start late
// because the SM is busy) take fewer pages and the launch ends together.
// Warp 8 is the producer: for every page it TMA-loads the page's K block and
// V block of this layer ([8 heads][16 slots][64 dims], 16 KB each in bf16)
// into a ring of shared-memory stages that runs on across splits and
// chunks, tagging each stage with its chunk; page ids come from the step's
// flat list (split order, uploaded with the step's plan), 32 per coalesced
// load; the next chunk's ticket is drawn while the current chunk's last
// pages go out, and the first chunk's pages that hold only earlier positions
// are requested before the kernel waits for its predecessor. After the last
// chunk it sends an end tag through the ring. Warps 0-7
// (one per head) consume each stage with the online softmax of
// attn_partial_kernel, release it, and write one partial per split. K/V
// loads carry an L2 evict-first hint. Tiles are loaded with SWIZZLE_128B
// (16-byte chunk index XOR row % 8), so the per-key row reads of the
// consumers are bank-conflict free. fp32 pages use two 128-byte column boxes
// per block. No multicast; every wait is bounded.
#pragma once

#include "phonon_gemm.cuh"
#include "phonon_kernels.cuh"

namespace phonon {

constexpr int kAttnHeadsPerCta = kHeads;            // consumer warps
constexpr int kAttnTmaThreads = 32 * (kAttnHeadsPerCta + 1);

template <bool kBf16>
struct AttnTma {
    static constexpr int kBoxes = kBf16 ? 1 : 2;            // 128-byte column boxes per block
    static constexpr int kBoxBytes = 128 * 128;             // 128 rows x 128 bytes
    static constexpr int kBlockBytes = kBoxes * kBoxBytes;  // K (or V) of one page, all heads
    static constexpr int kStageBytes = 2 * kBlockBytes;     // a page's K and V
    static constexpr int kStages = 3;
    // + barriers (2 per stage), the failure flag and the stage tags
    static constexpr int kSmem = 1024 + kStages * kStageBytes + 128;
    static_assert(2 * kStages * 8 + 4 + 4 * kStages <= 128, "ring bookkeeping exceeds its shared memory");
    static constexpr int kBoxCols = kBf16 ? 64 : 32;        // elements per 128-byte box row
};

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Address of 16-byte chunk `chunk` of row `row` in a SWIZZLE_128B box.
__device__ __forceinline__ const uint8_t* sw128(const uint8_t* box, int row, int chunk) {
    return box + row * 128 + ((chunk ^ (row & 7)) << 4);
}

// A consumer lane's byte offsets into a stage's K and V blocks, swizzle
// included. The swizzle of row r depends on r & 7 only, and the rows a lane
// reads are head*16 + key (K) and head*16 + j (V, j < 16): the offsets are
// fixed per lane, and V row j + 8 is V row j plus 8 rows of 128 bytes.
template <bool kBf16>
struct AttnLane {
    int k_off[kBf16 ? 4 : 8];  // the lane's 16-byte chunks of its key row
    int v_off[8];              // the lane's two dims in V rows head*16 + j, j < 8
};

template <bool kBf16>
__device__ __forceinline__ AttnLane<kBf16> attn_lane(int head, int lane) {
    using T = AttnTma<kBf16>;
    AttnLane<kBf16> a;
    const int half = lane >> 4, krow = head * kPage + (lane & 15);
#pragma unroll
    for (int c = 0; c < (kBf16 ? 4 : 8); ++c) {
        if constexpr (kBf16) a.k_off[c] = krow * 128 + (((half * 4 + c) ^ (krow & 7)) << 4);
        else a.k_off[c] = half * T::kBoxBytes + krow * 128 + ((c ^ (krow & 7)) << 4);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int vrow = head * kPage + j;
        if constexpr (kBf16) a.v_off[j] = vrow * 128 + (((lane >> 2) ^ (vrow & 7)) << 4) + (lane & 3) * 4;
        else a.v_off[j] = (lane >> 4) * T::kBoxBytes + vrow * 128 + ((((lane & 15) >> 1) ^ (vrow & 7)) << 4) + (lane & 1) * 8;
    }
    return a;
}

// One page of one head (the warp's) into the online softmax state (m, l,
// a0, a1), in two halves so that a ring can release the K block before the
// V block is read. attn_page_k: lane l scores key (l & 15) over dims
// (l >> 4)*32 .. +31, the two halves meet with one shuffle; keys key0 + k
// with key0 + k >= n_keys are masked (exp(-inf) = 0); the running max, sum
// and rescaled accumulators are updated and the key's probability pr (lane
// l: key l & 15) returned. attn_page_v: P.V, lane l owns output dims 2l,
// 2l+1. attn_page = both, for a ring holding K and V together; shared with
// the persistent step kernel.
template <bool kBf16>
__device__ __forceinline__ float attn_page_k(const uint8_t* sK, const AttnLane<kBf16>& ad, const float (&qh)[32],
                                             int key0, int n_keys, float& m, float& l, float& a0, float& a1,
                                             bool& finite_ok) {
    const int lane = threadIdx.x & 31;
    const bool valid = key0 + (lane & 15) < n_keys;
    // four independent partial dots (a quarter of the lane's 32 dims each),
    // summed pairwise: a short dependency chain per page
    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if constexpr (kBf16) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint4 v = *reinterpret_cast<const uint4*>(sK + ad.k_off[c]);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                d[c] = fmaf(qh[8 * c + 2 * k], __uint_as_float(w[k] << 16), d[c]);
                d[c] = fmaf(qh[8 * c + 2 * k + 1], __uint_as_float(w[k] & 0xffff0000u), d[c]);
            }
        }
    } else {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const float4 v = *reinterpret_cast<const float4*>(sK + ad.k_off[c]);
            d[c >> 1] = fmaf(qh[4 * c], v.x, d[c >> 1]);
            d[c >> 1] = fmaf(qh[4 * c + 1], v.y, d[c >> 1]);
            d[c >> 1] = fmaf(qh[4 * c + 2], v.z, d[c >> 1]);
            d[c >> 1] = fmaf(qh[4 * c + 3], v.w, d[c >> 1]);
        }
    }
    float dot = (d[0] + d[1]) + (d[2] + d[3]);
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
    m = m_new;
    return pr;
}

template <bool kBf16>
__device__ __forceinline__ float2 attn_v_pair(const uint8_t* vp) {
    if constexpr (kBf16) {
        const uint32_t w2 = *reinterpret_cast<const uint32_t*>(vp);
        return make_float2(__uint_as_float(w2 << 16), __uint_as_float(w2 & 0xffff0000u));
    } else {
        return *reinterpret_cast<const float2*>(vp);
    }
}

// P.V of one page: even and odd keys in two independent chains, added to
// the (rescaled) accumulators at the end.
template <bool kBf16>
__device__ __forceinline__ void attn_page_v(const uint8_t* sV, const AttnLane<kBf16>& ad, float pr, int key0,
                                            int n_keys, float& a0, float& a1) {
    const int n_valid = min(kPage, n_keys - key0);
    float e0 = 0.0f, e1 = 0.0f, o0 = 0.0f, o1 = 0.0f;
    if (n_valid == kPage) {  // full page: no per-key guard
#pragma unroll
        for (int j = 0; j < kPage; j += 2) {
            const float pe = __shfl_sync(kFull, pr, j), po = __shfl_sync(kFull, pr, j + 1);
            const float2 ve = attn_v_pair<kBf16>(sV + ad.v_off[j & 7] + (j >> 3) * 1024);
            const float2 vo = attn_v_pair<kBf16>(sV + ad.v_off[(j + 1) & 7] + ((j + 1) >> 3) * 1024);
            e0 = fmaf(pe, ve.x, e0);
            e1 = fmaf(pe, ve.y, e1);
            o0 = fmaf(po, vo.x, o0);
            o1 = fmaf(po, vo.y, o1);
        }
    } else {
#pragma unroll
        for (int j = 0; j < kPage; j += 2) {
            const float pe = __shfl_sync(kFull, pr, j), po = __shfl_sync(kFull, pr, j + 1);
            if (j < n_valid) {
                const float2 ve = attn_v_pair<kBf16>(sV + ad.v_off[j & 7] + (j >> 3) * 1024);
                e0 = fmaf(pe, ve.x, e0);
                e1 = fmaf(pe, ve.y, e1);
            }
            if (j + 1 < n_valid) {
                const float2 vo = attn_v_pair<kBf16>(sV + ad.v_off[(j + 1) & 7] + ((j + 1) >> 3) * 1024);
                o0 = fmaf(po, vo.x, o0);
                o1 = fmaf(po, vo.y, o1);
            }
        }
    }
    a0 += e0 + o0;
    a1 += e1 + o1;
}

// A bf16 page's share of one consumer lane in registers: its four 16-byte K
// chunks and its two dims of V for the 16 keys. attn_tma_kernel loads these
// and releases the ring stage before the math, so a stage is held only for
// the shared-memory loads. The math (attn_page_regs) is attn_page_k +
// attn_page_v operation for operation, on register data.
struct PageRegsBf16 {
    uint4 k[4];
    uint32_t v[kPage];
};

__device__ __forceinline__ void load_page_bf16(const uint8_t* sK, const uint8_t* sV, const AttnLane<true>& ad,
                                               PageRegsBf16& r) {
#pragma unroll
    for (int c = 0; c < 4; ++c) r.k[c] = *reinterpret_cast<const uint4*>(sK + ad.k_off[c]);
#pragma unroll
    for (int j = 0; j < kPage; ++j) r.v[j] = *reinterpret_cast<const uint32_t*>(sV + ad.v_off[j & 7] + (j >> 3) * 1024);
}

__device__ __forceinline__ void attn_page_regs(const PageRegsBf16& r, const float (&qh)[32], int key0, int n_keys,
                                               float& m, float& l, float& a0, float& a1, bool& finite_ok) {
    const int lane = threadIdx.x & 31;
    const bool valid = key0 + (lane & 15) < n_keys;
    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint32_t w[4] = {r.k[c].x, r.k[c].y, r.k[c].z, r.k[c].w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            d[c] = fmaf(qh[8 * c + 2 * k], __uint_as_float(w[k] << 16), d[c]);
            d[c] = fmaf(qh[8 * c + 2 * k + 1], __uint_as_float(w[k] & 0xffff0000u), d[c]);
        }
    }
    float dot = (d[0] + d[1]) + (d[2] + d[3]);
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
    m = m_new;
    const int n_valid = min(kPage, n_keys - key0);
    float e0 = 0.0f, e1 = 0.0f, o0 = 0.0f, o1 = 0.0f;
#pragma unroll
    for (int j = 0; j < kPage; j += 2) {
        const float pe = __shfl_sync(kFull, pr, j), po = __shfl_sync(kFull, pr, j + 1);
        if (j < n_valid) {  // keys past the stream's end may hold anything
            e0 = fmaf(pe, __uint_as_float(r.v[j] << 16), e0);
            e1 = fmaf(pe, __uint_as_float(r.v[j] & 0xffff0000u), e1);
        }
        if (j + 1 < n_valid) {
            o0 = fmaf(po, __uint_as_float(r.v[j + 1] << 16), o0);
            o1 = fmaf(po, __uint_as_float(r.v[j + 1] & 0xffff0000u), o1);
        }
    }
    a0 += e0 + o0;
    a1 += e1 + o1;
}

template <bool kBf16>
__device__ __forceinline__ void attn_page(const uint8_t* sK, const uint8_t* sV, const AttnLane<kBf16>& ad,
                                          const float (&qh)[32], int key0, int n_keys, float& m, float& l, float& a0,
                                          float& a1, bool& finite_ok) {
    const float pr = attn_page_k<kBf16>(sK, ad, qh, key0, n_keys, m, l, a0, a1, finite_ok);
    attn_page_v<kBf16>(sV, ad, pr, key0, n_keys, a0, a1);
}

template <bool kBf16>
__global__ void __launch_bounds__(kAttnTmaThreads, 2) attn_tma_kernel(const __grid_constant__ CUtensorMap tm_kv,
                                                                   AttnParams p, int32_t* error) {
    using T = AttnTma<kBf16>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + T::kStages * T::kStageBytes);
    volatile int* failed = reinterpret_cast<volatile int*>(bars + 2 * T::kStages);
    volatile int* stage_chunk = failed + 1;  // [kStages]: chunk of the stage's page; -1: no more chunks
    const uint32_t full0 = smem_addr(bars), empty0 = full0 + 8 * T::kStages;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < T::kStages; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, kAttnHeadsPerCta);
        }
        *failed = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    // The plan (header, chunk tables, page ids) is host data uploaded before
    // the step's first kernel, so it may be read before the wait; so may the
    // K/V of every page but a stream's last one (the page this layer's QKV
    // launch appends to, marked ~page in the id list): the producer starts
    // its first chunk's ring before the wait.
    const int n_chunks = __ldcg(p.plan + 1);
    const int32_t* cta_split = p.plan + __ldcg(p.plan + 2);
    const int32_t* cta_page = p.plan + __ldcg(p.plan + 3);
    const int32_t* ids = p.plan + __ldcg(p.plan + 4);

    if (warp == kAttnHeadsPerCta) {
        // Ring index n runs on across splits and chunks: stage n % kStages,
        // use n / kStages. Lane j holds the id of page i0 + j of the chunk;
        // lane 0 issues. The next chunk's ticket is drawn when this chunk
        // has kTicketLead pages left to issue, so that near the end no CTA
        // holds a chunk it has not started.
        constexpr int kTicketLead = 4;
        const uint64_t policy = l2_evict_first_policy();
        int n = 0;
        bool stop = false, waited = false;
        int c = blockIdx.x;
        int f0 = 0, np = 0;
        if (c < n_chunks) {
            f0 = __ldcg(cta_page + c);
            np = __ldcg(cta_page + c + 1) - f0;
        }
        while (c < n_chunks && !stop) {
            int c_next = n_chunks, f0n = 0, npn = 0;
            const int draw_at = max(0, np - kTicketLead);
            int id = 0;
            for (int i = 0; i < np; ++i, ++n) {
                if ((i & 31) == 0) id = i + lane < np ? __ldcg(ids + f0 + i + lane) : 0;
                if (i == draw_at) {
                    if (!waited) {
                        pdl_wait();  // the ticket counter is zeroed by the step's prep kernel
                        waited = true;
                    }
                    int ticket = 0;
                    if (lane == 0) ticket = atomicAdd(p.chunk_ctr, 1);
                    c_next = static_cast<int>(gridDim.x) + __shfl_sync(kFull, ticket, 0);
                    if (c_next < n_chunks) {
                        f0n = __ldcg(cta_page + c_next);
                        npn = __ldcg(cta_page + c_next + 1) - f0n;
                    }
                }
                const int raw = __shfl_sync(kFull, id, i & 31);
                if (raw < 0 && !waited) {
                    pdl_wait();  // a stream's last page: this layer's K/V row is being appended
                    waited = true;
                }
                const int page = raw < 0 ? ~raw : raw;
                if (lane == 0) {
                    const int st = n % T::kStages;
                    if (n < T::kStages || mbar_wait(empty0 + 8 * st, ((n / T::kStages) - 1) & 1, error, failed)) {
                        const int row0 = (p.layer * p.kv.pool_pages + page) * 256;  // K block; V block follows
                        uint8_t* stage = smem + st * T::kStageBytes;
                        stage_chunk[st] = c;
                        mbar_expect_tx(full0 + 8 * st, T::kStageBytes);
#pragma unroll
                        for (int bx = 0; bx < T::kBoxes; ++bx) {
                            tma_load_2d_hint(smem_addr(stage + bx * T::kBoxBytes), &tm_kv, bx * T::kBoxCols, row0,
                                             full0 + 8 * st, policy);
                            tma_load_2d_hint(smem_addr(stage + T::kBlockBytes + bx * T::kBoxBytes), &tm_kv,
                                             bx * T::kBoxCols, row0 + 128, full0 + 8 * st, policy);
                        }
                    }
                }
                // one decision for the whole warp (a wait that gave up sets *failed)
                stop = __any_sync(kFull, *failed != 0);
                if (stop) break;
            }
            c = c_next;
            f0 = f0n;
            np = npn;
        }
        if (!stop && lane == 0) {
            pdl_trigger();  // everything left of this CTA is in the ring
            const int st = n % T::kStages;
            if (n < T::kStages || mbar_wait(empty0 + 8 * st, ((n / T::kStages) - 1) & 1, error, failed)) {
                stage_chunk[st] = -1;  // end tag: completes the stage's phase without data
                mbar_arrive(full0 + 8 * st);
            }
        }
        return;
    }

    pdl_wait();  // q and the appended K/V rows come from earlier launches
    // Consumer: head = warp (attn_page).
    const int head = warp, half = lane >> 4;
    const AttnLane<kBf16> ad = attn_lane<kBf16>(head, lane);
    int n = 0;
    bool ok = true;
    while (ok) {
        const int st0 = n % T::kStages;
        if (!__all_sync(kFull, mbar_wait(full0 + 8 * st0, (n / T::kStages) & 1, error, failed))) break;
        const int c = stage_chunk[st0];
        if (c < 0) break;
        const int s_begin = __ldcg(cta_split + c), s_end = __ldcg(cta_split + c + 1);
        bool landed = true;  // stage n (the chunk's first K block) has been waited for
        for (int s = s_begin; s < s_end && ok; ++s) {
            const Split sp = p.splits[s];
            float qh[32];
            {
                const float4* qs = reinterpret_cast<const float4*>(p.q + static_cast<size_t>(sp.b) * kWidth +
                                                                   head * kHeadDim + half * 32);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float4 v = qs[i];
                    qh[4 * i] = v.x;
                    qh[4 * i + 1] = v.y;
                    qh[4 * i + 2] = v.z;
                    qh[4 * i + 3] = v.w;
                }
            }
            float m = -INFINITY, l = 0.0f, a0 = 0.0f, a1 = 0.0f;
            bool finite_ok = true;
            for (int i = 0; i < sp.page_count; ++i, ++n) {
                const int st = n % T::kStages;
                if (!landed && !__all_sync(kFull, mbar_wait(full0 + 8 * st, (n / T::kStages) & 1, error, failed))) {
                    ok = false;  // give up: the error flag is raised
                    break;
                }
                landed = false;
                const uint8_t* sK = smem + st * T::kStageBytes;
                if constexpr (kBf16) {
                    // the lane's share into registers, the stage back to the producer, then the math
                    PageRegsBf16 pr;
                    load_page_bf16(sK, sK + T::kBlockBytes, ad, pr);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(empty0 + 8 * st);
                    attn_page_regs(pr, qh, (sp.page_begin + i) * kPage, sp.n_keys, m, l, a0, a1, finite_ok);
                } else {
                    attn_page<kBf16>(sK, sK + T::kBlockBytes, ad, qh, (sp.page_begin + i) * kPage, sp.n_keys, m, l,
                                     a0, a1, finite_ok);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(empty0 + 8 * st);
                }
            }
            if (!ok) break;
            float* out = p.part + (static_cast<size_t>(s) * kHeads + head) * kPartStride;
            *reinterpret_cast<float2*>(out + 2 + 2 * lane) = make_float2(a0, a1);
            if (lane == 0) {
                out[0] = m;
                out[1] = l;
            }
            if (!__all_sync(kFull, finite_ok) && lane == 0) flag_nonfinite(p.status, sp.b);
        }
    }
}

}  // namespace phonon
