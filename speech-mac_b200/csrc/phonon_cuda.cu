// libphonon_cuda host runtime: contexts, KV page pool, step scheduling and
// the C ABI declared in include/phonon_cuda.h.
#include "phonon_cuda.h"
#include "phonon_attention.cuh"
#include "phonon_gemm.cuh"
#include "phonon_kernels.cuh"
#include "phonon_cluster.cuh"
#include "phonon_persist.cuh"
#include "phonon_head.cuh"
#include "phonon_mimi.cuh"

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <utility>
#include <vector>

using namespace phonon;

namespace {

constexpr int kMaxLayers = 64;
constexpr int kMaxDevices = 64;
constexpr int kMaxPagesPerStream = PHONON_CUDA_MAX_POSITIONS / kPage;  // 512
constexpr int kPrefillChunk = 256;  // rows per prefill pass
// Batch paths by measurement (bf16 K/V, contexts 1000, µs per step; per-stage
// GEMV / per-stage tcgen05 / persistent): 1 stream 374 / 526 / 451, 2: 550 /
// 531 / 481, 3: 634 / 548 / 532, 4: 793 / 570 / 628, 8: 1164 / 627 / 794,
// 16: 1683 / 624 / 730, 64: 4741 / 885 / 1106.
constexpr int kTensorMinBatch = 4;   // streams from which projections run on tcgen05
constexpr int kMaxSms = 1024;        // bound on the SM count (persistent split table)
constexpr int kSmCount = 148;        // B200 SMs (launch-shape heuristics only)
constexpr int kFusedMinBatch = 2;    // default window of the persistent step
constexpr int kFusedMaxBatch = 3;
constexpr int kPlanHeader = 8;       // ints of the step plan header in the metadata
constexpr int kGuide = 2;            // guided chunks: remaining pages / (kGuide * attention CTAs)
constexpr uint32_t kClusterMaxPosF32 = 1152;   // default cluster-step window (positions below), fp32 K/V
constexpr uint32_t kClusterMaxPosBf16 = 1248;  // ... bf16 K/V
constexpr int kTicketMinChunk = 8;   // pages per guided chunk, at least
constexpr int kMaxChunks = 8192;     // chunks per plan, at most
constexpr int kSplitMinBatch = 96;   // from here a step runs as two concurrent half batches

#define CUDA_TRY(expr)                                                                       \
    do {                                                                                     \
        cudaError_t err_ = (expr);                                                           \
        if (err_ != cudaSuccess) {                                                           \
            std::fprintf(stderr, "phonon_cuda: %s failed: %s (%s:%d)\n", #expr,              \
                         cudaGetErrorString(err_), __FILE__, __LINE__);                      \
            return PHONON_CUDA_DEVICE_ERROR;                                                 \
        }                                                                                    \
    } while (0)

// Launch with programmatic dependent launch allowed: the kernel may begin
// while the previous kernel of the stream drains (see pdl_wait/pdl_trigger).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// ------------------------------------------------------------ device linears
struct DevLinear {
    int kind = 0;
    int rows = 0, cols = 0;
    bool fast = false;  // lane-interleaved layout for the GEMV kernel
    void* plane = nullptr;
    __half* scales = nullptr;
    size_t bytes = 0;
    // Tensor-core copy of a Q8_0 linear: one natural row-major int8 plane
    // [rows][cols] when every 32-block of a row shares one scale (wd = 1),
    // else three weight digit planes [3][rows][cols] of the per-block-scaled
    // integers (wd = 3, phonon_gemm.cuh), and the fp32 row scales.
    bool tensor = false;
    int wd = 1;
    int8_t* nat = nullptr;       // [wd * rows][cols]
    float* row_scale = nullptr;  // [rows]
    CUtensorMap tmap;            // 128-byte x 128-row SWIZZLE_128B boxes over `nat`
};

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// 2-D tiled map over [rows][cols] elements, rows `pitch` bytes apart,
// boxes of box_cols x box_rows, SWIZZLE_128B.
bool make_map_2d(CUtensorMap* map, CUtensorMapDataType type, const void* base, uint64_t rows, uint64_t cols,
                 uint64_t pitch, uint32_t box_cols, uint32_t box_rows) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn || pitch % 16 || reinterpret_cast<uintptr_t>(base) % 16) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {pitch};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estride[2] = {1, 1};
    return fn(map, type, 2, const_cast<void*>(base), dims, strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// int8 [rows][cols] (cols bytes per row) in 128-byte x 128-row boxes.
bool make_i8_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols) {
    if (cols % kGemmKTile) return false;
    return make_map_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, base, rows, cols, cols, kGemmKTile, 128);
}

bool half_is_finite(uint16_t h) { return ((h >> 10) & 0x1f) != 0x1f; }

bool bf16_is_finite(uint16_t b) { return ((b >> 7) & 0xff) != 0xff; }

float bf16_host(uint16_t b) {
    uint32_t u = static_cast<uint32_t>(b) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

void free_linear(DevLinear& l) {
    if (l.plane) cudaFree(l.plane);
    if (l.scales) cudaFree(l.scales);
    if (l.nat) cudaFree(l.nat);
    if (l.row_scale) cudaFree(l.row_scale);
    l = DevLinear{};
}

// Repack a host Q8_0 (34-byte blocks) or bf16 [rows, cols] matrix into the
// device layout and upload it. The fast layout is described next to
// GemvParams in phonon_kernels.cuh; other shapes keep natural row-major order.
int upload_linear(int kind, const void* host, size_t rows, size_t cols, DevLinear* out) {
    if (!host || !rows || !cols || rows > (1u << 24) || cols > (1u << 20)) return PHONON_CUDA_INVALID_ARGUMENT;
    if (kind == PHONON_CUDA_LINEAR_Q8_0 && cols % 32) return PHONON_CUDA_INVALID_ARGUMENT;
    if (kind != PHONON_CUDA_LINEAR_Q8_0 && kind != PHONON_CUDA_LINEAR_BF16) return PHONON_CUDA_INVALID_ARGUMENT;
    DevLinear l;
    l.kind = kind;
    l.rows = static_cast<int>(rows);
    l.cols = static_cast<int>(cols);
    l.fast = cols % 512 == 0 && (cols == 512 || cols == 2048);
    const size_t n = rows * cols;
    auto logical = [&](size_t c) -> size_t {  // device column position -> logical column
        if (!l.fast) return c;
        const size_t chunk = c / 512, in = c % 512, lane = in / 16, j = (in % 16) / 4, e = in % 4;
        return chunk * 512 + j * 128 + lane * 4 + e;
    };
    if (kind == PHONON_CUDA_LINEAR_Q8_0) {
        const uint8_t* blocks = static_cast<const uint8_t*>(host);
        std::vector<int8_t> q(n);
        std::vector<uint16_t> s(n / 32);
        for (size_t r = 0; r < rows; ++r) {
            const uint8_t* row = blocks + r * (cols / 32) * 34;
            for (size_t b = 0; b < cols / 32; ++b) {
                const uint16_t h = static_cast<uint16_t>(row[b * 34] | (row[b * 34 + 1] << 8));
                if (!half_is_finite(h)) return PHONON_CUDA_NON_FINITE;
                size_t dst = b;
                if (l.fast) {  // block c*16 + j*4 + g stored at c*16 + g*4 + j
                    const size_t c = b / 16, k = b % 16, j = k / 4, g = k % 4;
                    dst = c * 16 + g * 4 + j;
                }
                s[r * (cols / 32) + dst] = h;
            }
            for (size_t c = 0; c < cols; ++c) {
                const size_t lc = logical(c);
                q[r * cols + c] = static_cast<int8_t>(row[(lc / 32) * 34 + 2 + lc % 32]);
            }
        }
        // Tensor-core eligibility: every 32-block of a row has the same scale.
        bool uniform = cols % kGemmKTile == 0;
        std::vector<int8_t> nat;
        std::vector<float> rs;
        if (uniform) {
            nat.resize(n);
            rs.resize(rows);
            for (size_t r = 0; r < rows && uniform; ++r) {
                const uint8_t* row = blocks + r * (cols / 32) * 34;
                const uint16_t h0 = static_cast<uint16_t>(row[0] | (row[1] << 8));
                for (size_t b = 0; b < cols / 32; ++b) {
                    if (static_cast<uint16_t>(row[b * 34] | (row[b * 34 + 1] << 8)) != h0) uniform = false;
                    std::memcpy(&nat[r * cols + b * 32], row + b * 34 + 2, 32);
                }
                __half_raw hr;
                hr.x = h0;
                rs[r] = __half2float(__half(hr));
            }
        }
        if (cudaMalloc(&l.plane, n) != cudaSuccess ||
            cudaMalloc(reinterpret_cast<void**>(&l.scales), s.size() * 2) != cudaSuccess ||
            (uniform && (cudaMalloc(&l.nat, n) != cudaSuccess || cudaMalloc(&l.row_scale, rows * 4) != cudaSuccess))) {
            free_linear(l);
            return PHONON_CUDA_OUT_OF_MEMORY;
        }
        if (uniform) {
            if (cudaMemcpy(l.nat, nat.data(), n, cudaMemcpyHostToDevice) != cudaSuccess ||
                cudaMemcpy(l.row_scale, rs.data(), rows * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
                free_linear(l);
                return PHONON_CUDA_DEVICE_ERROR;
            }
            l.tensor = make_i8_map(&l.tmap, l.nat, rows, cols);
        } else if (cols % kGemmKTile == 0 && rows % kGemmM == 0) {
            // Per-block scales: three weight digit planes (phonon_gemm.cuh).
            std::vector<int8_t> planes(3 * n);
            rs.assign(rows, 1.0f);
            for (size_t r = 0; r < rows; ++r) {
                const uint8_t* row = blocks + r * (cols / 32) * 34;
                int emax = INT32_MIN;
                for (size_t b = 0; b < cols / 32; ++b) {
                    const uint16_t h = static_cast<uint16_t>(row[b * 34] | (row[b * 34 + 1] << 8));
                    const int e5 = (h >> 10) & 0x1f, m = (e5 ? 1024 : 0) + (h & 0x3ff);
                    if (m) emax = std::max(emax, (e5 ? e5 : 1) - 25);
                }
                if (emax == INT32_MIN) continue;  // an all-zero row: zero planes
                rs[r] = std::ldexp(1.0f, emax - 2);
                for (size_t b = 0; b < cols / 32; ++b) {
                    const uint16_t h = static_cast<uint16_t>(row[b * 34] | (row[b * 34 + 1] << 8));
                    const int e5 = (h >> 10) & 0x1f, m = (e5 ? 1024 : 0) + (h & 0x3ff);
                    const int sign = (h & 0x8000) ? -1 : 1;
                    const int shift = (e5 ? e5 : 1) - 25 - emax + 2;  // <= 2
                    for (size_t i = 0; i < 32; ++i) {
                        const long long qm = static_cast<long long>(static_cast<int8_t>(row[b * 34 + 2 + i])) * m * sign;
                        const long long W = shift >= 0 ? qm << shift : std::llround(std::ldexp(static_cast<double>(qm), shift));
                        const long long w2 = ((W + 64) % 128 + 128) % 128 - 64;
                        const long long W1 = (W - w2) / 128;
                        const long long w1 = ((W1 + 64) % 128 + 128) % 128 - 64;
                        const long long w0 = (W1 - w1) / 128;
                        const size_t at = r * cols + b * 32 + i;
                        planes[at] = static_cast<int8_t>(w0);
                        planes[n + at] = static_cast<int8_t>(w1);
                        planes[2 * n + at] = static_cast<int8_t>(w2);
                    }
                }
            }
            if (cudaMalloc(&l.nat, 3 * n) != cudaSuccess || cudaMalloc(&l.row_scale, rows * 4) != cudaSuccess) {
                free_linear(l);
                return PHONON_CUDA_OUT_OF_MEMORY;
            }
            if (cudaMemcpy(l.nat, planes.data(), 3 * n, cudaMemcpyHostToDevice) != cudaSuccess ||
                cudaMemcpy(l.row_scale, rs.data(), rows * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
                free_linear(l);
                return PHONON_CUDA_DEVICE_ERROR;
            }
            l.wd = 3;
            l.tensor = make_i8_map(&l.tmap, l.nat, 3 * rows, cols);
        }
        if (cudaMemcpy(l.plane, q.data(), n, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(l.scales, s.data(), s.size() * 2, cudaMemcpyHostToDevice) != cudaSuccess) {
            free_linear(l);
            return PHONON_CUDA_DEVICE_ERROR;
        }
        l.bytes = n + s.size() * 2;
    } else {
        const uint16_t* src = static_cast<const uint16_t*>(host);
        std::vector<uint16_t> w(n);
        for (size_t r = 0; r < rows; ++r)
            for (size_t c = 0; c < cols; ++c) {
                const uint16_t v = src[r * cols + logical(c)];
                if (!bf16_is_finite(v)) return PHONON_CUDA_NON_FINITE;
                w[r * cols + c] = v;
            }
        if (cudaMalloc(&l.plane, n * 2) != cudaSuccess) return PHONON_CUDA_OUT_OF_MEMORY;
        if (cudaMemcpy(l.plane, w.data(), n * 2, cudaMemcpyHostToDevice) != cudaSuccess) {
            free_linear(l);
            return PHONON_CUDA_DEVICE_ERROR;
        }
        l.bytes = n * 2;
    }
    *out = l;
    return PHONON_CUDA_OK;
}

// ------------------------------------------------------------- GEMV launcher
// The opt-in shared memory size is a per-device function attribute: one bit
// per device of `configured` records that it is set (host threads may race
// here; setting the attribute twice is harmless).
cudaError_t opt_in_smem(const void* kern, int smem, std::atomic<uint64_t>& configured) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    const uint64_t bit = uint64_t{1} << dev;
    if (!(configured.load(std::memory_order_acquire) & bit)) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured.fetch_or(bit, std::memory_order_release);
    }
    return cudaSuccess;
}

template <bool kQ8, int kChunks, int kBT, int kSrc, int kEpi>
cudaError_t launch_gemv_t(const GemvParams& p, cudaStream_t s) {
    auto kern = gemv_kernel<kQ8, kChunks, kBT, kSrc, kEpi>;
    constexpr int smem = kBT * kChunks * 512 * 4;
    if constexpr (smem > 48 * 1024) {
        static std::atomic<uint64_t> configured{0};
        const cudaError_t e = opt_in_smem(reinterpret_cast<const void*>(kern), smem, configured);
        if (e != cudaSuccess) return e;
    }
    const int rows_per_cta = kGemvWarps * kRowsPerWarp;
    const int gx = (p.rows + rows_per_cta - 1) / rows_per_cta;
    // Large batches of a matrix with few row blocks: split the streams over
    // grid.y so that about two CTAs per SM run (each re-reads its rows'
    // weights, a few KB from L2).
    GemvParams q = p;
    int gy = 1;
    const int tiles = (p.B + kBT - 1) / kBT;
    const int want = (2 * kSmCount + gx - 1) / gx;
    if (want > 1 && tiles > 1) {
        gy = std::min(want, tiles);
        q.b_per_cta = ((tiles + gy - 1) / gy) * kBT;
        gy = (p.B + q.b_per_cta - 1) / q.b_per_cta;
    } else {
        q.b_per_cta = 0;
    }
    return launch_pdl(kern, dim3(gx, gy), dim3(kGemvWarps * 32), smem, s, q);
}

template <bool kQ8, int kChunks, int kSrc, int kEpi>
cudaError_t launch_gemv_bt(const GemvParams& p, cudaStream_t s) {
    if (p.B <= 1) return launch_gemv_t<kQ8, kChunks, 1, kSrc, kEpi>(p, s);
    if (p.B <= 2) return launch_gemv_t<kQ8, kChunks, 2, kSrc, kEpi>(p, s);
    if (p.B <= 4) return launch_gemv_t<kQ8, kChunks, 4, kSrc, kEpi>(p, s);
    return launch_gemv_t<kQ8, kChunks, 8, kSrc, kEpi>(p, s);
}

template <int kChunks, int kSrc, int kEpi>
cudaError_t launch_gemv(bool q8, const GemvParams& p, cudaStream_t s) {
    return q8 ? launch_gemv_bt<true, kChunks, kSrc, kEpi>(p, s) : launch_gemv_bt<false, kChunks, kSrc, kEpi>(p, s);
}

cudaError_t launch_linear(const DevLinear& l, const float* x, int B, const float* bias, float* y,
                          int32_t* status, cudaStream_t s) {
    const bool q8 = l.kind == PHONON_CUDA_LINEAR_Q8_0;
    if (l.fast) {
        GemvParams p{};
        p.w = l.plane;
        p.scales = l.scales;
        p.rows = l.rows;
        p.cols = l.cols;
        p.x = x;
        p.ldx = l.cols;
        p.B = B;
        p.bias = bias;
        p.y = y;
        p.ldy = l.rows;
        p.status = status;
        return l.cols == 512 ? launch_gemv<1, SRC_X, EPI_STORE>(q8, p, s) : launch_gemv<4, SRC_X, EPI_STORE>(q8, p, s);
    }
    const long long warps = static_cast<long long>(l.rows) * B;
    const int threads = 256;
    const long long blocks = (warps * 32 + threads - 1) / threads;
    if (q8)
        linear_generic_kernel<true><<<static_cast<unsigned>(blocks), threads, 0, s>>>(l.plane, l.scales, l.rows, l.cols, x, B, bias, y, status);
    else
        linear_generic_kernel<false><<<static_cast<unsigned>(blocks), threads, 0, s>>>(l.plane, nullptr, l.rows, l.cols, x, B, bias, y, status);
    return cudaGetLastError();
}

template <int kEpi, int kWD = 1>
cudaError_t launch_gemm(const CUtensorMap& tw, const CUtensorMap& tx, int rows, int n_digit_rows, const GemmParams& p,
                        cudaStream_t s) {
    static std::atomic<uint64_t> configured{0};
    constexpr int smem = gemm_smem(kWD);
    cudaError_t e = opt_in_smem(reinterpret_cast<const void*>(i8_gemm_kernel<kEpi, kWD>), smem, configured);
    if (e != cudaSuccess) return e;
    dim3 grid((rows + kGemmM - 1) / kGemmM, (n_digit_rows + kGemmN - 1) / kGemmN);
    return launch_pdl(i8_gemm_kernel<kEpi, kWD>, grid, dim3(kGemmThreads), smem, s, tw, tx, p);
}

// A projection of a linear on the tensor cores: one or three weight planes.
template <int kEpi>
cudaError_t launch_linear_gemm(const DevLinear& w, const CUtensorMap& tx, int n_digit_rows, const GemmParams& p,
                               cudaStream_t s) {
    return w.wd == 3 ? launch_gemm<kEpi, 3>(w.tmap, tx, w.rows, n_digit_rows, p, s)
                     : launch_gemm<kEpi, 1>(w.tmap, tx, w.rows, n_digit_rows, p, s);
}

template <bool kBf16>
cudaError_t launch_attn_tma(const CUtensorMap& tm, const AttnParams& p, int32_t* err, int n_ctas, cudaStream_t s) {
    static std::atomic<uint64_t> configured{0};
    cudaError_t e = opt_in_smem(reinterpret_cast<const void*>(attn_tma_kernel<kBf16>), AttnTma<kBf16>::kSmem, configured);
    if (e != cudaSuccess) return e;
    return launch_pdl(attn_tma_kernel<kBf16>, dim3(n_ctas), dim3(kAttnTmaThreads), AttnTma<kBf16>::kSmem, s, tm, p, err);
}

template <int kCols, bool kLN>
cudaError_t launch_digits(const float* x, int ldx, const float* ln_w, const float* ln_b, int B, int Bpad,
                          int8_t* digits, int32_t* exps, int32_t* status, cudaStream_t s) {
    if constexpr (kLN) {
        static_assert(kCols == kWidth, "LayerNorm rows are 512 wide");
        return launch_pdl(ln_digits_kernel, dim3((Bpad + 7) / 8), dim3(256), 0, s, x, ldx, ln_w, ln_b, B, Bpad,
                          digits, exps, status);
    } else {
        constexpr int rows_per_cta = 256 / (kCols / 8);
        return launch_pdl(digits_kernel<kCols>, dim3((Bpad + rows_per_cta - 1) / rows_per_cta), dim3(256), 0, s, x,
                          ldx, B, Bpad, digits, exps, status);
    }
}

}  // namespace

// ------------------------------------------------------------------- context
struct StreamSlot {
    bool used = false;
    uint32_t capacity = 0, length = 0;
    std::vector<int32_t> pages;
};

struct DevLayer {
    DevLinear qkv, out, up, down;
    float* norms = nullptr;  // fp32 [4][512]: norm1 w, norm1 b, norm2 w, norm2 b
    bool q8 = true;
};

// Per-step scratch and stream of one lane. A large batch can be split over
// two lanes that run concurrently (one half's attention overlaps the other
// half's projections); lane 0 uses the context's main stream and buffers.
struct Lane {
    cudaStream_t stream = nullptr;
    float *x0 = nullptr, *x1 = nullptr, *q = nullptr, *a = nullptr, *h = nullptr, *g = nullptr, *part = nullptr;
    int32_t *meta = nullptr, *h_meta = nullptr;
    int8_t *dig512 = nullptr, *dig2048 = nullptr;
    int32_t* exps = nullptr;
    CUtensorMap tm_dig512, tm_dig2048;
    float2* rope = nullptr;
    cudaEvent_t ready = nullptr;  // recorded when the lane's share of a step is enqueued
    int32_t* chunk_ctr = nullptr;  // [n_layers] attention chunk tickets, zeroed at step start
    std::vector<long long> h_cuts;  // host scratch of the split planner: chunk boundaries
    std::vector<int32_t> h_pages;   //   page ids in split order
    std::vector<int32_t> h_first_split;  //   first split of each chunk
};

struct PhononCuda {
    PhononCudaConfig cfg{};
    std::mutex mu;
    cudaStream_t stream = nullptr;
    std::vector<DevLayer> layers;
    void* kv_pool = nullptr;
    long long page_elems = 0;
    int32_t* d_table = nullptr;
    std::vector<int32_t> free_pages;
    std::vector<StreamSlot> streams;
    std::vector<int32_t> h_fresh_page;  // split planner scratch per stream slot (INT32_MAX between calls)
    float* d_freq = nullptr;
    int cap_rows = 0, max_splits = 0, meta_ints = 0;
    float2* d_rope = nullptr;
    float *d_x0 = nullptr, *d_x1 = nullptr, *d_y = nullptr, *d_q = nullptr, *d_a = nullptr,
          *d_h = nullptr, *d_g = nullptr, *d_part = nullptr, *d_stage = nullptr;
    int32_t *d_meta = nullptr, *d_status = nullptr;
    // tensor-core path: digit rows of the current batch and their exponents
    int8_t *d_dig512 = nullptr, *d_dig2048 = nullptr;
    int32_t *d_exps = nullptr, *d_err = nullptr;
    CUtensorMap tm_dig512, tm_dig2048;
    bool tensor_ok = false;
    // KV pool as rows of 64 head dims for TMA page staging
    CUtensorMap tm_kv;
    bool attn_tma = false;
    // Single-stream steps on one 16-CTA cluster (step_cluster_kernel): one
    // head's K/V blocks of a page as 16-row boxes; steps of one stream at a
    // position below cluster_max_pos take that path when cluster_ok.
    CUtensorMap tm_kv16;
    bool cluster_ok = false;
    // ... with every projection on the tensor cores when every layer's
    // weights have one scale per row (d_cltc: their K-slice units,
    // cluster_tc_pack_kernel)
    bool cluster_tc = false;
    uint8_t* d_cltc = nullptr;
    uint32_t cluster_max_pos = PHONON_CUDA_MAX_POSITIONS;  // set at creation from the K/V type
    Lane lanes[2];
    bool lane1_ok = false;  // second lane allocated
    // Whole-step persistent kernel (batches up to fused_max streams)
    int sms = 0, smem_optin = 0;
    bool persist_ok = false;         // device and weights allow it
    uint32_t fused_min = kFusedMinBatch, fused_max = kFusedMaxBatch;
    uint32_t split_min = kSplitMinBatch;  // batches from which a step runs on two lanes
    cudaEvent_t fork = nullptr, join = nullptr;
    uint32_t tensor_min = kTensorMinBatch;
    PersistLayer* d_players = nullptr;  // [n_layers]
    unsigned* d_bar = nullptr;
    unsigned bar_epoch = 0;
    int32_t* h_meta = nullptr;
    float *h_x = nullptr, *h_y = nullptr, *h_stage = nullptr;
    size_t stage_cap = 0;  // floats in d_stage / h_stage
    int32_t* h_status = nullptr;
    // Replay of repeated step shapes: the step's kernels are captured into a
    // CUDA graph the second time the same StepShape comes
    // in a row and replayed while it repeats (a batch-1 decode keeps its
    // split count for 16 positions).
    // Everything the captured launches depend on besides the metadata
    // contents: batch and split counts, attention grid, buffers.
    struct StepShape {
        int R = -1, S = -1, chunks = -1;
        const void* in = nullptr;
        const void* out = nullptr;
        bool operator==(const StepShape& o) const {
            return R == o.R && S == o.S && chunks == o.chunks && in == o.in && out == o.out;
        }
    };
    StepShape last_shape, graph_shape;
    cudaGraphExec_t graph_exec = nullptr;
    uint64_t graph_kernels = 0;
    // launch accounting and live profiling
    uint64_t launches = 0;
    bool prof_on = false;
    struct ProfRec {
        int cls;
        cudaEvent_t a, b;
        double bytes;
    };
    std::vector<ProfRec> prof_pending;
    std::vector<cudaEvent_t> prof_events;  // free list
    double prof_ms[PHONON_CUDA_K_COUNT] = {};
    double prof_bytes[PHONON_CUDA_K_COUNT] = {};
    uint64_t prof_launches[PHONON_CUDA_K_COUNT] = {};
    // per-layer output trace of decode steps (phonon_cuda_set_layer_trace)
    float* trace = nullptr;
    uint32_t trace_rows = 0;
    bool tracing = false;  // inside a traced decode step
    // pending phonon_cuda_step_device
    bool pending = false;
    std::vector<uint32_t> pending_streams;
    std::vector<int32_t> pending_new_pages;
};

namespace {

void free_layer(DevLayer& D) {
    free_linear(D.qkv);
    free_linear(D.out);
    free_linear(D.up);
    free_linear(D.down);
    if (D.norms) cudaFree(D.norms);
    D = DevLayer{};
}

// Upload one layer into `D` (freeing what it held only once the new copy is
// complete, so a failed upload leaves the old weights in place).
int load_layer(DevLayer* D, const PhononCudaLayer& w) {
    if (!w.qkv || !w.attention_out || !w.mlp_in || !w.mlp_out || !w.norm1_weight || !w.norm1_bias ||
        !w.norm2_weight || !w.norm2_bias ||
        (w.linear_kind != PHONON_CUDA_LINEAR_Q8_0 && w.linear_kind != PHONON_CUDA_LINEAR_BF16))
        return PHONON_CUDA_INVALID_ARGUMENT;
    float norms[4 * kWidth];
    const uint16_t* src[4] = {w.norm1_weight, w.norm1_bias, w.norm2_weight, w.norm2_bias};
    for (int k = 0; k < 4; ++k)
        for (int i = 0; i < kWidth; ++i) {
            if (!bf16_is_finite(src[k][i])) return PHONON_CUDA_NON_FINITE;
            norms[k * kWidth + i] = bf16_host(src[k][i]);
        }
    DevLayer N;
    N.q8 = w.linear_kind == PHONON_CUDA_LINEAR_Q8_0;
    int st;
    if ((st = upload_linear(w.linear_kind, w.qkv, 1536, 512, &N.qkv)) ||
        (st = upload_linear(w.linear_kind, w.attention_out, 512, 512, &N.out)) ||
        (st = upload_linear(w.linear_kind, w.mlp_in, 2048, 512, &N.up)) ||
        (st = upload_linear(w.linear_kind, w.mlp_out, 512, 2048, &N.down))) {
        free_layer(N);
        return st;
    }
    if (cudaMalloc(&N.norms, sizeof(norms)) != cudaSuccess) {
        free_layer(N);
        return PHONON_CUDA_OUT_OF_MEMORY;
    }
    if (cudaMemcpy(N.norms, norms, sizeof(norms), cudaMemcpyHostToDevice) != cudaSuccess) {
        free_layer(N);
        return PHONON_CUDA_DEVICE_ERROR;
    }
    free_layer(*D);
    *D = N;
    return PHONON_CUDA_OK;
}

KvView kv_view(const PhononCuda* c) {
    KvView kv;
    kv.pool = c->kv_pool;
    kv.pool_pages = static_cast<int>(c->cfg.pool_pages);
    kv.bf16 = c->cfg.kv_type == PHONON_CUDA_KV_BF16;
    kv.table = c->d_table;
    kv.max_pages = kMaxPagesPerStream;
    return kv;
}

bool valid_stream(const PhononCuda* c, uint32_t s) { return s < c->streams.size() && c->streams[s].used; }

cudaEvent_t prof_event(PhononCuda* c) {
    if (!c->prof_events.empty()) {
        cudaEvent_t e = c->prof_events.back();
        c->prof_events.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

// Bracket one kernel launch: count it and, when profiling, time it.
struct LaunchScope {
    PhononCuda* c;
    int cls;
    double bytes;
    cudaStream_t s;
    cudaEvent_t a = nullptr;
    LaunchScope(PhononCuda* c_, int cls_, double bytes_, cudaStream_t s_ = nullptr)
        : c(c_), cls(cls_), bytes(bytes_), s(s_ ? s_ : c_->stream) {
        c->launches++;
        if (c->prof_on) {
            a = prof_event(c);
            cudaEventRecord(a, s);
        }
    }
    ~LaunchScope() {
        if (!a) return;
        cudaEvent_t b = prof_event(c);
        cudaEventRecord(b, s);
        c->prof_pending.push_back({cls, a, b, bytes});
    }
};

// Fold finished launch timings into the totals (after a stream sync).
void prof_collect(PhononCuda* c) {
    for (auto& r : c->prof_pending) {
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, r.a, r.b) == cudaSuccess) {
            c->prof_ms[r.cls] += ms;
            c->prof_bytes[r.cls] += r.bytes;
            c->prof_launches[r.cls] += 1;
        }
        c->prof_events.push_back(r.a);
        c->prof_events.push_back(r.b);
    }
    c->prof_pending.clear();
}

// Device bytes of one linear's weights (int8 plane + fp16 scales, or bf16).
double linear_bytes(const DevLinear& l) { return static_cast<double>(l.bytes); }

// Row batch for one enqueue: entry e is (stream slot, position); splits are
// planned over the pages each entry attends.
struct Batch {
    int R = 0, S = 0, U = 0;
    bool persist = false;  // whole step in step_persist_kernel
    bool split = false;    // one lane's share of a step split over two lanes
    int row0 = 0;          // first row of this batch within the step (the second lane's half)
    Lane* lane = nullptr;
    int32_t* d_status = nullptr;  // status words of this batch's entries
    double keys = 0;  // sum over entries of (position + 1)
    float2* d_rope = nullptr;  // [R][32] (cos, sin) of this batch's positions
    int32_t *d_slot, *d_pos, *d_first, *d_count, *d_updates;
    int32_t* d_plan = nullptr;       // plan header (splits, chunks, table offsets)
    int32_t* d_cta_split = nullptr;  // split range of each chunk (chunk k = persistent CTA k)
    int n_chunks = 0;
    int attn_grid = 0;  // attention CTAs (chunks beyond the first attn_grid go by ticket)
    Split* d_splits;
};

// Pages the caller allocated in this call, so that a failure can return them.
struct PageUndo {
    PhononCuda* c;
    std::vector<std::pair<uint32_t, int32_t>> taken;  // (stream, page)
    void rollback() {
        for (auto it = taken.rbegin(); it != taken.rend(); ++it) {
            c->streams[it->first].pages.pop_back();
            c->free_pages.push_back(it->second);
        }
        taken.clear();
    }
};

// Grow stream s to at least n pages; records page-table updates.
int ensure_pages(PhononCuda* c, uint32_t s, uint32_t n, PageUndo& undo, std::vector<int32_t>& updates) {
    StreamSlot& st = c->streams[s];
    while (st.pages.size() < n) {
        if (c->free_pages.empty()) return PHONON_CUDA_POOL_EXHAUSTED;
        const int32_t page = c->free_pages.back();
        c->free_pages.pop_back();
        updates.push_back(static_cast<int32_t>(s));
        updates.push_back(static_cast<int32_t>(st.pages.size()));
        updates.push_back(page);
        st.pages.push_back(page);
        undo.taken.emplace_back(s, page);
    }
    return PHONON_CUDA_OK;
}

void release_pages(PhononCuda* c, uint32_t s) {
    StreamSlot& st = c->streams[s];
    for (auto it = st.pages.rbegin(); it != st.pages.rend(); ++it) c->free_pages.push_back(*it);
    st.pages.clear();
    st.length = 0;
}

// Shared-memory plan of step_persist_kernel for R streams on G SMs: the
// union of the stage-B page ring and the activation rows of a group, then
// the two weight buffers (QKV|up and out|down rows of one CTA), then the
// mbarriers and flags. False when it exceeds the per-CTA opt-in limit.
struct PersistShape {
    int n_groups = 0, smem = 0, off_x = 0, off_w0 = 0, off_w1 = 0, off_norm = 0, off_bar = 0, ring = 0;
};

bool persist_shape(int R, int G, int smem_limit, bool bf16, PersistShape* out) {
    PersistShape sh;
    sh.n_groups = (R + kPersistGroup - 1) / kPersistGroup;
    const int nct = G / sh.n_groups;
    if (R < 1 || nct < 1) return false;
    const int w0 = std::max(persist_cta_rows(PM_QKV, nct) * persist_row_bytes(PM_QKV),
                            persist_cta_rows(PM_UP, nct) * persist_row_bytes(PM_UP));
    const int w1 = std::max(persist_cta_rows(PM_OUT, nct) * persist_row_bytes(PM_OUT),
                            persist_cta_rows(PM_DOWN, nct) * persist_row_bytes(PM_DOWN));
    // Stage B's page ring spans the activation region (the GELU rows of a
    // group in stage E) and both weight buffers, which hold nothing in flight
    // then: up to kPersistMaxRing stages, at least 2.
    const int stage = bf16 ? PersistAttn<true>::kStageBytes : PersistAttn<false>::kStageBytes;
    const int left = smem_limit - (w0 + w1 + kPersistNormBytes + 128 + 1024);
    const int x_bytes = std::min(left, std::max(kPersistGroup * kFfn * 4, kPersistMaxRing * stage - w0 - w1));
    sh.ring = std::min(kPersistMaxRing, (x_bytes + w0 + w1) / stage);
    if (sh.ring < 2 || x_bytes < kPersistGroup * kFfn * 4) return false;
    sh.off_x = 0;
    sh.off_w0 = x_bytes;
    sh.off_w1 = sh.off_w0 + w0;
    sh.off_norm = sh.off_w1 + w1;
    sh.off_bar = sh.off_norm + kPersistNormBytes;
    sh.smem = sh.off_bar + 128 + 1024;  // barriers and flags; 1024-byte alignment slack
    *out = sh;
    return sh.smem <= smem_limit;
}

// The whole step of this batch runs as one persistent launch.
bool use_persist(const PhononCuda* c, int R, bool cancel) {
    if (!c->persist_ok || cancel || static_cast<uint32_t>(R) < c->fused_min || static_cast<uint32_t>(R) > c->fused_max)
        return false;
    PersistShape sh;
    return persist_shape(R, c->sms, c->smem_optin, c->cfg.kv_type == PHONON_CUDA_KV_BF16, &sh);
}

// Pack metadata for entries (slot[e], pos[e]) into pinned memory, upload it
// and apply page-table updates. Entry e attends over pos[e] + 1 keys. With
// device_prep false the RoPE table and the page updates are left to the
// persistent kernel.
int upload_batch(PhononCuda* c, const std::vector<int32_t>& slot, const std::vector<int32_t>& pos,
                 const std::vector<int32_t>& updates, Batch* out, bool device_prep = true, Lane* lane = nullptr,
                 int32_t* status = nullptr, int plan_grid = 0) {
    if (!lane) lane = &c->lanes[0];
    if (!status) status = c->d_status;
    const int R = static_cast<int>(slot.size());
    long long total_pages = 0;
    for (int e = 0; e < R; ++e) total_pages += pos[e] / kPage + 1;
    int32_t* m = lane->h_meta;
    int32_t *h_slot = m, *h_pos = m + R, *h_first = m + 2 * R, *h_count = m + 3 * R;
    int S = 0;
    for (int e = 0; e < R; ++e) {
        h_slot[e] = slot[e];
        h_pos[e] = pos[e];
        h_first[e] = 0;
        h_count[e] = 0;
    }
    // Split plan: the pages of all entries, in (entry, page) order, are cut
    // into chunks, and a chunk is one split per entry segment it covers, so
    // every entry's splits are consecutive and in page order; chunk k's
    // splits are [cta_split[k], cta_split[k+1]). Batches within the
    // persistent window (on any path, so that the persistent and per-stage
    // steps merge the same splits), and each half of a batch split over two
    // lanes (plan_grid: a static chunk per CTA leaves the SMs a CTA finishes
    // early with to the other lane's projections): at most `grid` balanced
    // chunks of at least kPersistMinChunk pages, chunk k run by CTA k, and at
    // most ~sqrt(2 x pages per stream) splits per stream: every split is one
    // more partial the merge folds in, one after the other (one stream at
    // 8000 positions in 125 four-page splits spent 0.64 ms of its 0.98 ms step
    // merging; in ~32 splits the step takes 0.57 ms, at 2048 positions in ~16
    // 0.41 ms against 0.46), while a longer chunk only costs when few
    // streams leave SMs idle. Other
    // batches: guided self-scheduling over two attention CTAs per SM, chunk
    // sizes ceil(remaining / (kGuide * grid)) pages, at least
    // kTicketMinChunk, the first `grid` chunks run by CTA k and the rest
    // taken by ticket.
    const bool guided = R > PHONON_CUDA_FUSED_MAX_BATCH && plan_grid == 0;
    const int grid = plan_grid > 0 ? plan_grid : (guided ? 2 : 1) * c->sms;
    std::vector<long long>& cuts = lane->h_cuts;
    cuts.clear();
    cuts.push_back(0);
    if (!guided) {
        const long long per_stream = std::max<long long>(
            1, std::llround(std::sqrt(2.0 * static_cast<double>(total_pages) / static_cast<double>(R))));
        const long long min_chunk =
            std::max<long long>(kPersistMinChunk, (total_pages + R * per_stream - 1) / (R * per_stream));
        const long long chunks = std::max<long long>(1, std::min<long long>(grid, total_pages / min_chunk));
        for (long long k = 1; k <= chunks; ++k) cuts.push_back(k * total_pages / chunks);
    } else {
        long long done = 0;
        const long long div = static_cast<long long>(kGuide) * grid;
        while (done < total_pages) {
            long long size = std::max<long long>((total_pages - done + div - 1) / div, kTicketMinChunk);
            if (static_cast<int>(cuts.size()) >= kMaxChunks) size = total_pages - done;  // the last one takes the rest
            done = std::min(total_pages, done + size);
            cuts.push_back(done);
        }
    }
    const int C = static_cast<int>(cuts.size()) - 1;
    const int G = std::max(C, c->sms);  // chunk table entries: at least one per CTA of a persistent grid
    // Metadata layout: slot, pos, first, count [R each], the plan header [8]
    // (splits S, chunks C, offsets from the header of cta_split [G+1],
    // cta_page [G+1] and the page ids [P] in split order, a stream's last
    // page as ~id), splits [4S], the
    // two chunk tables, the page ids, then page updates [3U]. The kernels of
    // a step read S, C and the tables through the header, so a replayed step
    // graph depends on R alone; the page updates are applied outside graphs.
    int32_t* hdr = m + 4 * R;
    Split* h_splits = reinterpret_cast<Split*>(hdr + kPlanHeader);
    const long long split_cap = c->max_splits;
    std::vector<int32_t>& flat = lane->h_pages;
    flat.clear();
    // first page of each stream that this batch appends to (its lowest position)
    for (int e = 0; e < R; ++e) c->h_fresh_page[slot[e]] = std::min(c->h_fresh_page[slot[e]], pos[e] / kPage);
    struct FreshReset {  // back to INT32_MAX on every way out
        PhononCuda* c;
        const std::vector<int32_t>& slot;
        ~FreshReset() {
            for (int32_t sl : slot) c->h_fresh_page[sl] = INT32_MAX;
        }
    } fresh_reset{c, slot};
    {
        long long done = 0;  // pages before entry e
        int e = 0, pb = 0;   // cursor: page pb of entry e
        std::vector<int32_t>& first_split = lane->h_first_split;
        first_split.resize(static_cast<size_t>(G) + 1);
        for (int k = 0; k < C; ++k) {
            first_split[k] = S;
            long long left = cuts[k + 1] - (done + pb);  // pages of chunk k
            while (left > 0) {
                const int n_pages = pos[e] / kPage + 1;
                const int take = static_cast<int>(std::min<long long>(left, n_pages - pb));
                const std::vector<int32_t>& pages = c->streams[slot[e]].pages;
                if (S >= split_cap || static_cast<int>(pages.size()) < pb + take) return PHONON_CUDA_INVALID_ARGUMENT;
                if (h_count[e] == 0) h_first[e] = S;
                h_splits[S++] = Split{e, pb, take, pos[e] + 1};
                flat.insert(flat.end(), pages.begin() + pb, pages.begin() + pb + take);
                // pages this launch appends to (from the stream's lowest position in the batch on) as ~id
                const int fresh = std::max(pb, c->h_fresh_page[slot[e]]);
                for (int q = fresh; q < pb + take; ++q) flat[flat.size() - (pb + take - q)] = ~pages[q];
                h_count[e]++;
                pb += take;
                left -= take;
                if (pb == n_pages) {
                    done += n_pages;
                    ++e;
                    pb = 0;
                }
            }
        }
        for (int k = C; k <= G; ++k) first_split[k] = S;
    }
    const int U = static_cast<int>(updates.size() / 3);
    const long long P = static_cast<long long>(flat.size());
    const long long off_split_table = kPlanHeader + 4ll * S;
    const long long off_page_table = off_split_table + G + 1;
    const long long off_ids = off_page_table + G + 1;
    const long long ints = 4ll * R + off_ids + P + 3ll * U;
    if (ints > c->meta_ints) return PHONON_CUDA_INVALID_ARGUMENT;
    hdr[0] = S;
    hdr[1] = C;
    hdr[2] = static_cast<int32_t>(off_split_table);
    hdr[3] = static_cast<int32_t>(off_page_table);
    hdr[4] = static_cast<int32_t>(off_ids);
    hdr[5] = hdr[6] = hdr[7] = 0;
    std::memcpy(hdr + off_split_table, lane->h_first_split.data(), static_cast<size_t>(G + 1) * 4);
    int32_t* h_cta_page = hdr + off_page_table;
    for (int k = 0; k <= G; ++k) h_cta_page[k] = static_cast<int32_t>(cuts[std::min(k, C)]);
    std::memcpy(hdr + off_ids, flat.data(), flat.size() * 4);
    std::memcpy(hdr + off_ids + P, updates.data(), updates.size() * 4);
    const size_t bytes = static_cast<size_t>(ints) * 4;
    CUDA_TRY(cudaMemcpyAsync(lane->meta, lane->h_meta, bytes, cudaMemcpyHostToDevice, lane->stream));
    Batch b;
    b.lane = lane;
    b.d_status = status;
    b.R = R;
    b.S = S;
    b.U = U;
    for (int e = 0; e < R; ++e) b.keys += pos[e] + 1;
    b.d_slot = lane->meta;
    b.d_pos = lane->meta + R;
    b.d_first = lane->meta + 2 * R;
    b.d_count = lane->meta + 3 * R;
    b.d_plan = lane->meta + 4 * R;
    b.d_splits = reinterpret_cast<Split*>(b.d_plan + kPlanHeader);
    b.d_cta_split = b.d_plan + off_split_table;
    b.d_updates = b.d_plan + off_ids + P;
    b.n_chunks = C;
    b.attn_grid = guided ? grid : C;
    b.d_rope = lane->rope;
    b.persist = !device_prep;
    if (!device_prep) {
        *out = b;
        return PHONON_CUDA_OK;
    }
    {
        LaunchScope ls(c, PHONON_CUDA_K_OTHER, R * 32 * 12.0 + U * 12.0, b.lane->stream);
        const int n_ctr = static_cast<int>(c->cfg.n_layers);
        const int threads = std::max({R * 32, U, n_ctr});
        CUDA_TRY(launch_pdl(step_prep_kernel, dim3((threads + 255) / 256), dim3(256), 0, lane->stream,
                            static_cast<const int32_t*>(b.d_pos), static_cast<const float*>(c->d_freq), R, b.d_rope,
                            c->d_table, kMaxPagesPerStream, static_cast<const int32_t*>(b.d_updates), U,
                            lane->chunk_ctr, n_ctr));
    }
    *out = b;
    return PHONON_CUDA_OK;
}

// Enqueue layer `l` for the batch: in -> out (out != in).
int enqueue_attention(PhononCuda* c, const Batch& b, int l, bool digits_out = false, bool no_merge = false);

// Split-K attention then the split merge. With digits_out the merge writes
// the digit rows of the attention output (tensor-core path) instead of fp32;
// with no_merge the consumer merges the partials itself.
int enqueue_attention(PhononCuda* c, const Batch& b, int l, bool digits_out, bool no_merge) {
    cudaStream_t s = b.lane->stream;
    const KvView kv = kv_view(c);
    const double act = 4.0 * b.R;
    const double esize = kv.bf16 ? 2.0 : 4.0;
    AttnParams ap{};
    ap.q = b.lane->q;
    ap.slot = b.d_slot;
    ap.splits = b.d_splits;
    ap.plan = b.d_plan;
    ap.chunk_ctr = b.lane->chunk_ctr + l;
    ap.n_splits = b.S;
    ap.kv = kv;
    ap.layer = l;
    ap.part = b.lane->part;
    ap.status = b.d_status;
    const long long warps = static_cast<long long>(b.S) * kHeads;
    const unsigned grid = static_cast<unsigned>((warps + kAttnWarps - 1) / kAttnWarps);
    {
        LaunchScope ls(c, PHONON_CUDA_K_ATTENTION,
                       b.keys * 2.0 * kWidth * esize + act * kWidth + b.S * kHeads * kPartStride * 4.0, b.lane->stream);
        if (c->attn_tma) {
            CUDA_TRY(kv.bf16 ? launch_attn_tma<true>(c->tm_kv, ap, c->d_err, b.attn_grid, s)
                             : launch_attn_tma<false>(c->tm_kv, ap, c->d_err, b.attn_grid, s));
        } else {
            CUDA_TRY(kv.bf16 ? launch_pdl(attn_partial_kernel<true>, dim3(grid), dim3(kAttnWarps * 32), 0, s, ap)
                             : launch_pdl(attn_partial_kernel<false>, dim3(grid), dim3(kAttnWarps * 32), 0, s, ap));
        }
    }
    if (no_merge) return PHONON_CUDA_OK;
    CombineParams cp{};
    cp.part = b.lane->part;
    cp.first = b.d_first;
    cp.count = b.d_count;
    cp.B = b.R;
    cp.out = b.lane->a;
    cp.status = b.d_status;
    if (digits_out) {
        const int Bpad = (b.R + 31) / 32 * 32;
        LaunchScope ls(c, PHONON_CUDA_K_COMBINE, b.S * kHeads * kPartStride * 4.0 + kDigits * Bpad * 512.0, b.lane->stream);
        CUDA_TRY(launch_pdl(attn_combine_digits_kernel, dim3(Bpad), dim3(256), 0, s, cp, Bpad, b.lane->dig512, b.lane->exps));
        return PHONON_CUDA_OK;
    }
    {
        LaunchScope ls(c, PHONON_CUDA_K_COMBINE, b.S * kHeads * kPartStride * 4.0 + act * kWidth, b.lane->stream);
        CUDA_TRY(launch_pdl(attn_combine_kernel,
                            dim3(static_cast<unsigned>((static_cast<long long>(b.R) * kHeads + kAttnWarps - 1) / kAttnWarps)),
                            dim3(kAttnWarps * 32), 0, s, cp));
    }
    return PHONON_CUDA_OK;
}

// The same layer with the four projections on tcgen05 (digit-sliced int8).
int enqueue_layer_tensor(PhononCuda* c, const Batch& b, int l, const float* in, float* out) {
    const DevLayer& L = c->layers[l];
    cudaStream_t s = b.lane->stream;
    const KvView kv = kv_view(c);
    const int B = b.R, Bpad = (b.R + 31) / 32 * 32, nd = kDigits * Bpad;
    const double act = 4.0 * B, esize = kv.bf16 ? 2.0 : 4.0, dig = kDigits * Bpad;
    GemmParams g{};
    g.B = B;
    g.exps = b.lane->exps;
    g.status = b.d_status;
    g.error = c->d_err;
    // 1. LN1 + digits, QKV + RoPE + KV append
    {
        LaunchScope ls(c, PHONON_CUDA_K_QKV, act * kWidth + dig * 512, b.lane->stream);
        CUDA_TRY((launch_digits<512, true>(in, kWidth, L.norms, L.norms + kWidth, B, Bpad, b.lane->dig512, b.lane->exps,
                                           b.d_status, s)));
    }
    g.rows = 1536;
    g.K = 512;
    g.row_scale = L.qkv.row_scale;
    g.q = b.lane->q;
    g.slot = b.d_slot;
    g.pos = b.d_pos;
    g.rope = b.d_rope;
    g.kv = kv;
    g.layer = l;
    {
        LaunchScope ls(c, PHONON_CUDA_K_QKV, 1536.0 * 512 + dig * 512 + act * kWidth + B * 2.0 * kWidth * esize, b.lane->stream);
        CUDA_TRY(launch_linear_gemm<GEPI_QKV>(L.qkv, b.lane->tm_dig512, nd, g, s));
    }
    // 2. attention; the combine writes the digit rows of the attention output
    int st = enqueue_attention(c, b, l, true);
    if (st) return st;
    // 3. h = x + attn Wout^T
    GemmParams go = g;
    go.rows = 512;
    go.K = 512;
    go.row_scale = L.out.row_scale;
    go.res = in;
    go.ldres = kWidth;
    go.y = b.lane->h;
    go.ldy = kWidth;
    {
        LaunchScope ls(c, PHONON_CUDA_K_OUT, 512.0 * 512 + dig * 512 + act * 2 * kWidth, b.lane->stream);
        CUDA_TRY(launch_linear_gemm<GEPI_RESID>(L.out, b.lane->tm_dig512, nd, go, s));
    }
    // 4. g = GELU(LN2(h) Wup^T)
    {
        LaunchScope ls(c, PHONON_CUDA_K_UP, act * kWidth + dig * 512, b.lane->stream);
        CUDA_TRY((launch_digits<512, true>(b.lane->h, kWidth, L.norms + 2 * kWidth, L.norms + 3 * kWidth, B, Bpad,
                                           b.lane->dig512, b.lane->exps, b.d_status, s)));
    }
    GemmParams gu = g;
    gu.rows = kFfn;
    gu.K = 512;
    gu.row_scale = L.up.row_scale;
    gu.y = b.lane->g;
    gu.ldy = kFfn;
    {
        LaunchScope ls(c, PHONON_CUDA_K_UP, 2048.0 * 512 + dig * 512 + act * kFfn, b.lane->stream);
        CUDA_TRY(launch_linear_gemm<GEPI_GELU>(L.up, b.lane->tm_dig512, nd, gu, s));
    }
    // 5. out = h + g Wdown^T
    {
        LaunchScope ls(c, PHONON_CUDA_K_DOWN, act * kFfn + dig * 2048, b.lane->stream);
        CUDA_TRY((launch_digits<2048, false>(b.lane->g, kFfn, nullptr, nullptr, B, Bpad, b.lane->dig2048, b.lane->exps,
                                             b.d_status, s)));
    }
    GemmParams gd = g;
    gd.rows = 512;
    gd.K = kFfn;
    gd.row_scale = L.down.row_scale;
    gd.res = b.lane->h;
    gd.ldres = kWidth;
    gd.y = out;
    gd.ldy = kWidth;
    {
        LaunchScope ls(c, PHONON_CUDA_K_DOWN, 512.0 * 2048 + dig * 2048 + act * 2 * kWidth, b.lane->stream);
        CUDA_TRY(launch_linear_gemm<GEPI_RESID>(L.down, b.lane->tm_dig2048, nd, gd, s));
    }
    return PHONON_CUDA_OK;
}

int enqueue_layer(PhononCuda* c, const Batch& b, int l, const float* in, float* out) {
    const DevLayer& L = c->layers[l];
    if (c->tensor_ok && b.R >= static_cast<int>(c->tensor_min) && L.qkv.tensor && L.out.tensor && L.up.tensor && L.down.tensor)
        return enqueue_layer_tensor(c, b, l, in, out);
    const bool q8 = L.q8;
    cudaStream_t s = b.lane->stream;
    const KvView kv = kv_view(c);
    GemvParams p{};
    p.B = b.R;
    p.status = b.d_status;
    // 1. LN1 -> QKV -> RoPE -> q scratch + KV append
    p.w = L.qkv.plane;
    p.scales = L.qkv.scales;
    p.rows = 1536;
    p.cols = 512;
    p.x = in;
    p.ldx = kWidth;
    p.ln_w = L.norms;
    p.ln_b = L.norms + kWidth;
    p.q = b.lane->q;
    p.slot = b.d_slot;
    p.pos = b.d_pos;
    p.rope = b.d_rope;
    p.kv = kv;
    p.layer = l;
    const double act = 4.0 * b.R;  // bytes per activation element across the batch
    const double esize = kv.bf16 ? 2.0 : 4.0;
    {
        LaunchScope ls(c, PHONON_CUDA_K_QKV, linear_bytes(L.qkv) + act * (kWidth + kWidth) + b.R * 2.0 * kWidth * esize, b.lane->stream);
        CUDA_TRY((launch_gemv<1, SRC_LN, EPI_QKV>(q8, p, s)));
    }
    // 2. split-K attention (the out projection merges the splits)
    {
        int st = enqueue_attention(c, b, l, false, true);
        if (st) return st;
    }
    // 3. h = x + attn Wout^T, attn merged from the split partials
    GemvParams po{};
    po.B = b.R;
    po.status = b.d_status;
    po.w = L.out.plane;
    po.scales = L.out.scales;
    po.rows = 512;
    po.cols = 512;
    po.part = b.lane->part;
    po.first = b.d_first;
    po.count = b.d_count;
    po.ldx = kWidth;
    po.res = in;
    po.ldres = kWidth;
    po.y = b.lane->h;
    po.ldy = kWidth;
    {
        LaunchScope ls(c, PHONON_CUDA_K_OUT, linear_bytes(L.out) + act * 3 * kWidth, b.lane->stream);
        CUDA_TRY((launch_gemv<1, SRC_MERGE, EPI_RESID>(q8, po, s)));
    }
    // 4. g = GELU(LN2(h) Wup^T)
    GemvParams pu{};
    pu.B = b.R;
    pu.status = b.d_status;
    pu.w = L.up.plane;
    pu.scales = L.up.scales;
    pu.rows = kFfn;
    pu.cols = 512;
    pu.x = b.lane->h;
    pu.ldx = kWidth;
    pu.ln_w = L.norms + 2 * kWidth;
    pu.ln_b = L.norms + 3 * kWidth;
    pu.y = b.lane->g;
    pu.ldy = kFfn;
    {
        LaunchScope ls(c, PHONON_CUDA_K_UP, linear_bytes(L.up) + act * (kWidth + kFfn), b.lane->stream);
        CUDA_TRY((launch_gemv<1, SRC_LN, EPI_GELU>(q8, pu, s)));
    }
    // 5. out = h + g Wdown^T
    GemvParams pd{};
    pd.B = b.R;
    pd.status = b.d_status;
    pd.w = L.down.plane;
    pd.scales = L.down.scales;
    pd.rows = 512;
    pd.cols = kFfn;
    pd.x = b.lane->g;
    pd.ldx = kFfn;
    pd.res = b.lane->h;
    pd.ldres = kWidth;
    pd.y = out;
    pd.ldy = kWidth;
    {
        LaunchScope ls(c, PHONON_CUDA_K_DOWN, linear_bytes(L.down) + act * (kFfn + 2 * kWidth), b.lane->stream);
        CUDA_TRY((launch_gemv<4, SRC_X, EPI_RESID>(q8, pd, s)));
    }
    return PHONON_CUDA_OK;
}

// Run layers [0, L) over the batch, reading `in` and leaving the result in
// `final_out`. cancel (optional) is polled before each layer and once after;
// `polls_per_layer` extra polls emulate the reference's in-layer schedule.
void drop_graph(PhononCuda* c) {
    if (c->graph_exec) cudaGraphExecDestroy(c->graph_exec);
    c->graph_exec = nullptr;
    c->graph_shape = PhononCuda::StepShape{};
    c->last_shape = PhononCuda::StepShape{};
}

// Test instrumentation (phonon_cuda_set_layer_trace): layer l's output rows
// of batch b into the trace, on the batch's stream.
int trace_layer(PhononCuda* c, const Batch& b, int l, const float* out) {
    if (!c->tracing) return PHONON_CUDA_OK;
    CUDA_TRY(cudaMemcpyAsync(c->trace + (static_cast<size_t>(l) * c->trace_rows + b.row0) * kWidth, out,
                             static_cast<size_t>(b.R) * kWidth * 4, cudaMemcpyDeviceToDevice, b.lane->stream));
    return PHONON_CUDA_OK;
}

int enqueue_layers_direct(PhononCuda* c, const Batch& b, const float* in, float* final_out) {
    const int L = static_cast<int>(c->cfg.n_layers);
    const float* cur = in;
    for (int l = 0; l < L; ++l) {
        float* out = (l == L - 1) ? final_out : ((cur == b.lane->x0) ? b.lane->x1 : b.lane->x0);
        int st = enqueue_layer(c, b, l, cur, out);
        if (st == PHONON_CUDA_OK) st = trace_layer(c, b, l, out);
        if (st != PHONON_CUDA_OK) return st;
        cur = out;
    }
    return PHONON_CUDA_OK;
}

// All layers of an uncancellable, unprofiled step, through the step graph
// when the shape repeats; any capture problem falls back to direct launches.
int enqueue_layers_graphed(PhononCuda* c, const Batch& b, const float* in, float* final_out) {
    PhononCuda::StepShape shape;
    shape.R = b.R;
    // Kernels read S and the chunk tables through the plan header; the TMA
    // attention grid is fixed except for small (static) plans.
    shape.S = c->attn_tma ? 0 : b.S;
    shape.chunks = b.attn_grid;
    shape.in = in;
    shape.out = final_out;
    if (c->graph_exec && c->graph_shape == shape) {
        CUDA_TRY(cudaGraphLaunch(c->graph_exec, c->stream));
        c->launches += c->graph_kernels;
        return PHONON_CUDA_OK;
    }
    if (!(c->last_shape == shape)) {
        c->last_shape = shape;
        return enqueue_layers_direct(c, b, in, final_out);
    }
    cudaGraph_t g = nullptr;
    const uint64_t before = c->launches;
    if (cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        cudaGetLastError();
        return enqueue_layers_direct(c, b, in, final_out);
    }
    const int st = enqueue_layers_direct(c, b, in, final_out);
    const cudaError_t end = cudaStreamEndCapture(c->stream, &g);
    cudaGraphExec_t exec = nullptr;
    if (st != PHONON_CUDA_OK || end != cudaSuccess || !g || cudaGraphInstantiate(&exec, g, 0) != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        c->launches = before;
        return enqueue_layers_direct(c, b, in, final_out);
    }
    cudaGraphDestroy(g);
    if (c->graph_exec) cudaGraphExecDestroy(c->graph_exec);
    c->graph_exec = exec;
    c->graph_shape = shape;
    c->graph_kernels = c->launches - before;
    c->launches = before;
    CUDA_TRY(cudaGraphLaunch(c->graph_exec, c->stream));
    c->launches += c->graph_kernels;
    return PHONON_CUDA_OK;
}

template <bool kBf16>
cudaError_t launch_persist_t(PhononCuda* c, const PersistParams& pp, int smem) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(c->sms));
    cfg.blockDim = dim3(kPersistThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cfg.stream = c->stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;  // all CTAs resident: the grid barriers rely on it
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, step_persist_kernel<kBf16>, c->tm_kv, pp);
}

// Every layer of the batch in one step_persist_kernel launch.
int enqueue_persist(PhononCuda* c, const Batch& b, const float* in, float* final_out) {
    const bool bf16 = c->cfg.kv_type == PHONON_CUDA_KV_BF16;
    PersistShape sh;
    if (!persist_shape(b.R, c->sms, c->smem_optin, bf16, &sh)) return PHONON_CUDA_INVALID_ARGUMENT;
    const int L = static_cast<int>(c->cfg.n_layers);
    PersistParams pp{};
    pp.layers = c->d_players;
    pp.n_layers = L;
    pp.R = b.R;
    pp.S = b.S;
    pp.U = b.U;
    pp.n_groups = sh.n_groups;
    pp.in = in;
    pp.out = final_out;
    pp.xbuf0 = in == b.lane->x1 ? b.lane->x0 : b.lane->x1;
    pp.xbuf1 = in == b.lane->x1 ? b.lane->x1 : b.lane->x0;
    pp.h = b.lane->h;
    pp.g = b.lane->g;
    pp.q = b.lane->q;
    pp.part = b.lane->part;
    pp.status = b.d_status;
    pp.error = c->d_err;
    pp.barrier = c->d_bar;
    pp.barrier_base = c->bar_epoch;
    pp.slot = b.d_slot;
    pp.pos = b.d_pos;
    pp.first = b.d_first;
    pp.count = b.d_count;
    pp.updates = b.d_updates;
    pp.splits = b.d_splits;
    pp.cta_split = b.d_cta_split;
    pp.freq = c->d_freq;
    pp.rope = b.lane->rope;
    pp.kv = kv_view(c);
    pp.off_x = sh.off_x;
    pp.off_w0 = sh.off_w0;
    pp.off_w1 = sh.off_w1;
    pp.off_norm = sh.off_norm;
    pp.off_bar = sh.off_bar;
    pp.ring = sh.ring;
    pp.trace = c->tracing ? c->trace : nullptr;
    pp.trace_rows = static_cast<int>(c->trace_rows);
    double weights = 0.0;
    for (const DevLayer& D : c->layers)
        weights += linear_bytes(D.qkv) + linear_bytes(D.out) + linear_bytes(D.up) + linear_bytes(D.down);
    const double esize = bf16 ? 2.0 : 4.0;
    const double bytes = weights + L * (b.keys + b.R) * 2.0 * kWidth * esize + b.R * 2.0 * kWidth * 4.0;
    {
        LaunchScope ls(c, PHONON_CUDA_K_FUSED, bytes, b.lane->stream);
        CUDA_TRY(bf16 ? launch_persist_t<true>(c, pp, sh.smem) : launch_persist_t<false>(c, pp, sh.smem));
    }
    c->bar_epoch += static_cast<unsigned>(c->sms) * static_cast<unsigned>(1 + 5 * L);
    return PHONON_CUDA_OK;
}

template <bool kBf16, bool kTc>
cudaLaunchConfig_t cluster_config(cudaStream_t s, cudaLaunchAttribute* at) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(kClusterCtas);
    cfg.blockDim = dim3(kClThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(ClShape<kBf16, kTc>::kSmem);
    cfg.stream = s;
    at[0].id = cudaLaunchAttributeClusterDimension;  // the whole grid is one cluster
    at[0].val.clusterDim.x = kClusterCtas;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cfg;
}

// Opt the cluster kernel into its shared memory and a 16-CTA cluster, and
// check that such a cluster can be resident on this device.
template <bool kBf16, bool kTc>
bool cluster_launchable() {
    const void* fn = reinterpret_cast<const void*>(step_cluster_kernel<kBf16, kTc>);
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, ClShape<kBf16, kTc>::kSmem) != cudaSuccess ||
        cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    cudaLaunchAttribute at[1];
    cudaLaunchConfig_t cfg = cluster_config<kBf16, kTc>(nullptr, at);
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, step_cluster_kernel<kBf16, kTc>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return clusters >= 1;
}

// A single-stream decode step (entry (slot, pos), page-table updates
// `updates`) as one launch of step_cluster_kernel.
bool use_cluster(const PhononCuda* c, int n, const std::vector<int32_t>& pos, const std::vector<int32_t>& updates,
                 bool cancel) {
    return c->cluster_ok && n == 1 && !cancel && static_cast<uint32_t>(pos[0]) < c->cluster_max_pos &&
           updates.size() <= 3u * kClMaxUpdates;
}

int enqueue_cluster(PhononCuda* c, int32_t slot, int32_t pos, const std::vector<int32_t>& updates, const float* in,
                    float* out) {
    const bool bf16 = c->cfg.kv_type == PHONON_CUDA_KV_BF16;
    ClusterParams cp{};
    cp.layers = c->d_players;
    cp.tc = c->d_cltc;
    cp.n_layers = static_cast<int>(c->cfg.n_layers);
    cp.in = in;
    cp.out = out;
    cp.status = c->d_status;
    cp.error = c->d_err;
    cp.slot = slot;
    cp.pos = pos;
    cp.last_page = c->streams[slot].pages[pos / kPage];
    cp.n_updates = static_cast<int>(updates.size() / 3);
    for (size_t i = 0; i < updates.size(); ++i) cp.updates[i] = updates[i];
    cp.freq = c->d_freq;
    cp.kv = kv_view(c);
    cp.trace = c->tracing ? c->trace : nullptr;
    cp.trace_stride = static_cast<int>(c->trace_rows) * kWidth;
    double weights = 0.0;
    for (const DevLayer& D : c->layers)
        weights += linear_bytes(D.qkv) + linear_bytes(D.out) + linear_bytes(D.up) + linear_bytes(D.down);
    const double esize = bf16 ? 2.0 : 4.0;
    const double bytes = weights + cp.n_layers * (pos + 2.0) * 2.0 * kWidth * esize + 2.0 * kWidth * 4.0;
    LaunchScope ls(c, PHONON_CUDA_K_FUSED, bytes, c->stream);
    cudaLaunchAttribute at[1];
    if (bf16 && c->cluster_tc) {
        cudaLaunchConfig_t cfg = cluster_config<true, true>(c->stream, at);
        CUDA_TRY(cudaLaunchKernelEx(&cfg, step_cluster_kernel<true, true>, c->tm_kv16, cp));
    } else if (bf16) {
        cudaLaunchConfig_t cfg = cluster_config<true, false>(c->stream, at);
        CUDA_TRY(cudaLaunchKernelEx(&cfg, step_cluster_kernel<true, false>, c->tm_kv16, cp));
    } else if (c->cluster_tc) {
        cudaLaunchConfig_t cfg = cluster_config<false, true>(c->stream, at);
        CUDA_TRY(cudaLaunchKernelEx(&cfg, step_cluster_kernel<false, true>, c->tm_kv16, cp));
    } else {
        cudaLaunchConfig_t cfg = cluster_config<false, false>(c->stream, at);
        CUDA_TRY(cudaLaunchKernelEx(&cfg, step_cluster_kernel<false, false>, c->tm_kv16, cp));
    }
    return PHONON_CUDA_OK;
}

int enqueue_stack(PhononCuda* c, const Batch& b, const float* in, float* final_out,
                  PhononCudaCancelPoll cancel, void* cctx, const std::vector<int>* polls_per_layer,
                  bool* cancelled) {
    if (b.persist) return enqueue_persist(c, b, in, final_out);
    if (!cancel && !c->prof_on && !b.split && !c->tracing) return enqueue_layers_graphed(c, b, in, final_out);
    if (!cancel) return enqueue_layers_direct(c, b, in, final_out);
    const int L = static_cast<int>(c->cfg.n_layers);
    const float* cur = in;
    for (int l = 0; l < L; ++l) {
        if (cancel) {
            const int polls = polls_per_layer ? (*polls_per_layer)[l] : 1;
            for (int k = 0; k < polls; ++k)
                if (cancel(cctx)) {
                    *cancelled = true;
                    return PHONON_CUDA_CANCELLED;
                }
        }
        float* out = (l == L - 1) ? final_out : ((cur == b.lane->x0) ? b.lane->x1 : b.lane->x0);
        int st = enqueue_layer(c, b, l, cur, out);
        if (st == PHONON_CUDA_OK) st = trace_layer(c, b, l, out);
        if (st != PHONON_CUDA_OK) return st;
        cur = out;
    }
    if (cancel && cancel(cctx)) {
        *cancelled = true;
        return PHONON_CUDA_CANCELLED;
    }
    return PHONON_CUDA_OK;
}

int set_device(int device) {
    CUDA_TRY(cudaSetDevice(device));
    return PHONON_CUDA_OK;
}

// A decode step of entries (slot, pos) from `in` to `out` (device rows).
// Small batches within the fused window run as one persistent launch;
// batches of at least split_min entries run as two half batches on two
// lanes, so that one half's attention (HBM-bound) overlaps the other half's
// projections (latency-bound); everything else runs one launch per stage.
// Page-table updates are applied by the first lane before the second starts.
int enqueue_decode_paths(PhononCuda* c, const std::vector<int32_t>& slot, const std::vector<int32_t>& pos,
                         const std::vector<int32_t>& updates, const float* in, float* out,
                         PhononCudaCancelPoll cancel, void* cctx, bool* cancelled) {
    const int n = static_cast<int>(slot.size());
    if (use_cluster(c, n, pos, updates, cancel != nullptr)) return enqueue_cluster(c, slot[0], pos[0], updates, in, out);
    const bool persist = use_persist(c, n, cancel != nullptr);
    int st;
    if (persist || cancel || !c->lane1_ok || static_cast<uint32_t>(n) < c->split_min) {
        Batch b;
        if ((st = upload_batch(c, slot, pos, updates, &b, !persist))) return st;
        return enqueue_stack(c, b, in, out, cancel, cctx, nullptr, cancelled);
    }
    const int n0 = n / 2;
    Lane& L1 = c->lanes[1];
    // Attention chunks (= CTAs) per half: 5/4 of the SM count. Measured at
    // 512 streams (ms per step): 0.65x SMs 3.20, 1x 2.73, 1.14x 2.57, 1.24x
    // 2.54, 1.3x 2.57, 1.62x 2.70, 2x 2.94: with one CTA per SM a half's
    // attention leaves SMs idle between its chunks, with two per SM it takes
    // the SMs the other half's projections need.
    const int grid = (c->sms * 5) / 4;
    const std::vector<int32_t> s0(slot.begin(), slot.begin() + n0), p0(pos.begin(), pos.begin() + n0);
    const std::vector<int32_t> s1(slot.begin() + n0, slot.end()), p1(pos.begin() + n0, pos.end());
    Batch b0, b1;
    if ((st = upload_batch(c, s0, p0, updates, &b0, true, &c->lanes[0], c->d_status, grid))) return st;
    CUDA_TRY(cudaEventRecord(c->fork, c->stream));  // page updates and everything before this step
    CUDA_TRY(cudaStreamWaitEvent(L1.stream, c->fork, 0));
    st = upload_batch(c, s1, p1, {}, &b1, true, &L1, c->d_status + n0, grid);
    if (st) return st;
    b0.split = b1.split = true;
    b1.row0 = n0;
    // The halves' launches are issued layer by layer, alternating, so that
    // the second half starts as soon as the first (issuing all of one half
    // first delays the other by the host time of ~100 launches).
    {
        const int L = static_cast<int>(c->cfg.n_layers);
        const float* cur[2] = {in, in + static_cast<size_t>(n0) * kWidth};
        float* fin[2] = {out, out + static_cast<size_t>(n0) * kWidth};
        const Batch* bs[2] = {&b0, &b1};
        for (int l = 0; l < L; ++l)
            for (int k = 0; k < 2; ++k) {
                const Batch& b = *bs[k];
                float* o = (l == L - 1) ? fin[k] : ((cur[k] == b.lane->x0) ? b.lane->x1 : b.lane->x0);
                if ((st = enqueue_layer(c, b, l, cur[k], o))) return st;
                if ((st = trace_layer(c, b, l, o))) return st;
                cur[k] = o;
            }
    }
    CUDA_TRY(cudaEventRecord(c->join, L1.stream));
    CUDA_TRY(cudaStreamWaitEvent(c->stream, c->join, 0));
    return PHONON_CUDA_OK;
}

// A decode step on the paths above; with a layer trace set, every layer's
// output rows are copied into it as well.
int enqueue_decode(PhononCuda* c, const std::vector<int32_t>& slot, const std::vector<int32_t>& pos,
                   const std::vector<int32_t>& updates, const float* in, float* out, PhononCudaCancelPoll cancel,
                   void* cctx, bool* cancelled) {
    if (c->trace && slot.size() > c->trace_rows) return PHONON_CUDA_INVALID_ARGUMENT;
    c->tracing = c->trace != nullptr;
    const int st = enqueue_decode_paths(c, slot, pos, updates, in, out, cancel, cctx, cancelled);
    c->tracing = false;
    return st;
}

// Upload the per-layer weight pointers of step_persist_kernel and decide
// whether it can run: Q8_0 weights in the GEMV layout, TMA page staging,
// cooperative launch, and one resident CTA per SM at the largest plan.
int refresh_persist(PhononCuda* c) {
    std::vector<PersistLayer> pl(c->layers.size());
    bool ok = c->attn_tma && c->sms > 0;
    for (size_t l = 0; l < c->layers.size(); ++l) {
        const DevLayer& D = c->layers[l];
        const DevLinear* lin[4] = {&D.qkv, &D.out, &D.up, &D.down};
        for (int m = 0; m < 4; ++m) {
            ok = ok && D.q8 && lin[m]->fast && lin[m]->plane && lin[m]->scales;
            pl[l].plane[m] = static_cast<const uint8_t*>(lin[m]->plane);
            pl[l].scales[m] = lin[m]->scales;
        }
        pl[l].norms = D.norms;
    }
    CUDA_TRY(cudaMemcpy(c->d_players, pl.data(), sizeof(PersistLayer) * pl.size(), cudaMemcpyHostToDevice));
    int coop = 0;
    CUDA_TRY(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, c->cfg.device));
    ok = ok && coop;
    if (ok) {
        const bool bf16 = c->cfg.kv_type == PHONON_CUDA_KV_BF16;
        const void* fn = bf16 ? reinterpret_cast<const void*>(step_persist_kernel<true>)
                              : reinterpret_cast<const void*>(step_persist_kernel<false>);
        int resident = 0;
        ok = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, c->smem_optin) == cudaSuccess &&
             cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, fn, kPersistThreads, c->smem_optin) == cudaSuccess &&
             resident >= 1;
        cudaGetLastError();
    }
    c->persist_ok = ok;
    // The single-stream cluster step needs the same weights (Q8_0 in the
    // GEMV layout), the 16-row K/V boxes and a resident 16-CTA cluster.
    bool cl = c->attn_tma && !c->layers.empty();
    for (const DevLayer& D : c->layers) {
        const DevLinear* lin[4] = {&D.qkv, &D.out, &D.up, &D.down};
        for (int m = 0; m < 4; ++m) cl = cl && D.q8 && lin[m]->fast && lin[m]->plane && lin[m]->scales;
    }
    const bool bf16 = c->cfg.kv_type == PHONON_CUDA_KV_BF16;
    if (cl) cl = bf16 ? cluster_launchable<true, false>() : cluster_launchable<false, false>();
    c->cluster_ok = cl;
    // Its tensor-core form: one scale per row in every layer's four linears.
    bool tc = cl && c->tensor_ok;
    for (const DevLayer& D : c->layers)
        tc = tc && D.qkv.tensor && D.qkv.wd == 1 && D.qkv.rows == 3 * kWidth && D.qkv.cols == kWidth && D.out.tensor &&
             D.out.wd == 1 && D.out.rows == kWidth && D.out.cols == kWidth && D.up.tensor && D.up.wd == 1 &&
             D.up.rows == kFfn && D.up.cols == kWidth && D.down.tensor && D.down.wd == 1 && D.down.rows == kWidth &&
             D.down.cols == kFfn;
    if (tc) tc = bf16 ? cluster_launchable<true, true>() : cluster_launchable<false, true>();
    if (tc && !c->d_cltc) {
        const size_t bytes = c->layers.size() * kClusterCtas * kClTcUnits * static_cast<size_t>(kClUnitBytes);
        if (cudaMalloc(&c->d_cltc, bytes) != cudaSuccess) {
            cudaGetLastError();
            c->d_cltc = nullptr;
            tc = false;
        }
    }
    if (tc) {
        for (size_t l = 0; l < c->layers.size(); ++l) {
            const DevLayer& D = c->layers[l];
            const ClTcSource src{{D.qkv.nat, D.out.nat, D.up.nat, D.down.nat},
                                 {D.qkv.row_scale, D.out.row_scale, D.up.row_scale, D.down.row_scale}};
            cluster_tc_pack_kernel<<<kClusterCtas * kClTcUnits, 256, 0, c->stream>>>(
                src, c->d_cltc + l * kClusterCtas * kClTcUnits * static_cast<size_t>(kClUnitBytes));
            CUDA_TRY(cudaGetLastError());
        }
        CUDA_TRY(cudaStreamSynchronize(c->stream));
    }
    c->cluster_tc = tc;
    return PHONON_CUDA_OK;
}

void destroy_context(PhononCuda* c) {
    if (!c) return;
    cudaSetDevice(c->cfg.device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    drop_graph(c);
    for (auto& L : c->layers) free_layer(L);
    for (auto& r : c->prof_pending) {
        cudaEventDestroy(r.a);
        cudaEventDestroy(r.b);
    }
    for (cudaEvent_t e : c->prof_events) cudaEventDestroy(e);
    void* dev[] = {c->kv_pool, c->d_table, c->d_freq, c->d_x0, c->d_x1, c->d_y, c->d_q, c->d_a,
                   c->d_h, c->d_g, c->d_part, c->d_stage, c->d_meta, c->d_status,
                   c->d_dig512, c->d_dig2048, c->d_exps, c->d_err, c->d_rope,
                   c->d_players, c->d_bar, c->d_cltc};
    for (void* p : dev)
        if (p) cudaFree(p);
    void* host[] = {c->h_meta, c->h_x, c->h_y, c->h_stage, c->h_status};
    for (void* p : host)
        if (p) cudaFreeHost(p);
    {
        Lane& L1 = c->lanes[1];
        if (L1.stream) cudaStreamSynchronize(L1.stream);
        void* dev1[] = {L1.x0, L1.x1, L1.q, L1.a, L1.h, L1.g, L1.part, L1.meta, L1.dig512, L1.dig2048, L1.exps, L1.rope,
                        L1.chunk_ctr, c->lanes[0].chunk_ctr};
        for (void* p : dev1)
            if (p) cudaFree(p);
        if (L1.h_meta) cudaFreeHost(L1.h_meta);
        if (L1.stream) cudaStreamDestroy(L1.stream);
        if (c->fork) cudaEventDestroy(c->fork);
        if (c->join) cudaEventDestroy(c->join);
    }
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

// RoPE inverse frequencies exactly as the reference builds them in fp32:
// freq_i = 1 / powf(theta, (float)(2i) / (float)head_width)
// (src/phonon_transformer.c:229-232).
void rope_frequencies(float theta, size_t head_width, float* freq) {
    for (size_t i = 0; i < head_width / 2; ++i) {
        const float exponent = static_cast<float>(2 * i) / static_cast<float>(head_width);
        freq[i] = 1.0f / powf(theta, exponent);
    }
}

// Poll schedule of the reference prefill for one layer: layer start, after
// LN1, one per (head, query block, 512-key block), after LN2
// (src/phonon_transformer.c:497-509, :644-680).
int prefill_polls_per_layer(size_t length) {
    const size_t qb = length >= 768 ? 256 : (length >= 192 ? 64 : 32);
    size_t attn = 0;
    for (size_t start = 0; start < length; start += qb) {
        const size_t rows = std::min(qb, length - start);
        attn += (start + rows + 511) / 512;
    }
    return static_cast<int>(3 + 8 * attn);
}

// Kind 2 of phonon_cuda_wait_expiry_probe (defined with the allocation-free
// entry point, whose scratch it uses).
int noalloc_expiry_probe(int device, uint32_t budget_us, uint64_t* elapsed_ns);

}  // namespace

// =================================================================== C ABI
extern "C" {

const char* phonon_cuda_status_string(int status) {
    switch (status) {
        case PHONON_CUDA_OK: return "ok";
        case PHONON_CUDA_INVALID_ARGUMENT: return "invalid argument";
        case PHONON_CUDA_NON_FINITE: return "non-finite value";
        case PHONON_CUDA_OUT_OF_MEMORY: return "out of memory";
        case PHONON_CUDA_POOL_EXHAUSTED: return "KV page pool exhausted";
        case PHONON_CUDA_CAPACITY: return "stream capacity exceeded";
        case PHONON_CUDA_BAD_POSITION: return "position is not the stream length";
        case PHONON_CUDA_CANCELLED: return "cancelled";
        case PHONON_CUDA_DEVICE_ERROR: return "CUDA error";
        default: return "unknown status";
    }
}

int phonon_cuda_create(const PhononCudaConfig* config, const PhononCudaLayer* layers, PhononCuda** out) {
    if (!config || !layers || !out) return PHONON_CUDA_INVALID_ARGUMENT;
    *out = nullptr;
    const PhononCudaConfig& cfg = *config;
    if (cfg.n_layers < 1 || cfg.n_layers > kMaxLayers || cfg.max_streams < 1 || cfg.max_batch < 1 ||
        cfg.max_batch > 65536 || cfg.pool_pages < 1 || cfg.kv_type > PHONON_CUDA_KV_BF16 ||
        !(cfg.theta > 0.0f) || !std::isfinite(cfg.theta))
        return PHONON_CUDA_INVALID_ARGUMENT;
    int st = set_device(cfg.device);
    if (st) return st;
    PhononCuda* c = new (std::nothrow) PhononCuda();
    if (!c) return PHONON_CUDA_OUT_OF_MEMORY;
    c->cfg = cfg;
    // The cluster step reads a stream's K/V on its 16 SMs, the per-stage path on
    // all of them: measured on B200 (one stream, L2 flushed), the per-stage path
    // is faster from ~1,150 positions with fp32 K/V (2,048: 0.60 vs 0.42 ms per
    // step) and from ~1,250 with bf16 K/V.
    c->cluster_max_pos = cfg.kv_type == PHONON_CUDA_KV_BF16 ? kClusterMaxPosBf16 : kClusterMaxPosF32;
    auto fail = [&](int code) {
        destroy_context(c);
        return code;
    };
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) return fail(PHONON_CUDA_DEVICE_ERROR);
    c->layers.resize(cfg.n_layers);
    for (uint32_t l = 0; l < cfg.n_layers; ++l)
        if ((st = load_layer(&c->layers[l], layers[l]))) return fail(st);
    float freq[32];
    rope_frequencies(cfg.theta, kHeadDim, freq);
    const size_t esize = cfg.kv_type == PHONON_CUDA_KV_BF16 ? 2 : 4;
    c->page_elems = static_cast<long long>(cfg.n_layers) * 2 * kHeads * kPage * kHeadDim;
    c->cap_rows = static_cast<int>(std::max<uint32_t>(cfg.max_batch, kPrefillChunk));
    c->max_splits = kMaxChunks + c->cap_rows + 16;  // at most one split per (chunk, entry) boundary
    const int U_max = c->cap_rows * 2 + kMaxPagesPerStream + 16;
    // page ids of a batch: every page of its streams, at most the pool
    const long long batch_pages = std::min<long long>(static_cast<long long>(c->cap_rows) * kMaxPagesPerStream,
                                                      cfg.pool_pages);
    c->meta_ints = static_cast<int>(4 * c->cap_rows + kPlanHeader + 4 * c->max_splits +
                                    2 * (std::max(kMaxChunks, kMaxSms) + 1) + batch_pages + 3 * U_max);
    const size_t rows = static_cast<size_t>(c->cap_rows);
    bool ok = cudaMalloc(&c->kv_pool, static_cast<size_t>(cfg.pool_pages) * c->page_elems * esize) == cudaSuccess &&
              cudaMalloc(&c->d_table, static_cast<size_t>(cfg.max_streams) * kMaxPagesPerStream * 4) == cudaSuccess &&
              cudaMalloc(&c->d_freq, sizeof(freq)) == cudaSuccess &&
              cudaMalloc(&c->d_x0, rows * kWidth * 4) == cudaSuccess &&
              cudaMalloc(&c->d_x1, rows * kWidth * 4) == cudaSuccess &&
              cudaMalloc(&c->d_y, rows * kWidth * 4) == cudaSuccess &&
              cudaMalloc(&c->d_q, rows * kWidth * 4) == cudaSuccess &&
              cudaMalloc(&c->d_a, rows * kWidth * 4) == cudaSuccess &&
              cudaMalloc(&c->d_h, rows * kWidth * 4) == cudaSuccess &&
              cudaMalloc(&c->d_g, rows * kFfn * 4) == cudaSuccess &&
              cudaMalloc(&c->d_part, static_cast<size_t>(c->max_splits) * kHeads * kPartStride * 4) == cudaSuccess &&
              cudaMalloc(&c->d_meta, static_cast<size_t>(c->meta_ints) * 4) == cudaSuccess &&
              cudaMalloc(&c->d_status, rows * 4) == cudaSuccess &&
              cudaMallocHost(&c->h_meta, static_cast<size_t>(c->meta_ints) * 4) == cudaSuccess &&
              cudaMallocHost(&c->h_x, rows * kWidth * 4) == cudaSuccess &&
              cudaMallocHost(&c->h_y, rows * kWidth * 4) == cudaSuccess &&
              cudaMallocHost(&c->h_status, rows * 4) == cudaSuccess;
    const size_t rows_pad = (rows + 31) / 32 * 32;
    ok = ok && cudaMalloc(&c->d_dig512, rows_pad * kDigits * 512) == cudaSuccess &&
         cudaMalloc(&c->d_dig2048, rows_pad * kDigits * 2048) == cudaSuccess &&
         cudaMalloc(&c->d_exps, rows_pad * 4) == cudaSuccess && cudaMalloc(&c->d_err, 4) == cudaSuccess &&
         cudaMalloc(&c->d_rope, rows * 32 * sizeof(float2)) == cudaSuccess;
    if (!ok) return fail(PHONON_CUDA_OUT_OF_MEMORY);
    if (cudaMemset(c->d_err, 0, 4) != cudaSuccess) return fail(PHONON_CUDA_DEVICE_ERROR);
    c->tensor_ok = make_i8_map(&c->tm_dig512, c->d_dig512, rows_pad * kDigits, 512) &&
                   make_i8_map(&c->tm_dig2048, c->d_dig2048, rows_pad * kDigits, 2048);
    {
        Lane& L0 = c->lanes[0];
        L0.stream = c->stream;
        L0.x0 = c->d_x0;
        L0.x1 = c->d_x1;
        L0.q = c->d_q;
        L0.a = c->d_a;
        L0.h = c->d_h;
        L0.g = c->d_g;
        L0.part = c->d_part;
        L0.meta = c->d_meta;
        L0.h_meta = c->h_meta;
        L0.dig512 = c->d_dig512;
        L0.dig2048 = c->d_dig2048;
        L0.exps = c->d_exps;
        L0.tm_dig512 = c->tm_dig512;
        L0.tm_dig2048 = c->tm_dig2048;
        L0.rope = c->d_rope;
        const size_t ctr_bytes = static_cast<size_t>(cfg.n_layers) * 4;
        if (cudaMalloc(&L0.chunk_ctr, ctr_bytes) != cudaSuccess || cudaMemset(L0.chunk_ctr, 0, ctr_bytes) != cudaSuccess)
            return fail(PHONON_CUDA_OUT_OF_MEMORY);
        if (cudaEventCreateWithFlags(&c->fork, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&c->join, cudaEventDisableTiming) != cudaSuccess)
            return fail(PHONON_CUDA_DEVICE_ERROR);
        // A second lane only when a step can hold two half batches.
        if (cfg.max_batch >= 96) {
            Lane& L1 = c->lanes[1];
            const bool ok1 =
                cudaStreamCreateWithFlags(&L1.stream, cudaStreamNonBlocking) == cudaSuccess &&
                cudaMalloc(&L1.x0, rows * kWidth * 4) == cudaSuccess && cudaMalloc(&L1.x1, rows * kWidth * 4) == cudaSuccess &&
                cudaMalloc(&L1.q, rows * kWidth * 4) == cudaSuccess && cudaMalloc(&L1.a, rows * kWidth * 4) == cudaSuccess &&
                cudaMalloc(&L1.h, rows * kWidth * 4) == cudaSuccess && cudaMalloc(&L1.g, rows * kFfn * 4) == cudaSuccess &&
                cudaMalloc(&L1.part, static_cast<size_t>(c->max_splits) * kHeads * kPartStride * 4) == cudaSuccess &&
                cudaMalloc(&L1.meta, static_cast<size_t>(c->meta_ints) * 4) == cudaSuccess &&
                cudaMallocHost(&L1.h_meta, static_cast<size_t>(c->meta_ints) * 4) == cudaSuccess &&
                cudaMalloc(&L1.dig512, rows_pad * kDigits * 512) == cudaSuccess &&
                cudaMalloc(&L1.dig2048, rows_pad * kDigits * 2048) == cudaSuccess &&
                cudaMalloc(&L1.exps, rows_pad * 4) == cudaSuccess &&
                cudaMalloc(&L1.rope, rows * 32 * sizeof(float2)) == cudaSuccess &&
                cudaMalloc(&L1.chunk_ctr, ctr_bytes) == cudaSuccess &&
                cudaMemset(L1.chunk_ctr, 0, ctr_bytes) == cudaSuccess;
            if (!ok1) return fail(PHONON_CUDA_OUT_OF_MEMORY);
            c->lane1_ok = c->tensor_ok && make_i8_map(&L1.tm_dig512, L1.dig512, rows_pad * kDigits, 512) &&
                          make_i8_map(&L1.tm_dig2048, L1.dig2048, rows_pad * kDigits, 2048);
        }
    }
    {
        // Row r of the pool = 64 dims of (layer, page, k|v, head, slot); a
        // layer-page K block is rows [(layer*pool_pages + page)*256, +128).
        const uint64_t kv_rows = static_cast<uint64_t>(cfg.pool_pages) * cfg.n_layers * 256;
        const bool bf16 = cfg.kv_type == PHONON_CUDA_KV_BF16;
        c->attn_tma = kv_rows < (1ull << 31) &&
                      make_map_2d(&c->tm_kv, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                                  c->kv_pool, kv_rows, kHeadDim, kHeadDim * esize, bf16 ? 64 : 32, 128) &&
                      make_map_2d(&c->tm_kv16, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                                  c->kv_pool, kv_rows, kHeadDim, kHeadDim * esize, bf16 ? 64 : 32, kPage);
    }
    if (cudaDeviceGetAttribute(&c->sms, cudaDevAttrMultiProcessorCount, cfg.device) != cudaSuccess ||
        cudaDeviceGetAttribute(&c->smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, cfg.device) != cudaSuccess ||
        cudaMalloc(&c->d_players, sizeof(PersistLayer) * cfg.n_layers) != cudaSuccess ||
        cudaMalloc(&c->d_bar, 4) != cudaSuccess || cudaMemset(c->d_bar, 0, 4) != cudaSuccess || c->sms > kMaxSms)
        return fail(PHONON_CUDA_OUT_OF_MEMORY);
    if ((st = refresh_persist(c))) return fail(st);
    if (cudaMemcpy(c->d_freq, freq, sizeof(freq), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemset(c->d_table, 0, static_cast<size_t>(cfg.max_streams) * kMaxPagesPerStream * 4) != cudaSuccess)
        return fail(PHONON_CUDA_DEVICE_ERROR);
    c->free_pages.reserve(cfg.pool_pages);
    for (int32_t p = static_cast<int32_t>(cfg.pool_pages) - 1; p >= 0; --p) c->free_pages.push_back(p);
    c->streams.resize(cfg.max_streams);
    c->h_fresh_page.assign(cfg.max_streams, INT32_MAX);
    *out = c;
    return PHONON_CUDA_OK;
}

void phonon_cuda_destroy(PhononCuda* ctx) { destroy_context(ctx); }

int phonon_cuda_set_theta(PhononCuda* c, float theta) {
    if (!c || !(theta > 0.0f) || !std::isfinite(theta)) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(c->mu);
    if (c->pending) return PHONON_CUDA_INVALID_ARGUMENT;
    if (theta == c->cfg.theta) return PHONON_CUDA_OK;
    int st = set_device(c->cfg.device);
    if (st) return st;
    float freq[32];
    rope_frequencies(theta, kHeadDim, freq);
    CUDA_TRY(cudaMemcpyAsync(c->d_freq, freq, sizeof(freq), cudaMemcpyHostToDevice, c->stream));
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    c->cfg.theta = theta;
    return PHONON_CUDA_OK;
}

int phonon_cuda_set_layer(PhononCuda* c, uint32_t layer, const PhononCudaLayer* weights) {
    if (!c || !weights) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(c->mu);
    if (c->pending || layer >= c->cfg.n_layers) return PHONON_CUDA_INVALID_ARGUMENT;
    int st = set_device(c->cfg.device);
    if (st) return st;
    if (cudaStreamSynchronize(c->stream) != cudaSuccess) return PHONON_CUDA_DEVICE_ERROR;
    drop_graph(c);  // captured kernels hold the old weight pointers
    if ((st = load_layer(&c->layers[layer], *weights))) return st;
    return refresh_persist(c);
}

int phonon_cuda_stream_alloc(PhononCuda* c, uint32_t capacity, uint32_t* stream) {
    if (!c || !stream || capacity == 0) return PHONON_CUDA_INVALID_ARGUMENT;
    if (capacity > PHONON_CUDA_MAX_POSITIONS) return PHONON_CUDA_CAPACITY;
    std::lock_guard<std::mutex> g(c->mu);
    for (uint32_t s = 0; s < c->streams.size(); ++s)
        if (!c->streams[s].used) {
            c->streams[s].used = true;
            c->streams[s].capacity = capacity;
            c->streams[s].length = 0;
            c->streams[s].pages.clear();
            *stream = s;
            return PHONON_CUDA_OK;
        }
    return PHONON_CUDA_CAPACITY;
}

int phonon_cuda_stream_reset(PhononCuda* c, uint32_t stream) {
    if (!c) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(c->mu);
    if (!valid_stream(c, stream)) return PHONON_CUDA_INVALID_ARGUMENT;
    release_pages(c, stream);
    return PHONON_CUDA_OK;
}

int phonon_cuda_stream_free(PhononCuda* c, uint32_t stream) {
    if (!c) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(c->mu);
    if (!valid_stream(c, stream)) return PHONON_CUDA_INVALID_ARGUMENT;
    release_pages(c, stream);
    c->streams[stream].used = false;
    return PHONON_CUDA_OK;
}

int phonon_cuda_stream_length(PhononCuda* c, uint32_t stream, uint32_t* length) {
    if (!c || !length) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(c->mu);
    if (!valid_stream(c, stream)) return PHONON_CUDA_INVALID_ARGUMENT;
    *length = c->streams[stream].length;
    return PHONON_CUDA_OK;
}

int phonon_cuda_stream_pages(PhononCuda* c, uint32_t stream, int32_t* pages, uint32_t max_pages, uint32_t* n_pages) {
    if (!c || !n_pages) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(c->mu);
    if (!valid_stream(c, stream)) return PHONON_CUDA_INVALID_ARGUMENT;
    const auto& v = c->streams[stream].pages;
    *n_pages = static_cast<uint32_t>(v.size());
    if (pages)
        for (uint32_t i = 0; i < std::min<uint32_t>(max_pages, *n_pages); ++i) pages[i] = v[i];
    return PHONON_CUDA_OK;
}

uint32_t phonon_cuda_free_pages(PhononCuda* c) {
    if (!c) return 0;
    std::lock_guard<std::mutex> g(c->mu);
    return static_cast<uint32_t>(c->free_pages.size());
}

void* phonon_cuda_cuda_stream(PhononCuda* c) { return c ? c->stream : nullptr; }

int phonon_cuda_profile_enable(PhononCuda* c, int enable) {
    if (!c) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(c->mu);
    if (c->pending) return PHONON_CUDA_INVALID_ARGUMENT;
    c->prof_on = enable != 0;
    if (c->prof_on)
        for (int k = 0; k < PHONON_CUDA_K_COUNT; ++k) {
            c->prof_ms[k] = c->prof_bytes[k] = 0.0;
            c->prof_launches[k] = 0;
        }
    return PHONON_CUDA_OK;
}

int phonon_cuda_profile_read(PhononCuda* c, double* ms, double* bytes, uint64_t* launches) {
    if (!c) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(c->mu);
    for (int k = 0; k < PHONON_CUDA_K_COUNT; ++k) {
        if (ms) ms[k] = c->prof_ms[k];
        if (bytes) bytes[k] = c->prof_bytes[k];
        if (launches) launches[k] = c->prof_launches[k];
    }
    return PHONON_CUDA_OK;
}

uint64_t phonon_cuda_launch_count(PhononCuda* c) {
    if (!c) return 0;
    std::lock_guard<std::mutex> g(c->mu);
    return c->launches;
}

int phonon_cuda_wait_expiry_probe(int device, int kind, uint32_t budget_us, uint64_t* elapsed_ns) {
    if (kind < 0 || kind > 2 || budget_us == 0 || budget_us > 1000000) return PHONON_CUDA_INVALID_ARGUMENT;
    int st = set_device(device);
    if (st) return st;
    if (kind == 2) return noalloc_expiry_probe(device, budget_us, elapsed_ns);
    int32_t* d_err = nullptr;
    unsigned* d_ctr = nullptr;
    cudaEvent_t a = nullptr, b = nullptr;
    int clock_khz = 0;
    int result = PHONON_CUDA_DEVICE_ERROR;
    if (cudaMalloc(&d_err, 4) == cudaSuccess && cudaMalloc(&d_ctr, 4) == cudaSuccess &&
        cudaMemset(d_err, 0, 4) == cudaSuccess && cudaMemset(d_ctr, 0, 4) == cudaSuccess &&
        cudaEventCreate(&a) == cudaSuccess && cudaEventCreate(&b) == cudaSuccess &&
        cudaDeviceGetAttribute(&clock_khz, cudaDevAttrClockRate, device) == cudaSuccess) {
        const long long budget = static_cast<long long>(budget_us) * clock_khz / 1000;
        // Two CTAs of one warp each fit on any device at once, which the
        // grid barrier needs (the counter target is 2 arrivals).
        cudaEventRecord(a);
        wait_expiry_kernel<<<2, 32>>>(kind, budget, d_err, d_ctr);
        cudaEventRecord(b);
        int32_t err = 0;
        float ms = 0.0f;
        if (cudaGetLastError() == cudaSuccess && cudaEventSynchronize(b) == cudaSuccess &&
            cudaMemcpy(&err, d_err, 4, cudaMemcpyDeviceToHost) == cudaSuccess &&
            cudaEventElapsedTime(&ms, a, b) == cudaSuccess) {
            if (elapsed_ns) *elapsed_ns = static_cast<uint64_t>(ms * 1e6);
            result = err ? PHONON_CUDA_DEVICE_ERROR : PHONON_CUDA_OK;
        }
    }
    if (a) cudaEventDestroy(a);
    if (b) cudaEventDestroy(b);
    if (d_err) cudaFree(d_err);
    if (d_ctr) cudaFree(d_ctr);
    return result;
}

int phonon_cuda_set_batch_paths(PhononCuda* c, uint32_t fused_min_batch, uint32_t fused_max_batch,
                                uint32_t tensor_min_batch, uint32_t split_min_batch) {
    if (!c || fused_min_batch < 1 || fused_max_batch > PHONON_CUDA_FUSED_MAX_BATCH || tensor_min_batch < 1 ||
        split_min_batch < 2)
        return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(c->mu);
    if (c->pending) return PHONON_CUDA_INVALID_ARGUMENT;
    c->fused_min = fused_min_batch;
    c->fused_max = fused_max_batch;
    c->split_min = split_min_batch;
    c->tensor_min = tensor_min_batch;
    drop_graph(c);  // a captured step holds the old path choice
    return PHONON_CUDA_OK;
}

#ifdef PHONON_CLUSTER_TRACE
// Profiling builds only: the cluster step's phase timestamps of the last launch.
int phonon_cuda_debug_cluster_trace(unsigned long long* out) {
    return cudaMemcpyFromSymbol(out, g_cluster_trace, sizeof(g_cluster_trace)) == cudaSuccess ? PHONON_CUDA_OK
                                                                                             : PHONON_CUDA_DEVICE_ERROR;
}
#endif

int phonon_cuda_set_layer_trace(PhononCuda* c, float* trace_dev, uint32_t max_rows) {
    if (!c || (trace_dev && (max_rows == 0 || max_rows > c->cfg.max_batch))) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(c->mu);
    if (c->pending) return PHONON_CUDA_INVALID_ARGUMENT;
    c->trace = trace_dev;
    c->trace_rows = trace_dev ? max_rows : 0;
    return PHONON_CUDA_OK;
}

int phonon_cuda_set_cluster_step(PhononCuda* c, uint32_t max_position, int* available) {
    if (!c) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(c->mu);
    if (c->pending) return PHONON_CUDA_INVALID_ARGUMENT;
    c->cluster_max_pos = max_position;
    if (available) *available = c->cluster_ok ? (c->cluster_tc ? 2 : 1) : 0;
    drop_graph(c);
    return PHONON_CUDA_OK;
}

}  // extern "C"

namespace {

// Validate a decode batch and allocate the pages it writes. On success the
// entries are in slot/pos and `undo` holds the new pages.
int prepare_decode(PhononCuda* c, uint32_t n, const uint32_t* streams, const uint32_t* positions,
                   std::vector<int32_t>& slot, std::vector<int32_t>& pos, std::vector<int32_t>& updates,
                   PageUndo& undo, bool require_length) {
    if (n < 1 || n > c->cfg.max_batch || !streams || !positions) return PHONON_CUDA_INVALID_ARGUMENT;
    slot.resize(n);
    pos.resize(n);
    for (uint32_t i = 0; i < n; ++i) {
        const uint32_t s = streams[i];
        if (!valid_stream(c, s)) return PHONON_CUDA_INVALID_ARGUMENT;
        for (uint32_t j = 0; j < i; ++j)
            if (streams[j] == s) return PHONON_CUDA_INVALID_ARGUMENT;
        const StreamSlot& st = c->streams[s];
        if (positions[i] >= st.capacity || positions[i] >= PHONON_CUDA_MAX_POSITIONS) return PHONON_CUDA_CAPACITY;
        if (require_length && positions[i] != st.length) return PHONON_CUDA_BAD_POSITION;
        slot[i] = static_cast<int32_t>(s);
        pos[i] = static_cast<int32_t>(positions[i]);
    }
    for (uint32_t i = 0; i < n; ++i) {
        const int st = ensure_pages(c, streams[i], positions[i] / kPage + 1, undo, updates);
        if (st != PHONON_CUDA_OK) {
            undo.rollback();
            return st;
        }
    }
    return PHONON_CUDA_OK;
}

int finish_sync(PhononCuda* c, uint32_t n) {
    CUDA_TRY(cudaMemcpyAsync(c->h_status, c->d_status, n * 4, cudaMemcpyDeviceToHost, c->stream));
    int32_t err = 0;
    CUDA_TRY(cudaMemcpyAsync(&err, c->d_err, 4, cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    prof_collect(c);
    if (err) {  // a bounded device wait expired: report, then clear for the next call
        cudaMemsetAsync(c->d_err, 0, 4, c->stream);
        if (c->d_bar) cudaMemsetAsync(c->d_bar, 0, 4, c->stream);
        c->bar_epoch = 0;
        cudaStreamSynchronize(c->stream);
        std::fprintf(stderr, "phonon_cuda: a device wait expired\n");
        return PHONON_CUDA_DEVICE_ERROR;
    }
    return PHONON_CUDA_OK;
}

}  // namespace

extern "C" {

// Host memory the driver has page-locked (cudaHostAlloc, cudaHostRegister):
// DMA can read it directly, without a staging copy.
static bool is_pinned_host(const void* p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

int phonon_cuda_step(PhononCuda* c, uint32_t n, const uint32_t* streams, const uint32_t* positions,
                     const float* x, float* y, int32_t* status, PhononCudaCancelPoll cancel, void* cctx) {
    if (!c || !x || !y || !status) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(c->mu);
    if (c->pending) return PHONON_CUDA_INVALID_ARGUMENT;
    int st = set_device(c->cfg.device);
    if (st) return st;
    std::vector<int32_t> slot, pos, updates;
    PageUndo undo{c, {}};
    if ((st = prepare_decode(c, n, streams, positions, slot, pos, updates, undo, true))) return st;
    const size_t x_bytes = static_cast<size_t>(n) * kWidth * 4;
    if (is_pinned_host(x)) {
        CUDA_TRY(cudaMemcpyAsync(c->d_x0, x, x_bytes, cudaMemcpyHostToDevice, c->stream));
    } else {
        std::memcpy(c->h_x, x, x_bytes);
        CUDA_TRY(cudaMemcpyAsync(c->d_x0, c->h_x, x_bytes, cudaMemcpyHostToDevice, c->stream));
    }
    cudaMemsetAsync(c->d_status, 0, n * 4, c->stream);
    bool cancelled = false;
    st = enqueue_decode(c, slot, pos, updates, c->d_x0, c->d_y, cancel, cctx, &cancelled);
    if (st && st != PHONON_CUDA_CANCELLED && !cancelled) undo.rollback();
    // Page-locked y: read the status words first, then DMA the rows of the
    // streams that succeeded straight into y (runs of consecutive rows), so
    // no host copy of the outputs is made. Other y: through the staging rows.
    const bool direct_y = is_pinned_host(y);
    if (st == PHONON_CUDA_OK && !direct_y)
        cudaMemcpyAsync(c->h_y, c->d_y, static_cast<size_t>(n) * kWidth * 4, cudaMemcpyDeviceToHost, c->stream);
    const int sync = finish_sync(c, n);
    if (cancelled) {
        for (uint32_t i = 0; i < n; ++i) release_pages(c, streams[i]);
        return PHONON_CUDA_CANCELLED;
    }
    if (st) return st;
    if (sync) return sync;
    for (uint32_t i = 0; i < n; ++i) status[i] = c->h_status[i] ? c->h_status[i] : PHONON_CUDA_OK;
    if (direct_y) {
        for (uint32_t i = 0; i < n;) {
            if (status[i] != PHONON_CUDA_OK) {
                ++i;
                continue;
            }
            uint32_t j = i;
            while (j < n && status[j] == PHONON_CUDA_OK) ++j;
            CUDA_TRY(cudaMemcpyAsync(y + static_cast<size_t>(i) * kWidth, c->d_y + static_cast<size_t>(i) * kWidth,
                                     static_cast<size_t>(j - i) * kWidth * 4, cudaMemcpyDeviceToHost, c->stream));
            i = j;
        }
        CUDA_TRY(cudaStreamSynchronize(c->stream));
    }
    for (uint32_t i = 0; i < n; ++i) {
        if (status[i] != PHONON_CUDA_OK) continue;
        c->streams[streams[i]].length++;
        if (!direct_y)
            std::memcpy(y + static_cast<size_t>(i) * kWidth, c->h_y + static_cast<size_t>(i) * kWidth, kWidth * 4);
    }
    return PHONON_CUDA_OK;
}

int phonon_cuda_step_device(PhononCuda* c, uint32_t n, const uint32_t* streams, const uint32_t* positions,
                            const float* x_dev, float* y_dev) {
    if (!c || !x_dev || !y_dev) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(c->mu);
    if (c->pending) return PHONON_CUDA_INVALID_ARGUMENT;
    int st = set_device(c->cfg.device);
    if (st) return st;
    std::vector<int32_t> slot, pos, updates;
    PageUndo undo{c, {}};
    if ((st = prepare_decode(c, n, streams, positions, slot, pos, updates, undo, true))) return st;
    cudaMemsetAsync(c->d_status, 0, n * 4, c->stream);
    bool cancelled = false;
    if ((st = enqueue_decode(c, slot, pos, updates, x_dev, y_dev, nullptr, nullptr, &cancelled))) {
        undo.rollback();
        return st;
    }
    c->pending = true;
    c->pending_streams.assign(streams, streams + n);
    return PHONON_CUDA_OK;
}

int phonon_cuda_sync(PhononCuda* c, int32_t* status) {
    if (!c) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(c->mu);
    if (!c->pending) return PHONON_CUDA_INVALID_ARGUMENT;
    int st = set_device(c->cfg.device);
    if (st) return st;
    const uint32_t n = static_cast<uint32_t>(c->pending_streams.size());
    c->pending = false;
    if ((st = finish_sync(c, n))) return st;
    for (uint32_t i = 0; i < n; ++i) {
        const int32_t s = c->h_status[i] ? c->h_status[i] : PHONON_CUDA_OK;
        if (status) status[i] = s;
        if (s == PHONON_CUDA_OK) c->streams[c->pending_streams[i]].length++;
    }
    return PHONON_CUDA_OK;
}

int phonon_cuda_layer_step(PhononCuda* c, uint32_t stream, uint32_t layer, uint32_t position, const float* x,
                           float* y) {
    if (!c || !x || !y) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(c->mu);
    if (c->pending || layer >= c->cfg.n_layers) return PHONON_CUDA_INVALID_ARGUMENT;
    int st = set_device(c->cfg.device);
    if (st) return st;
    std::vector<int32_t> slot, pos, updates;
    PageUndo undo{c, {}};
    if ((st = prepare_decode(c, 1, &stream, &position, slot, pos, updates, undo, true))) return st;
    Batch b;
    if ((st = upload_batch(c, slot, pos, updates, &b))) {
        undo.rollback();
        return st;
    }
    std::memcpy(c->h_x, x, kWidth * 4);
    cudaMemcpyAsync(c->d_x0, c->h_x, kWidth * 4, cudaMemcpyHostToDevice, c->stream);
    cudaMemsetAsync(c->d_status, 0, 4, c->stream);
    if ((st = enqueue_layer(c, b, static_cast<int>(layer), c->d_x0, c->d_y))) return st;
    cudaMemcpyAsync(c->h_y, c->d_y, kWidth * 4, cudaMemcpyDeviceToHost, c->stream);
    if ((st = finish_sync(c, 1))) return st;
    if (c->h_status[0]) return c->h_status[0];
    std::memcpy(y, c->h_y, kWidth * 4);
    return PHONON_CUDA_OK;
}

int phonon_cuda_commit(PhononCuda* c, uint32_t stream, uint32_t position) {
    if (!c) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(c->mu);
    if (!valid_stream(c, stream)) return PHONON_CUDA_INVALID_ARGUMENT;
    StreamSlot& s = c->streams[stream];
    if (position != s.length) return PHONON_CUDA_BAD_POSITION;
    if (position >= s.capacity) return PHONON_CUDA_CAPACITY;
    s.length++;
    return PHONON_CUDA_OK;
}

int phonon_cuda_append(PhononCuda* c, uint32_t stream, const float* rows, uint32_t length, float* last_output,
                       PhononCudaCancelPoll cancel, void* cctx) {
    if (!c || !rows || !last_output || length == 0) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(c->mu);
    if (c->pending || !valid_stream(c, stream)) return PHONON_CUDA_INVALID_ARGUMENT;
    StreamSlot& ss = c->streams[stream];
    if (ss.length != 0) return PHONON_CUDA_BAD_POSITION;
    if (length > ss.capacity || length > PHONON_CUDA_MAX_POSITIONS) return PHONON_CUDA_CAPACITY;
    int st = set_device(c->cfg.device);
    if (st) return st;
    std::vector<int32_t> updates;
    PageUndo undo{c, {}};
    if ((st = ensure_pages(c, stream, (length - 1) / kPage + 1, undo, updates))) {
        undo.rollback();
        return st;
    }
    // Emulated reference poll schedule: the full per-layer count on the first
    // pass over the layers, one poll per layer afterwards.
    std::vector<int> first_polls(c->cfg.n_layers, prefill_polls_per_layer(length));
    std::vector<int> later_polls(c->cfg.n_layers, 1);
    const int chunk = c->cap_rows;
    int result = PHONON_CUDA_OK;
    bool cancelled = false, bad = false;
    for (uint32_t p0 = 0; p0 < length && result == PHONON_CUDA_OK; p0 += chunk) {
        const int R = static_cast<int>(std::min<uint32_t>(chunk, length - p0));
        std::vector<int32_t> slot(R, static_cast<int32_t>(stream)), pos(R);
        for (int e = 0; e < R; ++e) pos[e] = static_cast<int32_t>(p0 + e);
        Batch b;
        result = upload_batch(c, slot, pos, p0 == 0 ? updates : std::vector<int32_t>{}, &b);
        if (result != PHONON_CUDA_OK) break;
        std::memcpy(c->h_x, rows + static_cast<size_t>(p0) * kWidth, static_cast<size_t>(R) * kWidth * 4);
        cudaMemcpyAsync(c->d_x0, c->h_x, static_cast<size_t>(R) * kWidth * 4, cudaMemcpyHostToDevice, c->stream);
        cudaMemsetAsync(c->d_status, 0, R * 4, c->stream);
        result = enqueue_stack(c, b, c->d_x0, c->d_y, cancel, cctx, p0 == 0 ? &first_polls : &later_polls, &cancelled);
        if (result == PHONON_CUDA_OK && p0 + R == length)
            cudaMemcpyAsync(c->h_y, c->d_y + static_cast<size_t>(R - 1) * kWidth, kWidth * 4, cudaMemcpyDeviceToHost,
                            c->stream);
        const int sync = finish_sync(c, R);
        if (result == PHONON_CUDA_OK && sync) result = sync;
        for (int e = 0; e < R && result == PHONON_CUDA_OK; ++e)
            if (c->h_status[e]) bad = true;
        if (bad) result = PHONON_CUDA_NON_FINITE;
    }
    if (result != PHONON_CUDA_OK) {
        release_pages(c, stream);
        return cancelled ? PHONON_CUDA_CANCELLED : result;
    }
    ss.length = length;
    std::memcpy(last_output, c->h_y, kWidth * 4);
    return PHONON_CUDA_OK;
}

// Grow the pinned/device staging rows for KV transfers to hold n floats.
static int reserve_stage(PhononCuda* c, size_t n) {
    if (n <= c->stage_cap) return PHONON_CUDA_OK;
    if (c->d_stage) cudaFree(c->d_stage);
    if (c->h_stage) cudaFreeHost(c->h_stage);
    c->d_stage = nullptr;
    c->h_stage = nullptr;
    c->stage_cap = 0;
    if (cudaMalloc(&c->d_stage, n * 4) != cudaSuccess || cudaMallocHost(&c->h_stage, n * 4) != cudaSuccess)
        return PHONON_CUDA_OUT_OF_MEMORY;
    c->stage_cap = n;
    return PHONON_CUDA_OK;
}

static int check_kv_range(PhononCuda* c, uint32_t stream, uint32_t layer_begin, uint32_t layer_count,
                          uint32_t position, uint32_t count) {
    if (c->pending || !valid_stream(c, stream) || layer_count == 0 || count == 0 ||
        layer_begin >= c->cfg.n_layers || layer_count > c->cfg.n_layers - layer_begin)
        return PHONON_CUDA_INVALID_ARGUMENT;
    if (position >= c->streams[stream].capacity || count > c->streams[stream].capacity - position)
        return PHONON_CUDA_CAPACITY;
    return PHONON_CUDA_OK;
}

int phonon_cuda_kv_write(PhononCuda* c, uint32_t stream, uint32_t layer_begin, uint32_t layer_count,
                         uint32_t position, uint32_t count, const float* keys, const float* values) {
    if (!c || !keys || !values) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(c->mu);
    int st = check_kv_range(c, stream, layer_begin, layer_count, position, count);
    if (st) return st;
    const size_t n = static_cast<size_t>(layer_count) * count * kWidth;
    for (size_t i = 0; i < n; ++i)
        if (!std::isfinite(keys[i]) || !std::isfinite(values[i])) return PHONON_CUDA_NON_FINITE;
    if ((st = set_device(c->cfg.device)) || (st = reserve_stage(c, 2 * n))) return st;
    std::vector<int32_t> updates;
    PageUndo undo{c, {}};
    if ((st = ensure_pages(c, stream, (position + count - 1) / kPage + 1, undo, updates))) {
        undo.rollback();
        return st;
    }
    if (!updates.empty()) {
        Batch b;
        std::vector<int32_t> slot{static_cast<int32_t>(stream)}, pos{static_cast<int32_t>(position)};
        if ((st = upload_batch(c, slot, pos, updates, &b))) {
            undo.rollback();
            return st;
        }
    }
    std::memcpy(c->h_stage, keys, n * 4);
    std::memcpy(c->h_stage + n, values, n * 4);
    CUDA_TRY(cudaMemcpyAsync(c->d_stage, c->h_stage, 2 * n * 4, cudaMemcpyHostToDevice, c->stream));
    kv_rows_kernel<<<static_cast<unsigned>(std::min<size_t>((2 * n + 255) / 256, 4096)), 256, 0, c->stream>>>(
        kv_view(c), static_cast<int>(stream), static_cast<int>(layer_begin), static_cast<int>(layer_count),
        static_cast<int>(position), static_cast<int>(count), c->d_stage, 1);
    CUDA_TRY(cudaGetLastError());
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    return PHONON_CUDA_OK;
}

int phonon_cuda_kv_read(PhononCuda* c, uint32_t stream, uint32_t layer_begin, uint32_t layer_count,
                        uint32_t position, uint32_t count, float* keys, float* values) {
    if (!c || !keys || !values) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(c->mu);
    int st = check_kv_range(c, stream, layer_begin, layer_count, position, count);
    if (st) return st;
    const size_t n = static_cast<size_t>(layer_count) * count * kWidth;
    const uint32_t allocated = static_cast<uint32_t>(c->streams[stream].pages.size()) * kPage;
    const uint32_t readable = position >= allocated ? 0 : std::min(count, allocated - position);
    if (readable < count) {  // never-allocated positions read as zeros
        for (uint32_t l = 0; l < layer_count; ++l) {
            std::memset(keys + (static_cast<size_t>(l) * count + readable) * kWidth, 0, (count - readable) * kWidth * 4);
            std::memset(values + (static_cast<size_t>(l) * count + readable) * kWidth, 0, (count - readable) * kWidth * 4);
        }
    }
    if (readable == 0) return PHONON_CUDA_OK;
    if ((st = set_device(c->cfg.device)) || (st = reserve_stage(c, 2 * n))) return st;
    kv_rows_kernel<<<static_cast<unsigned>(std::min<size_t>((2 * n + 255) / 256, 4096)), 256, 0, c->stream>>>(
        kv_view(c), static_cast<int>(stream), static_cast<int>(layer_begin), static_cast<int>(layer_count),
        static_cast<int>(position), static_cast<int>(readable), c->d_stage, 0);
    CUDA_TRY(cudaGetLastError());
    const size_t nr = static_cast<size_t>(layer_count) * readable * kWidth;
    CUDA_TRY(cudaMemcpyAsync(c->h_stage, c->d_stage, 2 * nr * 4, cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    for (uint32_t l = 0; l < layer_count; ++l) {
        std::memcpy(keys + static_cast<size_t>(l) * count * kWidth, c->h_stage + static_cast<size_t>(l) * readable * kWidth,
                    static_cast<size_t>(readable) * kWidth * 4);
        std::memcpy(values + static_cast<size_t>(l) * count * kWidth,
                    c->h_stage + nr + static_cast<size_t>(l) * readable * kWidth, static_cast<size_t>(readable) * kWidth * 4);
    }
    return PHONON_CUDA_OK;
}

int phonon_cuda_stream_fill_synthetic(PhononCuda* c, uint32_t stream, uint32_t length, uint64_t seed) {
    if (!c || length == 0) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(c->mu);
    if (c->pending || !valid_stream(c, stream)) return PHONON_CUDA_INVALID_ARGUMENT;
    StreamSlot& ss = c->streams[stream];
    if (ss.length != 0) return PHONON_CUDA_BAD_POSITION;
    if (length > ss.capacity) return PHONON_CUDA_CAPACITY;
    int st = set_device(c->cfg.device);
    if (st) return st;
    std::vector<int32_t> updates;
    PageUndo undo{c, {}};
    if ((st = ensure_pages(c, stream, (length - 1) / kPage + 1, undo, updates))) {
        undo.rollback();
        return st;
    }
    Batch b;
    std::vector<int32_t> slot{static_cast<int32_t>(stream)}, pos{0};
    if ((st = upload_batch(c, slot, pos, updates, &b))) {
        undo.rollback();
        return st;
    }
    {
        LaunchScope ls(c, PHONON_CUDA_K_OTHER, static_cast<double>(length) * c->page_elems / kPage *
                                                   (c->cfg.kv_type == PHONON_CUDA_KV_BF16 ? 2 : 4));
        kv_fill_kernel<<<296, 256, 0, c->stream>>>(kv_view(c), static_cast<int>(stream),
                                                   static_cast<int>(c->cfg.n_layers), static_cast<int>(length), seed);
        CUDA_TRY(cudaGetLastError());
    }
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    prof_collect(c);
    ss.length = length;
    return PHONON_CUDA_OK;
}

}  // extern "C"

// ========================================================= raw int8 GEMM
extern "C" int phonon_cuda_i8_gemm(int device, const int8_t* a, const int8_t* b, size_t m, size_t n, size_t k,
                                   int32_t* d) {
    if (!a || !b || !d || !m || !n || !k || k % kGemmKTile || m > (1u << 20) || n > (1u << 20) || k > (1u << 16))
        return PHONON_CUDA_INVALID_ARGUMENT;
    int st = set_device(device);
    if (st) return st;
    int8_t *da = nullptr, *db = nullptr;
    int32_t *dd = nullptr, *derr = nullptr;
    cudaStream_t s = nullptr;
    auto cleanup = [&](int code) {
        if (s) cudaStreamSynchronize(s);
        if (da) cudaFree(da);
        if (db) cudaFree(db);
        if (dd) cudaFree(dd);
        if (derr) cudaFree(derr);
        if (s) cudaStreamDestroy(s);
        return code;
    };
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess || cudaMalloc(&da, m * k) != cudaSuccess ||
        cudaMalloc(&db, n * k) != cudaSuccess || cudaMalloc(&dd, m * n * 4) != cudaSuccess ||
        cudaMalloc(&derr, 4) != cudaSuccess)
        return cleanup(PHONON_CUDA_OUT_OF_MEMORY);
    CUtensorMap ta, tb;
    if (!make_i8_map(&ta, da, m, k) || !make_i8_map(&tb, db, n, k)) return cleanup(PHONON_CUDA_DEVICE_ERROR);
    if (cudaMemcpy(da, a, m * k, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(db, b, n * k, cudaMemcpyHostToDevice) != cudaSuccess || cudaMemset(derr, 0, 4) != cudaSuccess)
        return cleanup(PHONON_CUDA_DEVICE_ERROR);
    GemmParams p{};
    p.rows = static_cast<int>(m);
    p.K = static_cast<int>(k);
    p.raw = dd;
    p.n_total = static_cast<int>(n);
    p.error = derr;
    if (launch_gemm<GEPI_RAW>(ta, tb, static_cast<int>(m), static_cast<int>(n), p, s) != cudaSuccess)
        return cleanup(PHONON_CUDA_DEVICE_ERROR);
    int32_t err = 0;
    if (cudaMemcpyAsync(&err, derr, 4, cudaMemcpyDeviceToHost, s) != cudaSuccess || cudaStreamSynchronize(s) != cudaSuccess)
        return cleanup(PHONON_CUDA_DEVICE_ERROR);
    if (err) return cleanup(PHONON_CUDA_DEVICE_ERROR);
    if (cudaMemcpy(d, dd, m * n * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return cleanup(PHONON_CUDA_DEVICE_ERROR);
    return cleanup(PHONON_CUDA_OK);
}

// ============================================================ linear handles
struct PhononCudaLinear {
    int device = 0;
    DevLinear lin;
    std::mutex mu;
    cudaStream_t stream = nullptr;
    size_t cap = 0;
    float *d_x = nullptr, *d_y = nullptr, *d_bias = nullptr;
    int32_t* d_status = nullptr;
};

extern "C" {

int phonon_cuda_linear_create(int device, int kind, const void* data, size_t rows, size_t cols,
                              PhononCudaLinear** out) {
    if (!out) return PHONON_CUDA_INVALID_ARGUMENT;
    *out = nullptr;
    int st = set_device(device);
    if (st) return st;
    PhononCudaLinear* l = new (std::nothrow) PhononCudaLinear();
    if (!l) return PHONON_CUDA_OUT_OF_MEMORY;
    l->device = device;
    if ((st = upload_linear(kind, data, rows, cols, &l->lin))) {
        delete l;
        return st;
    }
    if (cudaStreamCreateWithFlags(&l->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&l->d_bias, rows * 4) != cudaSuccess || cudaMalloc(&l->d_status, 4 * 4096) != cudaSuccess) {
        phonon_cuda_linear_destroy(l);
        return PHONON_CUDA_OUT_OF_MEMORY;
    }
    *out = l;
    return PHONON_CUDA_OK;
}

void phonon_cuda_linear_destroy(PhononCudaLinear* l) {
    if (!l) return;
    cudaSetDevice(l->device);
    if (l->stream) cudaStreamSynchronize(l->stream);
    free_linear(l->lin);
    void* dev[] = {l->d_x, l->d_y, l->d_bias, l->d_status};
    for (void* p : dev)
        if (p) cudaFree(p);
    if (l->stream) cudaStreamDestroy(l->stream);
    delete l;
}

size_t phonon_cuda_linear_bytes(const PhononCudaLinear* l) { return l ? l->lin.bytes : 0; }

int phonon_cuda_linear_apply(PhononCudaLinear* l, const float* x, size_t batch, const float* bias, float* y) {
    if (!l || !x || !y || batch == 0 || batch > 4096) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(l->mu);
    int st = set_device(l->device);
    if (st) return st;
    const size_t rows = l->lin.rows, cols = l->lin.cols;
    if (batch > l->cap) {
        if (l->d_x) cudaFree(l->d_x);
        if (l->d_y) cudaFree(l->d_y);
        l->d_x = l->d_y = nullptr;
        l->cap = 0;
        if (cudaMalloc(&l->d_x, batch * cols * 4) != cudaSuccess || cudaMalloc(&l->d_y, batch * rows * 4) != cudaSuccess)
            return PHONON_CUDA_OUT_OF_MEMORY;
        l->cap = batch;
    }
    CUDA_TRY(cudaMemcpyAsync(l->d_x, x, batch * cols * 4, cudaMemcpyHostToDevice, l->stream));
    if (bias) CUDA_TRY(cudaMemcpyAsync(l->d_bias, bias, rows * 4, cudaMemcpyHostToDevice, l->stream));
    CUDA_TRY(cudaMemsetAsync(l->d_status, 0, batch * 4, l->stream));
    CUDA_TRY(launch_linear(l->lin, l->d_x, static_cast<int>(batch), bias ? l->d_bias : nullptr, l->d_y, l->d_status,
                           l->stream));
    std::vector<int32_t> status(batch);
    CUDA_TRY(cudaMemcpyAsync(y, l->d_y, batch * rows * 4, cudaMemcpyDeviceToHost, l->stream));
    CUDA_TRY(cudaMemcpyAsync(status.data(), l->d_status, batch * 4, cudaMemcpyDeviceToHost, l->stream));
    CUDA_TRY(cudaStreamSynchronize(l->stream));
    for (size_t b = 0; b < batch; ++b)
        if (status[b]) return PHONON_CUDA_NON_FINITE;
    return PHONON_CUDA_OK;
}

}  // extern "C"

// ------------------------------------------- allocation-free tensor linear
// Scratch of phonon_cuda_linear_apply_device_noalloc: digit rows of up to
// PHONON_CUDA_NOALLOC_MAX_BATCH streams x 2048 columns, their exponents and
// the tile error flag. Host code must not use these names as addresses: the
// device address comes from cudaGetSymbolAddress on each device.
constexpr int kNoallocRows = kDigits * PHONON_CUDA_NOALLOC_MAX_BATCH;
static __device__ __align__(256) int8_t g_noalloc_digits[kNoallocRows * 2048];
static __device__ __align__(256) int32_t g_noalloc_exps[PHONON_CUDA_NOALLOC_MAX_BATCH];
static __device__ __align__(256) int32_t g_noalloc_error[1];

namespace {

// After the tensor-core kernel of an allocation-free call: when one of its
// bounded waits expired (the flag in the scratch), the rows of y were not
// written, and every status word of the call says so.
__global__ void noalloc_report_kernel(const int32_t* error, int32_t* status, int B) {
    pdl_wait();
    if (*error)
        for (int b = threadIdx.x; b < B; b += blockDim.x) status[b] = PHONON_CUDA_DEVICE_ERROR;
}

struct NoallocScratch {
    bool ready = false;
    int8_t* digits = nullptr;
    int32_t* exps = nullptr;
    int32_t* error = nullptr;
    CUtensorMap map512, map2048;
};

// One-time set-up per device (the device must be current): resolve the
// scratch addresses and describe the digit rows for TMA. Idempotent.
int noalloc_scratch(int device, NoallocScratch** out) {
    static std::mutex mu;
    static NoallocScratch table[kMaxDevices];
    if (device < 0 || device >= kMaxDevices) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(mu);
    NoallocScratch& t = table[device];
    if (!t.ready) {
        void* d = nullptr;
        void* e = nullptr;
        void* f = nullptr;
        if (cudaGetSymbolAddress(&d, g_noalloc_digits) != cudaSuccess ||
            cudaGetSymbolAddress(&e, g_noalloc_exps) != cudaSuccess ||
            cudaGetSymbolAddress(&f, g_noalloc_error) != cudaSuccess)
            return PHONON_CUDA_DEVICE_ERROR;
        t.digits = static_cast<int8_t*>(d);
        t.exps = static_cast<int32_t*>(e);
        t.error = static_cast<int32_t*>(f);
        if (!make_i8_map(&t.map512, t.digits, kNoallocRows, 512) ||
            !make_i8_map(&t.map2048, t.digits, kNoallocRows, 2048))
            return PHONON_CUDA_DEVICE_ERROR;
        t.ready = true;
    }
    *out = &t;
    return PHONON_CUDA_OK;
}

// An mbarrier wait that nothing completes expires against the scratch's error
// flag, then the report kernel marks the status words of a 4-row call: the
// path by which an expired wait inside the tensor-core kernel reaches the
// caller of phonon_cuda_linear_apply_device_noalloc. DEVICE_ERROR when every
// status word reads PHONON_CUDA_DEVICE_ERROR (the expected outcome).
int noalloc_expiry_probe(int device, uint32_t budget_us, uint64_t* elapsed_ns) {
    NoallocScratch* sc = nullptr;
    int st = noalloc_scratch(device, &sc);
    if (st) return st;
    constexpr int kRows = 4;
    int32_t* d_status = nullptr;
    cudaEvent_t a = nullptr, b = nullptr;
    int clock_khz = 0;
    int result = PHONON_CUDA_DEVICE_ERROR;
    if (cudaMalloc(&d_status, kRows * 4) == cudaSuccess && cudaMemset(d_status, 0, kRows * 4) == cudaSuccess &&
        cudaMemset(sc->error, 0, 4) == cudaSuccess && cudaEventCreate(&a) == cudaSuccess &&
        cudaEventCreate(&b) == cudaSuccess &&
        cudaDeviceGetAttribute(&clock_khz, cudaDevAttrClockRate, device) == cudaSuccess) {
        const long long budget = static_cast<long long>(budget_us) * clock_khz / 1000;
        cudaEventRecord(a);
        wait_expiry_kernel<<<2, 32>>>(0, budget, sc->error, nullptr);
        cudaEventRecord(b);
        noalloc_report_kernel<<<1, 64>>>(sc->error, d_status, kRows);
        int32_t status[kRows] = {};
        float ms = 0.0f;
        if (cudaGetLastError() == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess &&
            cudaMemcpy(status, d_status, sizeof(status), cudaMemcpyDeviceToHost) == cudaSuccess &&
            cudaEventElapsedTime(&ms, a, b) == cudaSuccess) {
            if (elapsed_ns) *elapsed_ns = static_cast<uint64_t>(ms * 1e6);
            bool all = true;
            for (int i = 0; i < kRows; ++i) all &= status[i] == PHONON_CUDA_DEVICE_ERROR;
            result = all ? PHONON_CUDA_DEVICE_ERROR : PHONON_CUDA_OK;
        }
        cudaMemset(sc->error, 0, 4);
    }
    if (a) cudaEventDestroy(a);
    if (b) cudaEventDestroy(b);
    if (d_status) cudaFree(d_status);
    return result;
}

}  // namespace

extern "C" {

int phonon_cuda_linear_apply_device_noalloc(PhononCudaLinear* l, const float* x_dev, size_t batch,
                                            const float* bias_dev, float* y_dev, int32_t* status_dev,
                                            void* cuda_stream) {
    if (!l || !x_dev || !y_dev || batch == 0) return PHONON_CUDA_INVALID_ARGUMENT;
    if (reinterpret_cast<uintptr_t>(x_dev) % 16) return PHONON_CUDA_INVALID_ARGUMENT;  // read as float4
    if (batch > PHONON_CUDA_NOALLOC_MAX_BATCH) {
        std::fprintf(stderr, "phonon_cuda_linear_apply_device_noalloc: batch %zu exceeds the scratch limit of %d\n",
                     batch, PHONON_CUDA_NOALLOC_MAX_BATCH);
        return PHONON_CUDA_CAPACITY;
    }
    const DevLinear& w = l->lin;
    if (!w.tensor || w.wd != 1 || (w.cols != 512 && w.cols != 2048)) return PHONON_CUDA_INVALID_ARGUMENT;
    int st = set_device(l->device);
    if (st) return st;
    NoallocScratch* sc = nullptr;
    if ((st = noalloc_scratch(l->device, &sc))) return st;
    cudaStream_t s = static_cast<cudaStream_t>(cuda_stream);
    const int B = static_cast<int>(batch), Bpad = (B + 31) / 32 * 32;
    // The scratch keeps the previous call's contents: clear the error flag.
    CUDA_TRY(cudaMemsetAsync(sc->error, 0, sizeof(int32_t), s));
    if (w.cols == 512)
        CUDA_TRY((launch_digits<512, false>(x_dev, 512, nullptr, nullptr, B, Bpad, sc->digits, sc->exps, status_dev, s)));
    else
        CUDA_TRY((launch_digits<2048, false>(x_dev, 2048, nullptr, nullptr, B, Bpad, sc->digits, sc->exps, status_dev, s)));
    GemmParams p{};
    p.rows = w.rows;
    p.K = w.cols;
    p.B = B;
    p.row_scale = w.row_scale;
    p.exps = sc->exps;
    p.y = y_dev;
    p.ldy = w.rows;
    p.status = status_dev;
    p.error = sc->error;
    p.bias = bias_dev;
    CUDA_TRY(launch_gemm<GEPI_STORE>(w.tmap, w.cols == 512 ? sc->map512 : sc->map2048, w.rows, kDigits * Bpad, p, s));
    if (status_dev) CUDA_TRY(launch_pdl(noalloc_report_kernel, dim3(1), dim3(64), 0, s, sc->error, status_dev, B));
    return PHONON_CUDA_OK;
}

int phonon_cuda_linear_apply_device(PhononCudaLinear* l, const float* x_dev, size_t batch, const float* bias_dev,
                                    float* y_dev, int32_t* status_dev, void* cuda_stream) {
    if (!l || !x_dev || !y_dev || batch == 0 || batch > 65536) return PHONON_CUDA_INVALID_ARGUMENT;
    if (reinterpret_cast<uintptr_t>(x_dev) % 16) return PHONON_CUDA_INVALID_ARGUMENT;  // rows are read as float4
    int st = set_device(l->device);
    if (st) return st;
    CUDA_TRY(launch_linear(l->lin, x_dev, static_cast<int>(batch), bias_dev, y_dev, status_dev,
                           static_cast<cudaStream_t>(cuda_stream)));
    return PHONON_CUDA_OK;
}

}  // extern "C"

// ============================================================== primitives
namespace {

__global__ void layernorm_any_kernel(const float* x, const float* w, const float* b, float* out, int width,
                                     float eps, int32_t* status) {
    // Widths other than 512: one thread, double mean and variance like the
    // reference (src/phonon_transformer.c:158-177), fp32 affine step.
    if (threadIdx.x != 0) return;
    double sum = 0.0;
    for (int i = 0; i < width; ++i) {
        if (!isfinite(x[i]) || !isfinite(w[i]) || !isfinite(b[i])) {
            *status = kStatusNonFinite;
            return;
        }
        sum += x[i];
    }
    const double mean = sum / static_cast<double>(width);
    double squares = 0.0;
    for (int i = 0; i < width; ++i) {
        const double centered = static_cast<double>(x[i]) - mean;
        squares = __dadd_rn(squares, __dmul_rn(centered, centered));
    }
    const float variance = __double2float_rn(squares / static_cast<double>(width));
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(variance, eps)));
    for (int i = 0; i < width; ++i) {
        const float v = __fadd_rn(__fmul_rn(__fmul_rn(__double2float_rn(static_cast<double>(x[i]) - mean), scale), w[i]), b[i]);
        if (!isfinite(v)) *status = kStatusNonFinite;
        out[i] = v;
    }
}

__global__ void layernorm512_eps_kernel(const float* x, const float* w, const float* b, float* out, float eps,
                                        int32_t* status) {
    if (!warp_layernorm512(x, w, b, out, eps) && threadIdx.x == 0) *status = kStatusNonFinite;
}

// x * scale * w, scale = 1/sqrtf(mean(x^2) + eps) with a double sum of squares
// (src/phonon_transformer.c:66-85). One thread: the reference order exactly.
__global__ void rmsnorm_kernel(const float* x, const float* w, float* out, int width, float eps, int32_t* status) {
    if (threadIdx.x != 0) return;
    double squares = 0.0;
    for (int i = 0; i < width; ++i) {
        if (!isfinite(x[i]) || !isfinite(w[i])) {
            *status = kStatusNonFinite;
            return;
        }
        squares = __dadd_rn(squares, __dmul_rn(static_cast<double>(x[i]), static_cast<double>(x[i])));
    }
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__double2float_rn(squares / static_cast<double>(width)), eps)));
    if (!isfinite(scale)) {
        *status = kStatusNonFinite;
        return;
    }
    for (int i = 0; i < width; ++i) {
        const float v = __fmul_rn(__fmul_rn(x[i], scale), w[i]);
        if (!isfinite(v)) *status = kStatusNonFinite;
        out[i] = v;
    }
}

// Elements in full groups of four use the polynomial erf; the count % 4 tail
// uses erf evaluated in double (the reference calls libm erff there).
__global__ void gelu_kernel(float* v, long long count, int32_t* status) {
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= count) return;
    const float x = v[i];
    if (!isfinite(x)) {
        *status = kStatusNonFinite;
        return;
    }
    float y;
    if (i < count - count % 4) {
        y = gelu_erf(x);
    } else {
        const float scaled = __fmul_rn(x, 0.7071067811865475244f);
        const float e = __double2float_rn(erf(static_cast<double>(scaled)));
        y = __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, e));
    }
    if (!isfinite(y)) *status = kStatusNonFinite;
    v[i] = y;
}

__global__ void rope_kernel(float* v, int width, int heads, int position, const float* freq, int32_t* status) {
    const int head_width = width / heads;
    const int pairs = width / 2;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= pairs) return;
    const int h = i / (head_width / 2), k = i % (head_width / 2);
    float a = v[h * head_width + 2 * k], b = v[h * head_width + 2 * k + 1];
    if (!isfinite(a) || !isfinite(b)) {
        *status = kStatusNonFinite;
        return;
    }
    rope_pair(a, b, position, freq[k]);
    if (!isfinite(a) || !isfinite(b)) *status = kStatusNonFinite;
    v[h * head_width + 2 * k] = a;
    v[h * head_width + 2 * k + 1] = b;
}

// Per-device scratch for the primitive calls.
struct PrimExec {
    std::mutex mu;
    cudaStream_t stream = nullptr;
    size_t cap = 0;  // floats per buffer
    float *d_a = nullptr, *d_b = nullptr, *d_c = nullptr, *d_d = nullptr;
    int32_t* d_status = nullptr;
};

PrimExec* prim_exec(int device) {
    static std::mutex table_mu;
    static std::vector<PrimExec*> table;
    std::lock_guard<std::mutex> g(table_mu);
    if (device < 0 || device > 1024) return nullptr;
    if (table.size() <= static_cast<size_t>(device)) table.resize(device + 1, nullptr);
    if (!table[device]) table[device] = new PrimExec();
    return table[device];
}

int prim_reserve(PrimExec* e, size_t n) {
    if (!e->stream && cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess)
        return PHONON_CUDA_DEVICE_ERROR;
    if (!e->d_status && cudaMalloc(&e->d_status, 4) != cudaSuccess) return PHONON_CUDA_OUT_OF_MEMORY;
    if (n <= e->cap) return PHONON_CUDA_OK;
    float** bufs[] = {&e->d_a, &e->d_b, &e->d_c, &e->d_d};
    for (float** b : bufs) {
        if (*b) cudaFree(*b);
        *b = nullptr;
    }
    e->cap = 0;
    for (float** b : bufs)
        if (cudaMalloc(b, n * 4) != cudaSuccess) return PHONON_CUDA_OUT_OF_MEMORY;
    e->cap = n;
    return PHONON_CUDA_OK;
}

int prim_finish(PrimExec* e) {
    int32_t status = 0;
    CUDA_TRY(cudaGetLastError());
    CUDA_TRY(cudaMemcpyAsync(&status, e->d_status, 4, cudaMemcpyDeviceToHost, e->stream));
    CUDA_TRY(cudaStreamSynchronize(e->stream));
    return status ? PHONON_CUDA_NON_FINITE : PHONON_CUDA_OK;
}

}  // namespace

extern "C" {

int phonon_cuda_layer_norm(int device, const float* x, const float* w, const float* b, size_t width, float eps,
                           float* out) {
    if (!x || !w || !b || !out || width == 0 || width > (1u << 24) || !(eps > 0.0f) || !std::isfinite(eps))
        return PHONON_CUDA_INVALID_ARGUMENT;
    int st = set_device(device);
    if (st) return st;
    PrimExec* e = prim_exec(device);
    if (!e) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(e->mu);
    if ((st = prim_reserve(e, width))) return st;
    CUDA_TRY(cudaMemcpyAsync(e->d_a, x, width * 4, cudaMemcpyHostToDevice, e->stream));
    CUDA_TRY(cudaMemcpyAsync(e->d_b, w, width * 4, cudaMemcpyHostToDevice, e->stream));
    CUDA_TRY(cudaMemcpyAsync(e->d_c, b, width * 4, cudaMemcpyHostToDevice, e->stream));
    CUDA_TRY(cudaMemsetAsync(e->d_status, 0, 4, e->stream));
    if (width == 512)
        layernorm512_eps_kernel<<<1, 32, 0, e->stream>>>(e->d_a, e->d_b, e->d_c, e->d_d, eps, e->d_status);
    else
        layernorm_any_kernel<<<1, 32, 0, e->stream>>>(e->d_a, e->d_b, e->d_c, e->d_d, static_cast<int>(width), eps,
                                                      e->d_status);
    if ((st = prim_finish(e))) return st;
    CUDA_TRY(cudaMemcpy(out, e->d_d, width * 4, cudaMemcpyDeviceToHost));
    return PHONON_CUDA_OK;
}

int phonon_cuda_rms_norm(int device, const float* x, const float* w, size_t width, float eps, float* out) {
    if (!x || !w || !out || width == 0 || width > (1u << 24) || !(eps > 0.0f) || !std::isfinite(eps))
        return PHONON_CUDA_INVALID_ARGUMENT;
    int st = set_device(device);
    if (st) return st;
    PrimExec* e = prim_exec(device);
    if (!e) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(e->mu);
    if ((st = prim_reserve(e, width))) return st;
    CUDA_TRY(cudaMemcpyAsync(e->d_a, x, width * 4, cudaMemcpyHostToDevice, e->stream));
    CUDA_TRY(cudaMemcpyAsync(e->d_b, w, width * 4, cudaMemcpyHostToDevice, e->stream));
    CUDA_TRY(cudaMemsetAsync(e->d_status, 0, 4, e->stream));
    rmsnorm_kernel<<<1, 32, 0, e->stream>>>(e->d_a, e->d_b, e->d_d, static_cast<int>(width), eps, e->d_status);
    if ((st = prim_finish(e))) return st;
    CUDA_TRY(cudaMemcpy(out, e->d_d, width * 4, cudaMemcpyDeviceToHost));
    return PHONON_CUDA_OK;
}

int phonon_cuda_erf_gelu(int device, float* values, size_t count) {
    if (count == 0) return PHONON_CUDA_OK;
    if (!values || count > (1u << 28)) return PHONON_CUDA_INVALID_ARGUMENT;
    int st = set_device(device);
    if (st) return st;
    PrimExec* e = prim_exec(device);
    if (!e) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(e->mu);
    if ((st = prim_reserve(e, count))) return st;
    CUDA_TRY(cudaMemcpyAsync(e->d_a, values, count * 4, cudaMemcpyHostToDevice, e->stream));
    CUDA_TRY(cudaMemsetAsync(e->d_status, 0, 4, e->stream));
    gelu_kernel<<<static_cast<unsigned>((count + 255) / 256), 256, 0, e->stream>>>(e->d_a, static_cast<long long>(count),
                                                                                   e->d_status);
    if ((st = prim_finish(e))) return st;
    CUDA_TRY(cudaMemcpy(values, e->d_a, count * 4, cudaMemcpyDeviceToHost));
    return PHONON_CUDA_OK;
}

int phonon_cuda_rope_interleaved(int device, float* values, size_t width, size_t heads, size_t position, float theta) {
    if (!values || !width || !heads || width % heads || (width / heads) % 2 || !(theta > 0.0f) ||
        !std::isfinite(theta) || width > (1u << 24) || position > (1u << 30))
        return PHONON_CUDA_INVALID_ARGUMENT;
    int st = set_device(device);
    if (st) return st;
    PrimExec* e = prim_exec(device);
    if (!e) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(e->mu);
    if ((st = prim_reserve(e, width))) return st;
    std::vector<float> freq(width / heads / 2);
    rope_frequencies(theta, width / heads, freq.data());
    CUDA_TRY(cudaMemcpyAsync(e->d_a, values, width * 4, cudaMemcpyHostToDevice, e->stream));
    CUDA_TRY(cudaMemcpyAsync(e->d_b, freq.data(), freq.size() * 4, cudaMemcpyHostToDevice, e->stream));
    CUDA_TRY(cudaMemsetAsync(e->d_status, 0, 4, e->stream));
    rope_kernel<<<static_cast<unsigned>((width / 2 + 255) / 256), 256, 0, e->stream>>>(
        e->d_a, static_cast<int>(width), static_cast<int>(heads), static_cast<int>(position), e->d_b, e->d_status);
    if ((st = prim_finish(e))) return st;
    CUDA_TRY(cudaMemcpy(values, e->d_a, width * 4, cudaMemcpyDeviceToHost));
    return PHONON_CUDA_OK;
}

}  // extern "C"

// ------------------------------------------------------------------ frame loop
// The flow head, EOS logit, embedding and output norm (phonon_head.cuh) on a
// context's stream and lock. Matrices fed to gemv_kernel use its
// lane-interleaved bf16 layout (upload_linear); the small ones the head's own
// kernels read stay natural row-major bf16.
struct PhononCudaHead {
    PhononCuda* c = nullptr;
    DevLinear cond;                    // [513][512]: cond_embed rows, then the EOS row
    DevLinear ada;                     // [kAdaRows][512]: every block's adaLN rows, the final layer's last
    DevLinear mlp[phonon::kHeadBlocks][2];
    uint16_t* w16 = nullptr;           // natural bf16 matrices (offsets below)
    const uint16_t *in_w = nullptr, *fin_w = nullptr, *embed_w = nullptr;
    const uint16_t* time_w[2][2] = {};
    float* f = nullptr;                // fp32 copies of the vectors (offsets below)
    float *cond_b = nullptr, *ada_b = nullptr, *mlp_b = nullptr, *in_b = nullptr, *norm_w = nullptr,
          *norm_b = nullptr, *fin_b = nullptr, *time_b = nullptr, *freqs = nullptr, *alpha = nullptr,
          *onorm_w = nullptr, *onorm_b = nullptr, *temb = nullptr;
    bool has_eos = false, has_embed = false, has_onorm = false;
    bool temb_ok = false;              // temb holds the embeddings of (temb_s, temb_t)
    float temb_s = 0.0f, temb_t = 0.0f;
    // scratch for max_batch rows
    uint32_t cap = 0;
    float *d_cond = nullptr, *d_y = nullptr, *d_x = nullptr, *d_sy = nullptr, *d_mod = nullptr, *d_h = nullptr,
          *d_first = nullptr, *d_noise = nullptr, *d_out = nullptr;
    int32_t* d_status = nullptr;       // [cap + 1]: per row, then the time embeddings'
    float *h_in = nullptr, *h_out = nullptr;
    int32_t* h_status = nullptr;
    // tensor-core path (head_gemm_kernel) for batches of at least tensor_min rows
    uint16_t* wn = nullptr;            // natural bf16 rows: cond + EOS (513), every adaLN row, the MLPs
    CUtensorMap tm_cond, tm_ada, tm_mlp[phonon::kHeadBlocks][2];
    uint16_t *sl_a = nullptr, *sl_h = nullptr, *sl_f = nullptr;  // [3 * cap_pad][512] bf16 slice rows
    CUtensorMap tm_sl_a, tm_sl_h, tm_sl_f;
    bool tensor_ok = false;
    uint32_t tensor_min = 32;
    // The frame step's head launches, captured into a CUDA graph once a frame
    // repeats the previous frame's shape (rows, path, caller buffers, noise
    // scale, scratch), and replayed from then on.
    struct FrameShape {
        int B = -1;
        bool tensor = false;
        const float *state = nullptr, *cond = nullptr, *x = nullptr, *x0 = nullptr;
        uint32_t scale_bits = 0;
        bool operator==(const FrameShape& o) const {
            return B == o.B && tensor == o.tensor && state == o.state && cond == o.cond && x == o.x && x0 == o.x0 &&
                   scale_bits == o.scale_bits;
        }
    };
    cudaGraphExec_t frame_graph = nullptr;
    FrameShape frame_shape, frame_last;
    uint64_t frame_graph_kernels = 0;
};

namespace {

void head_release(PhononCudaHead* h) {
    if (h->frame_graph) cudaGraphExecDestroy(h->frame_graph);
    h->frame_graph = nullptr;
    free_linear(h->cond);
    free_linear(h->ada);
    for (auto& m : h->mlp) {
        free_linear(m[0]);
        free_linear(m[1]);
    }
    for (void* p : {static_cast<void*>(h->wn), static_cast<void*>(h->sl_a), static_cast<void*>(h->sl_h),
                    static_cast<void*>(h->sl_f)})
        if (p) cudaFree(p);
    for (void* p : {static_cast<void*>(h->w16), static_cast<void*>(h->f), static_cast<void*>(h->d_cond),
                    static_cast<void*>(h->d_y), static_cast<void*>(h->d_x), static_cast<void*>(h->d_sy),
                    static_cast<void*>(h->d_mod), static_cast<void*>(h->d_h), static_cast<void*>(h->d_first),
                    static_cast<void*>(h->d_noise), static_cast<void*>(h->d_out), static_cast<void*>(h->d_status)})
        if (p) cudaFree(p);
    if (h->h_in) cudaFreeHost(h->h_in);
    if (h->h_out) cudaFreeHost(h->h_out);
    if (h->h_status) cudaFreeHost(h->h_status);
}

// bf16 bits -> float, false on a non-finite value or a missing vector.
bool head_vec(const uint16_t* bits, size_t n, float* out) {
    if (!bits) return false;
    for (size_t i = 0; i < n; ++i) {
        if (!bf16_is_finite(bits[i])) return false;
        const uint32_t u = static_cast<uint32_t>(bits[i]) << 16;
        std::memcpy(out + i, &u, 4);
    }
    return true;
}

bool head_mat(const uint16_t* bits, size_t n) {
    if (!bits) return false;
    for (size_t i = 0; i < n; ++i)
        if (!bf16_is_finite(bits[i])) return false;
    return true;
}

int head_upload(PhononCudaHead* h, const PhononCudaHeadWeights& w) {
    using namespace phonon;
    constexpr size_t W = kWidth;
    // fp32 vectors
    const size_t n_cond_b = kHeadCondLd, n_ada_b = kAdaRows, n_mlp_b = kHeadBlocks * 2 * W, n_in_b = W,
                 n_norm = kHeadBlocks * W, n_fin_b = kLatent, n_time_b = 4 * W, n_freqs = 2 * 128,
                 n_alpha = 2 * W, n_onorm = W, n_temb = 2 * W;
    std::vector<float> f(n_cond_b + n_ada_b + n_mlp_b + n_in_b + 2 * n_norm + n_fin_b + n_time_b + n_freqs +
                         n_alpha + 2 * n_onorm + n_temb, 0.0f);
    size_t o = 0;
    auto take = [&](size_t n) {
        const size_t at = o;
        o += n;
        return at;
    };
    const size_t o_cond_b = take(n_cond_b), o_ada_b = take(n_ada_b), o_mlp_b = take(n_mlp_b), o_in_b = take(n_in_b),
                 o_norm_w = take(n_norm), o_norm_b = take(n_norm), o_fin_b = take(n_fin_b), o_time_b = take(n_time_b),
                 o_freqs = take(n_freqs), o_alpha = take(n_alpha), o_onorm_w = take(n_onorm),
                 o_onorm_b = take(n_onorm), o_temb = take(n_temb);
    bool ok = head_vec(w.cond.bias, W, &f[o_cond_b]) && head_vec(w.input.bias, W, &f[o_in_b]) &&
              head_vec(w.final_out.bias, kLatent, &f[o_fin_b]) && head_vec(w.final_ada.bias, 2 * W,
                                                                           &f[o_ada_b + kHeadBlocks * kAdaBlockRows]);
    for (int b = 0; b < kHeadBlocks && ok; ++b)
        ok = head_vec(w.block_ada[b].bias, kAdaBlockRows, &f[o_ada_b + b * kAdaBlockRows]) &&
             head_vec(w.block_norm_w[b], W, &f[o_norm_w + b * W]) && head_vec(w.block_norm_b[b], W, &f[o_norm_b + b * W]) &&
             head_vec(w.block_mlp[b][0].bias, W, &f[o_mlp_b + (2 * b) * W]) &&
             head_vec(w.block_mlp[b][1].bias, W, &f[o_mlp_b + (2 * b + 1) * W]);
    for (int t = 0; t < 2 && ok; ++t)
        ok = head_vec(w.time[t][0].bias, W, &f[o_time_b + (2 * t) * W]) &&
             head_vec(w.time[t][1].bias, W, &f[o_time_b + (2 * t + 1) * W]) &&
             head_vec(w.time_freqs[t], 128, &f[o_freqs + t * 128]) && head_vec(w.time_alpha[t], W, &f[o_alpha + t * W]);
    if (!ok) return PHONON_CUDA_NON_FINITE;
    h->has_eos = w.eos.weight && w.eos.bias;
    if (h->has_eos && !head_vec(w.eos.bias, 1, &f[o_cond_b + W])) return PHONON_CUDA_NON_FINITE;
    h->has_onorm = w.out_norm_w && w.out_norm_b;
    if (h->has_onorm &&
        !(head_vec(w.out_norm_w, W, &f[o_onorm_w]) && head_vec(w.out_norm_b, W, &f[o_onorm_b])))
        return PHONON_CUDA_NON_FINITE;
    h->has_embed = w.embed != nullptr;
    // natural bf16 matrices: input [512][32], time mlp.0 [512][256] x2, time mlp.2 [512][512] x2,
    // final [32][512], embed [512][32]
    const size_t n_in = W * kLatent, n_t0 = W * 256, n_t1 = W * W, n_fin = kLatent * W, n_emb = W * kLatent;
    std::vector<uint16_t> m16(n_in + 2 * n_t0 + 2 * n_t1 + n_fin + n_emb, 0);
    if (!head_mat(w.input.weight, n_in) || !head_mat(w.final_out.weight, n_fin)) return PHONON_CUDA_NON_FINITE;
    std::memcpy(&m16[0], w.input.weight, n_in * 2);
    for (int t = 0; t < 2; ++t) {
        if (!head_mat(w.time[t][0].weight, n_t0) || !head_mat(w.time[t][1].weight, n_t1)) return PHONON_CUDA_NON_FINITE;
        std::memcpy(&m16[n_in + t * n_t0], w.time[t][0].weight, n_t0 * 2);
        std::memcpy(&m16[n_in + 2 * n_t0 + t * n_t1], w.time[t][1].weight, n_t1 * 2);
    }
    std::memcpy(&m16[n_in + 2 * n_t0 + 2 * n_t1], w.final_out.weight, n_fin * 2);
    if (h->has_embed) {
        if (!head_mat(w.embed, n_emb)) return PHONON_CUDA_NON_FINITE;
        std::memcpy(&m16[n_in + 2 * n_t0 + 2 * n_t1 + n_fin], w.embed, n_emb * 2);
    }
    // GEMV matrices: cond (+ EOS row), all modulation rows, the MLPs
    std::vector<uint16_t> cond((W + 1) * W, 0);
    if (!w.cond.weight) return PHONON_CUDA_NON_FINITE;
    std::memcpy(cond.data(), w.cond.weight, W * W * 2);
    if (h->has_eos) std::memcpy(&cond[W * W], w.eos.weight, W * 2);
    std::vector<uint16_t> ada(static_cast<size_t>(kAdaRows) * W);
    for (int b = 0; b < kHeadBlocks; ++b) {
        if (!w.block_ada[b].weight) return PHONON_CUDA_NON_FINITE;
        std::memcpy(&ada[static_cast<size_t>(b) * kAdaBlockRows * W], w.block_ada[b].weight, kAdaBlockRows * W * 2);
    }
    if (!w.final_ada.weight) return PHONON_CUDA_NON_FINITE;
    std::memcpy(&ada[static_cast<size_t>(kHeadBlocks) * kAdaBlockRows * W], w.final_ada.weight, 2 * W * W * 2);
    int st;
    if ((st = upload_linear(PHONON_CUDA_LINEAR_BF16, cond.data(), W + 1, W, &h->cond)) ||
        (st = upload_linear(PHONON_CUDA_LINEAR_BF16, ada.data(), kAdaRows, W, &h->ada)))
        return st;
    for (int b = 0; b < kHeadBlocks; ++b)
        for (int j = 0; j < 2; ++j) {
            if (!w.block_mlp[b][j].weight) return PHONON_CUDA_NON_FINITE;
            if ((st = upload_linear(PHONON_CUDA_LINEAR_BF16, w.block_mlp[b][j].weight, W, W, &h->mlp[b][j]))) return st;
        }
    // natural bf16 copies for the tensor-core path: [cond + EOS | adaLN rows | MLPs], 128-row TMA boxes
    const size_t rows_n = (W + 1) + static_cast<size_t>(kAdaRows) + kHeadBlocks * 2 * W;
    if (cudaMalloc(&h->wn, rows_n * W * 2) != cudaSuccess) return PHONON_CUDA_OUT_OF_MEMORY;
    CUDA_TRY(cudaMemcpy(h->wn, cond.data(), (W + 1) * W * 2, cudaMemcpyHostToDevice));
    uint16_t* wn_ada = h->wn + (W + 1) * W;
    CUDA_TRY(cudaMemcpy(wn_ada, ada.data(), ada.size() * 2, cudaMemcpyHostToDevice));
    uint16_t* wn_mlp = wn_ada + static_cast<size_t>(kAdaRows) * W;
    for (int b = 0; b < kHeadBlocks; ++b)
        for (int j = 0; j < 2; ++j)
            CUDA_TRY(cudaMemcpy(wn_mlp + (2 * b + j) * W * W, w.block_mlp[b][j].weight, W * W * 2, cudaMemcpyHostToDevice));
    // (the TMA alignment rules hold by construction: 1 KB rows, 16-byte aligned bases)
    bool maps = make_map_2d(&h->tm_cond, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, h->wn, W + 1, W, W * 2, kHgKTile, kHgM) &&
                make_map_2d(&h->tm_ada, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, wn_ada, kAdaRows, W, W * 2, kHgKTile, kHgM);
    for (int b = 0; b < kHeadBlocks && maps; ++b)
        for (int j = 0; j < 2 && maps; ++j)
            maps = make_map_2d(&h->tm_mlp[b][j], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, wn_mlp + (2 * b + j) * W * W, W, W,
                               W * 2, kHgKTile, kHgM);
    h->tensor_ok = maps;
    if (cudaMalloc(&h->w16, m16.size() * 2) != cudaSuccess || cudaMalloc(&h->f, f.size() * 4) != cudaSuccess)
        return PHONON_CUDA_OUT_OF_MEMORY;
    CUDA_TRY(cudaMemcpy(h->w16, m16.data(), m16.size() * 2, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(h->f, f.data(), f.size() * 4, cudaMemcpyHostToDevice));
    h->in_w = h->w16;
    for (int t = 0; t < 2; ++t) {
        h->time_w[t][0] = h->w16 + n_in + t * n_t0;
        h->time_w[t][1] = h->w16 + n_in + 2 * n_t0 + t * n_t1;
    }
    h->fin_w = h->w16 + n_in + 2 * n_t0 + 2 * n_t1;
    h->embed_w = h->has_embed ? h->fin_w + n_fin : nullptr;
    h->cond_b = h->f + o_cond_b;
    h->ada_b = h->f + o_ada_b;
    h->mlp_b = h->f + o_mlp_b;
    h->in_b = h->f + o_in_b;
    h->norm_w = h->f + o_norm_w;
    h->norm_b = h->f + o_norm_b;
    h->fin_b = h->f + o_fin_b;
    h->time_b = h->f + o_time_b;
    h->freqs = h->f + o_freqs;
    h->alpha = h->f + o_alpha;
    h->onorm_w = h->f + o_onorm_w;
    h->onorm_b = h->f + o_onorm_b;
    h->temb = h->f + o_temb;
    return PHONON_CUDA_OK;
}

int head_alloc(PhononCudaHead* h, uint32_t cap) {
    using namespace phonon;
    const size_t B = cap;
    h->cap = cap;
    if (cudaMalloc(&h->d_cond, B * kWidth * 4) != cudaSuccess || cudaMalloc(&h->d_y, B * kHeadCondLd * 4) != cudaSuccess ||
        cudaMalloc(&h->d_x, B * kWidth * 4) != cudaSuccess || cudaMalloc(&h->d_sy, B * kWidth * 4) != cudaSuccess ||
        cudaMalloc(&h->d_mod, B * kAdaRows * 4) != cudaSuccess || cudaMalloc(&h->d_h, B * kWidth * 4) != cudaSuccess ||
        cudaMalloc(&h->d_first, B * kWidth * 4) != cudaSuccess || cudaMalloc(&h->d_noise, B * kLatent * 4) != cudaSuccess ||
        cudaMalloc(&h->d_out, B * kLatent * 4) != cudaSuccess || cudaMalloc(&h->d_status, (B + 1) * 4) != cudaSuccess ||
        cudaMallocHost(&h->h_in, B * (kWidth + kLatent) * 4) != cudaSuccess ||
        cudaMallocHost(&h->h_out, B * (kLatent + 1) * 4) != cudaSuccess ||
        cudaMallocHost(&h->h_status, (B + 1) * 4) != cudaSuccess)
        return PHONON_CUDA_OUT_OF_MEMORY;
    const size_t slice_rows = 3 * ((B + kHgStreams - 1) / kHgStreams * kHgStreams);
    for (uint16_t** sl : {&h->sl_a, &h->sl_h, &h->sl_f}) {
        if (cudaMalloc(sl, slice_rows * kWidth * 2) != cudaSuccess) return PHONON_CUDA_OUT_OF_MEMORY;
        CUDA_TRY(cudaMemset(*sl, 0, slice_rows * kWidth * 2));
    }
    h->tensor_ok = h->tensor_ok &&
                   make_map_2d(&h->tm_sl_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, h->sl_a, slice_rows, kWidth, kWidth * 2,
                               kHgKTile, kHgN) &&
                   make_map_2d(&h->tm_sl_h, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, h->sl_h, slice_rows, kWidth, kWidth * 2,
                               kHgKTile, kHgN) &&
                   make_map_2d(&h->tm_sl_f, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, h->sl_f, slice_rows, kWidth, kWidth * 2,
                               kHgKTile, kHgN);
    return PHONON_CUDA_OK;
}

// A bf16 x three-slice linear (head_gemm_kernel) of `rows` outputs for B
// activation rows, on stream s; status and error words in p.
template <int kEpi, int kK = kHgK>
cudaError_t launch_bf16x3_gemm(const CUtensorMap& tw, const CUtensorMap& tx, int rows, int B, HeadGemmParams p,
                               cudaStream_t s) {
    static std::atomic<uint64_t> configured{0};
    const cudaError_t e = opt_in_smem(reinterpret_cast<const void*>(head_gemm_kernel<kEpi, kK>), kHgSmem, configured);
    if (e != cudaSuccess) return e;
    p.rows = rows;
    p.B = B;
    const dim3 grid((rows + kHgM - 1) / kHgM, (B + kHgStreams - 1) / kHgStreams);
    return launch_pdl(head_gemm_kernel<kEpi, kK>, grid, dim3(kHgThreads), kHgSmem, s, tw, tx, p);
}

template <int kEpi>
cudaError_t launch_head_gemm(PhononCudaHead* h, const CUtensorMap& tw, const CUtensorMap& tx, int rows, int B,
                             HeadGemmParams p) {
    p.status = h->d_status;
    p.error = h->c->d_err;
    return launch_bf16x3_gemm<kEpi>(tw, tx, rows, B, p, h->c->stream);
}

bool head_tensor(const PhononCudaHead* h, int B) {
    return h->tensor_ok && static_cast<uint32_t>(B) >= h->tensor_min;
}

// cond_embed (and the EOS row) of B condition rows at x_dev: h->d_y [B][520].
int enqueue_head_cond(PhononCudaHead* h, int B, const float* x_dev) {
    using namespace phonon;
    PhononCuda* c = h->c;
    GemvParams p{};
    p.w = h->cond.plane;
    p.rows = kWidth + 1;
    p.cols = kWidth;
    p.x = x_dev;
    p.ldx = kWidth;
    p.B = B;
    p.bias = h->cond_b;
    p.y = h->d_y;
    p.ldy = kHeadCondLd;
    p.status = h->d_status;
    if (head_tensor(h, B)) {
        {
            LaunchScope ls(c, PHONON_CUDA_K_HEAD, B * kWidth * 10.0);
            CUDA_TRY(launch_pdl(slice_rows_kernel, dim3(B), dim3(128), 0, c->stream, x_dev, static_cast<int>(kWidth), B,
                                h->sl_a));
        }
        HeadGemmParams g{};
        g.bias = h->cond_b;
        g.y = h->d_y;
        g.ldy = kHeadCondLd;
        LaunchScope ls(c, PHONON_CUDA_K_HEAD, (kWidth + 1) * kWidth * 2.0 + B * (3 * kWidth * 2.0 + (kWidth + 1) * 4.0));
        CUDA_TRY(launch_head_gemm<HG_STORE>(h, h->tm_cond, h->tm_sl_a, kWidth + 1, B, g));
        return PHONON_CUDA_OK;
    }
    LaunchScope ls(c, PHONON_CUDA_K_HEAD, (kWidth + 1) * kWidth * 2.0 + B * (kWidth + kWidth + 1) * 4.0);
    CUDA_TRY((launch_gemv_bt<false, 1, SRC_X, EPI_STORE>(p, c->stream)));
    return PHONON_CUDA_OK;
}

// The time embeddings of (s, t), unless temb holds them already.
int enqueue_head_time(PhononCudaHead* h, float s, float t) {
    using namespace phonon;
    if (h->temb_ok && h->temb_s == s && h->temb_t == t) return PHONON_CUDA_OK;
    PhononCuda* c = h->c;
    for (int k = 0; k < 2; ++k) {
        LaunchScope ls(c, PHONON_CUDA_K_HEAD, (kWidth * 256 + kWidth * kWidth) * 2.0);
        head_time_kernel<<<1, 512, 0, c->stream>>>(k == 0 ? s : t, h->freqs + k * 128, h->time_w[k][0],
                                                   h->time_b + (2 * k) * kWidth, h->time_w[k][1],
                                                   h->time_b + (2 * k + 1) * kWidth, h->alpha + k * kWidth,
                                                   h->temb + k * kWidth, h->d_status + h->cap);
        CUDA_TRY(cudaGetLastError());
    }
    h->temb_ok = true;  // withdrawn by the caller if the status word reports a non-finite embedding
    h->temb_s = s;
    h->temb_t = t;
    return PHONON_CUDA_OK;
}

// The head for B rows: conditions at x_dev (the cond GEMV's input, already
// enqueued by the caller through enqueue_head_cond), latents or raw noise
// in h->d_noise; the result goes to h->d_out. With embed_out, also the
// next input rows input_linear(result) + condition_rows.
int enqueue_head(PhononCudaHead* h, int B, bool lsd, float scale, float s, float t, float* embed_out,
                 const float* condition_rows) {
    using namespace phonon;
    PhononCuda* c = h->c;
    cudaStream_t st = c->stream;
    const bool tensor = head_tensor(h, B);
    if (int e = enqueue_head_time(h, s, t)) return e;
    {
        HeadInParams q{};
        q.noise = h->d_noise;
        q.noise_scale = scale;
        q.scaled = lsd ? 1 : 0;
        q.in_w = h->in_w;
        q.in_b = h->in_b;
        q.cond = h->d_y;
        q.ldc = kHeadCondLd;
        q.temb = h->temb;
        q.x = h->d_x;
        q.silu_y = h->d_sy;
        q.sy_slices = tensor ? h->sl_a : nullptr;
        q.B = B;
        q.status = h->d_status;
        LaunchScope ls(c, PHONON_CUDA_K_HEAD, kWidth * kLatent * 2.0 + B * kWidth * 12.0);
        CUDA_TRY(launch_pdl(head_in_kernel, dim3((B + kHeadInStreams - 1) / kHeadInStreams), dim3(512), 0, st, q));
    }
    if (tensor) {
        HeadGemmParams g{};
        g.bias = h->ada_b;
        g.y = h->d_mod;
        g.ldy = kAdaRows;
        LaunchScope ls(c, PHONON_CUDA_K_HEAD, kAdaRows * kWidth * 2.0 + B * (3 * kWidth * 2.0 + kAdaRows * 4.0));
        CUDA_TRY(launch_head_gemm<HG_STORE>(h, h->tm_ada, h->tm_sl_a, kAdaRows, B, g));
    } else {
        GemvParams p{};
        p.w = h->ada.plane;
        p.rows = kAdaRows;
        p.cols = kWidth;
        p.x = h->d_sy;
        p.ldx = kWidth;
        p.B = B;
        p.bias = h->ada_b;
        p.y = h->d_mod;
        p.ldy = kAdaRows;
        p.status = h->d_status;
        LaunchScope ls(c, PHONON_CUDA_K_HEAD, kAdaRows * kWidth * 2.0 + B * (kWidth + kAdaRows) * 4.0);
        CUDA_TRY((launch_gemv_bt<false, 1, SRC_X, EPI_STORE>(p, st)));
    }
    for (int blk = 0; blk < kHeadBlocks; ++blk) {
        if (tensor) {
            {
                LaunchScope ls(c, PHONON_CUDA_K_HEAD, B * kWidth * 16.0);
                CUDA_TRY(launch_pdl(head_block_kernel, dim3((B + 7) / 8), dim3(256), 0, st,
                                    static_cast<const float*>(h->d_x), static_cast<const float*>(h->d_mod), blk,
                                    static_cast<const float*>(h->norm_w + blk * kWidth),
                                    static_cast<const float*>(h->norm_b + blk * kWidth), h->d_h, B, h->d_status,
                                    h->sl_h));
            }
            HeadGemmParams g{};
            g.bias = h->mlp_b + (2 * blk) * kWidth;
            g.slices = h->sl_f;
            g.slice_ld = kWidth;
            {
                LaunchScope ls(c, PHONON_CUDA_K_HEAD, kWidth * kWidth * 2.0 + B * 12.0 * kWidth);
                CUDA_TRY(launch_head_gemm<HG_SILU>(h, h->tm_mlp[blk][0], h->tm_sl_h, kWidth, B, g));
            }
            g = HeadGemmParams{};
            g.bias = h->mlp_b + (2 * blk + 1) * kWidth;
            g.y = h->d_x;
            g.ldy = kWidth;
            g.gate = h->d_mod + static_cast<size_t>(blk) * kAdaBlockRows + 2 * kWidth;
            g.ldgate = kAdaRows;
            LaunchScope ls(c, PHONON_CUDA_K_HEAD, kWidth * kWidth * 2.0 + B * 18.0 * kWidth);
            CUDA_TRY(launch_head_gemm<HG_GATE>(h, h->tm_mlp[blk][1], h->tm_sl_f, kWidth, B, g));
            continue;
        }
        // the block LayerNorm + modulation in the first MLP GEMV's prologue
        // (SRC_HEADLN), in place of a head_block_kernel launch
        GemvParams p{};
        p.rows = kWidth;
        p.cols = kWidth;
        p.ldx = kWidth;
        p.B = B;
        p.ldy = kWidth;
        p.status = h->d_status;
        p.w = h->mlp[blk][0].plane;
        p.x = h->d_x;
        p.ln_w = h->norm_w + blk * kWidth;
        p.ln_b = h->norm_b + blk * kWidth;
        p.mod = h->d_mod + static_cast<size_t>(blk) * kAdaBlockRows;
        p.ldmod = kAdaRows;
        p.bias = h->mlp_b + (2 * blk) * kWidth;
        p.y = h->d_first;
        {
            LaunchScope ls(c, PHONON_CUDA_K_HEAD, kWidth * kWidth * 2.0 + B * kWidth * 24.0);
            CUDA_TRY((launch_gemv_bt<false, 1, SRC_HEADLN, EPI_SILU>(p, st)));
        }
        p.w = h->mlp[blk][1].plane;
        p.x = h->d_first;
        p.bias = h->mlp_b + (2 * blk + 1) * kWidth;
        p.y = h->d_x;
        p.res = h->d_x;
        p.ldres = kWidth;
        p.gate = h->d_mod + static_cast<size_t>(blk) * kAdaBlockRows + 2 * kWidth;
        p.ldgate = kAdaRows;
        {
            LaunchScope ls(c, PHONON_CUDA_K_HEAD, kWidth * kWidth * 2.0 + B * kWidth * 16.0);
            CUDA_TRY((launch_gemv_bt<false, 1, SRC_X, EPI_GATE>(p, st)));
        }
    }
    HeadFinalParams f{};
    f.x = h->d_x;
    f.mod = h->d_mod;
    f.fin_w = h->fin_w;
    f.fin_b = h->fin_b;
    f.noise = h->d_noise;
    f.noise_scale = scale;
    f.scaled = lsd ? 1 : 0;
    f.out = h->d_out;
    f.embed_w = embed_out ? h->embed_w : nullptr;
    f.condition = condition_rows;
    f.embed_out = embed_out;
    f.B = B;
    f.status = h->d_status;
    LaunchScope ls(c, PHONON_CUDA_K_HEAD, kLatent * kWidth * 2.0 + B * kWidth * 12.0);
    CUDA_TRY(launch_pdl(head_final_kernel, dim3(B), dim3(256), 0, st, f));
    return PHONON_CUDA_OK;
}

// The frame step's head: the cond GEMV from the state rows, then the LSD
// step (s, t) = (0, 1) with the embedding of the new latent into c->d_x0.
// From the second frame of a repeated shape on, one captured graph (the
// head is ~23 dependent launches at one stream, launch-bound); the time
// embeddings are computed before, outside the graph (they change only with
// (s, t)). Profiling and layer tracing launch directly.
int enqueue_head_frame(PhononCudaHead* h, int B, const float* state_dev, float scale, const float* cond_dev) {
    PhononCuda* c = h->c;
    if (int e = enqueue_head_time(h, 0.0f, 1.0f)) return e;
    auto direct = [&]() {
        int e = enqueue_head_cond(h, B, state_dev);
        return e ? e : enqueue_head(h, B, true, scale, 0.0f, 1.0f, c->d_x0, cond_dev);
    };
    if (c->prof_on || c->tracing) return direct();
    uint32_t bits = 0;
    std::memcpy(&bits, &scale, 4);
    PhononCudaHead::FrameShape shape;
    shape.B = B;
    shape.tensor = head_tensor(h, B);
    shape.state = state_dev;
    shape.cond = cond_dev;
    shape.x = h->d_x;
    shape.x0 = c->d_x0;
    shape.scale_bits = bits;
    if (h->frame_graph && h->frame_shape == shape) {
        CUDA_TRY(cudaGraphLaunch(h->frame_graph, c->stream));
        c->launches += h->frame_graph_kernels;
        return PHONON_CUDA_OK;
    }
    if (!(h->frame_last == shape)) {
        h->frame_last = shape;
        return direct();
    }
    cudaGraph_t g = nullptr;
    const uint64_t before = c->launches;
    if (cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        cudaGetLastError();
        return direct();
    }
    const int st = direct();
    const cudaError_t end = cudaStreamEndCapture(c->stream, &g);
    cudaGraphExec_t exec = nullptr;
    if (st != PHONON_CUDA_OK || end != cudaSuccess || !g || cudaGraphInstantiate(&exec, g, 0) != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        c->launches = before;
        return direct();
    }
    cudaGraphDestroy(g);
    if (h->frame_graph) cudaGraphExecDestroy(h->frame_graph);
    h->frame_graph = exec;
    h->frame_shape = shape;
    h->frame_graph_kernels = c->launches - before;
    c->launches = before;
    CUDA_TRY(cudaGraphLaunch(h->frame_graph, c->stream));
    c->launches += h->frame_graph_kernels;
    return PHONON_CUDA_OK;
}

// Wait for the head's work, read its row statuses (and the time embeddings'
// word, which fails every row); false if any row failed.
int head_finish(PhononCudaHead* h, uint32_t B, bool* any_bad) {
    PhononCuda* c = h->c;
    CUDA_TRY(cudaMemcpyAsync(h->h_status, h->d_status, B * 4, cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaMemcpyAsync(h->h_status + h->cap, h->d_status + h->cap, 4, cudaMemcpyDeviceToHost, c->stream));
    int st = finish_sync(c, 0);
    if (st) return st;
    if (h->h_status[h->cap]) {
        h->temb_ok = false;
        cudaMemsetAsync(h->d_status + h->cap, 0, 4, c->stream);
        for (uint32_t i = 0; i < B; ++i) h->h_status[i] |= PHONON_CUDA_NON_FINITE;
    }
    *any_bad = false;
    for (uint32_t i = 0; i < B; ++i)
        if (h->h_status[i]) *any_bad = true;
    return PHONON_CUDA_OK;
}

int head_begin(PhononCudaHead* h, uint32_t batch) {
    if (!h || batch < 1 || batch > h->cap) return PHONON_CUDA_INVALID_ARGUMENT;
    if (h->c->pending) return PHONON_CUDA_INVALID_ARGUMENT;
    int st = set_device(h->c->cfg.device);
    if (st) return st;
    CUDA_TRY(cudaMemsetAsync(h->d_status, 0, batch * 4, h->c->stream));
    return PHONON_CUDA_OK;
}

// Host rows -> device through the pinned staging buffer (at float offset
// `at`: condition rows at 0, latent rows after max_batch condition rows).
int head_upload_rows(PhononCudaHead* h, float* dst, const float* src, size_t floats, size_t at = 0) {
    std::memcpy(h->h_in + at, src, floats * 4);
    CUDA_TRY(cudaMemcpyAsync(dst, h->h_in + at, floats * 4, cudaMemcpyHostToDevice, h->c->stream));
    return PHONON_CUDA_OK;
}

int head_run_host(PhononCudaHead* h, uint32_t batch, const float* condition, const float* latent, bool lsd, float scale,
                  float s, float t, float* out) {
    std::lock_guard<std::mutex> g(h->c->mu);
    int st = head_begin(h, batch);
    if (st) return st;
    const int B = static_cast<int>(batch);
    if ((st = head_upload_rows(h, h->d_cond, condition, static_cast<size_t>(B) * phonon::kWidth)) ||
        (st = head_upload_rows(h, h->d_noise, latent, static_cast<size_t>(B) * phonon::kLatent,
                               static_cast<size_t>(h->cap) * phonon::kWidth)))
        return st;
    if ((st = enqueue_head_cond(h, B, h->d_cond))) return st;
    if ((st = enqueue_head(h, B, lsd, scale, s, t, nullptr, nullptr))) return st;
    CUDA_TRY(cudaMemcpyAsync(h->h_out, h->d_out, static_cast<size_t>(B) * phonon::kLatent * 4, cudaMemcpyDeviceToHost,
                             h->c->stream));
    bool bad = false;
    if ((st = head_finish(h, batch, &bad))) return st;
    if (bad) return PHONON_CUDA_NON_FINITE;
    std::memcpy(out, h->h_out, static_cast<size_t>(B) * phonon::kLatent * 4);
    return PHONON_CUDA_OK;
}

}  // namespace

extern "C" {

int phonon_cuda_head_create(PhononCuda* c, const PhononCudaHeadWeights* w, PhononCudaHead** out) {
    if (!c || !w || !out) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(c->mu);
    int st = set_device(c->cfg.device);
    if (st) return st;
    PhononCudaHead* h = new (std::nothrow) PhononCudaHead;
    if (!h) return PHONON_CUDA_OUT_OF_MEMORY;
    h->c = c;
    if ((st = head_upload(h, *w)) || (st = head_alloc(h, c->cfg.max_batch))) {
        head_release(h);
        delete h;
        return st;
    }
    CUDA_TRY(cudaMemset(h->d_status, 0, (h->cap + 1) * 4));
    *out = h;
    return PHONON_CUDA_OK;
}

void phonon_cuda_head_free(PhononCudaHead* h) {
    if (!h) return;
    {
        std::lock_guard<std::mutex> g(h->c->mu);
        set_device(h->c->cfg.device);
        cudaStreamSynchronize(h->c->stream);
        head_release(h);
    }
    delete h;
}

int phonon_cuda_head_set_tensor_min(PhononCudaHead* h, uint32_t min_batch, int* available) {
    if (!h) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(h->c->mu);
    h->tensor_min = min_batch;
    if (available) *available = h->tensor_ok ? 1 : 0;
    return PHONON_CUDA_OK;
}

int phonon_cuda_head_forward(PhononCudaHead* h, uint32_t batch, const float* condition, const float* state, float s,
                             float t, float* velocity) {
    if (!h || !condition || !state || !velocity) return PHONON_CUDA_INVALID_ARGUMENT;
    if (!std::isfinite(s) || !std::isfinite(t)) return PHONON_CUDA_NON_FINITE;
    return head_run_host(h, batch, condition, state, false, 1.0f, s, t, velocity);
}

int phonon_cuda_lsd_one_step(PhononCudaHead* h, uint32_t batch, const float* condition, const float* raw_noise,
                             float temperature, float* output) {
    if (!h || !condition || !raw_noise || !output) return PHONON_CUDA_INVALID_ARGUMENT;
    if (!std::isfinite(temperature) || !(temperature > 0.0f)) return PHONON_CUDA_INVALID_ARGUMENT;
    return head_run_host(h, batch, condition, raw_noise, true, std::sqrt(temperature), 0.0f, 1.0f, output);
}

int phonon_cuda_eos_logit(PhononCudaHead* h, uint32_t batch, const float* state, float* logit) {
    if (!h || !state || !logit) return PHONON_CUDA_INVALID_ARGUMENT;
    if (!h->has_eos) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(h->c->mu);
    int st = head_begin(h, batch);
    if (st) return st;
    if ((st = head_upload_rows(h, h->d_cond, state, static_cast<size_t>(batch) * phonon::kWidth))) return st;
    if ((st = enqueue_head_cond(h, static_cast<int>(batch), h->d_cond))) return st;
    CUDA_TRY(cudaMemcpy2DAsync(h->h_out, 4, h->d_y + phonon::kWidth, phonon::kHeadCondLd * 4, 4, batch,
                               cudaMemcpyDeviceToHost, h->c->stream));
    bool bad = false;
    if ((st = head_finish(h, batch, &bad))) return st;
    if (bad) return PHONON_CUDA_NON_FINITE;
    std::memcpy(logit, h->h_out, batch * 4);
    return PHONON_CUDA_OK;
}

int phonon_cuda_output_norm_device(PhononCudaHead* h, uint32_t batch, const float* x_dev, float* out_dev) {
    if (!h || !x_dev || !out_dev || !h->has_onorm) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(h->c->mu);
    int st = head_begin(h, batch);
    if (st) return st;
    {
        LaunchScope ls(h->c, PHONON_CUDA_K_HEAD, batch * phonon::kWidth * 8.0);
        CUDA_TRY(launch_pdl(output_norm_kernel, dim3((batch + 7) / 8), dim3(256), 0, h->c->stream, x_dev,
                            static_cast<const float*>(h->onorm_w), static_cast<const float*>(h->onorm_b), out_dev,
                            static_cast<int>(batch), h->d_status));
    }
    bool bad = false;
    if ((st = head_finish(h, batch, &bad))) return st;
    return bad ? PHONON_CUDA_NON_FINITE : PHONON_CUDA_OK;
}

int phonon_cuda_frame_step(PhononCudaHead* h, uint32_t batch, const uint32_t* streams, const uint32_t* positions,
                           float* state_dev, const float* condition_dev, const float* raw_noise, float temperature,
                           float* eos_logit, float* latent, int32_t* status) {
    if (!h || !state_dev || !condition_dev || !raw_noise || !eos_logit || !latent || !status)
        return PHONON_CUDA_INVALID_ARGUMENT;
    if (!h->has_eos || !h->has_embed || !h->has_onorm) return PHONON_CUDA_INVALID_ARGUMENT;
    if (!std::isfinite(temperature) || !(temperature > 0.0f)) return PHONON_CUDA_INVALID_ARGUMENT;
    PhononCuda* c = h->c;
    std::lock_guard<std::mutex> g(c->mu);
    int st = head_begin(h, batch);
    if (st) return st;
    std::vector<int32_t> slot, pos, updates;
    PageUndo undo{c, {}};
    if ((st = prepare_decode(c, batch, streams, positions, slot, pos, updates, undo, true))) return st;
    const int B = static_cast<int>(batch);
    if ((st = head_upload_rows(h, h->d_noise, raw_noise, static_cast<size_t>(B) * phonon::kLatent))) return st;
    bool cancelled = false;
    if ((st = enqueue_head_frame(h, B, state_dev, std::sqrt(temperature), condition_dev))) {
        undo.rollback();
        return st;
    }
    // A memset between the head and the step: the step's first kernels were
    // written to follow a copy, and this ordering point keeps any of them
    // that read their input before griddepcontrol.wait after the head's end.
    CUDA_TRY(cudaMemsetAsync(c->d_status, 0, batch * 4, c->stream));
    if ((st = enqueue_decode(c, slot, pos, updates, c->d_x0, c->d_y, nullptr, nullptr, &cancelled))) {
        undo.rollback();
        return st;
    }
    {
        LaunchScope ls(c, PHONON_CUDA_K_HEAD, B * phonon::kWidth * 8.0);
        CUDA_TRY(launch_pdl(output_norm_kernel, dim3((B + 7) / 8), dim3(256), 0, c->stream,
                            static_cast<const float*>(c->d_y), static_cast<const float*>(h->onorm_w),
                            static_cast<const float*>(h->onorm_b), state_dev, B, h->d_status));
    }
    CUDA_TRY(cudaMemcpyAsync(h->h_out, h->d_out, static_cast<size_t>(B) * phonon::kLatent * 4, cudaMemcpyDeviceToHost,
                             c->stream));
    CUDA_TRY(cudaMemcpy2DAsync(h->h_out + static_cast<size_t>(B) * phonon::kLatent, 4, h->d_y + phonon::kWidth,
                               phonon::kHeadCondLd * 4, 4, batch, cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaMemcpyAsync(c->h_status, c->d_status, batch * 4, cudaMemcpyDeviceToHost, c->stream));
    bool bad = false;
    if ((st = head_finish(h, batch, &bad))) return st;
    for (uint32_t i = 0; i < batch; ++i) {
        int32_t s = c->h_status[i] ? c->h_status[i] : PHONON_CUDA_OK;
        if (h->h_status[i]) s = PHONON_CUDA_NON_FINITE;
        status[i] = s;
        if (s != PHONON_CUDA_OK) continue;
        c->streams[streams[i]].length++;
        std::memcpy(latent + static_cast<size_t>(i) * phonon::kLatent,
                    h->h_out + static_cast<size_t>(i) * phonon::kLatent, phonon::kLatent * 4);
        eos_logit[i] = h->h_out[static_cast<size_t>(B) * phonon::kLatent + i];
    }
    return PHONON_CUDA_OK;
}

}  // extern "C"

// ------------------------------------------------------------------ Mimi
// The Mimi latent transformer (phonon_mimi.cuh): weights, per-request ring
// states and a step of one frame for a batch of states, on its own stream.
struct PhononCudaMimi {
    int device = 0;
    std::mutex mu;
    cudaStream_t stream = nullptr;
    uint32_t max_states = 0, max_batch = 0;
    DevLinear in_proj[phonon::kMimiLayers], out_proj[phonon::kMimiLayers], linear1[phonon::kMimiLayers],
        linear2[phonon::kMimiLayers];
    uint16_t* w16 = nullptr;   // projection [512][32], upsample [512][32]
    float* vec = nullptr;      // per layer: norm1 w, b, norm2 w, b, scale1, scale2 [512]; zeros [512]; freq [32]
    float* rings = nullptr;    // [state][layer][k|v][272][512]
    float* previous = nullptr; // [state][512]
    // scratch for max_batch states (16 rows each)
    float *d_lat = nullptr, *d_hidden = nullptr, *d_norm = nullptr, *d_qkv = nullptr, *d_att = nullptr,
          *d_mlp = nullptr;
    int32_t *d_meta = nullptr, *d_status = nullptr;  // meta: slots [max_batch], positions [max_batch]
    float *h_lat = nullptr, *h_out = nullptr;
    int32_t *h_meta = nullptr, *h_status = nullptr;
    // tensor-core linears (head_gemm_kernel) for steps of at least tensor_min states
    uint16_t* wn = nullptr;                       // natural bf16 copies of the eight matrices
    CUtensorMap tm_w[phonon::kMimiLayers][4];     // in_proj, out_proj, linear1, linear2
    uint16_t *sl_a = nullptr, *sl_g = nullptr;    // slice rows [3 * rows_pad][512], [3 * rows_pad][2048]
    CUtensorMap tm_sl_a, tm_sl_g;
    int32_t* d_err = nullptr;                     // bounded-wait expiry of the tensor-core linears
    bool tensor_ok = false;
    uint32_t tensor_min = 4;
    struct State {
        bool used = false, failed = false;
        uint64_t position = 0;
    };
    std::vector<State> states;
    // A step's launches depend on the batch size and the path alone: once a
    // step repeats the previous one's (n, path) they are captured into a CUDA
    // graph and replayed (one state: ~20 dependent launches per frame).
    cudaGraphExec_t graph = nullptr;
    int graph_n = -1, last_n = -1;
    bool graph_tensor = false, last_tensor = false;
};

namespace {

constexpr int kMimiVecPerLayer = 6;

void mimi_release(PhononCudaMimi* m) {
    if (m->graph) cudaGraphExecDestroy(m->graph);
    m->graph = nullptr;
    for (int l = 0; l < phonon::kMimiLayers; ++l) {
        free_linear(m->in_proj[l]);
        free_linear(m->out_proj[l]);
        free_linear(m->linear1[l]);
        free_linear(m->linear2[l]);
    }
    for (void* p : {static_cast<void*>(m->wn), static_cast<void*>(m->sl_a), static_cast<void*>(m->sl_g),
                    static_cast<void*>(m->d_err)})
        if (p) cudaFree(p);
    for (void* p : {static_cast<void*>(m->w16), static_cast<void*>(m->vec), static_cast<void*>(m->rings),
                    static_cast<void*>(m->previous), static_cast<void*>(m->d_lat), static_cast<void*>(m->d_hidden),
                    static_cast<void*>(m->d_norm), static_cast<void*>(m->d_qkv), static_cast<void*>(m->d_att),
                    static_cast<void*>(m->d_mlp), static_cast<void*>(m->d_meta), static_cast<void*>(m->d_status)})
        if (p) cudaFree(p);
    for (void* p : {static_cast<void*>(m->h_lat), static_cast<void*>(m->h_out), static_cast<void*>(m->h_meta),
                    static_cast<void*>(m->h_status)})
        if (p) cudaFreeHost(p);
    if (m->stream) cudaStreamDestroy(m->stream);
}

int mimi_setup(PhononCudaMimi* m, const PhononCudaMimiWeights& w) {
    using namespace phonon;
    constexpr size_t W = kWidth;
    // vectors
    std::vector<float> v(kMimiLayers * kMimiVecPerLayer * W + kFfn + 32, 0.0f);  // vectors, zeros [2048], freq [32]
    for (int l = 0; l < kMimiLayers; ++l) {
        const uint16_t* src[kMimiVecPerLayer] = {w.norm1_w[l], w.norm1_b[l], w.norm2_w[l],
                                                 w.norm2_b[l], w.scale1[l],  w.scale2[l]};
        for (int k = 0; k < kMimiVecPerLayer; ++k)
            if (!head_vec(src[k], W, &v[(l * kMimiVecPerLayer + k) * W])) return PHONON_CUDA_NON_FINITE;
    }
    rope_frequencies(10000.0f, kHeadDim, &v[kMimiLayers * kMimiVecPerLayer * W + kFfn]);
    // natural bf16 projection and upsample kernel
    if (!head_mat(w.projection, W * 32) || !head_mat(w.upsample, W * 32)) return PHONON_CUDA_NON_FINITE;
    CUDA_TRY(cudaMalloc(&m->w16, 2 * W * 32 * 2));
    CUDA_TRY(cudaMemcpy(m->w16, w.projection, W * 32 * 2, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(m->w16 + W * 32, w.upsample, W * 32 * 2, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMalloc(&m->vec, v.size() * 4));
    CUDA_TRY(cudaMemcpy(m->vec, v.data(), v.size() * 4, cudaMemcpyHostToDevice));
    int st;
    for (int l = 0; l < kMimiLayers; ++l) {
        if (!w.in_proj[l] || !w.out_proj[l] || !w.linear1[l] || !w.linear2[l]) return PHONON_CUDA_INVALID_ARGUMENT;
        if ((st = upload_linear(PHONON_CUDA_LINEAR_BF16, w.in_proj[l], 3 * W, W, &m->in_proj[l])) ||
            (st = upload_linear(PHONON_CUDA_LINEAR_BF16, w.out_proj[l], W, W, &m->out_proj[l])) ||
            (st = upload_linear(PHONON_CUDA_LINEAR_BF16, w.linear1[l], kFfn, W, &m->linear1[l])) ||
            (st = upload_linear(PHONON_CUDA_LINEAR_BF16, w.linear2[l], W, kFfn, &m->linear2[l])))
            return st;
    }
    const size_t S = m->max_states, rows = static_cast<size_t>(m->max_batch) * kMimiRows;
    if (cudaMalloc(&m->rings, S * kMimiLayers * 2 * kMimiRing * W * 4) != cudaSuccess ||
        cudaMalloc(&m->previous, S * W * 4) != cudaSuccess ||
        cudaMalloc(&m->d_lat, m->max_batch * 32 * 4) != cudaSuccess ||
        cudaMalloc(&m->d_hidden, rows * W * 4) != cudaSuccess || cudaMalloc(&m->d_norm, rows * W * 4) != cudaSuccess ||
        cudaMalloc(&m->d_qkv, rows * 3 * W * 4) != cudaSuccess || cudaMalloc(&m->d_att, rows * W * 4) != cudaSuccess ||
        cudaMalloc(&m->d_mlp, rows * kFfn * 4) != cudaSuccess ||
        cudaMalloc(&m->d_meta, 2 * m->max_batch * 4) != cudaSuccess ||
        cudaMalloc(&m->d_status, rows * 4) != cudaSuccess ||
        cudaMallocHost(&m->h_lat, m->max_batch * 32 * 4) != cudaSuccess ||
        cudaMallocHost(&m->h_out, rows * W * 4) != cudaSuccess ||
        cudaMallocHost(&m->h_meta, 2 * m->max_batch * 4) != cudaSuccess ||
        cudaMallocHost(&m->h_status, rows * 4) != cudaSuccess)
        return PHONON_CUDA_OUT_OF_MEMORY;
    CUDA_TRY(cudaMemset(m->previous, 0, S * W * 4));
    CUDA_TRY(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
    m->states.assign(S, PhononCudaMimi::State{});
    // tensor-core copies: natural bf16 rows in 128-row TMA boxes, slice rows in 96-row boxes
    const size_t mats = static_cast<size_t>(kMimiLayers) * (3 * W * W + W * W + kFfn * W + W * kFfn);
    const size_t rows_pad = (rows + kHgStreams - 1) / kHgStreams * kHgStreams;
    if (cudaMalloc(&m->wn, mats * 2) != cudaSuccess || cudaMalloc(&m->sl_a, 3 * rows_pad * W * 2) != cudaSuccess ||
        cudaMalloc(&m->sl_g, 3 * rows_pad * kFfn * 2) != cudaSuccess || cudaMalloc(&m->d_err, 4) != cudaSuccess)
        return PHONON_CUDA_OUT_OF_MEMORY;
    CUDA_TRY(cudaMemset(m->d_err, 0, 4));
    CUDA_TRY(cudaMemset(m->sl_a, 0, 3 * rows_pad * W * 2));
    CUDA_TRY(cudaMemset(m->sl_g, 0, 3 * rows_pad * kFfn * 2));
    bool maps = true;
    uint16_t* at = m->wn;
    for (int l = 0; l < kMimiLayers; ++l) {
        const uint16_t* src[4] = {w.in_proj[l], w.out_proj[l], w.linear1[l], w.linear2[l]};
        const size_t rws[4] = {3 * W, W, static_cast<size_t>(kFfn), W}, cls[4] = {W, W, W, static_cast<size_t>(kFfn)};
        for (int k = 0; k < 4; ++k) {
            CUDA_TRY(cudaMemcpy(at, src[k], rws[k] * cls[k] * 2, cudaMemcpyHostToDevice));
            maps = maps && make_map_2d(&m->tm_w[l][k], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, at, rws[k], cls[k], cls[k] * 2,
                                       kHgKTile, kHgM);
            at += rws[k] * cls[k];
        }
    }
    m->tensor_ok = maps &&
                   make_map_2d(&m->tm_sl_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, m->sl_a, 3 * rows_pad, W, W * 2, kHgKTile,
                               kHgN) &&
                   make_map_2d(&m->tm_sl_g, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, m->sl_g, 3 * rows_pad, kFfn, kFfn * 2,
                               kHgKTile, kHgN);
    return PHONON_CUDA_OK;
}

// One frame of n states whose latents are in m->d_lat and slot/position
// metadata in m->d_meta: features in m->d_hidden, per-row status.
int mimi_enqueue(PhononCudaMimi* m, int n) {
    using namespace phonon;
    cudaStream_t s = m->stream;
    const int rows = n * kMimiRows;
    const int32_t* slots = m->d_meta;
    const int32_t* pos = m->d_meta + m->max_batch;
    const float* zeros = m->vec + kMimiLayers * kMimiVecPerLayer * kWidth;
    const float* freq = zeros + kFfn;
    const bool tensor = m->tensor_ok && static_cast<uint32_t>(n) >= m->tensor_min;
    uint16_t* sl = tensor ? m->sl_a : nullptr;
    CUDA_TRY(launch_pdl(mimi_in_kernel, dim3(n), dim3(512), 0, s, static_cast<const float*>(m->d_lat), slots,
                        static_cast<const uint16_t*>(m->w16), static_cast<const uint16_t*>(m->w16 + kWidth * 32),
                        m->previous, m->d_hidden, m->d_status));
    for (int l = 0; l < kMimiLayers; ++l) {
        const float* v = m->vec + l * kMimiVecPerLayer * kWidth;
        HeadGemmParams g{};
        g.bias = zeros;
        g.status = m->d_status;
        g.error = m->d_err;
        CUDA_TRY(launch_pdl(mimi_ln_kernel, dim3((rows + 7) / 8), dim3(256), 0, s, static_cast<const float*>(m->d_hidden),
                            v, v + kWidth, m->d_norm, rows, m->d_status, sl));
        if (tensor) {
            HeadGemmParams q = g;
            q.y = m->d_qkv;
            q.ldy = 3 * kWidth;
            CUDA_TRY((launch_bf16x3_gemm<HG_STORE>(m->tm_w[l][0], m->tm_sl_a, 3 * kWidth, rows, q, s)));
        } else {
            GemvParams p{};
            p.rows = 3 * kWidth;
            p.cols = kWidth;
            p.w = m->in_proj[l].plane;
            p.x = m->d_norm;
            p.ldx = kWidth;
            p.B = rows;
            p.y = m->d_qkv;
            p.ldy = 3 * kWidth;
            p.status = m->d_status;
            CUDA_TRY((launch_gemv_bt<false, 1, SRC_X, EPI_STORE>(p, s)));
        }
        CUDA_TRY(launch_pdl(mimi_rope_kv_kernel, dim3(rows), dim3(256), 0, s, m->d_qkv, slots, pos, freq, m->rings, l));
        {
            static std::atomic<uint64_t> configured{0};
            CUDA_TRY(opt_in_smem(reinterpret_cast<const void*>(mimi_attn_kernel), kMimiAttnSmem, configured));
        }
        CUDA_TRY(launch_pdl(mimi_attn_kernel, dim3(n * kHeads), dim3(kMimiRows * 32), kMimiAttnSmem, s,
                            static_cast<const float*>(m->d_qkv), slots, pos, static_cast<const float*>(m->rings), l,
                            m->d_att, m->d_status, sl));
        if (tensor) {
            HeadGemmParams o = g;
            o.y = m->d_hidden;
            o.ldy = kWidth;
            o.gate = v + 4 * kWidth;  // layer_scale_1, the same for every row
            o.ldgate = 0;
            CUDA_TRY((launch_bf16x3_gemm<HG_GATE>(m->tm_w[l][1], m->tm_sl_a, kWidth, rows, o, s)));
        } else {
            GemvParams p{};
            p.rows = kWidth;
            p.cols = kWidth;
            p.w = m->out_proj[l].plane;
            p.x = m->d_att;
            p.ldx = kWidth;
            p.B = rows;
            p.bias = zeros;
            p.y = m->d_hidden;
            p.ldy = kWidth;
            p.res = m->d_hidden;
            p.ldres = kWidth;
            p.gate = v + 4 * kWidth;  // layer_scale_1, the same for every row
            p.ldgate = 0;
            p.status = m->d_status;
            CUDA_TRY((launch_gemv_bt<false, 1, SRC_X, EPI_GATE>(p, s)));
        }
        CUDA_TRY(launch_pdl(mimi_ln_kernel, dim3((rows + 7) / 8), dim3(256), 0, s, static_cast<const float*>(m->d_hidden),
                            v + 2 * kWidth, v + 3 * kWidth, m->d_norm, rows, m->d_status, sl));
        if (tensor) {
            HeadGemmParams u = g;
            u.slices = m->sl_g;
            u.slice_ld = kFfn;
            CUDA_TRY((launch_bf16x3_gemm<HG_GELU>(m->tm_w[l][2], m->tm_sl_a, kFfn, rows, u, s)));
            HeadGemmParams d = g;
            d.y = m->d_hidden;
            d.ldy = kWidth;
            d.gate = v + 5 * kWidth;  // layer_scale_2
            d.ldgate = 0;
            CUDA_TRY((launch_bf16x3_gemm<HG_GATE, kFfn>(m->tm_w[l][3], m->tm_sl_g, kWidth, rows, d, s)));
            continue;
        }
        GemvParams p{};
        p.rows = kFfn;
        p.cols = kWidth;
        p.w = m->linear1[l].plane;
        p.x = m->d_norm;
        p.ldx = kWidth;
        p.B = rows;
        p.y = m->d_mlp;
        p.ldy = kFfn;
        p.status = m->d_status;
        CUDA_TRY((launch_gemv_bt<false, 1, SRC_X, EPI_GELU>(p, s)));
        p = GemvParams{};
        p.rows = kWidth;
        p.cols = kFfn;
        p.w = m->linear2[l].plane;
        p.x = m->d_mlp;
        p.ldx = kFfn;
        p.B = rows;
        p.bias = zeros;
        p.y = m->d_hidden;
        p.ldy = kWidth;
        p.res = m->d_hidden;
        p.ldres = kWidth;
        p.gate = v + 5 * kWidth;  // layer_scale_2
        p.ldgate = 0;
        p.status = m->d_status;
        CUDA_TRY((launch_gemv_bt<false, 4, SRC_X, EPI_GATE>(p, s)));
    }
    return PHONON_CUDA_OK;
}

// One frame for n distinct live states (host latents [n][32] -> host
// features [n][16][512]); per-state status.
int mimi_enqueue_graphed(PhononCudaMimi* m, int n) {
    const bool tensor = m->tensor_ok && static_cast<uint32_t>(n) >= m->tensor_min;
    if (m->graph && m->graph_n == n && m->graph_tensor == tensor) {
        CUDA_TRY(cudaGraphLaunch(m->graph, m->stream));
        return PHONON_CUDA_OK;
    }
    if (m->last_n != n || m->last_tensor != tensor) {
        m->last_n = n;
        m->last_tensor = tensor;
        return mimi_enqueue(m, n);
    }
    cudaGraph_t g = nullptr;
    if (cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        cudaGetLastError();
        return mimi_enqueue(m, n);
    }
    const int st = mimi_enqueue(m, n);
    const cudaError_t end = cudaStreamEndCapture(m->stream, &g);
    cudaGraphExec_t exec = nullptr;
    if (st != PHONON_CUDA_OK || end != cudaSuccess || !g || cudaGraphInstantiate(&exec, g, 0) != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        return mimi_enqueue(m, n);
    }
    cudaGraphDestroy(g);
    if (m->graph) cudaGraphExecDestroy(m->graph);
    m->graph = exec;
    m->graph_n = n;
    m->graph_tensor = tensor;
    CUDA_TRY(cudaGraphLaunch(m->graph, m->stream));
    return PHONON_CUDA_OK;
}

int mimi_step_locked(PhononCudaMimi* m, uint32_t n, const uint32_t* states, const float* latents, float* features,
                     int32_t* status) {
    using namespace phonon;
    if (n < 1 || n > m->max_batch || !states || !latents || !features || !status) return PHONON_CUDA_INVALID_ARGUMENT;
    for (uint32_t i = 0; i < n; ++i) {
        if (states[i] >= m->max_states || !m->states[states[i]].used) return PHONON_CUDA_INVALID_ARGUMENT;
        for (uint32_t j = 0; j < i; ++j)
            if (states[j] == states[i]) return PHONON_CUDA_INVALID_ARGUMENT;
        if (m->states[states[i]].failed) return PHONON_CUDA_INVALID_ARGUMENT;
        if (m->states[states[i]].position / kMimiRows >= PHONON_CUDA_MIMI_MAX_FRAMES) return PHONON_CUDA_CAPACITY;
        if (m->states[states[i]].position + kMimiRows > static_cast<uint64_t>(INT32_MAX)) return PHONON_CUDA_CAPACITY;
    }
    for (size_t i = 0; i < static_cast<size_t>(n) * 32; ++i)
        if (!std::isfinite(latents[i])) return PHONON_CUDA_NON_FINITE;
    int st = set_device(m->device);
    if (st) return st;
    for (uint32_t i = 0; i < n; ++i) {
        m->h_meta[i] = static_cast<int32_t>(states[i]);
        m->h_meta[m->max_batch + i] = static_cast<int32_t>(m->states[states[i]].position);
    }
    std::memcpy(m->h_lat, latents, static_cast<size_t>(n) * 32 * 4);
    const size_t rows = static_cast<size_t>(n) * kMimiRows;
    CUDA_TRY(cudaMemcpyAsync(m->d_meta, m->h_meta, 2 * m->max_batch * 4, cudaMemcpyHostToDevice, m->stream));
    CUDA_TRY(cudaMemcpyAsync(m->d_lat, m->h_lat, static_cast<size_t>(n) * 32 * 4, cudaMemcpyHostToDevice, m->stream));
    CUDA_TRY(cudaMemsetAsync(m->d_status, 0, rows * 4, m->stream));
    if ((st = mimi_enqueue_graphed(m, static_cast<int>(n)))) return st;
    CUDA_TRY(cudaMemcpyAsync(m->h_out, m->d_hidden, rows * kWidth * 4, cudaMemcpyDeviceToHost, m->stream));
    CUDA_TRY(cudaMemcpyAsync(m->h_status, m->d_status, rows * 4, cudaMemcpyDeviceToHost, m->stream));
    int32_t err = 0;
    CUDA_TRY(cudaMemcpyAsync(&err, m->d_err, 4, cudaMemcpyDeviceToHost, m->stream));
    CUDA_TRY(cudaStreamSynchronize(m->stream));
    if (err) {  // a bounded device wait expired: report, clear for the next call
        CUDA_TRY(cudaMemset(m->d_err, 0, 4));
        return PHONON_CUDA_DEVICE_ERROR;
    }
    for (uint32_t i = 0; i < n; ++i) {
        bool bad = false;
        for (int r = 0; r < kMimiRows; ++r) bad |= m->h_status[i * kMimiRows + r] != 0;
        PhononCudaMimi::State& s = m->states[states[i]];
        if (bad) {
            s.failed = true;  // the reference marks the state unusable until reset
            status[i] = PHONON_CUDA_NON_FINITE;
            continue;
        }
        status[i] = PHONON_CUDA_OK;
        s.position += kMimiRows;
        std::memcpy(features + static_cast<size_t>(i) * kMimiRows * kWidth,
                    m->h_out + static_cast<size_t>(i) * kMimiRows * kWidth, kMimiRows * kWidth * 4);
    }
    return PHONON_CUDA_OK;
}

}  // namespace

extern "C" {

int phonon_cuda_mimi_create(int device, const PhononCudaMimiWeights* w, uint32_t max_states, uint32_t max_batch,
                            PhononCudaMimi** out) {
    if (!w || !out || !max_states || !max_batch || max_batch > max_states || max_states > 65536)
        return PHONON_CUDA_INVALID_ARGUMENT;
    int st = set_device(device);
    if (st) return st;
    PhononCudaMimi* m = new (std::nothrow) PhononCudaMimi;
    if (!m) return PHONON_CUDA_OUT_OF_MEMORY;
    m->device = device;
    m->max_states = max_states;
    m->max_batch = max_batch;
    if ((st = mimi_setup(m, *w))) {
        mimi_release(m);
        delete m;
        return st;
    }
    *out = m;
    return PHONON_CUDA_OK;
}

void phonon_cuda_mimi_destroy(PhononCudaMimi* m) {
    if (!m) return;
    set_device(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    mimi_release(m);
    delete m;
}

int phonon_cuda_mimi_state_alloc(PhononCudaMimi* m, uint32_t* state) {
    if (!m || !state) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(m->mu);
    for (uint32_t i = 0; i < m->max_states; ++i)
        if (!m->states[i].used) {
            int st = set_device(m->device);
            if (st) return st;
            CUDA_TRY(cudaMemsetAsync(m->previous + static_cast<size_t>(i) * phonon::kWidth, 0, phonon::kWidth * 4,
                                     m->stream));
            CUDA_TRY(cudaStreamSynchronize(m->stream));
            m->states[i] = PhononCudaMimi::State{true, false, 0};
            *state = i;
            return PHONON_CUDA_OK;
        }
    return PHONON_CUDA_CAPACITY;
}

int phonon_cuda_mimi_state_reset(PhononCudaMimi* m, uint32_t state) {
    if (!m || state >= m->max_states) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(m->mu);
    if (!m->states[state].used) return PHONON_CUDA_INVALID_ARGUMENT;
    int st = set_device(m->device);
    if (st) return st;
    CUDA_TRY(cudaMemsetAsync(m->previous + static_cast<size_t>(state) * phonon::kWidth, 0, phonon::kWidth * 4,
                             m->stream));
    CUDA_TRY(cudaStreamSynchronize(m->stream));
    m->states[state] = PhononCudaMimi::State{true, false, 0};
    return PHONON_CUDA_OK;
}

int phonon_cuda_mimi_state_free(PhononCudaMimi* m, uint32_t state) {
    if (!m || state >= m->max_states) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(m->mu);
    if (!m->states[state].used) return PHONON_CUDA_INVALID_ARGUMENT;
    m->states[state] = PhononCudaMimi::State{};
    return PHONON_CUDA_OK;
}

int phonon_cuda_mimi_positions(PhononCudaMimi* m, uint32_t state, uint64_t* positions) {
    if (!m || !positions || state >= m->max_states) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(m->mu);
    if (!m->states[state].used) return PHONON_CUDA_INVALID_ARGUMENT;
    *positions = m->states[state].position;
    return PHONON_CUDA_OK;
}

int phonon_cuda_mimi_set_tensor_min(PhononCudaMimi* m, uint32_t min_states, int* available) {
    if (!m) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(m->mu);
    m->tensor_min = min_states;
    if (available) *available = m->tensor_ok ? 1 : 0;
    return PHONON_CUDA_OK;
}

int phonon_cuda_mimi_step(PhononCudaMimi* m, uint32_t n, const uint32_t* states, const float* latents,
                          float* features, int32_t* status) {
    if (!m) return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(m->mu);
    return mimi_step_locked(m, n, states, latents, features, status);
}

int phonon_cuda_mimi_process(PhononCudaMimi* m, uint32_t state, const float* latents, size_t frames, float* features,
                             size_t capacity) {
    if (!m || !latents || !features || !frames || frames > PHONON_CUDA_MIMI_MAX_FRAMES ||
        capacity < frames * phonon::kMimiRows)
        return PHONON_CUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(m->mu);
    if (state >= m->max_states || !m->states[state].used || m->states[state].failed) return PHONON_CUDA_INVALID_ARGUMENT;
    if (m->states[state].position / phonon::kMimiRows > PHONON_CUDA_MIMI_MAX_FRAMES - frames)
        return PHONON_CUDA_CAPACITY;
    for (size_t i = 0; i < frames * 32; ++i)
        if (!std::isfinite(latents[i])) return PHONON_CUDA_NON_FINITE;
    for (size_t f = 0; f < frames; ++f) {
        int32_t st_row = 0;
        const int st = mimi_step_locked(m, 1, &state, latents + f * 32,
                                        features + f * phonon::kMimiRows * phonon::kWidth, &st_row);
        if (st) return st;
        if (st_row) return st_row;
    }
    return PHONON_CUDA_OK;
}

}  // extern "C"
