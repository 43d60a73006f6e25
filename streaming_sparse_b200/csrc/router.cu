// router.cu -- learned KV-block router for sm_100a in exact fp32.
//
//   1. pool_project: one CTA per (head, group of 16 blocks). The head's [128 x R] projection is
//      fetched into shared memory with one bulk copy; each thread sums 8 dimensions of one block
//      over the block's valid tokens (fp32 adds in token order, one correctly rounded divide),
//      then the block means are projected with fmaf in ascending row order. Query projections
//      are stored [H][qb][R]; key projections transposed [H][R][kb] for the score stage.
//      Reference: block pooling of migration/unified_router/opt19/prototype.py:11-49 (one
//      prototype = plain mean of the valid tokens) and the projection of opt8/projection.py:4-14.
//   2. score_select: one warp per (head, query block), eight query blocks per CTA sharing the
//      head's transposed key projections, staged into shared memory 256 key blocks at a time by
//      bulk copies. Scores S[j] = <qh, kh_j> (fmaf in ascending order, -0 -> +0, non-finite
//      flagged); the order-preserving uint32 of each unforced score is kept in shared memory.
//      The `extra`-th largest score T is found exactly by a 32-step bisection with warp-wide
//      counts; blocks above T are kept and ties at T go to the lowest block indices (ordered
//      ballot scan). Forced blocks (sink, current chunk) are always kept; ids are written
//      ascending. Reference: the block-score GEMM `_coarse` (opt16/route.py:34-47), `_chosen`/
//      `_top` (opt16/route.py:13-24,49-55), fixed_page_select (local_experiments/
//      video_runtime_v1/fixed_page_select.py:7-21) and the forced set of local_experiments/
//      video_runtime_v1/pipeline_graph.py:140-151.
// The fixed summation order makes every score bit-identical to the CPU oracle. The score GEMM is
// tens of MFMA per chunk-layer, so CUDA-core FFMA keeps it exact at a cost of microseconds.
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace ss {
namespace router {

constexpr int D = 128;
constexpr int MAX_R = 128;
constexpr int MAX_KB = 8192;
constexpr int BG = 16;               // blocks per pool_project CTA
constexpr int PP_THREADS = BG * 16;  // thread = (block, 8 dims)
constexpr int ROWS = 8;              // query blocks (warps) per score_select CTA
constexpr int TJ = 256;              // key blocks per staged tile

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}

// grid (tiles_q + tiles_k, H), BG*16 threads. Tiles [0, tiles_q) pool query blocks, the rest key
// blocks. Dynamic shared memory: W [128][R], means [BG][128], mbarrier.
__global__ void __launch_bounds__(PP_THREADS) pool_project_kernel(const uint16_t *__restrict__ q,
                                                                  const uint16_t *__restrict__ k, int H, int Lq,
                                                                  int Lk, int block, int R, int tiles_q,
                                                                  const float *__restrict__ wq,
                                                                  const float *__restrict__ wk,
                                                                  float *__restrict__ qh, float *__restrict__ khT,
                                                                  int kbp, int *status) {
    extern __shared__ __align__(16) uint8_t smr[];
    float *sw = reinterpret_cast<float *>(smr);                 // [128][R]
    float *smean = sw + D * R;                                   // [BG][128]
    uint64_t *mbar = reinterpret_cast<uint64_t *>(smean + BG * D);
    const int h = blockIdx.y, tid = threadIdx.x;
    const bool isq = (int)blockIdx.x < tiles_q;
    const int tile = isq ? blockIdx.x : blockIdx.x - tiles_q;
    const int L = isq ? Lq : Lk;
    const int nb = (L + block - 1) / block;
    const int b0 = tile * BG, nblk = min(BG, nb - b0);
    const uint32_t bar = smem_u32(mbar);
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
        mbar_arrive_expect_tx(bar, (uint32_t)(D * R * 4));
        bulk_g2s(smem_u32(sw), (isq ? wq : wk) + (size_t)h * D * R, (uint32_t)(D * R * 4), bar);
    }
    // pooling: thread (bi, c) sums dims [8c, 8c+8) of block b0+bi in token order
    const int bi = tid >> 4, c = tid & 15;
    if (bi < nblk) {
        const int t0 = (b0 + bi) * block;
        const int n = min(block, L - t0);
        const uint16_t *x = isq ? q : k;
        const size_t row_vec = (size_t)H * D / 8;
        const uint4 *src = reinterpret_cast<const uint4 *>(x + ((size_t)t0 * H + h) * D) + c;
        float s[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) s[i] = 0.f;
        int t = 0;
        for (; t + 8 <= n; t += 8) {
            uint4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = __ldg(src + (size_t)(t + u) * row_vec);
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                s[0] = __fadd_rn(s[0], bf16_lo(v[u].x));
                s[1] = __fadd_rn(s[1], bf16_hi(v[u].x));
                s[2] = __fadd_rn(s[2], bf16_lo(v[u].y));
                s[3] = __fadd_rn(s[3], bf16_hi(v[u].y));
                s[4] = __fadd_rn(s[4], bf16_lo(v[u].z));
                s[5] = __fadd_rn(s[5], bf16_hi(v[u].z));
                s[6] = __fadd_rn(s[6], bf16_lo(v[u].w));
                s[7] = __fadd_rn(s[7], bf16_hi(v[u].w));
            }
        }
        for (; t < n; ++t) {
            const uint4 v = __ldg(src + (size_t)t * row_vec);
            s[0] = __fadd_rn(s[0], bf16_lo(v.x));
            s[1] = __fadd_rn(s[1], bf16_hi(v.x));
            s[2] = __fadd_rn(s[2], bf16_lo(v.y));
            s[3] = __fadd_rn(s[3], bf16_hi(v.y));
            s[4] = __fadd_rn(s[4], bf16_lo(v.z));
            s[5] = __fadd_rn(s[5], bf16_hi(v.z));
            s[6] = __fadd_rn(s[6], bf16_lo(v.w));
            s[7] = __fadd_rn(s[7], bf16_hi(v.w));
        }
        const float fn = (float)n;
#pragma unroll
        for (int i = 0; i < 8; ++i) smean[bi * D + 8 * c + i] = __fdiv_rn(s[i], fn);
    }
    // wait for W (bounded), then project: thread (bi, e-group) owns R/16 consecutive outputs
    volatile int no_abort = 0;
    const bool have_w = mbar_wait(bar, 0, &no_abort);
    __syncthreads();
    if (!have_w) {
        if (tid == 0) report(status, SS_DEV_TIMEOUT);
        return;
    }
    const int per = R / 16;  // 4 for R = 64 (R is a multiple of 16, at most 128)
    if (bi < nblk) {
        float acc[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) acc[u] = 0.f;
        const int e0 = c * per;
#pragma unroll 4
        for (int d = 0; d < D; ++d) {
            const float xm = smean[bi * D + d];
            const float *wr = sw + d * R + e0;
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (u < per) acc[u] = __fmaf_rn(xm, wr[u], acc[u]);
        }
        const int b = b0 + bi;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            if (u >= per) break;
            if (isq) qh[((size_t)h * nb + b) * R + e0 + u] = acc[u];
            else khT[((size_t)h * R + e0 + u) * kbp + b] = acc[u];
        }
    }
}

__device__ __forceinline__ bool is_forced(int j, int block, int Lq, int Lk, int sink) {
    const int lo = j * block, hi = min(lo + block, Lk);
    return lo < sink || hi > Lk - Lq;
}

__device__ __forceinline__ uint32_t ordered_bits(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// grid (ceil(qb / ROWS), H), ROWS warps. khT rows have stride kbp (kb rounded up to a multiple of
// 4). Dynamic shared memory: khT tile [R][TJ], qh rows [ROWS][R], keys [ROWS][kbp] (ordered score
// bits; 0 = not a candidate, which no finite score maps to), mbarrier.
__global__ void __launch_bounds__(ROWS * 32) score_select_kernel(const float *__restrict__ qh,
                                                                 const float *__restrict__ khT, int qb, int kb,
                                                                 int kbp, int R,
                                                                 int block, int Lq, int Lk, int sink, int extra,
                                                                 int32_t *__restrict__ ids, int n_ids,
                                                                 uint8_t *__restrict__ mask,
                                                                 float *__restrict__ scores, int *status) {
    extern __shared__ __align__(16) uint8_t smr[];
    float *sk = reinterpret_cast<float *>(smr);               // [R][TJ]
    float *sq = sk + R * TJ;                                   // [ROWS][R]
    uint32_t *keys = reinterpret_cast<uint32_t *>(sq + ROWS * R);  // [ROWS][kb]
    uint64_t *mbar = reinterpret_cast<uint64_t *>(keys + (size_t)ROWS * kbp);
    const int h = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int i = blockIdx.x * ROWS + warp;
    const bool row_ok = i < qb;
    const uint32_t bar = smem_u32(mbar);
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    for (int x = threadIdx.x; x < ROWS * R; x += blockDim.x) {
        const int ii = blockIdx.x * ROWS + x / R;
        sq[x] = ii < qb ? qh[((size_t)h * qb + ii) * R + x % R] : 0.f;
    }
    __syncthreads();
    const float *myq = sq + warp * R;
    uint32_t *mykeys = keys + (size_t)warp * kbp;
    bool bad = false, ok = true;
    volatile int no_abort = 0;
    for (int t = 0, j0 = 0; j0 < kb; ++t, j0 += TJ) {
        const int nj = min(TJ, kb - j0);
        if (threadIdx.x == 0) {
            // rows e of the tile: khT[h][e][j0 .. j0+nj), 16-byte multiples (the host pads kb)
            const uint32_t rb = (uint32_t)(((nj * 4) + 15) & ~15);
            mbar_arrive_expect_tx(bar, rb * (uint32_t)R);
            for (int e = 0; e < R; ++e)
                bulk_g2s(smem_u32(sk + e * TJ), khT + ((size_t)h * R + e) * kbp + j0, rb, bar);
        }
        ok = mbar_wait(bar, t & 1, &no_abort);
        if (!ok) break;
        if (row_ok) {
            float acc[TJ / 32];
#pragma unroll
            for (int u = 0; u < TJ / 32; ++u) acc[u] = 0.f;
#pragma unroll 2
            for (int e = 0; e < R; ++e) {
                const float qe = myq[e];
                const float *kr = sk + e * TJ + lane;
#pragma unroll
                for (int u = 0; u < TJ / 32; ++u) acc[u] = __fmaf_rn(qe, kr[32 * u], acc[u]);
            }
#pragma unroll
            for (int u = 0; u < TJ / 32; ++u) {
                const int j = j0 + lane + 32 * u;
                if (j >= kb) continue;
                float a = acc[u];
                if (a == 0.f) a = 0.f;  // -0 -> +0
                bad |= !isfinite(a);
                if (scores) scores[((size_t)h * qb + i) * kb + j] = a;
                mykeys[j] = is_forced(j, block, Lq, Lk, sink) ? 0u : ordered_bits(a);
            }
        }
        __syncthreads();  // the tile buffer is refilled next iteration
    }
    if (bad) report(status, SS_DEV_NONFINITE);
    if (!ok) {
        if (threadIdx.x == 0) report(status, SS_DEV_TIMEOUT);
        return;
    }
    if (!row_ok) return;
    __syncwarp();
    // T = the extra-th largest candidate score (bisection on the order-preserving bits)
    uint32_t T = 0xffffffffu;
    int need = 0;
    if (extra > 0) {
        T = 0u;
        for (int bit = 31; bit >= 0; --bit) {
            const uint32_t cand = T | (1u << bit);
            int cnt = 0;
            for (int j = lane; j < kb; j += 32) cnt += mykeys[j] >= cand;
            if ((int)__reduce_add_sync(0xffffffffu, (unsigned)cnt) >= extra) T = cand;
        }
        int gt = 0;
        for (int j = lane; j < kb; j += 32) gt += mykeys[j] > T;
        need = extra - (int)__reduce_add_sync(0xffffffffu, (unsigned)gt);  // ties at T to keep, >= 1
    }
    // ascending compaction of forced | above T | the first `need` ties at T
    int32_t *out = ids + ((size_t)h * qb + i) * n_ids;
    int pos = 0, taken = 0;
    for (int j0 = 0; j0 < kb; j0 += 32) {
        const int j = j0 + lane;
        const uint32_t key = j < kb ? mykeys[j] : 0u;
        const bool tie = extra > 0 && j < kb && key == T;
        const unsigned tb = __ballot_sync(0xffffffffu, tie);
        const bool keep_tie = tie && taken + __popc(tb & ((1u << lane) - 1u)) < need;
        taken += __popc(tb);
        const bool sel = j < kb && (is_forced(j, block, Lq, Lk, sink) || (extra > 0 && key > T) || keep_tie);
        const unsigned bal = __ballot_sync(0xffffffffu, sel);
        const int off = pos + __popc(bal & ((1u << lane) - 1u));
        if (sel && off < n_ids) out[off] = j;
        if (mask && j < kb) mask[((size_t)h * qb + i) * kb + j] = sel ? 1 : 0;
        pos += __popc(bal);
    }
}

}  // namespace router

static size_t pp_smem(int R) { return (size_t)router::D * R * 4 + (size_t)router::BG * router::D * 4 + 16; }

static size_t select_smem(int kb, int R) {
    return (size_t)R * router::TJ * 4 + (size_t)router::ROWS * R * 4 + (size_t)router::ROWS * kb * 4 + 16;
}

static int g_router_configured[64] = {0};

int router_prepare(int device) {
    if (device < 0 || device >= 64) return SS_ERR_SHAPE;
    if (g_router_configured[device]) return 0;
    cudaError_t e = cudaFuncSetAttribute(router::pool_project_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         227 * 1024);
    if (e != cudaSuccess) return (int)e;
    e = cudaFuncSetAttribute(router::score_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return (int)e;
    g_router_configured[device] = 1;
    return 0;
}

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// key projections are stored transposed with rows padded to a multiple of 4 blocks, so every
// bulk copy of a row segment starts and ends on a 16-byte boundary
static int kb_padded(int kb) { return (kb + 3) & ~3; }

struct RouterLayout {
    size_t qh, khT, total;
};

static RouterLayout router_layout(int H, int Lq, int Lk, int R, int block) {
    const size_t qb = (size_t)((Lq + block - 1) / block);
    const size_t kbp = (size_t)kb_padded((Lk + block - 1) / block);
    RouterLayout L;
    L.qh = 0;
    L.khT = align256(L.qh + 4 * (size_t)H * qb * R);
    L.total = align256(L.khT + 4 * (size_t)H * R * kbp);
    return L;
}

size_t router_workspace_size(int H, int Lq, int Lk, int R, int block) { return router_layout(H, Lq, Lk, R, block).total; }

static int count_forced(int Lq, int Lk, int block, int sink) {
    const int kb = (Lk + block - 1) / block;
    int n = 0;
    for (int j = 0; j < kb; ++j) {
        const int lo = j * block, hi = std::min(lo + block, Lk);
        n += (lo < sink || hi > Lk - Lq);
    }
    return n;
}

int router_check(const void *q, const void *k, const float *wq, const float *wk, int H, int Lq, int Lk, int R,
                 int block, int sink_tokens, int extra, const int32_t *ids, int n_ids) {
    if (!q || !k || !wq || !wk || !ids) return SS_ERR_POINTER;
    if (H <= 0 || H > 65535 || Lq <= 0 || Lk < Lq || R <= 0 || R > router::MAX_R || (R % 16) ||
        (block != 64 && block != 128) || sink_tokens < 0)
        return SS_ERR_SHAPE;
    const int kb = (Lk + block - 1) / block;
    if (kb > router::MAX_KB || select_smem(kb_padded(kb), R) > 227 * 1024) return SS_ERR_SHAPE;
    const int nforced = count_forced(Lq, Lk, block, sink_tokens);
    if (extra < 0 || extra > kb - nforced) return SS_ERR_BUDGET;
    if (n_ids != nforced + extra) return SS_ERR_SHAPE;
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(wq) |
         reinterpret_cast<uintptr_t>(wk)) & 15u)
        return SS_ERR_POINTER;
    return 0;
}

// Launch the router kernels with the intermediates in `ws` (router_workspace_size bytes,
// 256-byte aligned).
int router_launch(const void *q, const void *k, const float *wq, const float *wk, int H, int Lq, int Lk, int R,
                  int block, int sink_tokens, int extra, int32_t *ids, int n_ids, uint8_t *mask, float *scores,
                  uint8_t *ws, int *status, cudaStream_t st) {
    const int qb = (Lq + block - 1) / block, kb = (Lk + block - 1) / block, kbp = kb_padded(kb);
    int device;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return (int)e;
    int rc = router_prepare(device);
    if (rc) return rc;
    const RouterLayout L = router_layout(H, Lq, Lk, R, block);
    float *qh = reinterpret_cast<float *>(ws + L.qh), *khT = reinterpret_cast<float *>(ws + L.khT);
    const int tq = (qb + router::BG - 1) / router::BG, tk = (kb + router::BG - 1) / router::BG;
    router::pool_project_kernel<<<dim3(tq + tk, H), router::PP_THREADS, pp_smem(R), st>>>(
        (const uint16_t *)q, (const uint16_t *)k, H, Lq, Lk, block, R, tq, wq, wk, qh, khT, kbp, status);
    router::score_select_kernel<<<dim3((qb + router::ROWS - 1) / router::ROWS, H), router::ROWS * 32,
                                  select_smem(kbp, R), st>>>(qh, khT, qb, kb, kbp, R, block, Lq, Lk, sink_tokens,
                                                             extra, ids, n_ids, mask, scores, status);
    return (int)cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------
// ss_router_noalloc: the router with its intermediates in a static device array.
// ---------------------------------------------------------------------------------------------
// For callers that cannot allocate device memory per call. Every call on a device shares this
// one array (it keeps the previous call's contents; nothing in it has to start at zero, because
// each call writes every value that affects its results -- the few padding entries of the
// transposed key rows are copied along but never used), so calls that may overlap on the GPU --
// two streams, or two host threads -- race and must be serialised by the caller.
static __device__ __align__(256) uint8_t g_router_scratch[SS_ROUTER_STATIC_SCRATCH_BYTES];

static std::mutex g_router_scratch_mutex;
static uint8_t *g_router_scratch_addr[64] = {nullptr};

// Device address of g_router_scratch on the current device. In host code the symbol is only a
// host-side stand-in; a kernel given it would fault (or, where the GPU can reach host memory,
// silently use the wrong memory), so the address is looked up once per device, with that device
// current, and cached.
static int router_scratch_address(int device, uint8_t **addr) {
    std::lock_guard<std::mutex> lock(g_router_scratch_mutex);
    if (!g_router_scratch_addr[device]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_router_scratch);
        if (e != cudaSuccess) return (int)e;
        if (!p) return SS_ERR_POINTER;
        g_router_scratch_addr[device] = static_cast<uint8_t *>(p);
    }
    *addr = g_router_scratch_addr[device];
    return 0;
}

}  // namespace ss

extern "C" int ss_router_noalloc(const void *q, const void *k, const float *wq, const float *wk, int H, int Lq, int Lk,
                                 int R, int block, int sink_tokens, int extra, int32_t *ids, int n_ids, uint8_t *mask,
                                 float *scores, int *status, void *stream) {
    int rc = ss::router_check(q, k, wq, wk, H, Lq, Lk, R, block, sink_tokens, extra, ids, n_ids);
    if (rc) return rc;
    if (ss::router_workspace_size(H, Lq, Lk, R, block) > (size_t)SS_ROUTER_STATIC_SCRATCH_BYTES) return SS_ERR_WORKSPACE;
    int device;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return (int)e;
    if (device < 0 || device >= 64) return SS_ERR_SHAPE;
    uint8_t *scratch = nullptr;
    rc = ss::router_scratch_address(device, &scratch);
    if (rc) return rc;
    return ss::router_launch(q, k, wq, wk, H, Lq, Lk, R, block, sink_tokens, extra, ids, n_ids, mask, scores, scratch,
                             status, static_cast<cudaStream_t>(stream));
}

extern "C" int ss_router_workspace_bytes(int H, int Lq, int Lk, int R, int block, size_t *bytes) {
    if (!bytes || H <= 0 || Lq <= 0 || Lk <= 0 || R <= 0 || (block != 64 && block != 128)) return SS_ERR_SHAPE;
    *bytes = ss::router_workspace_size(H, Lq, Lk, R, block);
    return 0;
}

extern "C" int ss_router(const void *q, const void *k, const float *wq, const float *wk, int H, int Lq, int Lk, int R,
                         int block, int sink_tokens, int extra, int32_t *ids, int n_ids, uint8_t *mask, float *scores,
                         void *workspace, size_t workspace_bytes, int *status, void *stream) {
    int rc = ss::router_check(q, k, wq, wk, H, Lq, Lk, R, block, sink_tokens, extra, ids, n_ids);
    if (rc) return rc;
    if (!workspace) return SS_ERR_POINTER;
    if (workspace_bytes < ss::router_workspace_size(H, Lq, Lk, R, block)) return SS_ERR_WORKSPACE;
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return SS_ERR_POINTER;
    return ss::router_launch(q, k, wq, wk, H, Lq, Lk, R, block, sink_tokens, extra, ids, n_ids, mask, scores,
                             static_cast<uint8_t *>(workspace), status, static_cast<cudaStream_t>(stream));
}
