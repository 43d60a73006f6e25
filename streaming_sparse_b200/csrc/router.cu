// router.cu -- learned KV-block router for sm_100a in exact fp32.
//
//   1. pool: per (head, block) the mean of the block's valid tokens -- fp32 adds in token order,
//      one correctly rounded divide. One CTA reads a whole block of token rows (all heads) with
//      coalesced 16-byte loads; thread (h, 8 dims) keeps 8 running sums.
//      Reference: block pooling of migration/unified_router/opt19/prototype.py:11-49 (one
//      prototype = plain mean of the valid tokens).
//   2. project: pooled [nb x 128] @ W [128 x R] per head with fmaf in ascending row order,
//      W staged in shared memory. Reference: opt8/projection.py:4-14.
//   3. score_select: one warp per (head, query block). Scores S[j] = <qh, kh_j> (fmaf in
//      ascending order, -0 -> +0, non-finite flagged) for every key block; the order-preserving
//      uint32 of each unforced score stays in registers. The `extra`-th largest score T is found
//      exactly by a 32-step bisection with warp-wide counts; blocks above T are kept and ties at
//      T go to the lowest block indices (ordered ballot scan). Forced blocks (sink, current
//      chunk) are always kept and ids are written ascending. Reference: the block-score GEMM
//      `_coarse` (opt16/route.py:34-47), `_chosen`/`_top` (opt16/route.py:13-24,49-55),
//      fixed_page_select (local_experiments/video_runtime_v1/fixed_page_select.py:7-21) and the
//      forced set of local_experiments/video_runtime_v1/pipeline_graph.py:140-151.
// The fixed summation order makes every score bit-identical to the CPU oracle. The score GEMM is
// tens of MFMA per chunk-layer, so CUDA-core FFMA keeps it exact at a cost of microseconds.
#include <algorithm>

#include "common.cuh"

namespace ss {
namespace router {

constexpr int D = 128;
constexpr int MAX_R = 128;
constexpr int MAX_KB = 2048;       // score bits of a row live in registers (64 per lane)
constexpr int PROJ_ROWS = 32;       // pooled rows per projection CTA
constexpr int TILE_J = 64;          // key blocks staged per score tile

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// grid (nq + nk), H*16 threads. Block b < nq pools q, otherwise k; means -> [H][nb][128].
__global__ void pool_kernel(const uint16_t *__restrict__ q, const uint16_t *__restrict__ k, int H, int Lq, int Lk,
                            int block, int nq, float *__restrict__ qmean, float *__restrict__ kmean) {
    const bool isq = (int)blockIdx.x < nq;
    const int b = isq ? blockIdx.x : blockIdx.x - nq;
    const uint16_t *x = isq ? q : k;
    const int L = isq ? Lq : Lk;
    const int nb = isq ? nq : (Lk + block - 1) / block;
    float *out = isq ? qmean : kmean;
    const int t0 = b * block;
    const int n = min(block, L - t0);
    const int tid = threadIdx.x;            // = h*16 + chunk of 8 dims
    const int row_vec = H * D / 8;          // uint4 per token row
    const uint4 *src = reinterpret_cast<const uint4 *>(x + (size_t)t0 * H * D) + tid;
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
    const int h = tid >> 4, d0 = (tid & 15) * 8;
    const float fn = (float)n;
    float4 *dst = reinterpret_cast<float4 *>(out + ((size_t)h * nb + b) * D + d0);
    dst[0] = make_float4(__fdiv_rn(s[0], fn), __fdiv_rn(s[1], fn), __fdiv_rn(s[2], fn), __fdiv_rn(s[3], fn));
    dst[1] = make_float4(__fdiv_rn(s[4], fn), __fdiv_rn(s[5], fn), __fdiv_rn(s[6], fn), __fdiv_rn(s[7], fn));
}

// Copy n rows of R floats from global (dense rows) to shared memory rows of stride `ld`,
// eight loads in flight per thread (a plain loop would wait out one L2 round trip per element).
__device__ __forceinline__ void stage_rows(float *dst, int ld, const float *__restrict__ src, int n, int R) {
    const int total = n * R;
    for (int x0 = threadIdx.x; x0 < total; x0 += 8 * blockDim.x) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int x = x0 + u * blockDim.x;
            v[u] = x < total ? __ldg(src + x) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int x = x0 + u * blockDim.x;
            if (x < total) dst[(x / R) * ld + x % R] = v[u];
        }
    }
}

// grid (tq + tk, H), 256 threads; tiles [0, tq) project q means with wq, the rest k means with wk.
// Thread t owns row t / (R/8) of the tile and 8 consecutive output columns: eight independent
// fmaf chains (each in ascending d order) keep the FMA pipe busy.
__global__ void __launch_bounds__(256) project_kernel(const float *__restrict__ qmean, const float *__restrict__ kmean,
                                                      const float *__restrict__ wq, const float *__restrict__ wk,
                                                      int qb, int kb, int tq, int R, float *__restrict__ qh,
                                                      float *__restrict__ kh) {
    extern __shared__ float sm[];
    float *sw = sm;                      // [128][R]
    float *sx = sm + D * R;              // [PROJ_ROWS][129]
    const int h = blockIdx.y;
    const bool isq = (int)blockIdx.x < tq;
    const int tile = isq ? blockIdx.x : blockIdx.x - tq;
    const int nb = isq ? qb : kb;
    const float *mean = (isq ? qmean : kmean) + (size_t)h * nb * D;
    const float *w = (isq ? wq : wk) + (size_t)h * D * R;
    float *out = (isq ? qh : kh) + (size_t)h * nb * R;
    const int r0 = tile * PROJ_ROWS, rows = min(PROJ_ROWS, nb - r0);
    stage_rows(sw, R, w, D, R);
    stage_rows(sx, D + 1, mean + (size_t)r0 * D, rows, D);
    for (int x = threadIdx.x; x < (PROJ_ROWS - rows) * D; x += 256)   // zero the unused rows
        sx[(rows + x / D) * (D + 1) + x % D] = 0.f;
    __syncthreads();
    const int groups = R / 8;            // 8-column groups per row
    for (int o = threadIdx.x; o < PROJ_ROWS * groups; o += 256) {
        const int rr = o / groups, e0 = (o % groups) * 8;
        float acc[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) acc[u] = 0.f;
#pragma unroll 4
        for (int d = 0; d < D; ++d) {
            const float x = sx[rr * (D + 1) + d];
            const float4 w0 = reinterpret_cast<const float4 *>(sw + d * R + e0)[0];
            const float4 w1 = reinterpret_cast<const float4 *>(sw + d * R + e0)[1];
            acc[0] = __fmaf_rn(x, w0.x, acc[0]);
            acc[1] = __fmaf_rn(x, w0.y, acc[1]);
            acc[2] = __fmaf_rn(x, w0.z, acc[2]);
            acc[3] = __fmaf_rn(x, w0.w, acc[3]);
            acc[4] = __fmaf_rn(x, w1.x, acc[4]);
            acc[5] = __fmaf_rn(x, w1.y, acc[5]);
            acc[6] = __fmaf_rn(x, w1.z, acc[6]);
            acc[7] = __fmaf_rn(x, w1.w, acc[7]);
        }
        if (rr < rows) {
            float4 *dst = reinterpret_cast<float4 *>(out + (size_t)(r0 + rr) * R + e0);
            dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
            dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
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

// One warp per (head, query block) row; `rows` warps per CTA share staged tiles of kh[h].
// Key order: (ordered score bits, lower block index first). Lane owns blocks j = 32*i + lane,
// i < NPL, with the score bits in registers (0 = not a candidate: forced or past kb; every
// finite score maps to >= 0x00800000).
//   1. T = the extra-th largest score value among candidates (32-step bisection on the bits).
//   2. Blocks scoring above T are kept; of the blocks scoring exactly T, the lowest-index ones
//      fill the remaining slots (ordered ballot scan).
template <int NPL>
__global__ void score_select_kernel(const float *__restrict__ qh, const float *__restrict__ kh, int qb, int kb, int R,
                                    int block, int Lq, int Lk, int sink, int extra, int32_t *__restrict__ ids,
                                    int n_ids, uint8_t *__restrict__ mask, float *__restrict__ scores, int *status) {
    extern __shared__ float sm[];
    const int rows = blockDim.x / 32;
    float *sq = sm;                      // [rows][R]
    float *sk = sm + rows * R;           // [TILE_J][R+1]
    const int h = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int i = blockIdx.x * rows + warp;
    const bool row_ok = i < qb;
    for (int x = threadIdx.x; x < rows * R; x += blockDim.x) {
        const int ii = blockIdx.x * rows + x / R;
        sq[x] = ii < qb ? qh[((size_t)h * qb + ii) * R + x % R] : 0.f;
    }
    const float *myq = sq + warp * R;
    uint32_t hi[NPL];
#pragma unroll
    for (int u = 0; u < NPL; ++u) hi[u] = 0u;
    bool bad = false;
    for (int j0 = 0; j0 < kb; j0 += TILE_J) {
        const int nj = min(TILE_J, kb - j0);
        __syncthreads();
        stage_rows(sk, R + 1, kh + ((size_t)h * kb + j0) * R, nj, R);
        __syncthreads();
        if (row_ok) {
            // lanes own columns lane and lane + 32 of this tile: two independent fmaf chains
            const float *k0 = sk + lane * (R + 1), *k1 = sk + (lane + 32) * (R + 1);
            float a0 = 0.f, a1 = 0.f;
#pragma unroll 8
            for (int e = 0; e < R; ++e) {
                const float qe = myq[e];
                a0 = __fmaf_rn(qe, k0[e], a0);
                a1 = __fmaf_rn(qe, k1[e], a1);
            }
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                float acc = c ? a1 : a0;
                const int jj = lane + 32 * c;
                const int j = j0 + jj;
                if (acc == 0.f) acc = 0.f;  // -0 -> +0
                const bool live = jj < nj;
                bad |= live && !isfinite(acc);
                if (live && scores) scores[((size_t)h * qb + i) * kb + j] = acc;
                const uint32_t o = (!live || is_forced(j, block, Lq, Lk, sink)) ? 0u : ordered_bits(acc);
                const int slot = (j0 >> 5) + c;   // = j >> 5, the same for all lanes
#pragma unroll
                for (int u = 0; u < NPL; ++u)
                    if (u == slot && live) hi[u] = o;
            }
        }
    }
    if (bad) report(status, SS_DEV_NONFINITE);
    if (!row_ok) return;
    uint32_t T = 0xffffffffu;
    int need = 0;
    if (extra > 0) {
        T = 0u;
        for (int bit = 31; bit >= 0; --bit) {
            const uint32_t cand = T | (1u << bit);
            int cnt = 0;
#pragma unroll
            for (int u = 0; u < NPL; ++u) cnt += hi[u] >= cand;
            if ((int)__reduce_add_sync(0xffffffffu, (unsigned)cnt) >= extra) T = cand;
        }
        int gt = 0;
#pragma unroll
        for (int u = 0; u < NPL; ++u) gt += hi[u] > T;
        need = extra - (int)__reduce_add_sync(0xffffffffu, (unsigned)gt);  // ties at T to keep, >= 1
    }
    // ascending compaction of forced | above T | the first `need` ties at T
    int32_t *out = ids + ((size_t)h * qb + i) * n_ids;
    int pos = 0, taken = 0;
#pragma unroll
    for (int u = 0; u < NPL; ++u) {
        const int j = 32 * u + lane;
        if (32 * u >= kb) continue;   // warp-uniform
        const bool tie = extra > 0 && j < kb && hi[u] == T;
        const unsigned tb = __ballot_sync(0xffffffffu, tie);
        const bool keep_tie = tie && taken + __popc(tb & ((1u << lane) - 1u)) < need;
        taken += __popc(tb);
        const bool sel = j < kb && (is_forced(j, block, Lq, Lk, sink) || (extra > 0 && hi[u] > T) || keep_tie);
        const unsigned bal = __ballot_sync(0xffffffffu, sel);
        const int off = pos + __popc(bal & ((1u << lane) - 1u));
        if (sel && off < n_ids) out[off] = j;
        if (mask && j < kb) mask[((size_t)h * qb + i) * kb + j] = sel ? 1 : 0;
        pos += __popc(bal);
    }
}

}  // namespace router

static size_t select_smem(int rows, int R) {
    return (size_t)rows * R * 4 + (size_t)router::TILE_J * (R + 1) * 4;
}

using SelectFn = void (*)(const float *, const float *, int, int, int, int, int, int, int, int, int32_t *, int,
                          uint8_t *, float *, int *);

static SelectFn select_kernel(int kb) {
    if (kb <= 128) return router::score_select_kernel<4>;
    if (kb <= 512) return router::score_select_kernel<16>;
    if (kb <= 1024) return router::score_select_kernel<32>;
    return router::score_select_kernel<64>;
}

static int g_router_configured[64] = {0};

int router_prepare(int device) {
    if (device < 0 || device >= 64) return SS_ERR_SHAPE;
    if (g_router_configured[device]) return 0;
    cudaError_t e = cudaFuncSetAttribute(router::project_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         227 * 1024);
    if (e != cudaSuccess) return (int)e;
    g_router_configured[device] = 1;
    return 0;
}

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct RouterLayout {
    size_t qmean, kmean, qh, kh, total;
};

static RouterLayout router_layout(int H, int Lq, int Lk, int R, int block) {
    const size_t qb = (size_t)((Lq + block - 1) / block), kb = (size_t)((Lk + block - 1) / block);
    RouterLayout L;
    L.qmean = 0;
    L.kmean = align256(L.qmean + 4 * (size_t)H * qb * router::D);
    L.qh = align256(L.kmean + 4 * (size_t)H * kb * router::D);
    L.kh = align256(L.qh + 4 * (size_t)H * qb * R);
    L.total = align256(L.kh + 4 * (size_t)H * kb * R);
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
    if (H <= 0 || H > 64 || Lq <= 0 || Lk < Lq || R <= 0 || R > router::MAX_R || (R & 7) ||
        (block != 64 && block != 128) || sink_tokens < 0)
        return SS_ERR_SHAPE;
    const int kb = (Lk + block - 1) / block;
    if (kb > router::MAX_KB) return SS_ERR_SHAPE;
    const int nforced = count_forced(Lq, Lk, block, sink_tokens);
    if (extra < 0 || extra > kb - nforced) return SS_ERR_BUDGET;
    if (n_ids != nforced + extra) return SS_ERR_SHAPE;
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k)) & 15u) return SS_ERR_POINTER;
    return 0;
}

// Launch the router kernels with the intermediates at the given device addresses
// (ws points at a buffer of router_workspace_size bytes, 256-byte aligned).
int router_launch(const void *q, const void *k, const float *wq, const float *wk, int H, int Lq, int Lk, int R,
                  int block, int sink_tokens, int extra, int32_t *ids, int n_ids, uint8_t *mask, float *scores,
                  uint8_t *ws, int *status, cudaStream_t st) {
    const int qb = (Lq + block - 1) / block, kb = (Lk + block - 1) / block;
    int device;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return (int)e;
    int rc = router_prepare(device);
    if (rc) return rc;
    const RouterLayout L = router_layout(H, Lq, Lk, R, block);
    float *qmean = reinterpret_cast<float *>(ws + L.qmean), *kmean = reinterpret_cast<float *>(ws + L.kmean);
    float *qh = reinterpret_cast<float *>(ws + L.qh), *kh = reinterpret_cast<float *>(ws + L.kh);
    router::pool_kernel<<<qb + kb, H * 16, 0, st>>>((const uint16_t *)q, (const uint16_t *)k, H, Lq, Lk, block, qb,
                                                   qmean, kmean);
    const int tq = (qb + router::PROJ_ROWS - 1) / router::PROJ_ROWS, tk = (kb + router::PROJ_ROWS - 1) / router::PROJ_ROWS;
    const size_t sm_proj = sizeof(float) * ((size_t)router::D * R + router::PROJ_ROWS * (router::D + 1));
    router::project_kernel<<<dim3(tq + tk, H), 256, sm_proj, st>>>(qmean, kmean, wq, wk, qb, kb, tq, R, qh, kh);
    const int rows = 4;
    select_kernel(kb)<<<dim3((qb + rows - 1) / rows, H), rows * 32, select_smem(rows, R), st>>>(
        qh, kh, qb, kb, R, block, Lq, Lk, sink_tokens, extra, ids, n_ids, mask, scores, status);
    return (int)cudaGetLastError();
}

}  // namespace ss

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
