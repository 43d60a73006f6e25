// router.cu -- learned KV-block router for sm_100a in exact fp32.
//
//   1. pool_project: per (head, block) the mean of the block's valid tokens (fp32 adds in token
//      order, one correctly rounded divide) projected by the head's [128 x R] matrix with fmaf in
//      ascending row order. Reference: block pooling of migration/unified_router/opt19/
//      prototype.py:11-49 (one prototype = plain mean), projection opt8/projection.py:4-14.
//   2. block_scores: S[h,i,j] = <qh_i, kh_j> with fmaf in ascending order, -0 -> +0, non-finite
//      scores flagged. Reference: the block-score GEMM `_coarse` of opt16/route.py:34-47.
//   3. select_topk: forced blocks (sink, current chunk) plus the `extra` highest-scoring others,
//      ties to the lower block index, ids written ascending. Reference: `_chosen`/`_top`
//      (opt16/route.py:13-24,49-55), fixed_page_select (local_experiments/video_runtime_v1/
//      fixed_page_select.py:7-21) and the forced set of pipeline_graph.py:140-151.
// The fixed summation order makes the result bit-identical to the CPU oracle; the score GEMM is
// a few tens of MFMA per chunk-layer, so CUDA-core FFMA costs microseconds.
#include <algorithm>

#include "common.cuh"

namespace ss {
namespace router {

constexpr int D = 128;
constexpr int MAX_R = 128;
constexpr int TOPK_THREADS = 256;
constexpr int MAX_KB = 8192;

__device__ __forceinline__ float bf16_to_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

// grid (nb, H), 128 threads: thread d owns dimension d of the block mean.
__global__ void __launch_bounds__(128) pool_project_kernel(const uint16_t *__restrict__ x, int64_t row_stride, int L,
                                                           int H, int block, const float *__restrict__ W, int R,
                                                           float *__restrict__ proj) {
    __shared__ float mean[D];
    const int b = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
    const int t0 = b * block;
    const int n = min(block, L - t0);
    const uint16_t *src = x + (int64_t)t0 * row_stride + (int64_t)h * D + d;
    float s = 0.f;
    int t = 0;
    for (; t + 8 <= n; t += 8) {
        uint16_t v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = __ldg(src + (int64_t)(t + u) * row_stride);
#pragma unroll
        for (int u = 0; u < 8; ++u) s = __fadd_rn(s, bf16_to_f32(v[u]));
    }
    for (; t < n; ++t) s = __fadd_rn(s, bf16_to_f32(__ldg(src + (int64_t)t * row_stride)));
    mean[d] = __fdiv_rn(s, (float)n);
    __syncthreads();
    const float *w = W + (int64_t)h * D * R;
    for (int e = d; e < R; e += 128) {
        float acc = 0.f;
#pragma unroll 8
        for (int k = 0; k < D; ++k) acc = __fmaf_rn(mean[k], __ldg(w + (int64_t)k * R + e), acc);
        proj[((int64_t)h * gridDim.x + b) * R + e] = acc;
    }
}

// grid (ceil(kb/64), ceil(qb/16), H), 256 threads: a 16 x 64 tile of scores, 4 per thread.
__global__ void __launch_bounds__(256) block_scores_kernel(const float *__restrict__ qh, const float *__restrict__ kh,
                                                           int qb, int kb, int R, float *__restrict__ S, int *status) {
    extern __shared__ float sm[];
    float *sq = sm;            // [16][R]
    float *sk = sm + 16 * R;   // [64][R+1]
    const int h = blockIdx.z, i0 = blockIdx.y * 16, j0 = blockIdx.x * 64, tid = threadIdx.x;
    for (int x = tid; x < 16 * R; x += 256) {
        int i = i0 + x / R;
        sq[x] = i < qb ? qh[((int64_t)h * qb + i) * R + x % R] : 0.f;
    }
    for (int x = tid; x < 64 * R; x += 256) {
        int j = j0 + x / R;
        sk[(x / R) * (R + 1) + x % R] = j < kb ? kh[((int64_t)h * kb + j) * R + x % R] : 0.f;
    }
    __syncthreads();
    const int jj = tid & 63, ib = (tid >> 6) * 4;
    const int j = j0 + jj;
    bool bad = false;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int i = i0 + ib + u;
        float acc = 0.f;
        for (int e = 0; e < R; ++e) acc = __fmaf_rn(sq[(ib + u) * R + e], sk[jj * (R + 1) + e], acc);
        if (acc == 0.f) acc = 0.f;  // -0 -> +0
        if (i < qb && j < kb) {
            bad |= !isfinite(acc);
            S[((int64_t)h * qb + i) * kb + j] = acc;
        }
    }
    if (bad) report(status, SS_DEV_NONFINITE);
}

__device__ __forceinline__ bool is_forced(int j, int block, int Lq, int Lk, int sink) {
    const int lo = j * block, hi = min(lo + block, Lk);
    return lo < sink || hi > Lk - Lq;
}

__device__ __forceinline__ uint64_t score_key(float f, int j) {
    if (f == 0.f) f = 0.f;
    uint32_t u = __float_as_uint(f);
    uint32_t o = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((uint64_t)o << 32) | (uint64_t)(0xffffffffu - (uint32_t)j);
}

// one CTA per (head, query block) row; dynamic smem: npow2 uint64 keys
__global__ void __launch_bounds__(TOPK_THREADS) select_topk_kernel(const float *__restrict__ S, int qb, int kb,
                                                                   int block, int Lq, int Lk, int sink, int extra,
                                                                   int npow2, int32_t *__restrict__ ids, int n_ids,
                                                                   uint8_t *__restrict__ mask) {
    extern __shared__ uint64_t keys[];
    __shared__ int warp_tot[TOPK_THREADS / 32];
    const int row = blockIdx.x, tid = threadIdx.x;
    const float *srow = S + (int64_t)row * kb;
    for (int j = tid; j < npow2; j += TOPK_THREADS)
        keys[j] = (j < kb && !is_forced(j, block, Lq, Lk, sink)) ? score_key(srow[j], j) : 0ull;
    __syncthreads();
    // bitonic sort, descending
    for (int size = 2; size <= npow2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int t = tid; t < npow2 / 2; t += TOPK_THREADS) {
                const int lo = 2 * t - (t & (stride - 1));
                const int hi = lo + stride;
                const bool desc = (lo & size) == 0;
                const uint64_t a = keys[lo], b = keys[hi];
                if ((a < b) == desc) {
                    keys[lo] = b;
                    keys[hi] = a;
                }
            }
            __syncthreads();
        }
    }
    const uint64_t cutoff = extra > 0 ? keys[extra - 1] : ~0ull;
    // ascending compaction: thread tid owns the contiguous range [c0, c1)
    const int per = (kb + TOPK_THREADS - 1) / TOPK_THREADS;
    const int c0 = min(kb, tid * per), c1 = min(kb, c0 + per);
    int cnt = 0;
    for (int j = c0; j < c1; ++j) {
        const bool f = is_forced(j, block, Lq, Lk, sink);
        const bool sel = f || (extra > 0 && score_key(srow[j], j) >= cutoff);
        cnt += sel;
    }
    int incl = cnt;
    const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    int off = 0;
    for (int w = 0; w < warp; ++w) off += warp_tot[w];
    int pos = off + incl - cnt;
    int32_t *out = ids + (int64_t)row * n_ids;
    for (int j = c0; j < c1; ++j) {
        const bool f = is_forced(j, block, Lq, Lk, sink);
        const bool sel = f || (extra > 0 && score_key(srow[j], j) >= cutoff);
        if (sel && pos < n_ids) out[pos++] = j;
        if (mask) mask[(int64_t)row * kb + j] = sel ? 1 : 0;
    }
}

}  // namespace router

static int g_router_configured[64] = {0};

int router_prepare(int device) {
    if (device < 0 || device >= 64) return SS_ERR_SHAPE;
    if (g_router_configured[device]) return 0;
    cudaError_t e = cudaFuncSetAttribute(router::select_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         router::MAX_KB * 8);
    if (e != cudaSuccess) return (int)e;
    g_router_configured[device] = 1;
    return 0;
}

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct RouterLayout {
    size_t qh, kh, s, total;
};

static RouterLayout router_layout(int H, int Lq, int Lk, int R, int block) {
    const size_t qb = (size_t)((Lq + block - 1) / block), kb = (size_t)((Lk + block - 1) / block);
    RouterLayout L;
    L.qh = 0;
    L.kh = align256(L.qh + 4 * (size_t)H * qb * R);
    L.s = align256(L.kh + 4 * (size_t)H * kb * R);
    L.total = align256(L.s + 4 * (size_t)H * qb * kb);
    return L;
}

static int count_forced(int Lq, int Lk, int block, int sink) {
    const int kb = (Lk + block - 1) / block;
    int n = 0;
    for (int j = 0; j < kb; ++j) {
        const int lo = j * block, hi = std::min(lo + block, Lk);
        n += (lo < sink || hi > Lk - Lq);
    }
    return n;
}

// Launch the three router kernels with the intermediate tensors at the given device addresses.
int router_launch(const void *q, const void *k, const float *wq, const float *wk, int H, int Lq, int Lk, int R,
                  int block, int sink_tokens, int extra, int32_t *ids, int n_ids, uint8_t *mask, float *scores_out,
                  float *qh, float *kh, float *S, int *status, cudaStream_t st) {
    const int qb = (Lq + block - 1) / block, kb = (Lk + block - 1) / block;
    int device;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return (int)e;
    int rc = router_prepare(device);
    if (rc) return rc;
    float *Sbuf = scores_out ? scores_out : S;
    const int64_t stride = (int64_t)H * router::D;
    router::pool_project_kernel<<<dim3(qb, H), 128, 0, st>>>((const uint16_t *)q, stride, Lq, H, block, wq, R, qh);
    router::pool_project_kernel<<<dim3(kb, H), 128, 0, st>>>((const uint16_t *)k, stride, Lk, H, block, wk, R, kh);
    const size_t sm_scores = sizeof(float) * (16 * R + 64 * (R + 1));
    router::block_scores_kernel<<<dim3((kb + 63) / 64, (qb + 15) / 16, H), 256, sm_scores, st>>>(qh, kh, qb, kb, R,
                                                                                               Sbuf, status);
    int npow2 = 1;
    while (npow2 < kb) npow2 <<= 1;
    router::select_topk_kernel<<<H * qb, router::TOPK_THREADS, (size_t)npow2 * 8, st>>>(
        Sbuf, qb, kb, block, Lq, Lk, sink_tokens, extra, npow2, ids, n_ids, mask);
    return (int)cudaGetLastError();
}

int router_check(const void *q, const void *k, const float *wq, const float *wk, int H, int Lq, int Lk, int R,
                 int block, int sink_tokens, int extra, const int32_t *ids, int n_ids) {
    if (!q || !k || !wq || !wk || !ids) return SS_ERR_POINTER;
    if (H <= 0 || Lq <= 0 || Lk < Lq || R <= 0 || R > router::MAX_R || (block != 64 && block != 128) ||
        sink_tokens < 0)
        return SS_ERR_SHAPE;
    const int kb = (Lk + block - 1) / block;
    if (kb > router::MAX_KB) return SS_ERR_SHAPE;
    const int nforced = count_forced(Lq, Lk, block, sink_tokens);
    if (extra < 0 || extra > kb - nforced) return SS_ERR_BUDGET;
    if (n_ids != nforced + extra) return SS_ERR_SHAPE;
    return 0;
}

}  // namespace ss

extern "C" int ss_router_workspace_bytes(int H, int Lq, int Lk, int R, int block, size_t *bytes) {
    if (!bytes || H <= 0 || Lq <= 0 || Lk <= 0 || R <= 0 || (block != 64 && block != 128)) return SS_ERR_SHAPE;
    *bytes = ss::router_layout(H, Lq, Lk, R, block).total;
    return 0;
}

extern "C" int ss_router(const void *q, const void *k, const float *wq, const float *wk, int H, int Lq, int Lk, int R,
                         int block, int sink_tokens, int extra, int32_t *ids, int n_ids, uint8_t *mask, float *scores,
                         void *workspace, size_t workspace_bytes, int *status, void *stream) {
    int rc = ss::router_check(q, k, wq, wk, H, Lq, Lk, R, block, sink_tokens, extra, ids, n_ids);
    if (rc) return rc;
    const ss::RouterLayout L = ss::router_layout(H, Lq, Lk, R, block);
    if (!workspace) return SS_ERR_POINTER;
    if (workspace_bytes < L.total) return SS_ERR_WORKSPACE;
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return SS_ERR_POINTER;
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    return ss::router_launch(q, k, wq, wk, H, Lq, Lk, R, block, sink_tokens, extra, ids, n_ids, mask, scores,
                             reinterpret_cast<float *>(ws + L.qh), reinterpret_cast<float *>(ws + L.kh),
                             reinterpret_cast<float *>(ws + L.s), status, static_cast<cudaStream_t>(stream));
}
