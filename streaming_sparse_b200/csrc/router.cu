// router.cu -- learned KV-block router for sm_100a in exact fp32.
//
//   1. pool_project: one CTA per SM, each pooling a tile of blocks of one head (query or key).
//      The head's [128 x R] projection is transposed into shared memory; the blocks' tokens
//      arrive by TMA, one block per 64-thread group at a time; each thread sums 2 dimensions over
//      the block's valid tokens (fp32 adds in token order, one correctly rounded divide), then
//      the block means are projected with fmaf in ascending row order. Query projections are
//      stored [H][qb][R], key projections [H][kbp][R] (kbp = kb rounded up to 4).
//      Reference: block pooling of migration/unified_router/opt19/prototype.py:11-49 (one
//      prototype = plain mean of the valid tokens) and the projection of opt8/projection.py:4-14.
//   2. score_select: eight query blocks per CTA. Every thread scores its key blocks against the
//      eight query blocks, reading its key blocks' projections straight from L2 (each value used
//      eight times); scores S[j] = <qh, kh_j> accumulate with fmaf in ascending order,
//      -0 -> +0, non-finite flagged; the order-preserving uint32 of each unforced score is kept
//      in shared memory. Then one warp per query block finds the `extra`-th largest score T
//      exactly by a 32-step bisection with warp-wide counts (keys in registers); blocks above T
//      are kept and ties at T go to the lowest block indices (ordered ballot scan). Forced blocks
//      (sink, current chunk) are always kept; ids are written ascending. Reference: the
//      block-score GEMM `_coarse` (opt16/route.py:34-47), `_chosen`/`_top` (opt16/route.py:13-24,
//      49-55), fixed_page_select (local_experiments/video_runtime_v1/fixed_page_select.py:7-21)
//      and the forced set of local_experiments/video_runtime_v1/pipeline_graph.py:140-151.
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
constexpr int PP_MAX_GROUPS = 12;    // 64-thread groups per pool_project CTA (one TMA stage each)
constexpr int WT_STRIDE = 132;       // padded row of the transposed projection in shared memory
constexpr int ROWS = 8;              // query blocks per score_select CTA (one warp each in the selection)
constexpr int SS_THREADS = 512;      // score_select threads (one key block each up to 512 key blocks)

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}

// grid (tiles_q + tiles_k, H), 64 * ng threads = ng groups of 64 (one CTA per SM). Tiles
// [0, tiles_q) pool query blocks, the rest key blocks, bg blocks per tile. Group g pools blocks
// g, g + ng, ... of the tile: the group's leader TMA-loads a block (block tokens x 128 dims of
// head h, plain rows) into the group's stage, the 64 threads sum 2 dimensions each in token
// order, the leader starts the next block's load, and the group projects the block mean (thread
// e: outputs e, e + 64) against W transposed in shared memory (rows padded to WT_STRIDE floats, so
// the float4 reads of 32 threads hit every bank the same number of times). ng stages of 16 KB keep
// about 190 KB in flight per SM. Dynamic shared memory: stages [ng][block][128] bf16,
// W^T [R][WT_STRIDE] fp32, means [ng][128] fp32, mbarriers, abort flag.
__global__ void __launch_bounds__(PP_MAX_GROUPS * 64, 1)
pool_project_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k, int H, int Lq,
                    int Lk, int block, int R, int tiles_q, int bg, const float *__restrict__ wq,
                    const float *__restrict__ wk, float *__restrict__ qh, float *__restrict__ kh, int kbp,
                    int *status) {
    extern __shared__ uint8_t smr_raw[];
    uint8_t *smr = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smr_raw) + 1023) & ~uintptr_t(1023));
    const int ng = blockDim.x / 64;
    const uint32_t stage_bytes = (uint32_t)block * D * 2;
    float *swt = reinterpret_cast<float *>(smr + ng * stage_bytes);   // [R][WT_STRIDE]
    float *smean = swt + R * WT_STRIDE;                                // [ng][128]
    uint64_t *mb = reinterpret_cast<uint64_t *>(smean + ng * D);      // full[ng]
    volatile int *abort_flag = reinterpret_cast<volatile int *>(mb + ng);
    const int h = blockIdx.y, tid = threadIdx.x, g = tid >> 6, gt = tid & 63;
    const bool isq = (int)blockIdx.x < tiles_q;
    const int tile = isq ? blockIdx.x : blockIdx.x - tiles_q;
    const int L = isq ? Lq : Lk;
    const int nb = (L + block - 1) / block;
    const int b0 = tile * bg, nblk = min(bg, nb - b0);
    const uint32_t full = smem_u32(mb + g);
    const uint32_t stage = smem_u32(smr) + g * stage_bytes;
    const CUtensorMap *tm = isq ? &tm_q : &tm_k;
    if (tid == 0) {
        *abort_flag = 0;
        for (int i = 0; i < ng; ++i) mbar_init(smem_u32(mb + i), 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (gt == 0 && g < nblk) {
        mbar_arrive_expect_tx(full, stage_bytes);
        tma_load_2d(stage, tm, h * D, (b0 + g) * block, full);
    }
    {   // W [128][R] of head h, transposed into shared memory while the first loads are in flight;
        // each thread's loads are all issued before any is stored (one round trip, not one each)
        const float *w = (isq ? wq : wk) + (size_t)h * D * R;
        const int nw = D * R, step = blockDim.x;
        for (int x0 = tid; x0 < nw; x0 += 16 * step) {
            float v[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) v[u] = x0 + u * step < nw ? __ldg(w + x0 + u * step) : 0.f;
#pragma unroll
            for (int u = 0; u < 16; ++u) {
                const int x = x0 + u * step;
                if (x < nw) swt[(x % R) * WT_STRIDE + x / R] = v[u];
            }
        }
    }
    __syncthreads();
    // Every thread of a group runs every group barrier (bar.sync is not bounded): after a failed
    // wait the work is skipped but the barriers are kept, and the shared abort flag makes the
    // remaining waits of the CTA return at once.
    bool ok = true;
    int issued = g < nblk ? 1 : 0, seen = 0;   // the leader's loads into the stage, and those waited on
    for (int it = 0; g + ng * it < nblk; ++it) {
        const int bi = g + ng * it;
        if (ok) {
            ok = mbar_wait(full, it & 1, abort_flag);
            seen = it + 1;
        }
        const int t0 = (b0 + bi) * block, n = min(block, L - t0);
        float s0 = 0.f, s1 = 0.f;
        if (ok) {
            // thread gt sums dimensions 2gt, 2gt+1 over the block's valid tokens, in token order
            const uint32_t *rows = reinterpret_cast<const uint32_t *>(smr + g * stage_bytes) + gt;
#pragma unroll 8
            for (int t = 0; t < n; ++t) {
                const uint32_t w = rows[t * (D / 2)];
                s0 = __fadd_rn(s0, bf16_lo(w));
                s1 = __fadd_rn(s1, bf16_hi(w));
            }
        }
        asm volatile("bar.sync %0, 64;" ::"r"(1 + g) : "memory");   // the stage has been read
        if (ok && gt == 0 && bi + ng < nblk) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive_expect_tx(full, stage_bytes);
            tma_load_2d(stage, tm, h * D, (b0 + bi + ng) * block, full);
            ++issued;
        }
        const float fn = (float)n;
        smean[g * D + 2 * gt] = __fdiv_rn(s0, fn);
        smean[g * D + 2 * gt + 1] = __fdiv_rn(s1, fn);
        asm volatile("bar.sync %0, 64;" ::"r"(1 + g) : "memory");
        if (ok) {
            // projection: outputs gt and gt + 64, fmaf over the 128 rows in ascending order
            const int b = b0 + bi;
            const float4 *m4 = reinterpret_cast<const float4 *>(smean + g * D);
#pragma unroll
            for (int e = gt; e < MAX_R; e += 64) {
                if (e >= R) break;
                const float4 *w4 = reinterpret_cast<const float4 *>(swt + e * WT_STRIDE);
                float acc = 0.f;
#pragma unroll 8
                for (int d4 = 0; d4 < D / 4; ++d4) {
                    const float4 mv = m4[d4], wv = w4[d4];
                    acc = __fmaf_rn(mv.x, wv.x, acc);
                    acc = __fmaf_rn(mv.y, wv.y, acc);
                    acc = __fmaf_rn(mv.z, wv.z, acc);
                    acc = __fmaf_rn(mv.w, wv.w, acc);
                }
                if (isq) qh[((size_t)h * nb + b) * R + e] = acc;
                else kh[((size_t)h * kbp + b) * R + e] = acc;
            }
        }
        asm volatile("bar.sync %0, 64;" ::"r"(1 + g) : "memory");   // smean is rewritten next block
    }
    if (*abort_flag) {
        // a copy may still be landing: the leader's last load
        volatile int never = 0;
        if (gt == 0) {
            for (int j = seen; j < issued; ++j) mbar_wait(full, j & 1, &never);
            if (g == 0) report(status, SS_DEV_TIMEOUT);
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

// Threshold of one query block's selection: T = the extra-th largest candidate key (bisection on
// the order-preserving bits) and `need` = how many keys equal to T are kept, run by one warp. NK
// keys per lane are held in registers (NK = 0: read from shared memory at every step).
template <int NK>
__device__ __forceinline__ void select_threshold(const uint32_t *mykeys, int kb, int extra, int lane, uint32_t &T,
                                                 int &need) {
    uint32_t kr[NK > 0 ? NK : 1];
#pragma unroll
    for (int u = 0; u < NK; ++u) {
        const int j = lane + 32 * u;
        kr[u] = j < kb ? mykeys[j] : 0u;
    }
    auto count = [&](uint32_t c, bool strict) -> int {
        int n = 0;
        if (NK > 0) {
            int n4[4] = {0, 0, 0, 0};   // independent partial counts keep the add chains short
#pragma unroll
            for (int u = 0; u < NK; ++u) n4[u & 3] += strict ? (kr[u] > c) : (kr[u] >= c);
            n = (n4[0] + n4[1]) + (n4[2] + n4[3]);
        } else {
            for (int j = lane; j < kb; j += 32) n += strict ? (mykeys[j] > c) : (mykeys[j] >= c);
        }
        return (int)__reduce_add_sync(0xffffffffu, (unsigned)n);
    };
    T = 0u;
    for (int bit = 31; bit >= 0; --bit) {
        const uint32_t cand = T | (1u << bit);
        if (count(cand, false) >= extra) T = cand;
    }
    need = extra - count(T, true);   // ties at T to keep, >= 1
}

// grid (ceil(qb / ROWS), H), SS_THREADS threads, ROWS = 8 query blocks per CTA.
// Phase 1: thread t scores key blocks t, t + SS_THREADS, ... against the CTA's 8 query blocks: the R
// projections of a key block are one contiguous row of kh (16 float4 loads in flight per thread),
// each value reused for the 8 query blocks, whose projections are
// read from shared memory ([R][8], two broadcast float4 per row). Scores accumulate with fmaf in
// ascending e, -0 becomes +0, non-finite scores are flagged; the order-preserving uint32 of each
// unforced score goes to shared memory (0 = not a candidate, which no finite score maps to).
// Phase 2: warp w selects for query block w: the `extra`-th largest key T (keys in registers for
// kb <= 1024), blocks above T kept, ties at T to the lowest block indices (ordered ballot scan),
// forced blocks always kept, ids written ascending.
__global__ void __launch_bounds__(SS_THREADS) score_select_kernel(const float *__restrict__ qh, const float *__restrict__ kh,
                                                           int qb, int kb, int kbp, int R, int block, int Lq, int Lk,
                                                           int sink, int extra, int32_t *__restrict__ ids, int n_ids,
                                                           uint8_t *__restrict__ mask, float *__restrict__ scores,
                                                           int *status) {
    extern __shared__ __align__(16) uint8_t smr[];
    float *sqT = reinterpret_cast<float *>(smr);                       // [R][ROWS]
    uint32_t *keys = reinterpret_cast<uint32_t *>(sqT + R * ROWS);     // [ROWS][kbp]
    const int h = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int i0 = blockIdx.x * ROWS;
    for (int x = tid; x < ROWS * R; x += blockDim.x) {
        const int ii = x / R, e = x % R;
        sqT[e * ROWS + ii] = i0 + ii < qb ? qh[((size_t)h * qb + i0 + ii) * R + e] : 0.f;
    }
    __syncthreads();
    static_assert(ROWS == 8, "two float4 of query projections per row");
    const float4 *q4 = reinterpret_cast<const float4 *>(sqT);
    bool bad = false;
    for (int j = tid; j < kb; j += blockDim.x) {
        float acc[ROWS];
#pragma unroll
        for (int r = 0; r < ROWS; ++r) acc[r] = 0.f;
        const float4 *krow = reinterpret_cast<const float4 *>(kh + ((size_t)h * kbp + j) * R);
        for (int e0 = 0; e0 < R; e0 += 64) {   // R is a multiple of 16
            float4 kv[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) kv[u] = e0 + 4 * u < R ? __ldg(krow + e0 / 4 + u) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int u = 0; u < 64; ++u) {
                if (e0 + u >= R) break;
                const float k = (u & 3) == 0 ? kv[u >> 2].x : (u & 3) == 1 ? kv[u >> 2].y : (u & 3) == 2 ? kv[u >> 2].z : kv[u >> 2].w;
                const float4 qa = q4[2 * (e0 + u)], qb4 = q4[2 * (e0 + u) + 1];
                acc[0] = __fmaf_rn(qa.x, k, acc[0]);
                acc[1] = __fmaf_rn(qa.y, k, acc[1]);
                acc[2] = __fmaf_rn(qa.z, k, acc[2]);
                acc[3] = __fmaf_rn(qa.w, k, acc[3]);
                acc[4] = __fmaf_rn(qb4.x, k, acc[4]);
                acc[5] = __fmaf_rn(qb4.y, k, acc[5]);
                acc[6] = __fmaf_rn(qb4.z, k, acc[6]);
                acc[7] = __fmaf_rn(qb4.w, k, acc[7]);
            }
        }
        const bool forced = is_forced(j, block, Lq, Lk, sink);
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
            if (i0 + r >= qb) break;
            float a = acc[r];
            if (a == 0.f) a = 0.f;  // -0 -> +0
            bad |= !isfinite(a);
            if (scores) scores[((size_t)h * qb + i0 + r) * kb + j] = a;
            keys[(size_t)r * kbp + j] = forced ? 0u : ordered_bits(a);
        }
    }
    if (bad) report(status, SS_DEV_NONFINITE);
    __syncthreads();
    const int i = i0 + warp;
    if (warp >= ROWS || i >= qb) return;
    const uint32_t *mykeys = keys + (size_t)warp * kbp;
    uint32_t T = 0xffffffffu;
    int need = 0;
    if (extra > 0) {
        if (kb <= 256) select_threshold<8>(mykeys, kb, extra, lane, T, need);
        else if (kb <= 512) select_threshold<16>(mykeys, kb, extra, lane, T, need);
        else if (kb <= 1024) select_threshold<32>(mykeys, kb, extra, lane, T, need);
        else select_threshold<0>(mykeys, kb, extra, lane, T, need);
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

// pool_project: groups per CTA (one 16 KB / 32 KB stage each) that fit beside W^T and the means
static int pp_groups(int R, int block) {
    const size_t fixed = 1024 + (size_t)R * router::WT_STRIDE * 4 + 64;
    const size_t per = (size_t)block * router::D * 2 + router::D * 4 + 8;
    const size_t budget = 227 * 1024;
    int ng = budget > fixed ? (int)((budget - fixed) / per) : 0;
    return std::min(ng, router::PP_MAX_GROUPS);
}

static size_t pp_smem(int R, int block, int ng) {
    return 1024 + (size_t)ng * block * router::D * 2 + (size_t)R * router::WT_STRIDE * 4 + (size_t)ng * router::D * 4 +
           8 * (size_t)ng + 16;
}

static size_t select_smem(int kb, int R) {
    return (size_t)R * router::ROWS * 4 + (size_t)router::ROWS * kb * 4 + 16;
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

// key-block count rounded up to a multiple of 4: the stride of the per-query-block key rows of
// score_select in shared memory and the row count of the key projections
static int kb_padded(int kb) { return (kb + 3) & ~3; }

struct RouterLayout {
    size_t qh, kh, total;
};

static RouterLayout router_layout(int H, int Lq, int Lk, int R, int block) {
    const size_t qb = (size_t)((Lq + block - 1) / block);
    const size_t kbp = (size_t)kb_padded((Lk + block - 1) / block);
    RouterLayout L;
    L.qh = 0;
    L.kh = align256(L.qh + 4 * (size_t)H * qb * R);
    L.total = align256(L.kh + 4 * (size_t)H * R * kbp);
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
    float *qh = reinterpret_cast<float *>(ws + L.qh), *kh = reinterpret_cast<float *>(ws + L.kh);
    // blocks per pool_project tile: the fewest that keep the grid within one wave
    int nsm = 148;
    if (cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) nsm = 148;
    int bg = std::max(1, (H * (qb + kb) + nsm - 1) / nsm);
    while (H * ((qb + bg - 1) / bg + (kb + bg - 1) / bg) > nsm && bg < std::max(qb, kb)) ++bg;
    const int tq = (qb + bg - 1) / bg, tk = (kb + bg - 1) / bg;
    const int ng = pp_groups(R, block);
    CUtensorMap tmq, tmk;
    const uint64_t row_bytes = (uint64_t)H * router::D * 2;
    if (encode_tmap_2d_bf16_rows(&tmq, q, (uint64_t)H * router::D, (uint64_t)Lq, row_bytes, router::D, (uint32_t)block))
        return SS_ERR_DRIVER;
    if (encode_tmap_2d_bf16_rows(&tmk, k, (uint64_t)H * router::D, (uint64_t)Lk, row_bytes, router::D, (uint32_t)block))
        return SS_ERR_DRIVER;
    router::pool_project_kernel<<<dim3(tq + tk, H), 64 * ng, pp_smem(R, block, ng), st>>>(
        tmq, tmk, H, Lq, Lk, block, R, tq, bg, wq, wk, qh, kh, kbp, status);
    router::score_select_kernel<<<dim3((qb + router::ROWS - 1) / router::ROWS, H), router::SS_THREADS,
                                  select_smem(kbp, R), st>>>(qh, kh, qb, kb, kbp, R, block, Lq, Lk, sink_tokens,
                                                             extra, ids, n_ids, mask, scores, status);
    return (int)cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------
// ss_router_noalloc: the router with its intermediates in a static device array.
// ---------------------------------------------------------------------------------------------
// For callers that cannot allocate device memory per call. Every call on a device shares this
// one array (it keeps the previous call's contents; nothing in it has to start at zero, because
// each call writes every value it reads), so calls that may overlap on the GPU -- two streams,
// or two host threads -- race and must be serialised by the caller.
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
