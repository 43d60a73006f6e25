// router.cu -- learned KV-block router for sm_100a in exact fp32.
//
//   1. pool_project: one CTA per SM, each pooling a tile of blocks of one head (query or key).
//      The head's [128 x R] projection is bulk-copied into shared memory first; the blocks' tokens
//      arrive by TMA, one block per warp at a time; each lane sums 4 dimensions over the block's
//      valid tokens (fp32 adds in token order, one correctly rounded divide), then the means of
//      two blocks are projected together with fmaf in ascending row order (f32x2 instructions:
//      two independent IEEE operations each, so every value is the scalar chain's). Query projections are
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
constexpr int PP_MAX_WARPS = 16;     // warps per pool_project CTA (one TMA stage each)
constexpr int ROWS = 8;              // query blocks per score_select CTA (one warp each in the selection)
constexpr int SS_THREADS = 512;      // score_select threads (one key block each up to 512 key blocks)

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}

__device__ __forceinline__ uint64_t pack2(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float2 unpack2(uint64_t r) {
    float2 v;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(r));
    return v;
}
// two independent IEEE fp32 operations (round to nearest) on the halves of a register pair
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

// grid (tiles_q + tiles_k, H), 32 * nw threads (one CTA per SM). Tiles [0, tiles_q) pool query
// blocks [0, qb), the rest key blocks [kj0, kj1), bg blocks per tile; key block j goes to row
// h * kh_ld + j of kh, so a caller can keep the history's rows from an earlier call and pool only
// the blocks after them. Thread 0 first starts one bulk copy of the
// head's projection W [128][R] into shared memory (ahead of the token loads, so the small copy is
// not queued behind megabytes of them). Warp w owns one TMA stage and pools blocks w, w + nw, ...
// of the tile in pairs: lane 0 TMA-loads a block (block tokens x 128 dims of head h, plain rows),
// lane l sums dimensions 4l..4l+3 over the valid tokens in token order (two f32x2 adds per token),
// lane 0 reloads the stage with the warp's next block, and once both blocks of a pair are summed
// the warp projects both means with one pass over W (lane l: outputs 2l, 2l+1 (+64 ...), one
// f32x2 fma per block per row, rows ascending). Dynamic shared memory: stages [nw][block][128]
// bf16, W [128][R] fp32, means [nw][128] x {A, A, B, B} fp32, mbarriers full[nw] and w, abort.
__global__ void __launch_bounds__(PP_MAX_WARPS * 32, 1)
pool_project_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k, int H, int Lq,
                    int Lk, int block, int R, int tiles_q, int bg, const float *__restrict__ wq,
                    const float *__restrict__ wk, float *__restrict__ qh, float *__restrict__ kh, int kh_ld,
                    int kj0, int kj1, int krow0, int *status) {
    extern __shared__ uint8_t smr_raw[];
    uint8_t *smr = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smr_raw) + 1023) & ~uintptr_t(1023));
    const int nw = blockDim.x / 32;
    const uint32_t stage_bytes = (uint32_t)block * D * 2;
    float *sw = reinterpret_cast<float *>(smr + nw * stage_bytes);   // [128][R]
    float4 *smean = reinterpret_cast<float4 *>(sw + D * R);          // [nw][128]
    uint64_t *mb = reinterpret_cast<uint64_t *>(smean + nw * D);     // full[nw], w
    volatile int *abort_flag = reinterpret_cast<volatile int *>(mb + nw + 1);
    const int h = blockIdx.y, tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
    const bool isq = (int)blockIdx.x < tiles_q;
    const int tile = isq ? blockIdx.x : blockIdx.x - tiles_q;
    const int L = isq ? Lq : Lk;
    const int nb = (L + block - 1) / block;
    const int b0 = (isq ? 0 : kj0) + tile * bg, nblk = min(bg, (isq ? nb : kj1) - b0);
    const uint32_t full = smem_u32(mb + w), wbar = smem_u32(mb + nw);
    const uint32_t stage = smem_u32(smr) + w * stage_bytes;
    const uint8_t *stage_p = smr + w * stage_bytes;
    float4 *md = smean + w * D;
    const CUtensorMap *tm = isq ? &tm_q : &tm_k;
    const int row0 = isq ? 0 : krow0;   // window row of the tensor map's first row
    if (tid == 0) {
        *abort_flag = 0;
        for (int i = 0; i <= nw; ++i) mbar_init(smem_u32(mb + i), 1);
        fence_mbar_init();
        const uint32_t wbytes = (uint32_t)(D * R * 4);
        mbar_arrive_expect_tx(wbar, wbytes);
        bulk_g2s(smem_u32(sw), (isq ? wq : wk) + (size_t)h * D * R, wbytes, wbar);
    }
    __syncthreads();
    int issued = 0, seen = 0;   // lane 0's loads into the stage, and those waited on
    if (lane == 0 && w < nblk) {
        mbar_arrive_expect_tx(full, stage_bytes);
        tma_load_2d(stage, tm, h * D, (b0 + w) * block - row0, full);
        issued = 1;
    }
    bool ok = true, w_seen = false;
    // sum block bi from the stage (the k-th load), then reload the stage with block `next`
    auto pool = [&](int bi, int k, int next, bool hi_half) {
        if (ok) {
            ok = mbar_wait(full, k & 1, abort_flag);
            seen = k + 1;
        }
        const int t0 = (b0 + bi) * block, n = min(block, L - t0);
        uint64_t s01 = 0, s23 = 0;
        if (ok) {
            const uint2 *rows = reinterpret_cast<const uint2 *>(stage_p) + lane;
#pragma unroll 8
            for (int t = 0; t < n; ++t) {
                const uint2 v = rows[t * (D / 4)];
                s01 = add2(s01, pack2(bf16_lo(v.x), bf16_hi(v.x)));
                s23 = add2(s23, pack2(bf16_lo(v.y), bf16_hi(v.y)));
            }
        }
        __syncwarp();
        if (ok && lane == 0 && next < nblk) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive_expect_tx(full, stage_bytes);
            tma_load_2d(stage, tm, h * D, (b0 + next) * block - row0, full);
            ++issued;
        }
        const float fn = (float)n;
        const float2 a = unpack2(s01), b = unpack2(s23);
        const float m[4] = {__fdiv_rn(a.x, fn), __fdiv_rn(a.y, fn), __fdiv_rn(b.x, fn), __fdiv_rn(b.y, fn)};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float2 *p = reinterpret_cast<float2 *>(md + 4 * lane + i) + (hi_half ? 1 : 0);
            *p = make_float2(m[i], m[i]);
        }
    };
    int k = 0;
    for (int bA = w; bA < nblk; bA += 2 * nw, k += 2) {
        const int bB = bA + nw;
        const bool hasB = bB < nblk;
        pool(bA, k, bB, false);
        if (hasB) pool(bB, k + 1, bB + nw, true);
        if (!w_seen && ok) {
            ok = mbar_wait(wbar, 0, abort_flag);
            w_seen = ok;
        }
        __syncwarp();
        if (ok) {
            // projection of both means: fmaf over the 128 rows in ascending order per output
            for (int e = 2 * lane; e < R; e += 64) {
                const float *wc = sw + e;
                uint64_t accA = 0, accB = 0;
#pragma unroll 8
                for (int d = 0; d < D; ++d) {
                    const float4 mv = md[d];
                    const uint64_t wv = *reinterpret_cast<const uint64_t *>(wc + d * R);
                    accA = fma2(pack2(mv.x, mv.y), wv, accA);
                    accB = fma2(pack2(mv.z, mv.w), wv, accB);
                }
                const float2 ra = unpack2(accA), rb = unpack2(accB);
                float *dst = isq ? qh + ((size_t)h * nb + b0) * R : kh + ((size_t)h * kh_ld + b0) * R;
                *reinterpret_cast<float2 *>(dst + (size_t)bA * R + e) = ra;
                if (hasB) *reinterpret_cast<float2 *>(dst + (size_t)bB * R + e) = rb;
            }
        }
        __syncwarp();   // the means are rewritten by the next pair
    }
    if (*abort_flag) {
        // copies may still be landing: W, and lane 0's last load
        volatile int never = 0;
        if (tid == 0 && !w_seen) mbar_wait(wbar, 0, &never);
        if (lane == 0) {
            for (int j = seen; j < issued; ++j) mbar_wait(full, j & 1, &never);
            if (w == 0) report(status, SS_DEV_TIMEOUT);
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
                                                           int kh_ld, int qb, int kb, int kbp, int R, int block, int Lq, int Lk,
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
        const float4 *krow = reinterpret_cast<const float4 *>(kh + ((size_t)h * kh_ld + j) * R);
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

// pool_project: warps per CTA (one 16 KB / 32 KB stage and 2 KB of means each) beside W
static int pp_warps(int R, int block) {
    const size_t fixed = 1024 + (size_t)R * router::D * 4 + 64;
    const size_t per = (size_t)block * router::D * 2 + router::D * 16 + 8;
    const size_t budget = 227 * 1024;
    int nw = budget > fixed ? (int)((budget - fixed) / per) : 0;
    return std::min(nw, router::PP_MAX_WARPS);
}

static size_t pp_smem(int R, int block, int nw) {
    return 1024 + (size_t)nw * block * router::D * 2 + (size_t)R * router::D * 4 + (size_t)nw * router::D * 16 +
           8 * ((size_t)nw + 1) + 16;
}

static size_t select_smem(int kb, int R) {
    return (size_t)R * router::ROWS * 4 + (size_t)router::ROWS * kb * 4 + 16;
}

static int g_router_configured[SS_MAX_DEVICES] = {0};
static void *g_router_ctx[SS_MAX_DEVICES] = {nullptr};
static int g_router_sms[SS_MAX_DEVICES] = {0};
static std::mutex g_router_mutex;

// Per (device, context): the kernels' shared-memory attributes and the SM count.
int router_prepare(int device) {
    if (device < 0 || device >= SS_MAX_DEVICES) return SS_ERR_DEVICE;
    void *ctx = nullptr;
    int rc = current_context(&ctx);
    if (rc) return rc;
    std::lock_guard<std::mutex> lock(g_router_mutex);
    if (g_router_configured[device] && g_router_ctx[device] == ctx) return 0;
    cudaError_t e = cudaFuncSetAttribute(router::pool_project_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         227 * 1024);
    if (e != cudaSuccess) return (int)e;
    e = cudaFuncSetAttribute(router::score_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return (int)e;
    int nsm = 0;
    e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess) return (int)e;
    g_router_sms[device] = nsm;
    g_router_ctx[device] = ctx;
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

// Pool and project query blocks [0, qb) (when with_q) and key blocks [kj0, kj1) in one launch of
// pool_project_kernel: blocks per CTA tile chosen as the fewest that keep the grid within one wave.
static int pool_launch(int device, const void *q, const void *k, const float *wq, const float *wk, int H, int Lq,
                       int Lk, int R, int block, bool with_q, float *qh, float *kh, int kh_ld, int kj0, int kj1,
                       int *status, cudaStream_t st, int krow0 = 0) {
    const int qb = with_q ? (Lq + block - 1) / block : 0, nk = kj1 - kj0;
    if (qb + nk <= 0) return 0;
    const int nsm = g_router_sms[device] > 0 ? g_router_sms[device] : 148;
    int bg = std::max(1, (H * (qb + nk) + nsm - 1) / nsm);
    while (H * ((qb + bg - 1) / bg + (nk + bg - 1) / bg) > nsm && bg < std::max(qb, nk)) ++bg;
    const int tq = (qb + bg - 1) / bg, tk = (nk + bg - 1) / bg;
    const int nw = pp_warps(R, block);
    CUtensorMap tmq, tmk;
    const uint64_t row_bytes = (uint64_t)H * router::D * 2;
    if (encode_tmap_2d_bf16_rows(&tmk, k, (uint64_t)H * router::D, (uint64_t)(Lk - krow0), row_bytes, router::D,
                                 (uint32_t)block))
        return SS_ERR_DRIVER;
    if (with_q) {
        if (encode_tmap_2d_bf16_rows(&tmq, q, (uint64_t)H * router::D, (uint64_t)Lq, row_bytes, router::D,
                                     (uint32_t)block))
            return SS_ERR_DRIVER;
    } else {
        tmq = tmk;   // no query tiles: the map is never read
    }
    router::pool_project_kernel<<<dim3(tq + tk, H), 32 * nw, pp_smem(R, block, nw), st>>>(
        tmq, tmk, H, Lq, Lk, block, R, tq, bg, wq, wk, qh, kh, kh_ld, kj0, kj1, krow0, status);
    return (int)cudaGetLastError();
}

// Launch the router kernels with the query projections in `ws` (router_workspace_size bytes,
// 256-byte aligned). The key projections go to the workspace too (kh_ext == nullptr), or to the
// caller's table kh_ext [H][kh_ld][R], whose rows [0, n_cached) already hold this window's first
// n_cached key blocks: only blocks [n_cached, kb) are pooled.
int router_launch(const void *q, const void *k, const float *wq, const float *wk, int H, int Lq, int Lk, int R,
                  int block, int sink_tokens, int extra, int32_t *ids, int n_ids, uint8_t *mask, float *scores,
                  uint8_t *ws, int *status, cudaStream_t st, float *kh_ext = nullptr, int kh_ld_ext = 0,
                  int n_cached = 0, int krow0 = 0) {
    const int qb = (Lq + block - 1) / block, kb = (Lk + block - 1) / block, kbp = kb_padded(kb);
    int device;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return (int)e;
    int rc = router_prepare(device);
    if (rc) return rc;
    const RouterLayout L = router_layout(H, Lq, Lk, R, block);
    float *qh = reinterpret_cast<float *>(ws + L.qh);
    float *kh = kh_ext ? kh_ext : reinterpret_cast<float *>(ws + L.kh);
    const int kh_ld = kh_ext ? kh_ld_ext : kbp;
    rc = pool_launch(device, q, k, wq, wk, H, Lq, Lk, R, block, true, qh, kh, kh_ld, kh_ext ? n_cached : 0, kb,
                     status, st, krow0);
    if (rc) return rc;
    router::score_select_kernel<<<dim3((qb + router::ROWS - 1) / router::ROWS, H), router::SS_THREADS,
                                  select_smem(kbp, R), st>>>(qh, kh, kh_ld, qb, kb, kbp, R, block, Lq, Lk, sink_tokens,
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
static uint8_t *g_router_scratch_addr[SS_MAX_DEVICES] = {nullptr};
static void *g_router_scratch_ctx[SS_MAX_DEVICES] = {nullptr};

// Device address of g_router_scratch on the current device. In host code the symbol is only a
// host-side stand-in; a kernel given it would fault (or, where the GPU can reach host memory,
// silently use the wrong memory), so the address is looked up with the device current and kept
// together with the context it belongs to. A new context on the device (after cudaDeviceReset the
// module is loaded again and the array may sit elsewhere) triggers a fresh lookup.
static int router_scratch_address(int device, uint8_t **addr) {
    void *ctx = nullptr;
    int rc = current_context(&ctx);
    if (rc) return rc;
    std::lock_guard<std::mutex> lock(g_router_scratch_mutex);
    if (!g_router_scratch_addr[device] || g_router_scratch_ctx[device] != ctx) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_router_scratch);
        if (e != cudaSuccess) return (int)e;
        if (!p) return SS_ERR_POINTER;
        g_router_scratch_addr[device] = static_cast<uint8_t *>(p);
        g_router_scratch_ctx[device] = ctx;
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
    if (device < 0 || device >= SS_MAX_DEVICES) return SS_ERR_DEVICE;
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

extern "C" int ss_router_pool_keys(const void *k, const float *wk, int H, int Lk, int R, int block, int j0, int j1,
                                   float *kh, int kh_rows, int *status, void *stream) {
    using namespace ss;
    if (!k || !wk || !kh) return SS_ERR_POINTER;
    if (H <= 0 || H > 65535 || Lk <= 0 || R <= 0 || R > router::MAX_R || (R % 16) || (block != 64 && block != 128))
        return SS_ERR_SHAPE;
    const int kb = (Lk + block - 1) / block;
    if (j0 < 0 || j1 < j0 || j1 > kb || kh_rows < kb) return SS_ERR_SHAPE;
    if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(wk) | reinterpret_cast<uintptr_t>(kh)) & 15u)
        return SS_ERR_POINTER;
    int device;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return (int)e;
    int rc = router_prepare(device);
    if (rc) return rc;
    return pool_launch(device, nullptr, k, nullptr, wk, H, 0, Lk, R, block, false, nullptr, kh, kh_rows, j0, j1,
                       status, static_cast<cudaStream_t>(stream));
}

extern "C" int ss_router_cached(const void *q, const void *k, int k_row0, const float *wq, const float *wk, int H,
                                int Lq, int Lk, int R, int block, int sink_tokens, int extra, float *kh, int kh_rows,
                                int n_cached, int32_t *ids, int n_ids, uint8_t *mask, float *scores, void *workspace,
                                size_t workspace_bytes, int *status, void *stream) {
    int rc = ss::router_check(q, k, wq, wk, H, Lq, Lk, R, block, sink_tokens, extra, ids, n_ids);
    if (rc) return rc;
    if (!workspace || !kh) return SS_ERR_POINTER;
    const int kb = (Lk + block - 1) / block;
    if (kh_rows < kb || n_cached < 0 || n_cached > kb) return SS_ERR_SHAPE;
    if (k_row0 < 0 || k_row0 > n_cached * block || k_row0 >= Lk) return SS_ERR_SHAPE;
    if (workspace_bytes < ss::router_workspace_size(H, Lq, Lk, R, block)) return SS_ERR_WORKSPACE;
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) || (reinterpret_cast<uintptr_t>(kh) & 15u))
        return SS_ERR_POINTER;
    return ss::router_launch(q, k, wq, wk, H, Lq, Lk, R, block, sink_tokens, extra, ids, n_ids, mask, scores,
                             static_cast<uint8_t *>(workspace), status, static_cast<cudaStream_t>(stream), kh,
                             kh_rows, n_cached, k_row0);
}
