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
                    int kj0, int kj1, int krow0, KvRing ring_arg, int *status) {
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
    const KvRing ring = ring_arg.resolved();
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
    // a block arrives as block / 64 boxes of 64 rows, each from its sub-block's physical row
    auto load_block = [&](int bi) {
        mbar_arrive_expect_tx(full, stage_bytes);
        for (int sb = 0; sb < block / 64; ++sb) {
            const int t = (b0 + bi) * block + 64 * sb;
            tma_load_2d(stage + (uint32_t)sb * 64 * D * 2, tm, h * D, (isq ? t : ring.sub_row(t)) - row0, full);
        }
    };
    if (lane == 0 && w < nblk) {
        load_block(w);
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
            load_block(next);
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
// keys per lane are held in registers (NK = 0: read from shared memory at every step). The search
// stops early once exactly `extra` keys are >= the candidate: T is then not necessarily a key, but
// {key >= T} is the same `extra` keys the full search keeps (its T is their minimum, with all of
// its ties among them).
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
        const int c = count(cand, false);
        if (c >= extra) {
            T = cand;
            if (c == extra) break;   // exactly `extra` keys >= cand: they are the selection, no tie across it
        }
    }
    need = extra - count(T, true);   // ties at T to keep (all keys equal to T when the search stopped early)
}

// Exclusive prefix sum of v over the warp's lanes (and the total in *total).
__device__ __forceinline__ int warp_exclusive_scan(int v, int lane, int *total) {
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    *total = __shfl_sync(0xffffffffu, x, 31);
    return x - v;
}

// select_threshold with the keys per lane chosen by the key-block count.
__device__ __forceinline__ void find_threshold(const uint32_t *mykeys, int kb, int extra, int lane, uint32_t &T,
                                               int &need) {
    if (kb <= 256) select_threshold<8>(mykeys, kb, extra, lane, T, need);
    else if (kb <= 512) select_threshold<16>(mykeys, kb, extra, lane, T, need);
    else if (kb <= 1024) select_threshold<32>(mykeys, kb, extra, lane, T, need);
    else select_threshold<0>(mykeys, kb, extra, lane, T, need);
}

// One query block's ids, run by one warp: the ascending compaction of forced blocks, keys above
// T and the first `need` keys equal to T (lowest block indices first) into out[0, n_ids); mrow
// (optional) receives the 0/1 selection of every key block.
__device__ __forceinline__ void write_selection(const uint32_t *mykeys, int kb, int extra, uint32_t T, int need,
                                                int lane, int block, int Lq, int Lk, int sink, int32_t *out, int n_ids,
                                                uint8_t *mrow) {
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
        if (mrow && j < kb) mrow[j] = sel ? 1 : 0;
        pos += __popc(bal);
    }
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
    if (extra > 0) find_threshold(mykeys, kb, extra, lane, T, need);
    write_selection(mykeys, kb, extra, T, need, lane, block, Lq, Lk, sink, ids + ((size_t)h * qb + i) * n_ids, n_ids,
                    mask ? mask + ((size_t)h * qb + i) * kb : nullptr);
}

// ---------------------------------------------------------------------------------------------
// Fast mode: the score GEMM on tcgen05, the exact scores only where the selection could differ.
// ---------------------------------------------------------------------------------------------
// Every score S = <qh_i, kh_j> is first computed on the tensor cores from the split operands
// x = hi + lo (hi = x with its 13 low mantissa bits cleared, exact in tf32; lo = x - hi, exact in
// fp32) as lo.hi + hi.lo + hi.hi (kind::tf32, fp32 accumulate), which leaves out lo.lo and the
// truncation of lo: |fast - S| <= 3 * 2^-20 * sum|q_e k_e| from the split, plus the accumulation's
// own rounding (at most one 2^-23-relative truncation of the running sum per K=8 instruction,
// 24 instructions for R = 64: below 2^-15 * sum|q_e k_e|). The exact mode's chain of R fmaf is
// within R * 2^-24 * sum|q_e k_e| of S. With sum|q_e k_e| <= |q| |k_j| (Cauchy-Schwarz), every
// exact score lies within
//     eps_j = FAST_BOUND * |q| * |k_j| + FAST_ABS,   FAST_BOUND = 2^-13 (over 3x the sum above),
// of its fast score (FAST_ABS covers tf32 denormals flushed to zero). A query block's selection
// from the fast scores is therefore the exact mode's whenever its threshold T is not tied and
// min over selected (fast - eps) > max over the unselected candidates (fast + eps): then every
// exact score of a selected block exceeds every exact score of an unselected one. Any other
// query block (and any with a non-finite value) is scored again in exact fp32 with the exact
// mode's arithmetic and selected by the exact mode's code, so the ids are bit-identical to it.
constexpr float FAST_BOUND = 1.0f / 8192.0f;
constexpr float FAST_ABS = 7.8886091e-31f;   // 2^-100
constexpr int TC_TILE = 128;                 // query blocks (M) and key blocks (N) of a score tile
constexpr uint32_t TC_REGION = TC_TILE * 128;   // one 128-byte K slice (32 fp32) of a 128-row tile
constexpr int FAST_WARPS = 4;                // query blocks (one warp each) per select_fast CTA

__device__ __forceinline__ void mma_tf32_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Instruction descriptor for kind::tf32 with fp32 D, both operands K-major.
__host__ __device__ constexpr uint32_t idesc_tf32_f32(int M, int N) {
    return (1u << 4)                       // D format: f32
           | (2u << 7)                     // A format: tf32
           | (2u << 10)                    // B format: tf32
           | ((uint32_t)(N >> 3) << 17)    // N / 8
           | ((uint32_t)(M >> 4) << 24);   // M / 16
}

__device__ __forceinline__ void split_tf32(float4 x, float4 &hi, float4 &lo) {
    hi.x = __uint_as_float(__float_as_uint(x.x) & 0xffffe000u);
    hi.y = __uint_as_float(__float_as_uint(x.y) & 0xffffe000u);
    hi.z = __uint_as_float(__float_as_uint(x.z) & 0xffffe000u);
    hi.w = __uint_as_float(__float_as_uint(x.w) & 0xffffe000u);
    lo = make_float4(x.x - hi.x, x.y - hi.y, x.z - hi.z, x.w - hi.w);
}

// grid (kbr / 64, ceil(qb / 128), H), TC_THREADS threads: the fast scores of query blocks
// [m0, m0 + 128) x key blocks [n0, n0 + 64) of head h into sfast [H][qb][kbr], and (from the first
// query tile) the norms |kh_j| into kn [H][kbr].
//   1. cp.async copies every 16-byte chunk of the fp32 projections straight to its place in the
//      UMMA K-major 128-byte-swizzle layout (a tile is R / 32 regions of rows x 128 B; chunk c of
//      row r sits at chunk c ^ (r & 7)); rows past qb / kb are zero-filled. All copies are in
//      flight together.
//   2. Each thread splits the chunks it copied: hi in place, lo = x - hi to the lo tile.
//   3. One elected thread issues the 3 * R / 8 MMAs (M = 128, N = 64, K = 8) into a 64-column
//      TMEM accumulator.
//   4. Warp w reads TMEM lanes 32 (w % 4) .. +31, columns 32 (w / 4) .. +31, into a padded
//      staging tile in the (now free) A tiles' shared memory; thread r < 128 then sends row r
//      (256 B) to sfast with one bulk copy.
constexpr int TC_THREADS = 256;
constexpr int TC_N = 64;                             // key blocks per score tile
constexpr uint32_t TC_STAGE_ROW = TC_N * 4 + 16;     // padded staging row: conflict-free 16-byte stores

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}

template <int R>
__global__ void __launch_bounds__(TC_THREADS, 1)
score_tc_kernel(const float *__restrict__ qh, const float *__restrict__ kh, int kh_ld, int qb, int kb, int kbr,
                float *__restrict__ sfast, float *__restrict__ kn, int *status) {
    constexpr int NREG = R / 32, C4N = R / 4;
    constexpr uint32_t A_BYTES = NREG * TC_TILE * 128, B_BYTES = NREG * TC_N * 128;
    constexpr uint32_t B_REGION = TC_N * 128;
    extern __shared__ uint8_t smr_raw[];
    uint8_t *smr = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smr_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *a_hi = smr, *a_lo = smr + A_BYTES, *b_hi = smr + 2 * A_BYTES, *b_lo = smr + 2 * A_BYTES + B_BYTES;
    uint64_t *bar = reinterpret_cast<uint64_t *>(smr + 2 * A_BYTES + 2 * B_BYTES);
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bar + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(bar + 2);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int h = blockIdx.z, m0 = blockIdx.y * TC_TILE, n0 = blockIdx.x * TC_N;
    if (tid == 0) {
        mbar_init(smem_u32(bar), 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(tslot), TC_N);
        tmem_relinquish();
    }
    // 1. chunk x of the A tile (x < 128 * C4N) is row x / C4N, float4 x % C4N; then the B tile
    constexpr int NA = TC_TILE * C4N / TC_THREADS, NB = TC_N * C4N / TC_THREADS;
    const float4 *q4 = reinterpret_cast<const float4 *>(qh) + (size_t)h * qb * C4N;
    const float4 *k4 = reinterpret_cast<const float4 *>(kh) + (size_t)h * kh_ld * C4N;
    auto a_off = [](int row, int c4) -> uint32_t {
        return (uint32_t)(c4 >> 3) * (TC_TILE * 128) + (uint32_t)row * 128 + ((uint32_t)((c4 & 7) ^ (row & 7)) << 4);
    };
    auto b_off = [](int row, int c4) -> uint32_t {
        return (uint32_t)(c4 >> 3) * B_REGION + (uint32_t)row * 128 + ((uint32_t)((c4 & 7) ^ (row & 7)) << 4);
    };
#pragma unroll
    for (int u = 0; u < NA; ++u) {
        const int x = tid + u * TC_THREADS, row = x / C4N, c4 = x % C4N;
        const bool in = m0 + row < qb;
        cp_async16(smem_u32(a_hi) + a_off(row, c4), q4 + (size_t)(in ? m0 + row : 0) * C4N + c4, in ? 16u : 0u);
    }
#pragma unroll
    for (int u = 0; u < NB; ++u) {
        const int x = tid + u * TC_THREADS, row = x / C4N, c4 = x % C4N;
        const bool in = n0 + row < kb;
        cp_async16(smem_u32(b_hi) + b_off(row, c4), k4 + (size_t)(in ? n0 + row : 0) * C4N + c4, in ? 16u : 0u);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    // 2. split the chunks this thread copied (its own writes: no barrier needed before)
#pragma unroll
    for (int u = 0; u < NA; ++u) {
        const int x = tid + u * TC_THREADS;
        const uint32_t off = a_off(x / C4N, x % C4N);
        float4 hi, lo;
        split_tf32(*reinterpret_cast<const float4 *>(a_hi + off), hi, lo);
        *reinterpret_cast<float4 *>(a_hi + off) = hi;
        *reinterpret_cast<float4 *>(a_lo + off) = lo;
    }
#pragma unroll
    for (int u = 0; u < NB; ++u) {
        const int x = tid + u * TC_THREADS, row = x / C4N;
        const uint32_t off = b_off(row, x % C4N);
        const float4 v = *reinterpret_cast<const float4 *>(b_hi + off);
        float4 hi, lo;
        split_tf32(v, hi, lo);
        *reinterpret_cast<float4 *>(b_hi + off) = hi;
        *reinterpret_cast<float4 *>(b_lo + off) = lo;
        float ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, v.w * v.w)));
#pragma unroll
        for (int o = C4N >> 1; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (blockIdx.y == 0 && x % C4N == 0) kn[(size_t)h * kbr + n0 + row] = sqrtf(ss);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // the stores above, to the MMA
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(tslot);
    // 3.
    if (warp == 0) {
        if (elect_one()) {
            constexpr uint32_t idesc = idesc_tf32_f32(TC_TILE, TC_N);
            const uint32_t ah = smem_u32(a_hi), al = smem_u32(a_lo), bh = smem_u32(b_hi), bl = smem_u32(b_lo);
            uint32_t acc = 0;
#pragma unroll 1
            for (int pass = 0; pass < 3; ++pass) {   // lo.hi, hi.lo, then hi.hi
                const uint32_t a = pass == 0 ? al : ah, b = pass == 1 ? bl : bh;
#pragma unroll
                for (int kk = 0; kk < R / 8; ++kk) {
                    const uint32_t ka = (uint32_t)(kk >> 2) * (TC_TILE * 128) + (uint32_t)(kk & 3) * 32;
                    const uint32_t kb_ = (uint32_t)(kk >> 2) * B_REGION + (uint32_t)(kk & 3) * 32;
                    mma_tf32_ss(tmem, smem_desc_sw128(a + ka, 16, 1024), smem_desc_sw128(b + kb_, 16, 1024), idesc,
                                acc);
                    acc = 1;
                }
            }
            tc_commit(smem_u32(bar));
        }
        __syncwarp();
    }
    bool ok = mbar_wait(smem_u32(bar), 0, abort_flag);
    tc_fence_after();
    // 4. (the MMAs have completed: the A tiles are free for the staging rows)
    uint8_t *stage = smr;
    if (ok) {
        const int r = 32 * (warp & 3) + (tid & 31), c0 = 32 * (warp >> 2);
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(32 * (warp & 3)) << 16) + c0, v);
        tmem_wait_ld();
        tmem_ld_fence32(v);
        float4 *dst = reinterpret_cast<float4 *>(stage + (uint32_t)r * TC_STAGE_ROW + c0 * 4);
#pragma unroll
        for (int x = 0; x < 8; ++x) dst[x] = make_float4(v[4 * x], v[4 * x + 1], v[4 * x + 2], v[4 * x + 3]);
    } else {
        if (tid == 0) report(status, SS_DEV_TIMEOUT);
        volatile int never = 0;
        mbar_wait(smem_u32(bar), 0, &never);   // the MMAs still own the accumulator (bounded)
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // the staging rows, to the bulk copies
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, TC_N);
    if (ok && tid < TC_TILE && m0 + tid < qb) {
        float *g = sfast + ((size_t)h * qb + m0 + tid) * kbr + n0;
        asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(g),
                     "r"(smem_u32(stage + (uint32_t)tid * TC_STAGE_ROW)), "r"((uint32_t)(TC_N * 4))
                     : "memory");
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");   // before the CTA's memory is released
    }
}

__device__ __forceinline__ float warp_sum(float v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float ordered_to_float(uint32_t key) {
    return __uint_as_float((key & 0x80000000u) ? (key & 0x7fffffffu) : ~key);
}

// The exact mode's score of key block j for the query projections sq (one fmaf chain in ascending
// e, -0 -> +0), as its order-preserving key; `nonfinite` set for NaN / inf.
__device__ __forceinline__ uint32_t exact_key(const float *sq, const float4 *krow, int R, bool &nonfinite) {
    const float4 *sq4 = reinterpret_cast<const float4 *>(sq);
    float4 kv[16];   // R <= 64: the whole row's loads in flight together
#pragma unroll
    for (int e4 = 0; e4 < 16; ++e4)
        if (e4 < R / 4) kv[e4] = __ldg(krow + e4);
    float a = 0.f;
#pragma unroll
    for (int e4 = 0; e4 < 16; ++e4) {
        if (e4 < R / 4) {
            const float4 qv = sq4[e4];
            a = __fmaf_rn(qv.x, kv[e4].x, a);
            a = __fmaf_rn(qv.y, kv[e4].y, a);
            a = __fmaf_rn(qv.z, kv[e4].z, a);
            a = __fmaf_rn(qv.w, kv[e4].w, a);
        }
    }
    if (a == 0.f) a = 0.f;
    nonfinite |= !isfinite(a);
    return ordered_bits(a);
}

// Warp-wide count of keys >= c (or > c when strict) over NK keys per lane in registers.
template <int NK>
__device__ __forceinline__ int count_keys(const uint32_t (&kr)[NK], uint32_t c, bool strict) {
    int n4[4] = {0, 0, 0, 0};   // independent partial counts keep the add chains short
#pragma unroll
    for (int u = 0; u < NK; ++u) n4[u & 3] += strict ? (kr[u] > c) : (kr[u] >= c);
    return (int)__reduce_add_sync(0xffffffffu, (unsigned)((n4[0] + n4[1]) + (n4[2] + n4[3])));
}

// The threshold of the exact mode's selection from keys in registers: T with need = the keys
// equal to T to keep (lowest indices first), by bisection on the order-preserving bits. The
// search stops as soon as exactly `extra` keys are >= the candidate: those are then the `extra`
// largest with no tie across the boundary, the set the full search selects. (A radix select with
// shared-memory histograms measured slower here: most keys share their top digits, so the
// histogram atomics serialise.)
template <int NK>
__device__ __forceinline__ void threshold_regs(const uint32_t (&kr)[NK], int extra, uint32_t &T, int &need) {
    T = 0u;
    for (int bit = 31; bit >= 0; --bit) {
        const uint32_t cand = T | (1u << bit);
        const int c = count_keys(kr, cand, false);
        if (c >= extra) {
            T = cand;
            if (c == extra) break;
        }
    }
    need = extra - count_keys(kr, T, true);
}

// grid ceil(H * qb / FAST_WARPS), 32 * FAST_WARPS threads; NK keys per lane (kb <= 32 * NK, the
// fast scores' row stride kbr a multiple of 32 * NK): warp w of the grid selects for query block
// (h, i) = (w / qb, w % qb), lane l holding key blocks j = NK l + u in kr[u] (ascending block order
// runs lane by lane, so an ordered compaction is one prefix sum of per-lane counts). Dynamic
// shared memory: the query projections [FAST_WARPS][R] fp32, then [FAST_WARPS][32] block indices.
// With t the exact mode's threshold search run on the fast keys (t lies between the (extra+1)-th
// and the extra-th largest fast score) and e = 2 * max_j eps_j over the query block's candidates,
// every candidate is
//   in        if fast > t + e: any block that could precede it in the exact order (higher exact
//             score, or equal and lower index) has fast >= fast_j - e > t, and at most `extra`
//             blocks have fast > t;
//   out       if fast < t - e: the >= `extra` blocks with fast >= t all precede it;
//   uncertain otherwise.
// The selection is `in` plus the best r = extra - |in| uncertain blocks in the exact order: all of
// them when r equals their count, none when r = 0, else the uncertain blocks (up to 32) get exact
// scores, one per lane, ranked by (exact key descending, index ascending). A query block with
// more uncertain blocks than that, or any non-finite value, is scored again in full with the
// exact mode's arithmetic and selected by its rule. `scores` (optional) receives the fast scores;
// `rescored` (optional) counts the query blocks that needed any exact score.
template <int NK>
__global__ void __launch_bounds__(32 * FAST_WARPS) select_fast_kernel(
    const float *__restrict__ qh, const float *__restrict__ kh, int kh_ld, const float *__restrict__ sfast,
    const float *__restrict__ kn, int H, int qb, int kb, int kbr, int R, int block, int Lq, int Lk, int sink,
    int extra, int32_t *__restrict__ ids, int n_ids, uint8_t *__restrict__ mask, float *__restrict__ scores,
    int *rescored, int *status) {
    extern __shared__ __align__(16) uint8_t smr[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gw = blockIdx.x * FAST_WARPS + warp;   // = h * qb + i
    if (gw >= H * qb) return;
    const int h = gw / qb, jl = NK * lane;
    float *sq = reinterpret_cast<float *>(smr) + warp * R;
    int *uidx = reinterpret_cast<int *>(reinterpret_cast<float *>(smr) + FAST_WARPS * R) + warp * 32;
    const float4 *khh = reinterpret_cast<const float4 *>(kh + (size_t)h * kh_ld * R);
    const float4 *srow4 = reinterpret_cast<const float4 *>(sfast + (size_t)gw * kbr + jl);
    const float4 *knh4 = reinterpret_cast<const float4 *>(kn + (size_t)h * kbr + jl);
    uint32_t kr[NK];
    float kv[NK];
#pragma unroll
    for (int x = 0; x < NK / 4; ++x) {
        const float4 a = srow4[x], b = knh4[x];
        kr[4 * x] = __float_as_uint(a.x);
        kr[4 * x + 1] = __float_as_uint(a.y);
        kr[4 * x + 2] = __float_as_uint(a.z);
        kr[4 * x + 3] = __float_as_uint(a.w);
        kv[4 * x] = b.x;
        kv[4 * x + 1] = b.y;
        kv[4 * x + 2] = b.z;
        kv[4 * x + 3] = b.w;
    }
    float qn2 = 0.f;
    for (int e = lane; e < R; e += 32) {
        const float x = qh[(size_t)gw * R + e];
        sq[e] = x;
        qn2 = fmaf(x, x, qn2);
    }
    qn2 = warp_sum(qn2);
    bool bad = !(qn2 <= 3.0e38f);   // also NaN
    float knmax = 0.f;
#pragma unroll
    for (int u = 0; u < NK; ++u) {
        const int j = jl + u;
        const float sv = __uint_as_float(kr[u]);
        if (j < kb) {
            if (scores) scores[(size_t)gw * kb + j] = sv;
            bad |= !isfinite(sv);
        }
        const bool cand = j < kb && !is_forced(j, block, Lq, Lk, sink);
        kr[u] = cand ? ordered_bits(sv == 0.f ? 0.f : sv) : 0u;
        if (cand) knmax = fmaxf(knmax, kv[u]);
    }
    for (int o = 16; o > 0; o >>= 1) knmax = fmaxf(knmax, __shfl_xor_sync(0xffffffffu, knmax, o));
    bool full = __any_sync(0xffffffffu, bad);
    __syncwarp();   // sq
    int32_t *out = ids + (size_t)gw * n_ids;
    uint8_t *mrow = mask ? mask + (size_t)gw * kb : nullptr;
    bool touched = false;
    if (extra > 0 && !full) {
        uint32_t T;
        int need;
        threshold_regs(kr, extra, T, need);
        const float t = ordered_to_float(T);
        const float e = 2.f * fmaf(FAST_BOUND * sqrtf(qn2), knmax, FAST_ABS);
        const float up = t + e, dn = t - e;
        full = !(e <= 1.0e38f);
        int nin_l = 0, nu_l = 0;
#pragma unroll
        for (int u = 0; u < NK; ++u) {
            const float sv = ordered_to_float(kr[u]);
            const bool cand = kr[u] != 0u;
            nin_l += cand && sv > up;
            nu_l += cand && sv >= dn && sv <= up;
        }
        const int nin = (int)__reduce_add_sync(0xffffffffu, (unsigned)nin_l);
        int nu;
        const int ubase = warp_exclusive_scan(nu_l, lane, &nu);
        const int r = extra - nin;
        const bool take_all = r == nu, take_none = r == 0;
        unsigned takemask = 0u;
        if (!full && !take_all && !take_none) {
            if (nu > 32) {
                full = true;
            } else {
                int k = ubase;
#pragma unroll
                for (int u = 0; u < NK; ++u) {
                    const float sv = ordered_to_float(kr[u]);
                    if (kr[u] != 0u && sv >= dn && sv <= up) uidx[k++] = jl + u;
                }
                __syncwarp();   // uidx
                touched = true;
                const int j = lane < nu ? uidx[lane] : 0;
                bool nonfinite = false;
                const uint32_t ek = lane < nu ? exact_key(sq, khh + (size_t)j * (R / 4), R, nonfinite) : 0u;
                if (__any_sync(0xffffffffu, nonfinite)) {
                    full = true;
                } else {
                    int rank = 0;
                    for (int x = 0; x < nu; ++x) {
                        const uint32_t kx = __shfl_sync(0xffffffffu, ek, x);
                        const int jx = __shfl_sync(0xffffffffu, j, x);
                        rank += kx > ek || (kx == ek && jx < j);
                    }
                    takemask = __ballot_sync(0xffffffffu, lane < nu && rank < r);
                }
            }
        }
        if (!full) {
            // selected: forced, in, and the taken uncertain ones; then the ordered compaction
            uint64_t selbits = 0u;   // bit u: key block jl + u selected
            int k = ubase;
#pragma unroll
            for (int u = 0; u < NK; ++u) {
                const int j = jl + u;
                const float sv = ordered_to_float(kr[u]);
                const bool cand = kr[u] != 0u;
                const bool unc = cand && sv >= dn && sv <= up;
                const bool take = unc && (take_all || (!take_none && k < 32 && ((takemask >> k) & 1u)));
                k += unc;
                const bool sel = j < kb && ((!cand && is_forced(j, block, Lq, Lk, sink)) || (cand && sv > up) || take);
                selbits |= (uint64_t)sel << u;
            }
            int total;
            int o = warp_exclusive_scan(__popcll(selbits), lane, &total);
#pragma unroll
            for (int u = 0; u < NK; ++u) {
                const int j = jl + u;
                if ((selbits >> u) & 1u) {
                    if (o < n_ids) out[o] = j;
                    ++o;
                }
                if (mrow && j < kb) mrow[j] = (uint8_t)((selbits >> u) & 1u);
            }
        }
    }
    if (full || extra == 0) {
        // the exact mode: every key block scored with its arithmetic (only to select when extra > 0,
        // and always to flag non-finite scores as it does), then its threshold and its ordered
        // compaction with the ties at T kept from the lowest index
        uint32_t T = 0xffffffffu;
        int need = 0;
        if (full) {
            bool nonfinite = false;
#pragma unroll
            for (int u = 0; u < NK; ++u) {   // unrolled: kr stays in registers
                const int j = jl + u;
                if (j < kb) {
                    const uint32_t key = exact_key(sq, khh + (size_t)j * (R / 4), R, nonfinite);
                    kr[u] = is_forced(j, block, Lq, Lk, sink) ? 0u : key;
                }
            }
            if (__any_sync(0xffffffffu, nonfinite) && lane == 0) report(status, SS_DEV_NONFINITE);
            touched = true;
            if (extra > 0) threshold_regs(kr, extra, T, need);
        }
        int ties_l = 0;
#pragma unroll
        for (int u = 0; u < NK; ++u) ties_l += extra > 0 && jl + u < kb && kr[u] == T;
        int ties;
        int tie_rank = warp_exclusive_scan(ties_l, lane, &ties);
        uint64_t selbits = 0u;   // bit u: key block jl + u selected
#pragma unroll
        for (int u = 0; u < NK; ++u) {
            const int j = jl + u;
            const bool tie = extra > 0 && j < kb && kr[u] == T;
            const bool keep_tie = tie && tie_rank < need;
            tie_rank += tie;
            const bool sel = j < kb && (is_forced(j, block, Lq, Lk, sink) || (extra > 0 && kr[u] > T) || keep_tie);
            selbits |= (uint64_t)sel << u;
        }
        int total;
        int o = warp_exclusive_scan(__popcll(selbits), lane, &total);
#pragma unroll
        for (int u = 0; u < NK; ++u) {
            const int j = jl + u;
            if ((selbits >> u) & 1u) {
                if (o < n_ids) out[o] = j;
                ++o;
            }
            if (mrow && j < kb) mrow[j] = (uint8_t)((selbits >> u) & 1u);
        }
    }
    if (touched && rescored && lane == 0) atomicAdd(rescored, 1);
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
    e = cudaFuncSetAttribute(router::score_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return (int)e;
    e = cudaFuncSetAttribute(router::score_tc_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
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

// the fast mode's score row stride: 32 lanes x the selector's keys per lane (256, 512, 1024, 2048),
// so a lane's keys are whole float4s of one row
static int kb_tiles(int kb) { return kb <= 256 ? 256 : kb <= 512 ? 512 : kb <= 1024 ? 1024 : 2048; }

// Workspace: query projections [H][qb][R], key projections [H][kbp][R] (when no caller table),
// then for the fast mode its scores [H][qb][kbr] and key norms [H][kbr] (kbr = kb_tiles(kb)).
struct RouterLayout {
    size_t qh, kh, total, sf, kn, total_fast;
};

static RouterLayout router_layout(int H, int Lq, int Lk, int R, int block) {
    const size_t qb = (size_t)((Lq + block - 1) / block);
    const int kb = (Lk + block - 1) / block;
    const size_t kbp = (size_t)kb_padded(kb), kbr = (size_t)kb_tiles(kb);
    RouterLayout L;
    L.qh = 0;
    L.kh = align256(L.qh + 4 * (size_t)H * qb * R);
    L.total = align256(L.kh + 4 * (size_t)H * R * kbp);
    L.sf = L.total;
    L.kn = align256(L.sf + 4 * (size_t)H * qb * kbr);
    L.total_fast = align256(L.kn + 4 * (size_t)H * kbr);
    return L;
}

size_t router_workspace_size(int H, int Lq, int Lk, int R, int block) { return router_layout(H, Lq, Lk, R, block).total; }
size_t router_fast_workspace_size(int H, int Lq, int Lk, int R, int block) {
    return router_layout(H, Lq, Lk, R, block).total_fast;
}

static size_t tc_smem(int R) {
    return 1024 + 2 * (size_t)(R / 32) * (router::TC_TILE + router::TC_N) * 128 + 64;
}
constexpr int FAST_MAX_KB = 2048;   // 64 keys per lane
static size_t fast_smem(int R) { return (size_t)router::FAST_WARPS * ((size_t)R + 32) * 4; }

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
                       int *status, cudaStream_t st, int krow0 = 0, KvRing ring = KvRing()) {
    const int qb = with_q ? (Lq + block - 1) / block : 0, nk = kj1 - kj0;
    if (qb + nk <= 0) return 0;
    const int nsm = g_router_sms[device] > 0 ? g_router_sms[device] : 148;
    int bg = std::max(1, (H * (qb + nk) + nsm - 1) / nsm);
    while (H * ((qb + bg - 1) / bg + (nk + bg - 1) / bg) > nsm && bg < std::max(qb, nk)) ++bg;
    const int tq = (qb + bg - 1) / bg, tk = (nk + bg - 1) / bg;
    const int nw = pp_warps(R, block);
    CUtensorMap tmq, tmk;
    const uint64_t row_bytes = (uint64_t)H * router::D * 2;
    if (encode_tmap_2d_bf16_rows(&tmk, k, (uint64_t)H * router::D, (uint64_t)(ring.phys_rows(Lk) - krow0), row_bytes,
                                 router::D, 64u))
        return SS_ERR_DRIVER;
    if (with_q) {
        if (encode_tmap_2d_bf16_rows(&tmq, q, (uint64_t)H * router::D, (uint64_t)Lq, row_bytes, router::D, 64u))
            return SS_ERR_DRIVER;
    } else {
        tmq = tmk;   // no query tiles: the map is never read
    }
    router::pool_project_kernel<<<dim3(tq + tk, H), 32 * nw, pp_smem(R, block, nw), st>>>(
        tmq, tmk, H, Lq, Lk, block, R, tq, bg, wq, wk, qh, kh, kh_ld, kj0, kj1, krow0, ring, status);
    return (int)cudaGetLastError();
}

// Launch the router kernels with the query projections in `ws` (router_workspace_size bytes,
// 256-byte aligned). The key projections go to the workspace too (kh_ext == nullptr), or to the
// caller's table kh_ext [H][kh_ld][R], whose rows [0, n_cached) already hold this window's first
// n_cached key blocks: only blocks [n_cached, kb) are pooled.
int router_launch(const void *q, const void *k, const float *wq, const float *wk, int H, int Lq, int Lk, int R,
                  int block, int sink_tokens, int extra, int32_t *ids, int n_ids, uint8_t *mask, float *scores,
                  uint8_t *ws, int *status, cudaStream_t st, float *kh_ext = nullptr, int kh_ld_ext = 0,
                  int n_cached = 0, int krow0 = 0, KvRing ring = KvRing()) {
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
                     status, st, krow0, ring);
    if (rc) return rc;
    router::score_select_kernel<<<dim3((qb + router::ROWS - 1) / router::ROWS, H), router::SS_THREADS,
                                  select_smem(kbp, R), st>>>(qh, kh, kh_ld, qb, kb, kbp, R, block, Lq, Lk, sink_tokens,
                                                             extra, ids, n_ids, mask, scores, status);
    return (int)cudaGetLastError();
}

// router_launch in the fast mode: pooling as there, then score_tc_kernel and select_fast_kernel
// (the fast scores and key norms in the workspace's fast-mode part). R must be 32 or 64.
int router_fast_launch(const void *q, const void *k, const float *wq, const float *wk, int H, int Lq, int Lk, int R,
                       int block, int sink_tokens, int extra, int32_t *ids, int n_ids, uint8_t *mask, float *scores,
                       int *rescored, uint8_t *ws, int *status, cudaStream_t st, float *kh_ext, int kh_ld_ext,
                       int n_cached, int krow0, KvRing ring = KvRing()) {
    const int qb = (Lq + block - 1) / block, kb = (Lk + block - 1) / block, kbp = kb_padded(kb), kbr = kb_tiles(kb);
    int device;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return (int)e;
    int rc = router_prepare(device);
    if (rc) return rc;
    const RouterLayout L = router_layout(H, Lq, Lk, R, block);
    float *qh = reinterpret_cast<float *>(ws + L.qh);
    float *kh = kh_ext ? kh_ext : reinterpret_cast<float *>(ws + L.kh);
    const int kh_ld = kh_ext ? kh_ld_ext : kbp;
    float *sf = reinterpret_cast<float *>(ws + L.sf), *kn = reinterpret_cast<float *>(ws + L.kn);
    rc = pool_launch(device, q, k, wq, wk, H, Lq, Lk, R, block, true, qh, kh, kh_ld, kh_ext ? n_cached : 0, kb,
                     status, st, krow0, ring);
    if (rc) return rc;
    const dim3 tg(kbr / router::TC_N, (qb + router::TC_TILE - 1) / router::TC_TILE, H);
    if (R == 64)
        router::score_tc_kernel<64><<<tg, router::TC_THREADS, tc_smem(R), st>>>(qh, kh, kh_ld, qb, kb, kbr, sf, kn,
                                                                              status);
    else
        router::score_tc_kernel<32><<<tg, router::TC_THREADS, tc_smem(R), st>>>(qh, kh, kh_ld, qb, kb, kbr, sf, kn,
                                                                              status);
    e = cudaGetLastError();
    if (e != cudaSuccess) return (int)e;
    const int rows = H * qb, grid = (rows + router::FAST_WARPS - 1) / router::FAST_WARPS;
    const size_t sm = fast_smem(R);
#define SS_SELECT_FAST(NK)                                                                                           \
    router::select_fast_kernel<NK><<<grid, 32 * router::FAST_WARPS, sm, st>>>(                                        \
        qh, kh, kh_ld, sf, kn, H, qb, kb, kbr, R, block, Lq, Lk, sink_tokens, extra, ids, n_ids, mask, scores, rescored, \
        status)
    if (kb <= 256) SS_SELECT_FAST(8);
    else if (kb <= 512) SS_SELECT_FAST(16);
    else if (kb <= 1024) SS_SELECT_FAST(32);
    else SS_SELECT_FAST(64);
#undef SS_SELECT_FAST
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

extern "C" int ss_router_fast_workspace_bytes(int H, int Lq, int Lk, int R, int block, size_t *bytes) {
    if (!bytes || H <= 0 || Lq <= 0 || Lk <= 0 || R <= 0 || (block != 64 && block != 128)) return SS_ERR_SHAPE;
    *bytes = ss::router_fast_workspace_size(H, Lq, Lk, R, block);   // the exact mode's part, then the fast scores
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

extern "C" int ss_router_fast(const void *q, const void *k, int k_row0, const float *wq, const float *wk, int H, int Lq,
                              int Lk, int R, int block, int sink_tokens, int extra, float *kh, int kh_rows,
                              int n_cached, int32_t *ids, int n_ids, uint8_t *mask, float *scores, int *rescored,
                              void *workspace, size_t workspace_bytes, int *status, void *stream) {
    int rc = ss::router_check(q, k, wq, wk, H, Lq, Lk, R, block, sink_tokens, extra, ids, n_ids);
    if (rc) return rc;
    if (R != 32 && R != 64) return SS_ERR_SHAPE;
    if (!workspace) return SS_ERR_POINTER;
    const int kb = (Lk + block - 1) / block;
    if (kh) {
        if (kh_rows < kb || n_cached < 0 || n_cached > kb) return SS_ERR_SHAPE;
        if (k_row0 < 0 || k_row0 > n_cached * block || k_row0 >= Lk) return SS_ERR_SHAPE;
        if (reinterpret_cast<uintptr_t>(kh) & 15u) return SS_ERR_POINTER;
    } else if (n_cached != 0 || k_row0 != 0) {
        return SS_ERR_SHAPE;
    }
    if (workspace_bytes < ss::router_fast_workspace_size(H, Lq, Lk, R, block)) return SS_ERR_WORKSPACE;
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return SS_ERR_POINTER;
    if (kb > ss::FAST_MAX_KB)   // beyond the fast selector's keys in registers: the exact kernels
        return ss::router_launch(q, k, wq, wk, H, Lq, Lk, R, block, sink_tokens, extra, ids, n_ids, mask, scores,
                                 static_cast<uint8_t *>(workspace), status, static_cast<cudaStream_t>(stream), kh,
                                 kh ? kh_rows : 0, n_cached, k_row0);
    return ss::router_fast_launch(q, k, wq, wk, H, Lq, Lk, R, block, sink_tokens, extra, ids, n_ids, mask, scores,
                                  rescored, static_cast<uint8_t *>(workspace), status, static_cast<cudaStream_t>(stream),
                                  kh, kh_rows, n_cached, k_row0);
}

extern "C" int ss_router_pool_keys_ring(const void *k, const float *wk, int H, int Lk, int R, int block, int j0,
                                        int j1, float *kh, int kh_rows, int ring_sink, int ring_cap, int ring_head,
                                        const int *ring_head_dev, int *status, void *stream) {
    using namespace ss;
    KvRing ring;
    ring.S = ring_sink;
    ring.C = ring_cap;
    ring.head = ring_head;
    ring.head_dev = ring_head_dev;
    if (ring_cap <= 0 || ring_check(ring, Lk)) return SS_ERR_SHAPE;
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
                       status, static_cast<cudaStream_t>(stream), 0, ring);
}

extern "C" int ss_router_ring(const void *q, const void *k, const float *wq, const float *wk, int H, int Lq, int Lk,
                              int R, int block, int sink_tokens, int extra, float *kh, int kh_rows, int n_cached,
                              int32_t *ids, int n_ids, uint8_t *mask, float *scores, int *rescored, int fast,
                              int ring_sink, int ring_cap, int ring_head, const int *ring_head_dev, void *workspace,
                              size_t workspace_bytes, int *status, void *stream) {
    ss::KvRing ring;
    ring.S = ring_sink;
    ring.C = ring_cap;
    ring.head = ring_head;
    ring.head_dev = ring_head_dev;
    if (ring_cap <= 0 || ss::ring_check(ring, Lk)) return SS_ERR_SHAPE;
    int rc = ss::router_check(q, k, wq, wk, H, Lq, Lk, R, block, sink_tokens, extra, ids, n_ids);
    if (rc) return rc;
    if (!workspace) return SS_ERR_POINTER;
    const int kb = (Lk + block - 1) / block;
    if (kh) {
        if (kh_rows < kb || n_cached < 0 || n_cached > kb) return SS_ERR_SHAPE;
        if (reinterpret_cast<uintptr_t>(kh) & 15u) return SS_ERR_POINTER;
    } else if (n_cached != 0) {
        return SS_ERR_SHAPE;
    }
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return SS_ERR_POINTER;
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (fast && kb <= ss::FAST_MAX_KB) {
        if (R != 32 && R != 64) return SS_ERR_SHAPE;
        if (workspace_bytes < ss::router_fast_workspace_size(H, Lq, Lk, R, block)) return SS_ERR_WORKSPACE;
        return ss::router_fast_launch(q, k, wq, wk, H, Lq, Lk, R, block, sink_tokens, extra, ids, n_ids, mask, scores,
                                      rescored, ws, status, st, kh, kh ? kh_rows : 0, n_cached, 0, ring);
    }
    if (workspace_bytes < ss::router_workspace_size(H, Lq, Lk, R, block)) return SS_ERR_WORKSPACE;
    return ss::router_launch(q, k, wq, wk, H, Lq, Lk, R, block, sink_tokens, extra, ids, n_ids, mask, scores, ws,
                             status, st, kh, kh ? kh_rows : 0, n_cached, 0, ring);
}
