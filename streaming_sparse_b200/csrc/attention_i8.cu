// attention_i8.cu -- INT8-QK block-sparse attention on sm_100a and its K page quantiser.
//
// The arithmetic is that of the reference's INT8 path (migration/unified_router/opt23/attention.py:
// `_quant` :6-14 and `_shared` with INT8=True :30-58, used with 32-row query groups by
// opt24/pipeline.py:24-25): K is quantised per 64-token page and head, Q per 32-row group and head
// (scale = max(max|x| / 127, 1e-10), x_i8 = round-half-even(x / scale)); the logits are the exact
// int32 dot products times (qs * ks[page]) times scale * log2(e); softmax in base 2; P is rounded
// to bf16 (V's type here) for the P.V product, accumulated in fp32.
//
// B200 layout of the kernel (one CTA per 128-row query tile and head, 192 threads):
//   warps 0-3  one query row per thread (TMEM lane = row): quantise the tile's Q into shared memory
//              (128-byte swizzled rows, the K-major UMMA layout), then per step read the int32
//              scores from TMEM, scale, softmax, write P (bf16) over its own S columns;
//   warp 4     TMA producer: each 64-token page's int8 K (8 KB) and bf16 V (16 KB) into a 3-stage ring;
//   warp 5     MMA issuer: S = Q K^T as tcgen05.mma kind::i8 (M 128, N 64, K 32, both operands in
//              shared memory, s32 accumulator in TMEM), O += P V as kind::f16 (P from TMEM).
// TMEM (256 columns, two CTAs per SM): S0/P0 [0, 64), S1/P1 [64, 128), O [128, 256). The two S
// buffers let QK(s+1) run while the rows exponentiate step s. The running maximum is only raised
// when a row's maximum grows by more than 8 (log2 units), so O is rescaled in TMEM rarely; the
// result is the same softmax (the same maximum scales both O and the row sum).
// A 128-row tile covers one 128-token or two 64-token query blocks; its steps are the union of the
// blocks' pages in ascending order, each with a bit per query block, and a row ignores the pages
// its own block did not select. Every wait is bounded; on expiry SS_DEV_TIMEOUT is reported, loads
// and MMAs in flight are drained and TMEM is freed.
#include <climits>
#include <mutex>

#include "common.cuh"

namespace ss {
namespace i8 {

constexpr int D = 128;
constexpr int PAGE = 64;
constexpr int QGROUP = 32;
static_assert(QGROUP == 32, "a query scale group is one warp's 32 rows");
constexpr int NSTAGE = 3;
constexpr int MAX_PAGES = 4096;
constexpr int NTHREADS = 192;
constexpr uint32_t Q_BYTES = 128 * 128;
constexpr uint32_t K_BYTES = PAGE * 128;
constexpr uint32_t V_REGION = PAGE * 128;                  // 64 tokens x 64 dims bf16
constexpr uint32_t STAGE_BYTES = K_BYTES + 2 * V_REGION;
constexpr uint32_t OFF_Q = 0;
constexpr uint32_t OFF_STAGE = OFF_Q + Q_BYTES;
constexpr uint32_t OFF_BAR = OFF_STAGE + NSTAGE * STAGE_BYTES;
constexpr int NBAR = 16;
constexpr uint32_t OFF_MISC = OFF_BAR + NBAR * 8;
constexpr uint32_t OFF_BITS = OFF_MISC + 64;
constexpr uint32_t OFF_LIST = OFF_BITS + 2 * (MAX_PAGES / 32) * 4;
constexpr uint32_t SMEM_BYTES = OFF_LIST + MAX_PAGES * 4 + 1024;   // + alignment slack
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t TMEM_O = 128;
static_assert(OFF_STAGE % 1024 == 0 && STAGE_BYTES % 1024 == 0, "swizzle atoms are 1024-byte aligned");

enum Bar { Q_FULL = 0, KV_FULL = 1, KV_EMPTY = KV_FULL + NSTAGE, S_FULL = KV_EMPTY + NSTAGE, P_FULL = S_FULL + 2,
           PV_DONE = P_FULL + 2, DRAIN = PV_DONE + 2, NBAR_USED = DRAIN + 1 };
static_assert(NBAR_USED <= NBAR, "barrier space");

// kind::i8 instruction descriptor: D s32, A and B signed 8-bit, both K-major, M = 128, N = 64.
constexpr uint32_t IDESC_QK = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(PAGE >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint32_t IDESC_PV = idesc_bf16_f32(128, 128, false, true);

struct Params {
    const __nv_bfloat16 *q;
    const float *ks;
    const int32_t *ids;
    void *out;
    float *lse;
    int *status;
    int H, Lq, Lk, block, n_ids, nqb, nkb, npages, out_fp32;
    float c;   // scale * log2(e)
    int pieces;        // > 1: CTA z of a tile takes steps [z n / pieces, (z + 1) n / pieces)
    float *ws_o;       // pieces > 1: [pieces][Lq][H][128] fp32 normalised partials
    float *ws_lse;     //             [pieces][H][Lq] natural-log LSE (-inf: no token)
    KvRing ring;       // k_i8 / v as a ring cache (C = 0: a plain window); a page is one 64-row range
};

// D[tmem] (+)= A[smem] * B[smem], kind::i8 (s8 inputs, s32 accumulate)
__device__ __forceinline__ void mma_i8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem], kind::f16 (bf16 inputs, fp32 accumulate)
__device__ __forceinline__ void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ bool warp_all(bool ok) { return __all_sync(0xffffffffu, ok); }

// two fp32 lanes in one 64-bit register: fma.rn.f32x2 / add.rn.f32x2 (two IEEE operations each)
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    return ((uint64_t)__float_as_uint(hi) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ float f2_lo(uint64_t x) { return __uint_as_float((uint32_t)x); }
__device__ __forceinline__ float f2_hi(uint64_t x) { return __uint_as_float((uint32_t)(x >> 32)); }


// A wait that ignores the abort flag (used only to drain work this CTA itself issued).
__device__ __forceinline__ bool drain_wait(uint32_t bar, uint32_t parity) {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - t0 > kWaitLimitCycles) return false;
    return true;
}

__global__ void __launch_bounds__(NTHREADS, 2)
attention_i8_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                    const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + OFF_BAR;
    auto bar = [&](int i) -> uint32_t { return bar0 + 8u * (uint32_t)i; };
    volatile uint32_t *misc = reinterpret_cast<volatile uint32_t *>(smem + OFF_MISC);   // [0] tmem, [1] steps, [2] abort
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_MISC + 8);
    uint32_t *bits = reinterpret_cast<uint32_t *>(smem + OFF_BITS);
    uint32_t *list = reinterpret_cast<uint32_t *>(smem + OFF_LIST);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tile = blockIdx.x, h = blockIdx.y;
    const int nq = 128 / p.block;               // query blocks in the tile (2 or 1)
    const int nwords = (p.npages + 31) / 32;

    if (tid == 0) {
        for (int i = 0; i < NBAR_USED; ++i) {
            uint32_t cnt = 1;
            if (i == Q_FULL || i == P_FULL || i == P_FULL + 1) cnt = 128;
            mbar_init(bar(i), cnt);
        }
        fence_mbar_init();
        misc[2] = 0;
        prefetch_tmap(&tm_k);
        prefetch_tmap(&tm_v);
    }
    for (int i = tid; i < 2 * nwords; i += NTHREADS) bits[(i / nwords) * (MAX_PAGES / 32) + i % nwords] = 0u;
    if (warp == 0) {
        tmem_alloc(sbase + OFF_MISC, TMEM_COLS);
        tmem_relinquish();
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();

    // the tile's page lists: one bitmap per query block, then their ascending union
    const int ppb = p.block / PAGE;
    for (int idx = tid; idx < nq * p.n_ids; idx += NTHREADS) {
        const int i = idx / p.n_ids, qb = tile * nq + i;
        if (qb >= p.nqb) continue;
        const int id = p.ids[((size_t)h * p.nqb + qb) * p.n_ids + idx % p.n_ids];
        if (id < 0) continue;
        if (id >= p.nkb) {
            report(p.status, SS_DEV_BADID);
            continue;
        }
        for (int u = 0; u < ppb; ++u) {
            const int pg = id * ppb + u;
            if (pg < p.npages) atomicOr(&bits[i * (MAX_PAGES / 32) + (pg >> 5)], 1u << (pg & 31));
        }
    }
    __syncthreads();
    if (warp == 0) {
        int base = 0;
        for (int w0 = 0; w0 < nwords; w0 += 32) {
            const int w = w0 + lane;
            const uint32_t u0 = w < nwords ? bits[w] : 0u;
            const uint32_t u1 = w < nwords ? bits[MAX_PAGES / 32 + w] : 0u;
            uint32_t u = u0 | u1;
            const int cnt = __popc(u);
            int incl = cnt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += t;
            }
            int off = base + incl - cnt;
            while (u) {
                const int b = __ffs(u) - 1;
                u &= u - 1;
                const uint32_t m = ((u0 >> b) & 1u) | (((u1 >> b) & 1u) << 1);
                list[off++] = (uint32_t)(32 * w + b) | (m << 16);
            }
            base += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (lane == 0) misc[1] = (uint32_t)base;
    }
    __syncthreads();
    const int n_all = (int)misc[1];
    const int z = blockIdx.z;
    const int s_lo = (int)(((long)z * n_all) / p.pieces), s_hi = (int)(((long)(z + 1) * n_all) / p.pieces);
    const int n = s_hi - s_lo;                  // this CTA's steps: list[s_lo .. s_hi)
    const uint32_t *steps = list + s_lo;
    const uint32_t tmem = misc[0];
    const uint32_t sQ = sbase + OFF_Q;

    if (warp < 4) {
        // ---------------- query rows ----------------
        const int r = tid;                        // tile row = TMEM lane
        const int row = tile * 128 + r;
        const bool live = row < p.Lq;
        float x[D];
        {
            const uint4 *src = reinterpret_cast<const uint4 *>(p.q + ((size_t)(live ? row : 0) * p.H + h) * D);
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                const uint4 v = live ? src[c] : make_uint4(0u, 0u, 0u, 0u);
                const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    x[8 * c + 2 * j] = __uint_as_float(w4[j] << 16);
                    x[8 * c + 2 * j + 1] = __uint_as_float(w4[j] & 0xFFFF0000u);
                }
            }
        }
        float amax = 0.f;
#pragma unroll
        for (int j = 0; j < D; ++j) amax = fmaxf(amax, fabsf(x[j]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float qs = fmaxf(__fdiv_rn(amax, 127.f), 1e-10f);   // this warp's 32 rows are one group
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            uint32_t w4[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t acc = 0u;
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const int qv = (int)rintf(__fdiv_rn(x[16 * c + 4 * j + b], qs));
                    acc |= ((uint32_t)qv & 0xFFu) << (8 * b);
                }
                w4[j] = acc;
            }
            *reinterpret_cast<uint4 *>(smem + OFF_Q + r * 128 + ((c ^ (r & 7)) << 4)) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive(bar(Q_FULL));

        const uint32_t lane_base = tmem + ((uint32_t)(32 * warp) << 16);
        const int qi = r / p.block;               // which of the tile's query blocks this row is in
        const float *ksh = p.ks + (size_t)h * p.npages;
        float m_run = -INFINITY, l = 0.f;
        bool ok = true;
        float ks_next = n > 0 ? __ldg(ksh + (steps[0] & 0xFFFFu)) : 0.f;
        for (int s = 0; s < n && ok; ++s) {
            const uint32_t e = steps[s];
            const int page = (int)(e & 0xFFFFu);
            const bool sel = (e >> (16 + qi)) & 1u;
            const float ksv = ks_next;
            if (s + 1 < n) ks_next = __ldg(ksh + (steps[s + 1] & 0xFFFFu));
            const int b = s & 1;
            ok = warp_all(mbar_wait(bar(S_FULL + b), (s >> 1) & 1, abort_flag));
            if (!ok) break;
            tc_fence_after();
            uint32_t pk[32];
            if (sel) {   // warp-uniform: a warp's 32 rows lie in one query block
                float sv[64];
                tmem_ld32(lane_base + 64 * b, sv);
                tmem_ld32(lane_base + 64 * b + 32, sv + 32);
                tmem_wait_ld();
                tmem_ld_fence32(sv);
                tmem_ld_fence32(sv + 32);
                const int nvalid = min(PAGE, p.Lk - page * PAGE);
                // logit = score * tc with tc = (qs * ks) * scale * log2(e) > 0, so the row's largest
                // logit comes from its largest integer score
                const float tc = __fmul_rn(__fmul_rn(qs, ksv), p.c);
                int smax = INT_MIN;
                if (nvalid == PAGE) {   // every page but a window's last: no bounds in the loops
                    int m0 = INT_MIN, m1 = INT_MIN, m2 = INT_MIN, m3 = INT_MIN;   // four independent chains
#pragma unroll
                    for (int j = 0; j < 64; j += 8) {
                        m0 = __vimax3_s32(m0, __float_as_int(sv[j]), __float_as_int(sv[j + 1]));
                        m1 = __vimax3_s32(m1, __float_as_int(sv[j + 2]), __float_as_int(sv[j + 3]));
                        m2 = __vimax3_s32(m2, __float_as_int(sv[j + 4]), __float_as_int(sv[j + 5]));
                        m3 = __vimax3_s32(m3, __float_as_int(sv[j + 6]), __float_as_int(sv[j + 7]));
                    }
                    smax = max(__vimax3_s32(m0, m1, m2), m3);
                } else {
#pragma unroll
                    for (int j = 0; j < 64; ++j)
                        if (j < nvalid) smax = max(smax, __float_as_int(sv[j]));
                }
                const float mx = __fmul_rn((float)smax, tc);
                // raise the running maximum only when it grows by more than 8 (P stays <= 256)
                float alpha = 1.f;
                if (mx > m_run + 8.f) {
                    if (m_run != -INFINITY) alpha = ex2(m_run - mx);
                    m_run = mx;
                }
                if (__any_sync(0xffffffffu, alpha != 1.f)) {
                    // O holds PV(0 .. s-1): wait for the last one, then rescale this warp's rows
                    ok = warp_all(mbar_wait(bar(PV_DONE + ((s - 1) & 1)), ((s - 1) >> 1) & 1, abort_flag));
                    if (!ok) break;
                    tc_fence_after();
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc) {
                        float ov[32];
                        tmem_ld32(lane_base + TMEM_O + 32 * cc, ov);
                        tmem_wait_ld();
                        tmem_ld_fence32(ov);
#pragma unroll
                        for (int j = 0; j < 32; ++j) ov[j] *= alpha;
                        tmem_st32(lane_base + TMEM_O + 32 * cc, ov);
                        tmem_wait_st();
                        tmem_st_fence32(ov);
                    }
                    l *= alpha;
                }
                const float neg = -m_run;
                float sum0 = 0.f, sum1 = 0.f;
                if (nvalid == PAGE) {   // packed: one fma and one add instruction per two scores
                    const uint64_t tc2 = f2_pack(tc, tc), nb2 = f2_pack(neg, neg);
                    uint64_t sa = 0ull, sb = 0ull;
#pragma unroll
                    for (int c = 0; c < 64; c += 4) {
                        const uint64_t x0 = f2_fma(f2_pack((float)__float_as_int(sv[c]), (float)__float_as_int(sv[c + 1])),
                                                   tc2, nb2);
                        const uint64_t x1 = f2_fma(
                            f2_pack((float)__float_as_int(sv[c + 2]), (float)__float_as_int(sv[c + 3])), tc2, nb2);
                        const float p0 = ex2(f2_lo(x0)), p1 = ex2(f2_hi(x0));
                        const float p2 = ex2(f2_lo(x1)), p3 = ex2(f2_hi(x1));
                        sa = f2_add(sa, f2_pack(p0, p1));
                        sb = f2_add(sb, f2_pack(p2, p3));
                        pk[c >> 1] = pack_bf16x2(p0, p1);
                        pk[(c >> 1) + 1] = pack_bf16x2(p2, p3);
                    }
                    const uint64_t st2 = f2_add(sa, sb);
                    sum0 = f2_lo(st2);
                    sum1 = f2_hi(st2);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const float p0 = 2 * j < nvalid ? ex2(fmaf((float)__float_as_int(sv[2 * j]), tc, neg)) : 0.f;
                        const float p1 =
                            2 * j + 1 < nvalid ? ex2(fmaf((float)__float_as_int(sv[2 * j + 1]), tc, neg)) : 0.f;
                        sum0 += p0;
                        sum1 += p1;
                        pk[j] = pack_bf16x2(p0, p1);
                    }
                }
                l += sum0 + sum1;
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j) pk[j] = 0u;
            }
            tmem_st32(lane_base + 64 * b, reinterpret_cast<const float *>(pk));
            tmem_wait_st();
            tmem_st_fence32(reinterpret_cast<const float *>(pk));
            tc_fence_before();
            mbar_arrive(bar(P_FULL + b));
        }
        if (ok && n > 0) ok = warp_all(mbar_wait(bar(PV_DONE + ((n - 1) & 1)), ((n - 1) >> 1) & 1, abort_flag));
        if (ok) {
            tc_fence_after();
            const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                float ov[32];
                if (n > 0) {
                    tmem_ld32(lane_base + TMEM_O + 32 * cc, ov);
                    tmem_wait_ld();
                    tmem_ld_fence32(ov);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) ov[j] = 0.f;
                }
                if (live && p.pieces > 1) {
                    float4 *dst = reinterpret_cast<float4 *>(p.ws_o + (((size_t)z * p.Lq + row) * p.H + h) * D + 32 * cc);
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        dst[j] = make_float4(ov[4 * j] * inv, ov[4 * j + 1] * inv, ov[4 * j + 2] * inv,
                                             ov[4 * j + 3] * inv);
                } else if (live) {
                    if (p.out_fp32) {
                        float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(p.out) +
                                                                 ((size_t)row * p.H + h) * D + 32 * cc);
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            dst[j] = make_float4(ov[4 * j] * inv, ov[4 * j + 1] * inv, ov[4 * j + 2] * inv,
                                                 ov[4 * j + 3] * inv);
                    } else {
                        uint4 *dst = reinterpret_cast<uint4 *>(static_cast<__nv_bfloat16 *>(p.out) +
                                                               ((size_t)row * p.H + h) * D + 32 * cc);
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            dst[j] = make_uint4(pack_bf16x2(ov[8 * j] * inv, ov[8 * j + 1] * inv),
                                                pack_bf16x2(ov[8 * j + 2] * inv, ov[8 * j + 3] * inv),
                                                pack_bf16x2(ov[8 * j + 4] * inv, ov[8 * j + 5] * inv),
                                                pack_bf16x2(ov[8 * j + 6] * inv, ov[8 * j + 7] * inv));
                    }
                }
            }
            const float lse_row = l > 0.f ? (m_run + __log2f(l)) * 0.6931471805599453f : -INFINITY;
            if (live && p.pieces > 1) p.ws_lse[((size_t)z * p.H + h) * p.Lq + row] = lse_row;
            else if (live && p.lse) p.lse[(size_t)h * p.Lq + row] = lse_row;
        }
        if (!ok) report(p.status, SS_DEV_TIMEOUT);
    } else if (warp == 4) {
        // ---------------- TMA producer ----------------
        int issued = 0;
        bool ok = true;
        const KvRing rg = p.ring.resolved();
        for (int s = 0; s < n; ++s) {
            const int st = s % NSTAGE;
            if (s >= NSTAGE) {
                ok = warp_all(mbar_wait(bar(KV_EMPTY + st), ((s / NSTAGE) - 1) & 1, abort_flag));
                if (!ok) break;
            }
            const int page = (int)(steps[s] & 0xFFFFu);
            if (elect_one()) {
                const uint32_t dst = sbase + OFF_STAGE + (uint32_t)st * STAGE_BYTES;
                mbar_arrive_expect_tx(bar(KV_FULL + st), STAGE_BYTES);
                const int y = rg.sub_row(page * PAGE);   // the page's first physical row
                tma_load_2d(dst, &tm_k, h * D, y, bar(KV_FULL + st));
                tma_load_2d(dst + K_BYTES, &tm_v, h * D, y, bar(KV_FULL + st));
                tma_load_2d(dst + K_BYTES + V_REGION, &tm_v, h * D + 64, y, bar(KV_FULL + st));
            }
            __syncwarp();
            issued = s + 1;
        }
        if (!ok) report(p.status, SS_DEV_TIMEOUT);
        if (!ok || *abort_flag) {
            // the loads still in flight land before the CTA's shared memory goes away
            for (int s = issued > NSTAGE ? issued - NSTAGE : 0; s < issued; ++s)
                drain_wait(bar(KV_FULL + s % NSTAGE), (s / NSTAGE) & 1);
        }
    } else {
        // ---------------- MMA issuer ----------------
        const uint64_t dq = smem_desc_sw128(sQ, 16, 1024);
        const uint32_t sStage = sbase + OFF_STAGE;
        bool ok = warp_all(mbar_wait(bar(Q_FULL), 0, abort_flag));
        auto qk = [&](int s) -> bool {
            const int st = s % NSTAGE, b = s & 1;
            if (!warp_all(mbar_wait(bar(KV_FULL + st), (s / NSTAGE) & 1, abort_flag))) return false;
            tc_fence_after();
            const uint64_t dk = smem_desc_sw128(sStage + (uint32_t)st * STAGE_BYTES, 16, 1024);
            if (elect_one()) {
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)   // K = 32 int8 = 32 bytes per instruction
                    mma_i8_ss(tmem + 64 * b, dq + 2 * kk, dk + 2 * kk, IDESC_QK, kk > 0 ? 1u : 0u);
                tc_commit(bar(S_FULL + b));
            }
            __syncwarp();
            return true;
        };
        if (ok) tc_fence_after();
        if (ok && n > 0) ok = qk(0);
        if (ok && n > 1) ok = qk(1);
        for (int s = 0; s < n && ok; ++s) {
            const int st = s % NSTAGE, b = s & 1;
            ok = warp_all(mbar_wait(bar(P_FULL + b), (s >> 1) & 1, abort_flag));
            if (!ok) break;
            tc_fence_after();
            const uint64_t dv = smem_desc_sw128(sStage + (uint32_t)st * STAGE_BYTES + K_BYTES, V_REGION, 1024);
            if (elect_one()) {
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)   // tokens 16kk.. : P columns 8kk.. (bf16 pairs)
                    mma_bf16_ts(tmem + TMEM_O, tmem + 64 * b + 8 * kk, dv + ((kk * 2048) >> 4), IDESC_PV,
                                (s > 0 || kk > 0) ? 1u : 0u);
                tc_commit(bar(KV_EMPTY + st));
                tc_commit(bar(PV_DONE + b));
            }
            __syncwarp();
            if (s + 2 < n) {
                // S buffer b holds P(s) until PV(s) has read it
                ok = warp_all(mbar_wait(bar(PV_DONE + b), (s >> 1) & 1, abort_flag));
                if (ok) ok = qk(s + 2);
            }
        }
        if (!ok) report(p.status, SS_DEV_TIMEOUT);
        if (!ok || *abort_flag) {
            if (elect_one()) tc_commit(bar(DRAIN));   // arrives once every MMA issued so far is done
            __syncwarp();
            drain_wait(bar(DRAIN), 0);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------------------------
// K page quantiser: one CTA of 256 threads per (page, head); thread t takes row t/4 of the page,
// dims 32 (t%4) .. +32.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
quant_k_pages_kernel(const __nv_bfloat16 *k, int H, int Lk, int p0, int npages, int8_t *ki, float *ks, KvRing ring) {
    __shared__ float red[8];
    const int pg = p0 + blockIdx.x, h = blockIdx.y;
    const int t = threadIdx.x, d0 = 32 * (t & 3);
    const bool live = pg * PAGE + (t >> 2) < Lk;
    const int row = ring.resolved().sub_row(pg * PAGE) + (t >> 2);   // physical row (a ring keeps pages contiguous)
    float x[32];
    const uint4 *src = reinterpret_cast<const uint4 *>(k + ((size_t)(live ? row : 0) * H + h) * D + d0);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint4 v = live ? src[c] : make_uint4(0u, 0u, 0u, 0u);
        const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            x[8 * c + 2 * j] = __uint_as_float(w4[j] << 16);
            x[8 * c + 2 * j + 1] = __uint_as_float(w4[j] & 0xFFFF0000u);
        }
    }
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(x[j]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((t & 31) == 0) red[t >> 5] = amax;
    __syncthreads();
    amax = red[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) amax = fmaxf(amax, red[w]);
    const float scale = fmaxf(__fdiv_rn(amax, 127.f), 1e-10f);
    if (t == 0) ks[(size_t)h * npages + pg] = scale;
    if (!live) return;
    uint32_t w8[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        uint32_t acc = 0u;
#pragma unroll
        for (int b = 0; b < 4; ++b) acc |= ((uint32_t)(int)rintf(__fdiv_rn(x[4 * j + b], scale)) & 0xFFu) << (8 * b);
        w8[j] = acc;
    }
    uint4 *dst = reinterpret_cast<uint4 *>(ki + ((size_t)row * H + h) * D + d0);
    dst[0] = make_uint4(w8[0], w8[1], w8[2], w8[3]);
    dst[1] = make_uint4(w8[4], w8[5], w8[6], w8[7]);
}

}  // namespace i8

static std::mutex g_i8_mutex;
static int g_i8_configured[SS_MAX_DEVICES];
static void *g_i8_ctx[SS_MAX_DEVICES];
static int g_i8_nsm[SS_MAX_DEVICES];

int attention_i8_prepare(int device) {
    if (device < 0 || device >= SS_MAX_DEVICES) return SS_ERR_DEVICE;
    void *ctx = nullptr;
    int rc = current_context(&ctx);
    if (rc) return rc;
    std::lock_guard<std::mutex> lock(g_i8_mutex);
    if (g_i8_configured[device] && g_i8_ctx[device] == ctx) return 0;
    cudaError_t e = cudaFuncSetAttribute(i8::attention_i8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)i8::SMEM_BYTES);
    if (e != cudaSuccess) return (int)e;
    int nsm = 0;
    e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess) return (int)e;
    g_i8_nsm[device] = nsm;
    g_i8_ctx[device] = ctx;
    g_i8_configured[device] = 1;
    return 0;
}

// Pieces per tile (1-4): the fewest that minimise the waves of two-CTA-per-SM slots a tile-time
// each, e.g. 444 tiles on 148 SMs: whole tiles take 2 waves, halves 3 waves of half a tile (1.5).
static int i8_pieces(long T, int nsm) {
    const long slots = 2L * nsm;
    int best = 1;
    double cost = (double)((T + slots - 1) / slots);
    for (int P = 2; P <= 4; ++P) {
        const double c = (double)((P * T + slots - 1) / slots) / P;
        if (c < cost - 1e-9) {
            cost = c;
            best = P;
        }
    }
    return best;
}
static size_t i8_ws_bytes(int P, int H, int Lq) { return (size_t)P * Lq * H * (i8::D + 1) * sizeof(float); }

int encode_tmap_2d_u8(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                      uint32_t box_inner, uint32_t box_outer);

}  // namespace ss

namespace ss {

static int quant_launch(const void *k, int H, int Lk, int p0, int p1, int8_t *k_i8, float *ks, cudaStream_t stream,
                        KvRing ring) {
    if (!k || !k_i8 || !ks) return SS_ERR_POINTER;
    const int npages = (Lk + i8::PAGE - 1) / i8::PAGE;
    if (H <= 0 || Lk <= 0 || p0 < 0 || p1 > npages || p0 > p1 || H > 65535) return SS_ERR_SHAPE;
    if (ring_check(ring, Lk) || ring.phys_rows(Lk) * H * i8::D >= (1L << 31)) return SS_ERR_SHAPE;
    if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(k_i8)) & 15u) return SS_ERR_POINTER;
    if (reinterpret_cast<uintptr_t>(ks) & 3u) return SS_ERR_POINTER;
    if (p0 == p1) return 0;
    i8::quant_k_pages_kernel<<<dim3((unsigned)(p1 - p0), (unsigned)H), 256, 0, stream>>>(
        static_cast<const __nv_bfloat16 *>(k), H, Lk, p0, npages, k_i8, ks, ring);
    return (int)cudaGetLastError();
}

}  // namespace ss

extern "C" int ss_quant_k_pages(const void *k, int H, int Lk, int p0, int p1, int8_t *k_i8, float *ks, void *stream) {
    return ss::quant_launch(k, H, Lk, p0, p1, k_i8, ks, static_cast<cudaStream_t>(stream), ss::KvRing());
}

extern "C" int ss_quant_k_pages_ring(const void *k, int H, int Lk, int p0, int p1, int8_t *k_i8, float *ks,
                                     int ring_sink, int ring_cap, int ring_head, const int *ring_head_dev,
                                     void *stream) {
    ss::KvRing ring;
    ring.S = ring_sink;
    ring.C = ring_cap;
    ring.head = ring_head;
    ring.head_dev = ring_head_dev;
    if (ring_cap <= 0) return SS_ERR_SHAPE;
    return ss::quant_launch(k, H, Lk, p0, p1, k_i8, ks, static_cast<cudaStream_t>(stream), ring);
}

extern "C" int ss_attention_i8_workspace_bytes(int H, int Lq, size_t *bytes) {
    if (!bytes || H <= 0 || Lq <= 0) return SS_ERR_SHAPE;
    int device;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return (int)e;
    int rc = ss::attention_i8_prepare(device);
    if (rc) return rc;
    const int P = ss::i8_pieces((long)((Lq + 127) / 128) * H, ss::g_i8_nsm[device]);
    *bytes = P > 1 ? ss::i8_ws_bytes(P, H, Lq) : 0;
    return 0;
}

namespace ss {

static int attention_i8_launch(const void *q, const int8_t *k_i8, const float *ks, const void *v, const int32_t *ids,
                               int H, int Lq, int Lk, int block, int n_ids, float scale, void *out, int out_dtype,
                               float *lse, int *status, void *workspace, size_t workspace_bytes, void *stream,
                               KvRing ring) {
    using namespace ss::i8;
    if (!q || !k_i8 || !ks || !v || !ids || !out) return SS_ERR_POINTER;
    if (H <= 0 || Lq <= 0 || Lk <= 0 || n_ids <= 0 || (block != 64 && block != 128) || H > 65535) return SS_ERR_SHAPE;
    if (out_dtype != 0 && out_dtype != 1) return SS_ERR_SHAPE;
    const int npages = (Lk + PAGE - 1) / PAGE;
    if (npages > MAX_PAGES || (long)Lq * H * D >= (1L << 31)) return SS_ERR_SHAPE;
    if (ring_check(ring, Lk) || ring.phys_rows(Lk) * H * D >= (1L << 31)) return SS_ERR_SHAPE;
    const uint64_t kv_rows = (uint64_t)ring.phys_rows(Lk);
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_i8) | reinterpret_cast<uintptr_t>(v) |
         reinterpret_cast<uintptr_t>(out)) & 15u)
        return SS_ERR_POINTER;
    if ((reinterpret_cast<uintptr_t>(ks) | reinterpret_cast<uintptr_t>(lse)) & 3u) return SS_ERR_POINTER;
    int device;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return (int)e;
    int rc = ss::attention_i8_prepare(device);
    if (rc) return rc;

    Params prm;
    prm.q = static_cast<const __nv_bfloat16 *>(q);
    prm.ks = ks;
    prm.ids = ids;
    prm.out = out;
    prm.lse = lse;
    prm.status = status;
    prm.H = H;
    prm.Lq = Lq;
    prm.Lk = Lk;
    prm.block = block;
    prm.n_ids = n_ids;
    prm.nqb = (Lq + block - 1) / block;
    prm.nkb = (Lk + block - 1) / block;
    prm.npages = npages;
    prm.out_fp32 = out_dtype;
    prm.c = (float)((double)scale * 1.4426950408889634);
    prm.ring = ring;
    const unsigned ntiles = (unsigned)((Lq + 127) / 128);
    int P = workspace ? ss::i8_pieces((long)ntiles * H, ss::g_i8_nsm[device]) : 1;
    if (P > 1 && workspace_bytes < ss::i8_ws_bytes(P, H, Lq)) return SS_ERR_WORKSPACE;
    if (P > 1 && (reinterpret_cast<uintptr_t>(workspace) & 255u)) return SS_ERR_POINTER;
    prm.pieces = P;
    prm.ws_o = P > 1 ? static_cast<float *>(workspace) : nullptr;
    prm.ws_lse = P > 1 ? prm.ws_o + (size_t)P * Lq * H * D : nullptr;

    CUtensorMap tk, tv;
    if (ss::encode_tmap_2d_u8(&tk, k_i8, (uint64_t)H * D, kv_rows, (uint64_t)H * D, 128, PAGE))
        return SS_ERR_DRIVER;
    if (ss::encode_tmap_2d_bf16(&tv, v, (uint64_t)H * D, kv_rows, (uint64_t)H * D * 2, 64, PAGE))
        return SS_ERR_DRIVER;
    attention_i8_kernel<<<dim3(ntiles, (unsigned)H, (unsigned)P), NTHREADS, SMEM_BYTES,
                          static_cast<cudaStream_t>(stream)>>>(tk, tv, prm);
    e = cudaGetLastError();
    if (e != cudaSuccess || P == 1) return (int)e;
    return ss_lse_merge(prm.ws_o, prm.ws_lse, P, H, Lq, out, out_dtype, lse, stream);
}

}  // namespace ss

extern "C" int ss_attention_i8(const void *q, const int8_t *k_i8, const float *ks, const void *v, const int32_t *ids,
                               int H, int Lq, int Lk, int block, int n_ids, float scale, void *out, int out_dtype,
                               float *lse, int *status, void *workspace, size_t workspace_bytes, void *stream) {
    return ss::attention_i8_launch(q, k_i8, ks, v, ids, H, Lq, Lk, block, n_ids, scale, out, out_dtype, lse, status,
                                   workspace, workspace_bytes, stream, ss::KvRing());
}

extern "C" int ss_attention_i8_ring(const void *q, const int8_t *k_i8, const float *ks, const void *v,
                                    const int32_t *ids, int H, int Lq, int Lk, int block, int n_ids, float scale,
                                    void *out, int out_dtype, float *lse, int *status, int ring_sink, int ring_cap,
                                    int ring_head, const int *ring_head_dev, void *workspace, size_t workspace_bytes,
                                    void *stream) {
    ss::KvRing ring;
    ring.S = ring_sink;
    ring.C = ring_cap;
    ring.head = ring_head;
    ring.head_dev = ring_head_dev;
    if (ring_cap <= 0) return SS_ERR_SHAPE;
    return ss::attention_i8_launch(q, k_i8, ks, v, ids, H, Lq, Lk, block, n_ids, scale, out, out_dtype, lse, status,
                                   workspace, workspace_bytes, stream, ring);
}
