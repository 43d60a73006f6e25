// attention_sm100.cu -- block-sparse flash attention for sm_100a (tcgen05 + TMEM + TMA).
//
// Computes, for every query row t and head h,
//     out[t,h,:] = softmax(scale * q[t,h,:] . K_S^T) V_S,   lse[h,t] = ln sum exp(scale * q.K_S^T)
// where S is the set of valid tokens of the KV blocks listed for t's query block. This is the
// operation of the reference's page-LUT kernel `_attn_fwd` (local_experiments/
// gap_exact_round_kernel.py:4-137, wrapped by `exact` in local_experiments/video_runtime_v1/
// attention.py:15-24) and of the sm_80 CUDA `exact<>` kernel (local_experiments/video_runtime_v1/
// csrc/fixed15_attention.cu:248-387); the design below is sm_100a-specific.
//
// Work decomposition
//   One CTA per (head, 128-row query tile). With 64-token router blocks a tile holds two query
//   blocks; the CTA walks the union of their block lists and masks, per 64-row half, the blocks
//   that half did not select. With 128-token blocks a tile is exactly one query block.
//   The union is walked in steps of 128 KV tokens (two 64-token sub-blocks, each gathered by
//   TMA at its own row offset, so the two need not be adjacent). CTAs are ordered head-major
//   so the CTAs resident at one time share a few heads' K/V in L2.
//
// Warp roles (384 threads; every role runs on a whole converged warp and issues its
// single-thread instructions -- TMA, tcgen05.mma, tcgen05.commit -- from an elected lane)
//   warp 0      K producer: TMA loads of K steps into a 3-stage ring
//   warp 1      TMEM allocator + tcgen05.mma issuer
//   warp 2      V producer: TMA loads of V steps into a 3-stage ring
//   warp 3      block-list construction in the prologue, idle afterwards
//   warps 4-11  softmax: group g (warps 4+4g .. 7+4g) owns sub-block g of every step, i.e. score
//               columns [64g, 64g+64). In the prologue the groups copy the Q tile into TMEM (the QK
//               MMA reads Q from TMEM, so shared-memory bandwidth goes to K and V only). Thread r
//               of a group owns query row r (TMEM lane r). Per step both groups copy all 128 scores
//               of their row to registers and release the S buffer at once (the QK MMA two steps
//               ahead can start), derive the same running max (no exchange needed), exponentiate
//               their 64 columns, write P (bf16) to their P columns in TMEM (the PV MMA reads P
//               from TMEM) and rescale their half of the shared O accumulator when the running
//               max grows by more than 2^8.
//
// TMEM (512 columns): S of step parity b at [128b, 128b+128); Q (bf16 pairs) at [256, 320); P of
// group g at [320+32g, 352+32g); O at [384, 512).
// MMAs: S = Q K^T (M=128, N=128, K=128; A = Q in TMEM, B = K K-major in shared memory, 128-byte
//       swizzle), O += P V (M=128, N=128, K=128 tokens; A = P in TMEM, B = V MN-major in shared
//       memory). tcgen05.mma instructions of one thread execute in order, so the QK MMA that
//       reuses an S buffer (issued after the PV MMA that reads P from it) cannot overtake that read.
// Every mbarrier wait is bounded (common.cuh); on timeout the CTA drains its TMA loads and MMAs,
// frees TMEM, sets SS_DEV_TIMEOUT in *status and exits.
#include "common.cuh"

namespace ss {
namespace attn {

constexpr int D = 128;
constexpr int TILE_M = 128;
constexpr int SUB = 64;
constexpr int KSTAGES = 3;
constexpr int VSTAGES = 3;
constexpr int NTHREADS = 384;
constexpr uint32_t REGION = 16384;                 // 128 rows x 128 B: one 64-column half of a step
constexpr uint32_t KV_BYTES = 2 * REGION;          // 128 tokens x 128 dims bf16
constexpr uint32_t OFF_K = 0;
constexpr uint32_t OFF_V = OFF_K + KSTAGES * KV_BYTES;
constexpr uint32_t OFF_BAR = OFF_V + VSTAGES * KV_BYTES;
constexpr int NBAR = 24;
constexpr uint32_t OFF_MISC = OFF_BAR + NBAR * 8;
constexpr uint32_t OFF_LSUM = OFF_MISC + 64;       // [2 groups][128 rows] partial row sums
constexpr uint32_t OFF_DYN = OFF_LSUM + 2 * 128 * 4;   // bitmaps, then the sub-block list
constexpr uint32_t SMEM_LIMIT = 232448;            // 227 KB opt-in maximum per CTA
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t TMEM_S = 0, TMEM_Q = 256, TMEM_P = 320, TMEM_O = 384;

enum Bar {
    Q_FULL = 0,                  // Q tile copied into TMEM (256 softmax threads)
    K_FULL = 1,
    K_EMPTY = K_FULL + KSTAGES,
    V_FULL = K_EMPTY + KSTAGES,
    V_EMPTY = V_FULL + VSTAGES,
    S_FULL = V_EMPTY + VSTAGES,  // per S buffer (step parity): QK result ready
    S_FREE = S_FULL + 2,         // per S buffer: both groups copied the scores out (256 arrivals)
    P_FULL = S_FREE + 2,         // per step parity: P written by both groups (256 arrivals)
    O_DONE = P_FULL + 2,         // PV of a step completed (O up to date, P consumed)
    XSUM = O_DONE + 1,           // epilogue: both groups' row sums written (256 arrivals)
    DRAIN = XSUM + 1,
    NBAR_USED
};
static_assert(NBAR_USED <= NBAR, "barrier space");

constexpr uint32_t IDESC_QK = idesc_bf16_f32(128, 128, false, false);
constexpr uint32_t IDESC_PV = idesc_bf16_f32(128, 128, false, true);

// sub-block entry: bits 0-19 first token, bits 20-26 valid tokens (0..64), bits 27-28 row-half mask
__device__ __forceinline__ uint32_t entry(uint32_t start, uint32_t valid, uint32_t mask) {
    return start | (valid << 20) | (mask << 27);
}
__device__ __forceinline__ int e_start(uint32_t e) { return (int)(e & 0xFFFFFu); }
__device__ __forceinline__ int e_valid(uint32_t e) { return (int)((e >> 20) & 127u); }

struct Params {
    const __nv_bfloat16 *q;
    const int32_t *ids;
    void *out;
    float *lse;
    int *status;
    int H, Lq, Lk, block, n_ids, qb, kb, ntiles, nwords, out_fp32;
    float scale_log2;  // scale * log2(e)
};

__device__ __forceinline__ bool warp_all_ok(bool ok) { return __all_sync(0xffffffffu, ok) != 0; }

__device__ __forceinline__ float max3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
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
    asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ float f2_lo(uint64_t x) { return __uint_as_float((uint32_t)x); }
__device__ __forceinline__ float f2_hi(uint64_t x) { return __uint_as_float((uint32_t)(x >> 32)); }

// 2^x on the FMA pipe for a pair of arguments (x <= 8 here; x below -125 is clamped, giving
// ~2^-125 instead of 0). x = n + f with n = round(x), f in [-0.5, 0.5]; 2^f by the minimax cubic
// for relative error on [-0.5, 0.5] (coefficients fitted by the Remez exchange algorithm, max
// relative error 7.5e-5, below bf16 rounding of P); 2^n is added to the exponent bits.
// Offloading a share of the exponentials from the MUFU unit keeps it from bounding the softmax.
__device__ __forceinline__ void exp2_poly2(float x0, float x1, float &y0, float &y1) {
    constexpr float kRound = 12582912.0f;  // 1.5 * 2^23: x + kRound rounds x to an integer
    const uint64_t x = f2_pack(fmaxf(x0, -125.f), fmaxf(x1, -125.f));
    const uint64_t t = f2_add(x, f2_pack(kRound, kRound));
    const uint64_t n = f2_add(t, f2_pack(-kRound, -kRound));
    const uint64_t f = f2_fma(n, f2_pack(-1.f, -1.f), x);
    uint64_t p = f2_fma(f2_pack(0.0551716685f, 0.0551716685f), f, f2_pack(0.2426111251f, 0.2426111251f));
    p = f2_fma(p, f, f2_pack(0.6932609677f, 0.6932609677f));
    p = f2_fma(p, f, f2_pack(0.9999280572f, 0.9999280572f));
    const int n0 = (int)(uint32_t)t - 0x4B400000, n1 = (int)(uint32_t)(t >> 32) - 0x4B400000;
    y0 = __int_as_float(__float_as_int(f2_lo(p)) + (n0 << 23));
    y1 = __int_as_float(__float_as_int(f2_hi(p)) + (n1 << 23));
}

// D[tmem] (+)= A[tmem] * B[smem]
__device__ __forceinline__ void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t *r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

__global__ void __launch_bounds__(NTHREADS, 1)
sparse_attention_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                        const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t sK = sbase + OFF_K, sV = sbase + OFF_V;
    const uint32_t bar0 = sbase + OFF_BAR;
    auto bar = [&](int i) -> uint32_t { return bar0 + 8u * (uint32_t)i; };
    volatile uint32_t *tmem_slot = reinterpret_cast<volatile uint32_t *>(smem + OFF_MISC);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_MISC + 4);
    volatile int *nsub_slot = reinterpret_cast<volatile int *>(smem + OFF_MISC + 8);
    volatile int *badid_flag = reinterpret_cast<volatile int *>(smem + OFF_MISC + 12);
    float *lsum = reinterpret_cast<float *>(smem + OFF_LSUM);
    uint32_t *bmA = reinterpret_cast<uint32_t *>(smem + OFF_DYN);
    uint32_t *bmB = bmA + p.nwords;
    uint32_t *steps = bmB + p.nwords;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.x / p.ntiles;
    const int tile = blockIdx.x % p.ntiles;
    const bool pair = (p.block == 64);
    const int qblkA = pair ? 2 * tile : tile;
    const int qblkB = pair ? 2 * tile + 1 : -1;

    // ---------------- prologue: barriers, TMEM, the tile's sub-block list ----------------
    if (tid == 0) {
        *abort_flag = 0;
        *badid_flag = 0;
        mbar_init(bar(Q_FULL), 256);
        for (int s = 0; s < KSTAGES; ++s) {
            mbar_init(bar(K_FULL + s), 1);
            mbar_init(bar(K_EMPTY + s), 1);
        }
        for (int s = 0; s < VSTAGES; ++s) {
            mbar_init(bar(V_FULL + s), 1);
            mbar_init(bar(V_EMPTY + s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(bar(S_FULL + b), 1);
            mbar_init(bar(S_FREE + b), 256);
            mbar_init(bar(P_FULL + b), 256);
        }
        mbar_init(bar(O_DONE), 1);
        mbar_init(bar(XSUM), 256);
        mbar_init(bar(DRAIN), 1);
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tm_k);
        prefetch_tmap(&tm_v);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32((const void *)tmem_slot), TMEM_COLS);
        tmem_relinquish();
    }
    for (int w = tid; w < 2 * p.nwords; w += NTHREADS) bmA[w] = 0u;
    __syncthreads();
    {
        const int32_t *la = p.ids + ((size_t)h * p.qb + qblkA) * p.n_ids;
        const int32_t *lb = (qblkB >= 0 && qblkB < p.qb) ? p.ids + ((size_t)h * p.qb + qblkB) * p.n_ids : nullptr;
        for (int i = tid; i < p.n_ids; i += NTHREADS) {
            int a = la[i];
            if (a >= p.kb) *badid_flag = 1;
            else if (a >= 0) atomicOr(&bmA[a >> 5], 1u << (a & 31));
            if (lb) {
                int b = lb[i];
                if (b >= p.kb) *badid_flag = 1;
                else if (b >= 0) atomicOr(&bmB[b >> 5], 1u << (b & 31));
            }
        }
    }
    __syncthreads();
    if (warp == 3) {
        // ascending compaction of the union bitmap into sub-block entries
        const int per = p.block / SUB;  // sub-blocks per router block
        int carry = 0;
        for (int w0 = 0; w0 < p.nwords; w0 += 32) {
            int w = w0 + lane;
            uint32_t a = w < p.nwords ? bmA[w] : 0u, b = w < p.nwords ? bmB[w] : 0u, u = a | b;
            int cnt = __popc(u) * per, incl = cnt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                int y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            int pos = carry + incl - cnt;
            while (u) {
                int bit = __ffs(u) - 1;
                u &= u - 1;
                int j = w * 32 + bit;
                uint32_t m = pair ? (((a >> bit) & 1u) | (((b >> bit) & 1u) << 1)) : 3u;
                for (int s = 0; s < per; ++s) {
                    int t0 = j * p.block + s * SUB;
                    int valid = min(SUB, max(0, p.Lk - t0));
                    steps[pos++] = entry((uint32_t)t0, (uint32_t)valid, m);
                }
            }
            carry += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (lane == 0) {
            if (carry & 1) steps[carry++] = entry(0u, 0u, 0u);  // pad to whole 128-token steps
            *nsub_slot = carry;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int nsteps = *nsub_slot / 2;
    const int xh = h * D;

    if (warp == 0 || warp == 2) {
        // ---------------- K (warp 0) / V (warp 2) producer ----------------
        const bool isk = warp == 0;
        const CUtensorMap *tm = isk ? &tm_k : &tm_v;
        const uint32_t ring = isk ? sK : sV;
        const int stages = isk ? KSTAGES : VSTAGES;
        const int full = isk ? K_FULL : V_FULL, empty = isk ? K_EMPTY : V_EMPTY;
        int issued = 0;
        bool ok = true;
        for (int j = 0; j < nsteps; ++j) {
            const int st = j % stages, it = j / stages;
            if (it > 0) ok = warp_all_ok(mbar_wait(bar(empty + st), (it - 1) & 1, abort_flag));
            if (!ok) break;
            const int t0 = e_start(steps[2 * j]), t1 = e_start(steps[2 * j + 1]);
            const uint32_t dst = ring + st * KV_BYTES;
            if (elect_one()) {
                mbar_arrive_expect_tx(bar(full + st), KV_BYTES);
                tma_load_2d(dst, tm, xh, t0, bar(full + st));
                tma_load_2d(dst + REGION, tm, xh + 64, t0, bar(full + st));
                tma_load_2d(dst + REGION / 2, tm, xh, t1, bar(full + st));
                tma_load_2d(dst + REGION + REGION / 2, tm, xh + 64, t1, bar(full + st));
            }
            __syncwarp();
            issued = j + 1;
        }
        if (!ok) {  // drain: loads still landing in shared memory
            volatile int never = 0;
            for (int j = max(0, issued - stages); j < issued; ++j)
                mbar_wait(bar(full + j % stages), (j / stages) & 1, &never);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (nsteps > 0) {
            bool ok = warp_all_ok(mbar_wait(bar(Q_FULL), 0, abort_flag));
            tc_fence_after();
            auto issue_qk = [&](int j) -> bool {  // S_(j&1) = Q K_j^T
                const int st = j % KSTAGES, it = j / KSTAGES, b = j & 1;
                if (!warp_all_ok(mbar_wait(bar(K_FULL + st), it & 1, abort_flag))) return false;
                tc_fence_after();
                const uint32_t dk = sK + st * KV_BYTES;
                if (elect_one()) {
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk)
                        mma_bf16_ts(tmem + TMEM_S + 128 * b, tmem + TMEM_Q + kk * 8,
                                    smem_desc_sw128(dk + (kk >> 2) * REGION + (kk & 3) * 32, 16, 1024), IDESC_QK,
                                    kk > 0 ? 1u : 0u);
                    tc_commit(bar(S_FULL + b));
                    tc_commit(bar(K_EMPTY + st));
                }
                __syncwarp();
                return true;
            };
            auto issue_pv = [&](int j) -> bool {  // O += P_j V_j
                const int st = j % VSTAGES, it = j / VSTAGES, b = j & 1;
                if (!warp_all_ok(mbar_wait(bar(P_FULL + b), (j >> 1) & 1, abort_flag))) return false;
                if (!warp_all_ok(mbar_wait(bar(V_FULL + st), it & 1, abort_flag))) return false;
                tc_fence_after();
                const uint32_t dv = sV + st * KV_BYTES;
                if (elect_one()) {
                    // tokens 16kk.. of the step: P of sub-block kk/4 sits in the P columns of group kk/4
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk)
                        mma_bf16_ts(tmem + TMEM_O, tmem + TMEM_P + 8 * kk,
                                    smem_desc_sw128(dv + kk * 2048, REGION, 1024), IDESC_PV,
                                    (j > 0 || kk > 0) ? 1u : 0u);
                    tc_commit(bar(O_DONE));
                    tc_commit(bar(V_EMPTY + st));
                }
                __syncwarp();
                return true;
            };
            if (ok) ok = issue_qk(0);
            if (ok && nsteps > 1) ok = issue_qk(1);
            for (int j = 0; j < nsteps && ok; ++j) {
                if (j + 2 < nsteps) {
                    // S_(j&1) is free once both groups copied step j's scores out
                    ok = warp_all_ok(mbar_wait(bar(S_FREE + (j & 1)), (j >> 1) & 1, abort_flag));
                    if (ok) ok = issue_qk(j + 2);
                }
                if (ok) ok = issue_pv(j);
            }
            // every MMA issued above has completed once DRAIN fires
            if (elect_one()) tc_commit(bar(DRAIN));
            __syncwarp();
            volatile int never = 0;
            mbar_wait(bar(DRAIN), 0, &never);
        }
    } else if (warp >= 4) {
        // ---------------- softmax groups + epilogue ----------------
        const int grp = (warp - 4) >> 2;    // sub-block (score columns [64g, 64g+64)) of each step
        const int r = (tid - 128) & 127;    // row within the tile == TMEM lane
        const int half = r >> 6;            // which 64-row query block of the pair
        const uint32_t lane_base = tmem + ((uint32_t)((r >> 5) * 32) << 16);
        const int row = tile * TILE_M + r;
        // Q tile -> TMEM: group g copies dims [64g, 64g + 64) of row r as bf16 pairs
        {
            uint32_t qv[32];
            if (row < p.Lq) {
                const uint4 *src = reinterpret_cast<const uint4 *>(p.q + ((size_t)row * p.H + h) * D + 64 * grp);
#pragma unroll
                for (int x = 0; x < 8; ++x) {
                    const uint4 v = src[x];
                    qv[4 * x] = v.x;
                    qv[4 * x + 1] = v.y;
                    qv[4 * x + 2] = v.z;
                    qv[4 * x + 3] = v.w;
                }
            } else {
#pragma unroll
                for (int x = 0; x < 32; ++x) qv[x] = 0u;
            }
            tmem_st32(lane_base + TMEM_Q + 32 * grp, reinterpret_cast<const float *>(qv));
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar(Q_FULL));
        }
        const uint32_t o_addr = lane_base + TMEM_O + 64 * grp;   // this group's half of O
        const float sl2 = p.scale_log2;
        const uint64_t sl2x2 = f2_pack(sl2, sl2);
        float m = -INFINITY, l = 0.f;        // m identical in both groups; l partial per group
        bool ok = true;
        int j = 0;
        for (; j < nsteps && ok; ++j) {
            const int b = j & 1;
            ok = warp_all_ok(mbar_wait(bar(S_FULL + b), (j >> 1) & 1, abort_flag));
            if (!ok) break;
            tc_fence_after();
            const uint32_t s_addr = lane_base + TMEM_S + 128 * b + 64 * grp;
            const uint32_t e = steps[2 * j + grp], eo = steps[2 * j + (grp ^ 1)];
            // selection and valid length, warp-uniform (a warp lies within one 64-row half)
            const bool sel = (e >> (27 + half)) & 1u, selo = (eo >> (27 + half)) & 1u;
            const int valid = sel ? e_valid(e) : 0, valido = selo ? e_valid(eo) : 0;
            // row max over the whole step: both groups read all 128 columns, so both derive the
            // same running max without exchanging it; each keeps the 64 scores it exponentiates.
            float s[64];
            float mx = -INFINITY;
            if (sel) {
                tmem_ld32(s_addr, s);
                tmem_ld32(s_addr + 32, s + 32);
            }
            if (selo) {
                float t[64];
                const uint32_t o_s = lane_base + TMEM_S + 128 * b + 64 * (grp ^ 1);
                tmem_ld32(o_s, t);
                tmem_ld32(o_s + 32, t + 32);
                tmem_wait_ld();
                if (valido == SUB) {
                    float m0 = t[0], m1 = t[1], m2 = t[2], m3 = t[3];
#pragma unroll
                    for (int c = 4; c < 64; c += 8) {
                        m0 = max3(m0, t[c], t[c + 1]);
                        m1 = max3(m1, t[c + 2], t[c + 3]);
                        m2 = max3(m2, t[c + 4], t[c + 5]);
                        m3 = max3(m3, t[c + 6], t[c + 7]);
                    }
                    mx = max3(fmaxf(m0, m1), m2, m3);
                } else {
#pragma unroll
                    for (int c = 0; c < 64; ++c) mx = fmaxf(mx, c < valido ? t[c] : -INFINITY);
                }
            }
            if (sel) tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(bar(S_FREE + b));
            if (sel) {
                if (valid == SUB) {
                    float m0 = s[0], m1 = s[1], m2 = s[2], m3 = s[3];
#pragma unroll
                    for (int c = 4; c < 64; c += 8) {
                        m0 = max3(m0, s[c], s[c + 1]);
                        m1 = max3(m1, s[c + 2], s[c + 3]);
                        m2 = max3(m2, s[c + 4], s[c + 5]);
                        m3 = max3(m3, s[c + 6], s[c + 7]);
                    }
                    mx = max3(mx, fmaxf(m0, m1), fmaxf(m2, m3));
                } else {
#pragma unroll
                    for (int c = 0; c < 64; ++c) {
                        s[c] = c < valid ? s[c] : -INFINITY;
                        mx = fmaxf(mx, s[c]);
                    }
                }
            }
            // lazy rescale: move the reference max only when the row max grew by more than 2^8
            const float mnew = mx * sl2;
            float alpha = 1.f;
            bool grow = false;                   // an O row that is not all zeros must be scaled
            if (mnew > m + 8.0f) {
                grow = m != -INFINITY;
                alpha = grow ? ex2(m - mnew) : 0.f;
                l *= alpha;
                m = mnew;
            }
            // O and the P columns change through the previous step's PV; tcgen05.ld/st are
            // warp-collective, so the whole warp rescales its half of O if any of its rows must.
            bool o_ready = j == 0;
            if (j > 0 && __any_sync(0xffffffffu, grow)) {
                ok = warp_all_ok(mbar_wait(bar(O_DONE), (j - 1) & 1, abort_flag));
                if (!ok) break;
                tc_fence_after();
                o_ready = true;
#pragma unroll 1
                for (int c = 0; c < 2; ++c) {
                    float o[32];
                    tmem_ld32(o_addr + 32 * c, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int x = 0; x < 32; ++x) o[x] *= (grow ? alpha : 1.f);
                    tmem_st32(o_addr + 32 * c, o);
                }
            }
            // P = 2^(s*sl2 - m) as bf16 pairs over the first 32 columns this group read
            uint32_t pk[32];
            if (sel) {
                const float base = (m == -INFINITY) ? 0.f : m;
                const uint64_t nbx2 = f2_pack(-base, -base);
                uint64_t sa = 0, sb = 0;
#pragma unroll
                for (int c = 0; c < 64; c += 4) {
                    const uint64_t x0 = f2_fma(f2_pack(s[c], s[c + 1]), sl2x2, nbx2);
                    const uint64_t x1 = f2_fma(f2_pack(s[c + 2], s[c + 3]), sl2x2, nbx2);
                    float p0, p1, p2, p3;
                    if (c < 48) {   // MUFU
                        p0 = ex2(f2_lo(x0));
                        p1 = ex2(f2_hi(x0));
                        p2 = ex2(f2_lo(x1));
                        p3 = ex2(f2_hi(x1));
                    } else {        // FMA pipe (a quarter of the exponentials)
                        exp2_poly2(f2_lo(x0), f2_hi(x0), p0, p1);
                        exp2_poly2(f2_lo(x1), f2_hi(x1), p2, p3);
                    }
                    sa = f2_add(sa, f2_pack(p0, p1));
                    sb = f2_add(sb, f2_pack(p2, p3));
                    pk[c >> 1] = pack_bf16x2(p0, p1);
                    pk[(c >> 1) + 1] = pack_bf16x2(p2, p3);
                }
                const uint64_t st2 = f2_add(sa, sb);
                l += f2_lo(st2) + f2_hi(st2);
            } else {
#pragma unroll
                for (int x = 0; x < 32; ++x) pk[x] = 0u;
            }
            // the P columns are free once the previous step's PV has read them
            if (!o_ready) {
                ok = warp_all_ok(mbar_wait(bar(O_DONE), (j - 1) & 1, abort_flag));
                if (!ok) break;
                tc_fence_after();
            }
            const uint32_t p_addr = lane_base + TMEM_P + 32 * grp;
            tmem_st16(p_addr, pk);
            tmem_st16(p_addr + 16, pk + 16);
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar(P_FULL + b));
        }
        // epilogue: O is final once the last PV has completed
        bool have = ok && nsteps > 0;
        if (have) have = warp_all_ok(mbar_wait(bar(O_DONE), (nsteps - 1) & 1, abort_flag));
        if (have) tc_fence_after();
        lsum[grp * 128 + r] = l;
        mbar_arrive(bar(XSUM));
        const bool summed = warp_all_ok(mbar_wait(bar(XSUM), 0, abort_flag));
        const float lt = summed ? l + lsum[(grp ^ 1) * 128 + r] : 0.f;
        const float inv = lt > 0.f ? 1.f / lt : 0.f;
        const bool live = row < p.Lq && (pair ? (half == 0 ? qblkA < p.qb : qblkB < p.qb) : true);
        // warp-uniform conditions only: tcgen05.ld is warp-collective
        const bool fin = __all_sync(0xffffffffu, have && summed && !*abort_flag) != 0;
        // group g writes output columns [64g, 64g + 64) of its row
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
            const int col = 64 * grp + 32 * c;
            float o[32];
            if (fin) {
                tmem_ld32(lane_base + TMEM_O + col, o);
                tmem_wait_ld();
            }
#pragma unroll
            for (int x = 0; x < 32; ++x) o[x] = fin ? o[x] * inv : 0.f;
            if (live && (fin || nsteps == 0)) {
                if (p.out_fp32) {
                    float4 *dst = reinterpret_cast<float4 *>(reinterpret_cast<float *>(p.out) +
                                                             ((size_t)row * p.H + h) * D + col);
#pragma unroll
                    for (int x = 0; x < 8; ++x) dst[x] = make_float4(o[4 * x], o[4 * x + 1], o[4 * x + 2], o[4 * x + 3]);
                } else {
                    uint4 *dst = reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(p.out) +
                                                           ((size_t)row * p.H + h) * D + col);
#pragma unroll
                    for (int x = 0; x < 4; ++x)
                        dst[x] = make_uint4(pack_bf16x2(o[8 * x], o[8 * x + 1]), pack_bf16x2(o[8 * x + 2], o[8 * x + 3]),
                                            pack_bf16x2(o[8 * x + 4], o[8 * x + 5]),
                                            pack_bf16x2(o[8 * x + 6], o[8 * x + 7]));
                }
            }
        }
        if (live && (fin || nsteps == 0) && grp == 0 && p.lse)
            p.lse[(size_t)h * p.Lq + row] = lt > 0.f ? (m + __log2f(lt)) * 0.69314718055994530942f : -INFINITY;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
    if (tid == 0) {
        if (*abort_flag) report(p.status, SS_DEV_TIMEOUT);
        if (*badid_flag) report(p.status, SS_DEV_BADID);
    }
}

}  // namespace attn

int attention_smem_bytes(int Lk, int block, int n_ids, uint32_t *bytes) {
    const int kb = (Lk + block - 1) / block;
    const int nwords = (kb + 31) / 32;
    long max_sub = (block == 64) ? (long)std::min(2 * n_ids, kb) + 1 : 2L * std::min(n_ids, kb);
    long total = 1024 + attn::OFF_DYN + 8L * nwords + 4L * (max_sub + 2);
    *bytes = (uint32_t)total;
    return total <= (long)attn::SMEM_LIMIT ? 0 : SS_ERR_SMEM;
}

static int g_attn_configured[64] = {0};

int attention_prepare(int device) {
    if (device < 0 || device >= 64) return SS_ERR_SHAPE;
    if (g_attn_configured[device]) return 0;
    cudaError_t e = cudaFuncSetAttribute(attn::sparse_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)attn::SMEM_LIMIT);
    if (e != cudaSuccess) return (int)e;
    g_attn_configured[device] = 1;
    return 0;
}

}  // namespace ss

extern "C" int ss_attention_max_ids(int Lk, int block, int *max_ids) {
    if (!max_ids || Lk <= 0 || (block != 64 && block != 128)) return SS_ERR_SHAPE;
    int lo = 0, hi = (Lk + block - 1) / block;
    uint32_t b;
    while (lo < hi) {  // largest n that fits
        int mid = (lo + hi + 1) / 2;
        if (ss::attention_smem_bytes(Lk, block, mid, &b) == 0) lo = mid; else hi = mid - 1;
    }
    *max_ids = lo;
    return 0;
}

extern "C" int ss_attention(const void *q, const void *k, const void *v, const int32_t *ids, int H, int Lq, int Lk,
                            int block, int n_ids, float scale, void *out, int out_dtype, float *lse, int *status,
                            void *stream) {
    using namespace ss;
    if (!q || !k || !v || !ids || !out) return SS_ERR_POINTER;
    if (H <= 0 || Lq <= 0 || Lk <= 0 || n_ids <= 0 || (block != 64 && block != 128)) return SS_ERR_SHAPE;
    if (Lk >= (1 << 20) - 128 || (long)Lq * H * attn::D >= (1L << 31) || (long)Lk * H * attn::D >= (1L << 31))
        return SS_ERR_SHAPE;
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
         reinterpret_cast<uintptr_t>(out)) & 15u)
        return SS_ERR_POINTER;
    if (out_dtype != 0 && out_dtype != 1) return SS_ERR_SHAPE;
    uint32_t smem;
    int rc = attention_smem_bytes(Lk, block, n_ids, &smem);
    if (rc) return rc;
    int device;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return (int)e;
    rc = attention_prepare(device);
    if (rc) return rc;

    CUtensorMap tk, tv;
    const uint64_t row_bytes = (uint64_t)H * attn::D * 2;
    if (encode_tmap_2d_bf16(&tk, k, (uint64_t)H * attn::D, (uint64_t)Lk, row_bytes, 64, 64)) return SS_ERR_DRIVER;
    if (encode_tmap_2d_bf16(&tv, v, (uint64_t)H * attn::D, (uint64_t)Lk, row_bytes, 64, 64)) return SS_ERR_DRIVER;

    attn::Params prm;
    prm.q = static_cast<const __nv_bfloat16 *>(q);
    prm.ids = ids;
    prm.out = out;
    prm.lse = lse;
    prm.status = status;
    prm.H = H;
    prm.Lq = Lq;
    prm.Lk = Lk;
    prm.block = block;
    prm.n_ids = n_ids;
    prm.qb = (Lq + block - 1) / block;
    prm.kb = (Lk + block - 1) / block;
    prm.ntiles = (block == 64) ? (prm.qb + 1) / 2 : prm.qb;
    prm.nwords = (prm.kb + 31) / 32;
    prm.out_fp32 = out_dtype;
    prm.scale_log2 = scale * 1.4426950408889634f;
    dim3 grid((unsigned)(prm.ntiles * H));
    attn::sparse_attention_kernel<<<grid, attn::NTHREADS, smem, static_cast<cudaStream_t>(stream)>>>(tk, tv, prm);
    return (int)cudaGetLastError();
}
