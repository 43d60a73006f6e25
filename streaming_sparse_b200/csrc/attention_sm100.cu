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
//   its own TMA loads, so the two need not be adjacent). CTAs are ordered head-major so the
//   CTAs resident at one time share a few heads' K/V in L2.
//
// Warp roles (256 threads)
//   warp 0      TMA producer: Q once, then K and V sub-blocks into a 2-stage ring
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2-3   block-list construction in the prologue, idle afterwards
//   warps 4-7   softmax: thread r owns query row r (TMEM lane r); reads S from TMEM, applies the
//               masks, keeps the running max/sum, writes P (bf16) to shared memory, rescales the
//               O accumulator in TMEM when the running max grows by more than 2^8, and runs the
//               epilogue.
//
// TMEM (512 columns): S double buffer at columns [0,128) and [128,256); O at [256,384).
// MMAs: S = Q K^T (M=128, N=128, K=128, both K-major, 128-byte swizzle) and
//       O += P V   (M=128, N=128, K=128 tokens; P K-major, V MN-major).
// Every mbarrier wait is bounded (common.cuh); on timeout the CTA drains its TMA loads and MMAs,
// frees TMEM, sets SS_DEV_TIMEOUT in *status and exits.
#include "common.cuh"

namespace ss {
namespace attn {

constexpr int D = 128;
constexpr int TILE_M = 128;
constexpr int SUB = 64;
constexpr int STAGES = 2;
constexpr int NTHREADS = 256;
constexpr uint32_t REGION = 16384;                 // 128 rows x 128 B: one 64-column half
constexpr uint32_t Q_BYTES = 2 * REGION;           // 128 rows x 128 dims bf16
constexpr uint32_t KV_BYTES = 2 * REGION;          // 128 tokens x 128 dims bf16
constexpr uint32_t P_BYTES = 2 * REGION;           // 128 rows x 128 tokens bf16
constexpr uint32_t OFF_Q = 0;
constexpr uint32_t OFF_K = OFF_Q + Q_BYTES;
constexpr uint32_t OFF_V = OFF_K + STAGES * KV_BYTES;
constexpr uint32_t OFF_P = OFF_V + STAGES * KV_BYTES;
constexpr uint32_t OFF_BAR = OFF_P + P_BYTES;
constexpr int NBAR = 16;
constexpr uint32_t OFF_MISC = OFF_BAR + NBAR * 8;
constexpr uint32_t OFF_DYN = OFF_MISC + 64;        // bitmaps, then the sub-block list
constexpr uint32_t SMEM_LIMIT = 232448;            // 227 KB opt-in maximum per CTA
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t TMEM_O = 256;

enum Bar { Q_FULL = 0, K_FULL = 1, V_FULL = 3, K_EMPTY = 5, V_EMPTY = 7, S_FULL = 9, S_FREE = 11,
           P_FULL = 13, O_DONE = 14, DRAIN = 15 };

constexpr uint32_t IDESC_QK = idesc_bf16_f32(128, 128, false, false);
constexpr uint32_t IDESC_PV = idesc_bf16_f32(128, 128, false, true);

// sub-block entry: bits 0-19 first token, bits 20-26 valid tokens (0..64), bits 27-28 row-half mask
__device__ __forceinline__ uint32_t entry(uint32_t start, uint32_t valid, uint32_t mask) {
    return start | (valid << 20) | (mask << 27);
}
__device__ __forceinline__ int e_start(uint32_t e) { return (int)(e & 0xFFFFFu); }
__device__ __forceinline__ int e_valid(uint32_t e) { return (int)((e >> 20) & 127u); }

struct Params {
    const int32_t *ids;
    void *out;
    float *lse;
    int *status;
    int H, Lq, Lk, block, n_ids, qb, kb, ntiles, nwords, out_fp32;
    float scale_log2;  // scale * log2(e)
};

__device__ __forceinline__ bool warp_all_ok(bool ok) { return __all_sync(0xffffffffu, ok) != 0; }

__global__ void __launch_bounds__(NTHREADS, 1)
sparse_attention_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t sQ = sbase + OFF_Q, sK = sbase + OFF_K, sV = sbase + OFF_V, sP = sbase + OFF_P;
    const uint32_t bar0 = sbase + OFF_BAR;
    auto bar = [&](int i) -> uint32_t { return bar0 + 8u * (uint32_t)i; };
    volatile uint32_t *tmem_slot = reinterpret_cast<volatile uint32_t *>(smem + OFF_MISC);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_MISC + 4);
    volatile int *nsub_slot = reinterpret_cast<volatile int *>(smem + OFF_MISC + 8);
    volatile int *badid_flag = reinterpret_cast<volatile int *>(smem + OFF_MISC + 12);
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
        mbar_init(bar(Q_FULL), 1);
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(bar(K_FULL + s), 1);
            mbar_init(bar(V_FULL + s), 1);
            mbar_init(bar(K_EMPTY + s), 1);
            mbar_init(bar(V_EMPTY + s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(bar(S_FULL + b), 1);
            mbar_init(bar(S_FREE + b), 128);
        }
        mbar_init(bar(P_FULL), 128);
        mbar_init(bar(O_DONE), 1);
        mbar_init(bar(DRAIN), 1);
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tm_q);
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
    if (warp == 2) {
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

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0 && nsteps > 0) {
            const int q0 = tile * TILE_M;
            const int xh = h * D;
            mbar_arrive_expect_tx(bar(Q_FULL), Q_BYTES);
            tma_load_2d(sQ, &tm_q, xh, q0, bar(Q_FULL));
            tma_load_2d(sQ + REGION, &tm_q, xh + 64, q0, bar(Q_FULL));
            int issued = 0;
            bool ok = true;
            for (int j = 0; j < nsteps && ok; ++j) {
                const int st = j % STAGES, it = j / STAGES;
                const int t0 = e_start(steps[2 * j]), t1 = e_start(steps[2 * j + 1]);
                if (it > 0) ok = mbar_wait(bar(K_EMPTY + st), (it - 1) & 1, abort_flag);
                if (!ok) break;
                const uint32_t dk = sK + st * KV_BYTES;
                mbar_arrive_expect_tx(bar(K_FULL + st), KV_BYTES);
                tma_load_2d(dk, &tm_k, xh, t0, bar(K_FULL + st));
                tma_load_2d(dk + REGION, &tm_k, xh + 64, t0, bar(K_FULL + st));
                tma_load_2d(dk + REGION / 2, &tm_k, xh, t1, bar(K_FULL + st));
                tma_load_2d(dk + REGION + REGION / 2, &tm_k, xh + 64, t1, bar(K_FULL + st));
                if (it > 0) ok = mbar_wait(bar(V_EMPTY + st), (it - 1) & 1, abort_flag);
                const uint32_t dv = sV + st * KV_BYTES;
                if (ok) {
                    mbar_arrive_expect_tx(bar(V_FULL + st), KV_BYTES);
                    tma_load_2d(dv, &tm_v, xh, t0, bar(V_FULL + st));
                    tma_load_2d(dv + REGION, &tm_v, xh + 64, t0, bar(V_FULL + st));
                    tma_load_2d(dv + REGION / 2, &tm_v, xh, t1, bar(V_FULL + st));
                    tma_load_2d(dv + REGION + REGION / 2, &tm_v, xh + 64, t1, bar(V_FULL + st));
                }
                issued = j + 1;
            }
            if (!ok) {
                // drain: the loads of the last STAGES steps may still be landing in shared memory
                volatile int never = 0;
                for (int j = max(0, issued - STAGES); j < issued; ++j) {
                    const int st = j % STAGES, it = j / STAGES;
                    mbar_wait(bar(K_FULL + st), it & 1, &never);
                    mbar_wait(bar(V_FULL + st), it & 1, &never);
                }
                mbar_wait(bar(Q_FULL), 0, &never);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0 && nsteps > 0) {
            bool ok = mbar_wait(bar(Q_FULL), 0, abort_flag);
            tc_fence_after();
            auto issue_pv = [&](int i) -> bool {
                const int st = i % STAGES, it = i / STAGES;
                if (!mbar_wait(bar(P_FULL), i & 1, abort_flag)) return false;
                if (!mbar_wait(bar(V_FULL + st), it & 1, abort_flag)) return false;
                tc_fence_after();
                const uint32_t dv = sV + st * KV_BYTES;
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint64_t a = smem_desc_sw128(sP + (kk >> 2) * REGION + (kk & 3) * 32, 16, 1024);
                    const uint64_t b = smem_desc_sw128(dv + kk * 2048, REGION, 1024);
                    mma_bf16_ss(tmem + TMEM_O, a, b, IDESC_PV, (i > 0 || kk > 0) ? 1u : 0u);
                }
                tc_commit(bar(O_DONE));
                tc_commit(bar(V_EMPTY + st));
                return true;
            };
            for (int j = 0; j < nsteps && ok; ++j) {
                const int st = j % STAGES, it = j / STAGES, b = j & 1;
                ok = mbar_wait(bar(K_FULL + st), it & 1, abort_flag);
                if (ok && j >= 2) ok = mbar_wait(bar(S_FREE + b), ((j - 2) >> 1) & 1, abort_flag);
                if (!ok) break;
                tc_fence_after();
                const uint32_t dk = sK + st * KV_BYTES;
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint32_t off = (kk >> 2) * REGION + (kk & 3) * 32;
                    const uint64_t a = smem_desc_sw128(sQ + off, 16, 1024);
                    const uint64_t bd = smem_desc_sw128(dk + off, 16, 1024);
                    mma_bf16_ss(tmem + b * 128, a, bd, IDESC_QK, kk > 0 ? 1u : 0u);
                }
                tc_commit(bar(S_FULL + b));
                tc_commit(bar(K_EMPTY + st));
                if (j >= 1) ok = issue_pv(j - 1);
            }
            if (ok) issue_pv(nsteps - 1);
            // every MMA issued above has completed once DRAIN fires
            tc_commit(bar(DRAIN));
            volatile int never = 0;
            mbar_wait(bar(DRAIN), 0, &never);
        }
    } else if (warp >= 4) {
        // ---------------- softmax + epilogue ----------------
        const int r = tid - 128;            // row within the tile == TMEM lane
        const int half = r >> 6;            // which 64-row query block of the pair
        const uint32_t lane_addr = tmem + ((uint32_t)((r >> 5) * 32) << 16);
        const float sl2 = p.scale_log2;
        float m = -INFINITY, l = 0.f;
        bool ok = nsteps > 0;
        for (int j = 0; j < nsteps && ok; ++j) {
            const int b = j & 1;
            ok = warp_all_ok(mbar_wait(bar(S_FULL + b), (j >> 1) & 1, abort_flag));
            if (!ok) break;
            tc_fence_after();
            float s[128];
            tmem_ld32(lane_addr + b * 128 + 0, s + 0);
            tmem_ld32(lane_addr + b * 128 + 32, s + 32);
            tmem_ld32(lane_addr + b * 128 + 64, s + 64);
            tmem_ld32(lane_addr + b * 128 + 96, s + 96);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(bar(S_FREE + b));

            const uint32_t e0 = steps[2 * j], e1 = steps[2 * j + 1];
            const bool sel0 = (e0 >> (27 + half)) & 1u, sel1 = (e1 >> (27 + half)) & 1u;
            const int v0 = sel0 ? e_valid(e0) : 0, v1 = sel1 ? e_valid(e1) : 0;
            float mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < 64; ++c) {
                s[c] = c < v0 ? s[c] : -INFINITY;
                s[64 + c] = c < v1 ? s[64 + c] : -INFINITY;
                mx = fmaxf(mx, fmaxf(s[c], s[64 + c]));
            }
            const float mnew = mx * sl2;
            // P and O are single-buffered: PV of the previous step must be complete
            if (j > 0) {
                ok = warp_all_ok(mbar_wait(bar(O_DONE), (j - 1) & 1, abort_flag));
                if (!ok) break;
                tc_fence_after();
            }
            // lazy rescale: move the reference max only when the row max grew by more than 2^8
            float alpha = 1.f;
            if (mnew > m + 8.0f) {
                alpha = (m == -INFINITY) ? 0.f : ex2(m - mnew);
                l *= alpha;
                m = mnew;
            }
            // tcgen05.ld/st are warp-collective: the whole warp rescales if any of its rows must
            const bool rescale = (j > 0) && __any_sync(0xffffffffu, alpha != 1.f);
            if (rescale) {
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    float o[32];
                    tmem_ld32(lane_addr + TMEM_O + 32 * c, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int x = 0; x < 32; ++x) o[x] *= alpha;
                    tmem_st32(lane_addr + TMEM_O + 32 * c, o);
                }
            }
            const float base = (m == -INFINITY) ? 0.f : m;
            float rs = 0.f;
            // P row r: tokens 0-63 in region 0, 64-127 in region 1; 16-byte chunks swizzled by r&7
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                const bool sel = c < 8 ? sel0 : sel1;
                float pv[8];
#pragma unroll
                for (int x = 0; x < 8; ++x) pv[x] = sel ? ex2(fmaf(s[8 * c + x], sl2, -base)) : 0.f;
                rs += ((pv[0] + pv[1]) + (pv[2] + pv[3])) + ((pv[4] + pv[5]) + (pv[6] + pv[7]));
                const uint32_t addr = sP + (c >> 3) * REGION + r * 128 + (((c & 7) ^ (r & 7)) << 4);
                asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(pack_bf16x2(pv[0], pv[1])),
                             "r"(pack_bf16x2(pv[2], pv[3])), "r"(pack_bf16x2(pv[4], pv[5])),
                             "r"(pack_bf16x2(pv[6], pv[7]))
                             : "memory");
            }
            l += rs;
            if (rescale) tmem_wait_st();
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc_fence_before();
            mbar_arrive(bar(P_FULL));
        }
        bool have = ok && nsteps > 0;
        if (have) have = warp_all_ok(mbar_wait(bar(O_DONE), (nsteps - 1) & 1, abort_flag));
        const int row = tile * TILE_M + r;
        const bool live = row < p.Lq && (pair ? (half == 0 ? qblkA < p.qb : qblkB < p.qb) : true);
        if (have || nsteps == 0) {
            if (have) tc_fence_after();
            const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                float o[32];
                if (have) {
                    tmem_ld32(lane_addr + TMEM_O + 32 * c, o);
                    tmem_wait_ld();
                } else {
#pragma unroll
                    for (int x = 0; x < 32; ++x) o[x] = 0.f;
                }
                if (live) {
                    if (p.out_fp32) {
                        float4 *dst = reinterpret_cast<float4 *>(reinterpret_cast<float *>(p.out) +
                                                                 ((size_t)row * p.H + h) * D + 32 * c);
#pragma unroll
                        for (int x = 0; x < 8; ++x)
                            dst[x] = make_float4(o[4 * x] * inv, o[4 * x + 1] * inv, o[4 * x + 2] * inv, o[4 * x + 3] * inv);
                    } else {
                        uint4 *dst = reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(p.out) +
                                                               ((size_t)row * p.H + h) * D + 32 * c);
#pragma unroll
                        for (int x = 0; x < 4; ++x)
                            dst[x] = make_uint4(pack_bf16x2(o[8 * x] * inv, o[8 * x + 1] * inv),
                                                pack_bf16x2(o[8 * x + 2] * inv, o[8 * x + 3] * inv),
                                                pack_bf16x2(o[8 * x + 4] * inv, o[8 * x + 5] * inv),
                                                pack_bf16x2(o[8 * x + 6] * inv, o[8 * x + 7] * inv));
                    }
                }
            }
            if (live && p.lse)
                p.lse[(size_t)h * p.Lq + row] = l > 0.f ? (m + __log2f(l)) * 0.69314718055994530942f : -INFINITY;
        }
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

    CUtensorMap tq, tk, tv;
    const uint64_t row_bytes = (uint64_t)H * attn::D * 2;
    if (encode_tmap_2d_bf16(&tq, q, (uint64_t)H * attn::D, (uint64_t)Lq, row_bytes, 64, 128)) return SS_ERR_DRIVER;
    if (encode_tmap_2d_bf16(&tk, k, (uint64_t)H * attn::D, (uint64_t)Lk, row_bytes, 64, 64)) return SS_ERR_DRIVER;
    if (encode_tmap_2d_bf16(&tv, v, (uint64_t)H * attn::D, (uint64_t)Lk, row_bytes, 64, 64)) return SS_ERR_DRIVER;

    attn::Params prm;
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
    attn::sparse_attention_kernel<<<grid, attn::NTHREADS, smem, static_cast<cudaStream_t>(stream)>>>(tq, tk, tv, prm);
    return (int)cudaGetLastError();
}
