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
//   A tile is 128 query rows of one head: two 64-token query blocks (router block 64; the tile
//   walks the union of their block lists and masks, per 64-row half, the blocks that half did
//   not select) or one 128-token query block. The union is walked in steps of 128 KV tokens
//   (two 64-token sub-blocks, each gathered by TMA at its own row offset).
//   The grid is persistent: G <= #SMs CTAs; CTA c runs tiles c, c+G, c+2G, ... of the
//   head-major tile order, so at any time the CTAs of the grid share a few heads' K/V in L2.
//   Both softmax warpgroups work on the same tile: warpgroup w takes the steps of parity w,
//   with its own O accumulator and running max; the halves are merged by log-sum-exp at the
//   end of the tile. Two independent softmax streams let the tensor pipe run one warpgroup's
//   MMAs while the other exponentiates.
//
// Warp roles (384 threads; every role runs on a whole converged warp and issues its
// single-thread instructions -- TMA, tcgen05.mma, tcgen05.commit -- from an elected lane)
//   warp 0      list construction (prologue), then the TMA producer of the K/V ring
//   warp 1      TMEM allocator + tcgen05.mma issuer for warpgroup 0's QKs and PVs
//   warp 2      tcgen05.mma issuer for warpgroup 1
//   warp 3      after the prologue, L2 prefetch of the next tile's first K/V steps
//   warps 4-7   softmax warpgroup 0,   warps 8-11  softmax warpgroup 1
//               After the prologue the control warpgroup (warps 0-3) gives registers up
//               (setmaxnreg 56) and the softmax warpgroups take them (224): a softmax thread
//               holds the 128 scores of its row.
//               Thread r (r = 32*(warp%4) + lane) owns query row r of the tile (TMEM lane r).
//               Per step: copy the 128 scores of its row from TMEM and release S, mask, row
//               max, lazy rescale (only when the running max grows by more than 2^8),
//               exponentiate (MUFU ex2), write P (bf16) once the previous PV
//               has read the P buffer, release P.
//
// TMEM (512 columns): S [0,128) (one buffer, used by the warpgroups' QKs in turn); P [128,192)
// (bf16 pairs, one buffer in turn); Q [192,256) (bf16 pairs, the tile's queries, written by the
// softmax threads); O of warpgroup w at [256+128w, 384+128w).
// MMAs: S = Q K^T (M=128, N=128, K=128; A = Q in TMEM, B = K entry, K-major, 128-byte swizzle),
//       O_w += P V (M=128, N=128, K=128 tokens; A = P in TMEM, B = V entry, MN-major).
// Each warpgroup's MMAs are issued by its own warp in the order QK(0), QK(1), PV(0), QK(2), PV(1),
// ...: a warpgroup's next QK needs only the S buffer (P has its own), so it is issued ahead of its
// PV and the next scores are ready when the warpgroup finishes its exponentials. The K/V ring is
// filled in the interleaved order K0(0), K1(0), K0(1), V0(0), K1(1), V1(0), ...
// Shared memory: barriers and tables, then a ring of NST K/V entries (128 tokens x 128 dims
// bf16 each), the block bitmaps and the step lists.
// Every mbarrier wait is bounded (common.cuh); on timeout the CTA drains its TMA loads and MMAs,
// frees TMEM, sets SS_DEV_TIMEOUT in *status and exits.
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace ss {
namespace attn {

constexpr int D = 128;
constexpr int NTHREADS = 384;
constexpr int REG_CTRL = 56, REG_SOFTMAX = 224;    // setmaxnreg split of the 384 x 168 launch registers
static_assert(128 * REG_CTRL + 256 * REG_SOFTMAX <= NTHREADS * 168, "register split exceeds the launch");
constexpr int NST = 6;                             // K/V ring entries
constexpr int MAXT = 16;                           // tiles per CTA
constexpr uint32_t REGION = 16384;                 // 128 rows x 128 B: one 64-column half of a tile
constexpr uint32_t TILE_BYTES = 2 * REGION;        // 128 rows x 128 dims bf16
constexpr uint32_t OFF_BAR = 0;
constexpr int NBAR = 32;
constexpr uint32_t OFF_MISC = OFF_BAR + NBAR * 8;  // flags and counters
constexpr uint32_t OFF_TILES = OFF_MISC + 64;      // Tile table [MAXT]
constexpr uint32_t OFF_TINFO = OFF_TILES + MAXT * 16;  // prologue: per candidate tile 4 ints
constexpr uint32_t OFF_XCH = 1024;                 // log-sum-exp merge: [2 wg][m, l][128 rows]
constexpr uint32_t OFF_RING = OFF_XCH + 2 * 2 * 128 * 4;  // 1024-aligned
constexpr uint32_t SMEM_LIMIT = 232448;            // 227 KB opt-in maximum per CTA
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t TMEM_S = 0, TMEM_P = 128, TMEM_Q = 192, TMEM_O = 256;
static_assert(OFF_TINFO + MAXT * 16 <= OFF_XCH, "table space");
static_assert(OFF_RING % 1024 == 0, "ring alignment");

enum Bar {
    Q_FULL = 0,                  // the tile's Q written to TMEM (256 arrivals)
    S_FULL = 1,                  // per warpgroup: its QK completed
    S_FREE = 3,                  // per warpgroup: S copied to registers (128 arrivals)
    P_FULL = 5,                  // per warpgroup: P written (128 arrivals)
    PV_DONE = 7,                 // per warpgroup: its PV completed
    XSUM = 9,                    // tile end: both warpgroups posted m, l (256 arrivals)
    XDONE = 10,                  // tile end: both warpgroups read both O accumulators (256 arrivals)
    DRAIN = 11,
    FULL = 12,                   // per ring entry
    EMPTY = FULL + NST,
    NBAR_USED = EMPTY + NST
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

struct Tile {
    int first, n, tile, slot;    // steps [first, first+n) of the step array (n even, >= 2); tile id;
                                 // slot: -1 = the whole tile (written to out), else the workspace
                                 // slot of this CTA's piece of a split tile
};

// Position in the K/V ring: entry index and the parity of its use.
struct Ring {
    int e = 0, ph = 0;
    __device__ __forceinline__ void next() {
        if (++e == NST) {
            e = 0;
            ph ^= 1;
        }
    }
};

// Where the output rows go: row r of head h (this call's head numbering) is stored at element
// ((r * heads) + h0 + h) * D of every p[d], d < n. A plain call: n = 1 and heads = H, h0 = 0 (the
// caller's [Lq, H, D] buffer). Head sharding: p[] are every rank's [Lq, heads, D] buffers (this
// rank's and the peers' mapped with CUDA IPC), so the epilogue's stores are the all-gather.
// Owner mode (rows > 0, KV-block sharding): row r belongs to rank d = r / rows and goes to p[d]
// only, a [n][rows][heads][D] partial buffer, at slot `slot` (this rank), local row r - d * rows;
// its LSE goes to lse[d], [n][heads][rows] -- the epilogue's stores are the reduce-scatter.
struct OutRows {
    void *p[SS_MAX_PEERS];
    float *lse[SS_MAX_PEERS];
    int n, heads, h0, rows, slot;
};

struct Params {
    const __nv_bfloat16 *q;
    const int32_t *ids;
    OutRows out;
    float *lse;
    int *status;
    int H, Lq, Lk, block, n_ids, qb, kb, ntiles, nwords, T, G, tmax, step_cap, out_fp32;
    float scale_log2;  // scale * log2(e)
    // split mode (fewer than two tiles per CTA): CTA c takes tile-units [c*T, (c+1)*T) of the
    // T*G units (G per tile); a tile spanning several CTAs is split at step pairs in proportion,
    // each piece writing its normalised partial and LSE to slot 2c (the first tile of c's range)
    // or 2c + 1 (the last) of ws_o [2G][128][128] / ws_lse [2G][128], merged by split_merge_kernel
    int split;
    float *ws_o, *ws_lse;
    KvRing ring;   // where K/V rows live (C = 0: the window's rows in order)
    // ids name window blocks of which this rank stores those with id % own_n == own_r, packed in
    // order (local block id / own_n); own_n = 1: the ids are the k/v blocks themselves
    int own_n, own_r;
};

// Pieces of one tile at most in split mode: the grid has at most 8 CTAs per tile, and a tile
// meets at most one more CTA than that.
constexpr int MAXSPLIT_PIECES = 9;

// Tile range of CTA c in split mode: tiles [first, last] meet its units [c*T, (c+1)*T).
__host__ __device__ __forceinline__ int split_first(int c, int T, int G) { return (int)(((long)c * T) / G); }
__host__ __device__ __forceinline__ int split_last(int c, int T, int G) { return (int)(((long)(c + 1) * T - 1) / G); }
__host__ __device__ __forceinline__ int split_slot(int c, int t, int T, int G) {
    return 2 * c + (t == split_first(c, T, G) ? 0 : 1);
}

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

// Ascending compaction of the set bits of word(w) (w < nwords) into sub-block entries, run by
// one warp; sub-block k of the output is stored by put(k, entry). Returns the number written.
template <class W, class M, class P>
__device__ __forceinline__ void compact(int nwords, int block, int Lk, const KvRing &ring, int lane, W &&word,
                                        M &&maskof, P &&put) {
    // the set bits of word(0), word(1), ... in ascending block order: lane l takes bit l of each
    // word, its rank among the word's set bits is the popcount of the bits below it
    const int per = block / 64;
    const uint32_t below = (1u << lane) - 1u;
    int carry = 0;
    for (int w = 0; w < nwords; ++w) {
        const uint32_t u = word(w);
        if ((u >> lane) & 1u) {
            const int j = w * 32 + lane;
            const uint32_t m = maskof(w, lane);
            const int pos = carry + __popc(u & below) * per;
            for (int s = 0; s < per; ++s) {
                const int t0 = j * block + s * 64;
                const int valid = min(64, max(0, Lk - t0));
                put(pos + s, entry((uint32_t)ring.sub_row(t0), (uint32_t)valid, m));
            }
        }
        carry += __popc(u) * per;
    }
}

__device__ __forceinline__ int warp_count_bits(int nwords, int lane, int per, const uint32_t *a, const uint32_t *b,
                                               uint32_t ka, uint32_t kb_) {
    // number of set bits of (a ^ ka) & (b ^ kb_) over nwords words, times per (warp reduction)
    int c = 0;
    for (int w = lane; w < nwords; w += 32) c += __popc((a[w] ^ ka) & (b[w] ^ kb_));
    return (int)__reduce_add_sync(0xffffffffu, (unsigned)c) * per;
}

// Q rows of the tile for one warpgroup: dims [64w, 64w + 64) of row `row` as 32 bf16 pairs.
// One 32-byte store (sm_100 st.global.v8): each lane writes whole 32-byte sectors. Measured on B200
// against 16-byte stores of the same rows: 1-5% faster kernels, most for fp32 and split outputs.
__device__ __forceinline__ void st_v8(void *p, const uint32_t *w) {
    asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(w[0]), "r"(w[1]), "r"(w[2]),
                 "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7]) : "memory");
}

__device__ __forceinline__ void load_q(const Params &p, int h, int row, int w, uint32_t *qv) {
    if (row < p.Lq) {
        const uint4 *src = reinterpret_cast<const uint4 *>(p.q + ((size_t)row * p.H + h) * D + 64 * w);
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
}

// MMA issuer of warpgroup W. The ring order (shared with the producer) per tile of m steps per
// warpgroup: K0(0), K1(0), then for j < m-1: K0(j+1), V0(j), K1(j+1), V1(j), then V0(m-1), V1(m-1)
// (4m entries). Warpgroup W's operations sit at fixed positions of that order.
template <int W>
__device__ __forceinline__ bool mma_issuer(uint32_t tmem, uint32_t sRing, uint32_t bar0, const Tile *tiles, int nt,
                                        volatile int *abort_flag) {
    auto bar = [&](int i) -> uint32_t { return bar0 + 8u * (uint32_t)i; };
    const uint64_t dk0 = smem_desc_sw128(sRing, 16, 1024), dv0 = smem_desc_sw128(sRing, REGION, 1024);
    int qc = 0, pc = 0;     // QKs and PVs issued by this warpgroup
    int base = 0;           // ring position of the tile's first entry
    auto qk = [&](int pos) -> bool {         // S = Q K^T into the shared S buffer
        // the QK before ours in the alternating QK order belongs to the other warpgroup:
        // S is free once that warpgroup copied its scores out
        if (W == 1 || qc > 0) {
            const int other = W == 0 ? qc - 1 : qc;
            if (!warp_all_ok(mbar_wait(bar(S_FREE + (W ^ 1)), other & 1, abort_flag))) return false;
        }
        const int e = pos % NST;
        if (!warp_all_ok(mbar_wait(bar(FULL + e), (pos / NST) & 1, abort_flag))) return false;
        tc_fence_after();
        const uint64_t db = dk0 + (uint32_t)e * (TILE_BYTES >> 4);
        if (elect_one()) {
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
                mma_bf16_ts(tmem + TMEM_S, tmem + TMEM_Q + 8 * kk, db + ((((kk >> 2) * REGION) + (kk & 3) * 32) >> 4),
                            IDESC_QK, kk > 0 ? 1u : 0u);
            tc_commit(bar(S_FULL + W));
            tc_commit(bar(EMPTY + e));
        }
        __syncwarp();
        ++qc;
        return true;
    };
    auto pv = [&](int pos, bool first) -> bool {   // O_W (+)= P V
        if (!warp_all_ok(mbar_wait(bar(P_FULL + W), pc & 1, abort_flag))) return false;
        const int e = pos % NST;
        if (!warp_all_ok(mbar_wait(bar(FULL + e), (pos / NST) & 1, abort_flag))) return false;
        tc_fence_after();
        const uint64_t db = dv0 + (uint32_t)e * (TILE_BYTES >> 4);
        if (elect_one()) {
            // tokens 16kk.. of the step: P columns 8kk.. (bf16 pairs)
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
                mma_bf16_ts(tmem + TMEM_O + 128 * W, tmem + TMEM_P + 8 * kk, db + ((kk * 2048) >> 4), IDESC_PV,
                            (first && kk == 0) ? 0u : 1u);
            tc_commit(bar(EMPTY + e));
            tc_commit(bar(PV_DONE + W));
        }
        __syncwarp();
        ++pc;
        return true;
    };
    bool ok = true;
    for (int lt = 0; lt < nt && ok; ++lt) {
        const int m = tiles[lt].n / 2;
        ok = warp_all_ok(mbar_wait(bar(Q_FULL), lt & 1, abort_flag));   // the tile's Q is in TMEM
        ok = ok && qk(base + W);
        for (int j = 0; j + 1 < m && ok; ++j)
            ok = qk(base + 2 + 2 * W + 4 * j) && pv(base + 3 + 2 * W + 4 * j, j == 0);
        ok = ok && pv(base + 4 * m - 2 + W, m == 1);
        base += 4 * m;
    }
    return ok;
}

// NDST: the most output buffers a row is stored to (1, or SS_MAX_PEERS for head sharding).
template <int NDST>
__global__ void __launch_bounds__(NTHREADS, 1)
sparse_attention_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                        const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t sRing = sbase + OFF_RING;
    const uint32_t bar0 = sbase + OFF_BAR;
    auto bar = [&](int i) -> uint32_t { return bar0 + 8u * (uint32_t)i; };
    volatile uint32_t *tmem_slot = reinterpret_cast<volatile uint32_t *>(smem + OFF_MISC);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_MISC + 4);
    volatile int *badid_flag = reinterpret_cast<volatile int *>(smem + OFF_MISC + 8);
    volatile int *progress = reinterpret_cast<volatile int *>(smem + OFF_MISC + 12);   // (tile << 16) | half-way
    volatile int *nt_slot = reinterpret_cast<volatile int *>(smem + OFF_MISC + 16);    // pieces with steps
    Tile *tiles = reinterpret_cast<Tile *>(smem + OFF_TILES);
    float *xch = reinterpret_cast<float *>(smem + OFF_XCH);                              // [2][2][128]
    uint32_t *bm = reinterpret_cast<uint32_t *>(smem + OFF_RING + NST * TILE_BYTES);     // [tmax][2][nwords]
    uint2 *steps = reinterpret_cast<uint2 *>(bm + 2 * p.tmax * p.nwords);                // [step_cap]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // candidate tiles of this CTA: blockIdx.x + k*G < T, or in split mode the tiles its units meet
    const int c_first = p.split ? split_first((int)blockIdx.x, p.T, p.G) : 0;
    const int ntc = p.split ? split_last((int)blockIdx.x, p.T, p.G) - c_first + 1
                            : (p.T - (int)blockIdx.x + p.G - 1) / p.G;
    auto cand_tile = [&](int lt) { return p.split ? c_first + lt : (int)blockIdx.x + lt * p.G; };
    const bool pairq = (p.block == 64);

    // ---------------- prologue: barriers, TMEM, block bitmaps, step lists ----------------
    if (tid == 0) {
        *abort_flag = 0;
        *badid_flag = 0;
        *progress = 0;
        mbar_init(bar(Q_FULL), 256);
        for (int s = 0; s < 2; ++s) {
            mbar_init(bar(S_FULL + s), 1);
            mbar_init(bar(S_FREE + s), 128);
            mbar_init(bar(P_FULL + s), 128);
            mbar_init(bar(PV_DONE + s), 1);
        }
        mbar_init(bar(XSUM), 256);
        mbar_init(bar(XDONE), 256);
        mbar_init(bar(DRAIN), 2);
        for (int s = 0; s < NST; ++s) {
            mbar_init(bar(FULL + s), 1);
            mbar_init(bar(EMPTY + s), 1);
        }
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
    for (int w = tid; w < 2 * ntc * p.nwords; w += NTHREADS) bm[w] = 0u;
    __syncthreads();
    {
        // bitmap (lt, half) <- ids of query block (pair ? 2*tile + half : tile) of head h
        const int per_tile = (pairq ? 2 : 1) * p.n_ids;
        for (int x = tid; x < ntc * per_tile; x += NTHREADS) {
            const int lt = x / per_tile, rem = x % per_tile, half = rem / p.n_ids, i = rem % p.n_ids;
            const int t = cand_tile(lt), h = t / p.ntiles, tile = t % p.ntiles;
            const int qblk = pairq ? 2 * tile + half : tile;
            if (qblk >= p.qb) continue;
            int a = p.ids[((size_t)h * p.qb + qblk) * p.n_ids + i];
            if (p.own_n > 1 && a >= 0) {
                // KV-block sharding: window block a is stored by rank a % own_n, as local block a / own_n
                if ((int)((unsigned)a % (unsigned)p.own_n) != p.own_r) continue;
                a = (int)((unsigned)a / (unsigned)p.own_n);
            }
            if (a >= p.kb) *badid_flag = 1;
            else if (a >= 0) atomicOr(&bm[(2 * lt + half) * p.nwords + (a >> 5)], 1u << (a & 31));
        }
    }
    __syncthreads();
    {
        // Per tile, the union's sub-blocks, padded to a whole, even number (>= 2) of steps. A
        // 64-row half of the tile runs on two fixed SM sub-partitions (TMEM lane quarters), so a
        // step whose sub-blocks only one half selected keeps the other half's sub-partitions
        // idle while the first exponentiate 128 columns per row. The blocks only the first
        // half selected are therefore paired with blocks only the second half selected (each
        // row then exponentiates 64 columns). The blocks both halves selected come first: they
        // are mostly the forced current-chunk blocks, the same for every tile of a head, so the
        // start of a tile reads K/V that the head's other tiles (and warp 3's L2 prefetch) have
        // already brought into L2. Order: both (an even count), the pairs, the unpaired rest, the
        // odd "both" sub-block if there is one; each group ascending.
        // Built in three passes over the warps: the piece counts (one warp per tile), the list
        // offsets and tile table (warp 0), the entries (one warp per tile and group).
        uint32_t *sub = reinterpret_cast<uint32_t *>(steps);
        int *tinfo = reinterpret_cast<int *>(smem + OFF_TINFO);   // per tile: A only, B only, both, offset
        const int per = p.block / 64;
        for (int lt = warp; lt < ntc; lt += NTHREADS / 32) {
            const uint32_t *A = bm + (2 * lt) * p.nwords, *B = A + p.nwords;
            const int na = warp_count_bits(p.nwords, lane, per, A, B, 0u, 0xffffffffu);   // A only
            const int nb = warp_count_bits(p.nwords, lane, per, B, A, 0u, 0xffffffffu);   // B only
            const int nboth = warp_count_bits(p.nwords, lane, per, A, B, 0u, 0u);         // both
            if (lane == 0) {
                tinfo[4 * lt] = na;
                tinfo[4 * lt + 1] = nb;
                tinfo[4 * lt + 2] = nboth;
            }
        }
        __syncthreads();
        if (warp == 0) {
            int pos = 0;   // sub-blocks before the tile's list
            int nout = 0;  // table entries (pieces with steps)
            for (int lt = 0; lt < ntc; ++lt) {
                const int n = tinfo[4 * lt] + tinfo[4 * lt + 1] + tinfo[4 * lt + 2];
                const int padded = max(4, (n + 3) & ~3);
                if (lane == 0) tinfo[4 * lt + 3] = pos;
                // the steps this CTA runs: the whole list, or in split mode its share of the tile's
                // step pairs (the same cut for every CTA holding a piece of the tile)
                const int t = cand_tile(lt), tsteps = padded / 2;
                int s0 = 0, s1 = tsteps, slot = -1;
                if (p.split) {
                    const long g0 = (long)t * p.G, u0 = (long)blockIdx.x * p.T;
                    const long a = max(u0, g0) - g0, b = min(u0 + p.T, g0 + p.G) - g0;
                    if (a > 0 || b < p.G) {
                        const long pairs = tsteps / 2;
                        s0 = 2 * (int)(a * pairs / p.G);
                        s1 = 2 * (int)(b * pairs / p.G);
                        slot = split_slot((int)blockIdx.x, t, p.T, p.G);
                    }
                }
                if (s1 > s0) {
                    if (lane == 0) {
                        Tile tl;
                        tl.first = pos / 2 + s0;
                        tl.n = s1 - s0;
                        tl.tile = t;
                        tl.slot = slot;
                        tiles[nout] = tl;
                    }
                    ++nout;
                } else {   // a piece without steps: an empty partial for the merge
                    for (int r = lane; r < 128; r += 32) p.ws_lse[(size_t)slot * 128 + r] = -INFINITY;
                }
                pos += padded;
            }
            if (lane == 0) *nt_slot = nout;
        }
        __syncthreads();
        const KvRing ring = p.ring.resolved();
        for (int job = warp; job < 3 * ntc; job += NTHREADS / 32) {
            const int lt = job / 3, grp = job % 3;
            const uint32_t *A = bm + (2 * lt) * p.nwords, *B = A + p.nwords;
            auto maskof = [&](int w, int bit) -> uint32_t {
                if (!pairq) return 3u;
                return ((A[w] >> bit) & 1u) | (((B[w] >> bit) & 1u) << 1);
            };
            const int na = tinfo[4 * lt], nb = tinfo[4 * lt + 1], nboth = tinfo[4 * lt + 2];
            const int mp = min(na, nb), nb2 = nboth & ~1;
            const int n = na + nb + nboth;
            uint32_t *base = sub + tinfo[4 * lt + 3];
            if (grp == 0) {
                compact(p.nwords, p.block, p.Lk, ring, lane, [&](int w) { return A[w] & B[w]; }, maskof,
                        [&](int k, uint32_t e) { base[k < nb2 ? k : n - 1] = e; });
                const int padded = max(4, (n + 3) & ~3);
                for (int k = n + lane; k < padded; k += 32) base[k] = entry(0u, 0u, 0u);
            } else if (grp == 1) {
                compact(p.nwords, p.block, p.Lk, ring, lane, [&](int w) { return A[w] & ~B[w]; }, maskof,
                        [&](int k, uint32_t e) { base[nb2 + (k < mp ? 2 * k : mp + k)] = e; });
            } else {
                compact(p.nwords, p.block, p.Lk, ring, lane, [&](int w) { return B[w] & ~A[w]; }, maskof,
                        [&](int k, uint32_t e) { base[nb2 + (k < mp ? 2 * k + 1 : mp + k)] = e; });
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int nt = *nt_slot;

    if (warp >= 4) {
        // The softmax warpgroups and the control warpgroup run with different register budgets
        // and never share code after this point (each branch ends with its own teardown).
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REG_SOFTMAX));
        // ---------------- softmax warpgroups + epilogues ----------------
        const int wg = (warp - 4) >> 2;
        const int q4 = warp & 3;
        const int r = q4 * 32 + lane;                // row within the tile == TMEM lane
        const int half = r >> 6;                     // which 64-row query block of the pair
        const uint32_t lane_base = tmem + ((uint32_t)(q4 * 32) << 16);
        const uint32_t s_addr = lane_base + TMEM_S, p_addr = lane_base + TMEM_P;
        const uint32_t o_addr = lane_base + TMEM_O + 128 * wg;
        const float sl2 = p.scale_log2;
        const uint64_t sl2x2 = f2_pack(sl2, sl2);
        bool ok = true;
        int k = 0;                                   // steps of this warpgroup so far
        uint32_t qv[32];
        if (nt > 0) {   // (a CTA whose split pieces all came out empty has no tile at all)
            const int t0 = tiles[0].tile;
            load_q(p, t0 / p.ntiles, (t0 % p.ntiles) * 128 + r, wg, qv);
            tmem_st32(lane_base + TMEM_Q + 32 * wg, reinterpret_cast<const float *>(qv));
            tmem_wait_st();
            tmem_st_fence32(reinterpret_cast<const float *>(qv));
            tc_fence_before();
            mbar_arrive(bar(Q_FULL));
        }
        for (int lt = 0; lt < nt && ok; ++lt) {
            const Tile tl = tiles[lt];
            const bool more = lt + 1 < nt;
            if (more) {   // the next tile's Q row slice (128 B) into L2, a whole tile ahead of its use
                const int tn = tiles[lt + 1].tile, rn = (tn % p.ntiles) * 128 + r;
                if (rn < p.Lq)
                    asm volatile("prefetch.global.L2 [%0];" ::"l"(p.q + ((size_t)rn * p.H + tn / p.ntiles) * D + 64 * wg));
            }
            if (warp == 4 && lane == 0) *progress = lt << 16;
            float m = -INFINITY, l = 0.f;
            for (int j = 0; j < tl.n / 2; ++j, ++k) {
                if (warp == 4 && lane == 0 && j == tl.n / 4) *progress = (lt << 16) | 1;   // half-way
                const uint2 st = steps[tl.first + 2 * j + wg];
                ok = warp_all_ok(mbar_wait(bar(S_FULL + wg), k & 1, abort_flag));
                if (!ok) break;
                tc_fence_after();
                float s[128];
                tmem_ld32(s_addr, s);
                tmem_ld32(s_addr + 32, s + 32);
                tmem_ld32(s_addr + 64, s + 64);
                tmem_ld32(s_addr + 96, s + 96);
                // selection and valid length per sub-block, warp-uniform (a warp lies in one half)
                const bool sel0 = (st.x >> (27 + half)) & 1u, sel1 = (st.y >> (27 + half)) & 1u;
                const int v0 = sel0 ? e_valid(st.x) : 0, v1 = sel1 ? e_valid(st.y) : 0;
                tmem_wait_ld();
                tmem_ld_fence32(s);
                tmem_ld_fence32(s + 32);
                tmem_ld_fence32(s + 64);
                tmem_ld_fence32(s + 96);
                tc_fence_before();
                mbar_arrive(bar(S_FREE + wg));       // the next QK may overwrite S
                float mx = -INFINITY;
                if (v0 == 64) {
                    float m0 = s[0], m1 = s[1], m2 = s[2], m3 = s[3];
#pragma unroll
                    for (int c = 4; c < 64; c += 8) {
                        m0 = max3(m0, s[c], s[c + 1]);
                        m1 = max3(m1, s[c + 2], s[c + 3]);
                        m2 = max3(m2, s[c + 4], s[c + 5]);
                        m3 = max3(m3, s[c + 6], s[c + 7]);
                    }
                    mx = max3(fmaxf(m0, m1), m2, m3);
                } else if (v0 > 0) {
#pragma unroll
                    for (int c = 0; c < 64; ++c) {
                        s[c] = c < v0 ? s[c] : -INFINITY;
                        mx = fmaxf(mx, s[c]);
                    }
                }
                if (v1 == 64) {
                    float m0 = s[64], m1 = s[65], m2 = s[66], m3 = s[67];
#pragma unroll
                    for (int c = 68; c < 128; c += 8) {
                        m0 = max3(m0, s[c], s[c + 1]);
                        m1 = max3(m1, s[c + 2], s[c + 3]);
                        m2 = max3(m2, s[c + 4], s[c + 5]);
                        m3 = max3(m3, s[c + 6], s[c + 7]);
                    }
                    mx = max3(mx, fmaxf(m0, m1), fmaxf(m2, m3));
                } else if (v1 > 0) {
#pragma unroll
                    for (int c = 64; c < 128; ++c) {
                        s[c] = c - 64 < v1 ? s[c] : -INFINITY;
                        mx = fmaxf(mx, s[c]);
                    }
                }
                // lazy rescale: move the reference max only when the row max grew by more than 2^8
                const float mnew = mx * sl2;
                float alpha = 1.f;
                bool grow = false;                   // an O row holding earlier steps must be scaled
                if (mnew > m + 8.0f) {
                    grow = m != -INFINITY;
                    alpha = grow ? ex2(m - mnew) : 0.f;
                    l *= alpha;
                    m = mnew;
                }
                // O_w holds the previous steps once this warpgroup's previous PV completed;
                // tcgen05.ld/st are warp-collective, so the whole warp rescales if any row must.
                if (__any_sync(0xffffffffu, grow)) {
                    ok = warp_all_ok(mbar_wait(bar(PV_DONE + wg), (k - 1) & 1, abort_flag));
                    if (!ok) break;
                    tc_fence_after();
#pragma unroll 1
                    for (int c = 0; c < 4; ++c) {
                        float o[32];
                        tmem_ld32(o_addr + 32 * c, o);
                        tmem_wait_ld();
                        tmem_ld_fence32(o);
#pragma unroll
                        for (int x = 0; x < 32; ++x) o[x] *= (grow ? alpha : 1.f);
                        tmem_st32(o_addr + 32 * c, o);
                        tmem_wait_st();            // o is reloaded by the next chunk
                        tmem_st_fence32(o);
                    }
                }
                // P = 2^(s*sl2 - m) as bf16 pairs, all on MUFU ex2: measured on B200, moving a
                // share of the exponentials to an FMA-pipe polynomial (a quarter or a half,
                // grouped or interleaved) made the step slower, the extra instructions costing
                // more issue slots than the MUFU time they saved.
                const float base = (m == -INFINITY) ? 0.f : m;
                const uint64_t nbx2 = f2_pack(-base, -base);
                uint64_t sa = 0, sb = 0;
                uint32_t pk[64];
#pragma unroll
                for (int g = 0; g < 2; ++g) {
                    const bool on = g == 0 ? v0 > 0 : v1 > 0;
                    if (on) {
#pragma unroll
                        for (int c = 0; c < 64; c += 4) {
                            const int cc = 64 * g + c;
                            const uint64_t x0 = f2_fma(f2_pack(s[cc], s[cc + 1]), sl2x2, nbx2);
                            const uint64_t x1 = f2_fma(f2_pack(s[cc + 2], s[cc + 3]), sl2x2, nbx2);
                            const float p0 = ex2(f2_lo(x0)), p1 = ex2(f2_hi(x0));
                            const float p2 = ex2(f2_lo(x1)), p3 = ex2(f2_hi(x1));
                            sa = f2_add(sa, f2_pack(p0, p1));
                            sb = f2_add(sb, f2_pack(p2, p3));
                            pk[cc >> 1] = pack_bf16x2(p0, p1);
                            pk[(cc >> 1) + 1] = pack_bf16x2(p2, p3);
                        }
                    } else {
#pragma unroll
                        for (int x = 0; x < 32; ++x) pk[32 * g + x] = 0u;
                    }
                }
                const uint64_t st2 = f2_add(sa, sb);
                l += f2_lo(st2) + f2_hi(st2);
                // the P buffer is free once the PV issued before ours has read it: PV1(k-1) for
                // warpgroup 0, PV0(k) for warpgroup 1
                if (wg == 0) {
                    if (k > 0) ok = warp_all_ok(mbar_wait(bar(PV_DONE + 1), (k - 1) & 1, abort_flag));
                } else {
                    ok = warp_all_ok(mbar_wait(bar(PV_DONE + 0), k & 1, abort_flag));
                }
                if (!ok) break;
                tc_fence_after();
                tmem_st32(p_addr, reinterpret_cast<const float *>(pk));
                tmem_st32(p_addr + 32, reinterpret_cast<const float *>(pk + 32));
                tmem_wait_st();
                tmem_st_fence32(reinterpret_cast<const float *>(pk));
                tmem_st_fence32(reinterpret_cast<const float *>(pk + 32));
                tc_fence_before();
                mbar_arrive(bar(P_FULL + wg));
            }
            if (!ok) break;
            if (more) {
                // The next tile's Q goes into TMEM as soon as this tile's last QK (warpgroup 1's)
                // has completed, so its first QKs run while the epilogue below merges and writes.
                const int tn = tiles[lt + 1].tile;
                load_q(p, tn / p.ntiles, (tn % p.ntiles) * 128 + r, wg, qv);
                ok = warp_all_ok(mbar_wait(bar(S_FULL + 1), (k - 1) & 1, abort_flag));
                if (!ok) break;
                tc_fence_after();
                tmem_st32(lane_base + TMEM_Q + 32 * wg, reinterpret_cast<const float *>(qv));
                tmem_wait_st();
                tmem_st_fence32(reinterpret_cast<const float *>(qv));
                tc_fence_before();
                mbar_arrive(bar(Q_FULL));
            }
            // ---------------- tile epilogue: merge the two halves, write ----------------
            const int h = tl.tile / p.ntiles, row = (tl.tile % p.ntiles) * 128 + r;
            const bool live = row < p.Lq;
            ok = warp_all_ok(mbar_wait(bar(PV_DONE + wg), (k - 1) & 1, abort_flag));   // our last PV
            if (!ok) break;
            xch[(wg * 2 + 0) * 128 + r] = m;
            xch[(wg * 2 + 1) * 128 + r] = l;
            tc_fence_before();
            mbar_arrive(bar(XSUM));
            ok = warp_all_ok(mbar_wait(bar(XSUM), lt & 1, abort_flag));   // every MMA of the tile done
            if (!ok) break;
            tc_fence_after();
            const float mo = xch[((wg ^ 1) * 2 + 0) * 128 + r], lo = xch[((wg ^ 1) * 2 + 1) * 128 + r];
            const float M = fmaxf(m, mo);
            const float a_s = (m == -INFINITY) ? 0.f : ex2(m - M);
            const float a_o = (mo == -INFINITY) ? 0.f : ex2(mo - M);
            const float L = l * a_s + lo * a_o;
            const float inv = L > 0.f ? 1.f / L : 0.f;
            // warpgroup w writes output columns [64w, 64w + 64): O0 and O1 are both read here
            const uint32_t o_self = o_addr, o_oth = lane_base + TMEM_O + 128 * (wg ^ 1);
            float res[64];
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                float o[32], t[32];
                tmem_ld32(o_self + 64 * wg + 32 * c, o);
                tmem_ld32(o_oth + 64 * wg + 32 * c, t);
                tmem_wait_ld();
                tmem_ld_fence32(o);
                tmem_ld_fence32(t);
#pragma unroll
                for (int x = 0; x < 32; ++x)
                    res[32 * c + x] = ((a_s > 0.f ? o[x] * a_s : 0.f) + (a_o > 0.f ? t[x] * a_o : 0.f)) * inv;
            }
            tc_fence_before();
            mbar_arrive(bar(XDONE));
            if (tl.slot >= 0) {
                // a piece of a split tile: the normalised partial and its LSE, merged later
                float *dst = p.ws_o + ((size_t)tl.slot * 128 + r) * D + 64 * wg;
#pragma unroll
                for (int x = 0; x < 8; ++x) st_v8(dst + 8 * x, reinterpret_cast<const uint32_t *>(res + 8 * x));
                if (wg == 0)
                    p.ws_lse[(size_t)tl.slot * 128 + r] =
                        L > 0.f ? (M + __log2f(L)) * 0.69314718055994530942f : -INFINITY;
            } else if (live) {
                size_t off = ((size_t)row * p.out.heads + p.out.h0 + h) * D + 64 * wg;
                int d_lo = 0, d_hi = NDST;     // destinations [d_lo, d_hi) of those below p.out.n
                if (NDST > 1 && p.out.rows > 0) {
                    // owner mode: the row goes to its owner's buffer only, at slot p.out.slot
                    const int d = row / p.out.rows, rl = row - d * p.out.rows;
                    off = (((size_t)p.out.slot * p.out.rows + rl) * p.out.heads + p.out.h0 + h) * D + 64 * wg;
                    d_lo = d;
                    d_hi = d + 1;
                    if (wg == 0) {
                        const float l_row = L > 0.f ? (M + __log2f(L)) * 0.69314718055994530942f : -INFINITY;
                        const size_t li = ((size_t)p.out.slot * p.out.heads + p.out.h0 + h) * p.out.rows + rl;
#pragma unroll
                        for (int i = 0; i < NDST; ++i)
                            if (i == d) p.out.lse[i][li] = l_row;
                    }
                }
                if (p.out_fp32) {
#pragma unroll
                    for (int d = 0; d < NDST; ++d) {
                        if (NDST == 1 || (d >= d_lo && d < d_hi && d < p.out.n)) {
                            float *dst = reinterpret_cast<float *>(p.out.p[d]) + off;
#pragma unroll
                            for (int x = 0; x < 8; ++x)
                                st_v8(dst + 8 * x, reinterpret_cast<const uint32_t *>(res + 8 * x));
                        }
                    }
                } else if (NDST == 1) {
                    __nv_bfloat16 *dst = reinterpret_cast<__nv_bfloat16 *>(p.out.p[0]) + off;
#pragma unroll
                    for (int x = 0; x < 4; ++x) {
                        uint32_t w[8];
#pragma unroll
                        for (int y = 0; y < 8; ++y) w[y] = pack_bf16x2(res[16 * x + 2 * y], res[16 * x + 2 * y + 1]);
                        st_v8(dst + 16 * x, w);
                    }
                } else {
                    // packed once, then stored to this rank's buffer and over NVLink to the peers'
                    uint32_t w[32];
#pragma unroll
                    for (int y = 0; y < 32; ++y) w[y] = pack_bf16x2(res[2 * y], res[2 * y + 1]);
#pragma unroll
                    for (int d = 0; d < NDST; ++d) {
                        if (d >= d_lo && d < d_hi && d < p.out.n) {
                            __nv_bfloat16 *dst = reinterpret_cast<__nv_bfloat16 *>(p.out.p[d]) + off;
#pragma unroll
                            for (int x = 0; x < 4; ++x) st_v8(dst + 16 * x, w + 8 * x);
                        }
                    }
                }
                if (p.lse && wg == 0)
                    p.lse[(size_t)h * p.Lq + row] = L > 0.f ? (M + __log2f(L)) * 0.69314718055994530942f : -INFINITY;
            }
            // the next tile's first PV overwrites O: both warpgroups must have read it
            ok = warp_all_ok(mbar_wait(bar(XDONE), lt & 1, abort_flag));
        }
        tc_fence_before();
        __syncthreads();
        return;
    }
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_CTRL));
    if (warp == 0) {
        // ---------------- TMA producer: K/V steps in MMA order ----------------
        // Per tile: K of QK0(0), K of QK1(0), then for each i and w: K of QKw(i+1), V of PVw(i).
        Ring ring;
        int loaded = 0;
        bool ok = true;
        auto load = [&](const CUtensorMap *tm, int h, uint2 st) -> bool {
            if (loaded >= NST && !warp_all_ok(mbar_wait(bar(EMPTY + ring.e), ring.ph ^ 1, abort_flag))) return false;
            const uint32_t dst = sRing + ring.e * TILE_BYTES, fb = bar(FULL + ring.e);
            const int t0 = e_start(st.x), t1 = e_start(st.y);
            if (elect_one()) {
                mbar_arrive_expect_tx(fb, TILE_BYTES);
                tma_load_2d(dst, tm, h * D, t0, fb);
                tma_load_2d(dst + REGION, tm, h * D + 64, t0, fb);
                tma_load_2d(dst + REGION / 2, tm, h * D, t1, fb);
                tma_load_2d(dst + REGION + REGION / 2, tm, h * D + 64, t1, fb);
            }
            __syncwarp();
            ring.next();
            ++loaded;
            return true;
        };
        for (int lt = 0; lt < nt && ok; ++lt) {
            const Tile tl = tiles[lt];
            const int h = tl.tile / p.ntiles, m = tl.n / 2;
            const uint2 *sp = steps + tl.first;
            ok = load(&tm_k, h, sp[0]) && load(&tm_k, h, sp[1]);
            for (int j = 0; j < m && ok; ++j) {
#pragma unroll
                for (int w = 0; w < 2; ++w) {
                    if (ok && j + 1 < m) ok = load(&tm_k, h, sp[2 * j + 2 + w]);
                    if (ok) ok = load(&tm_v, h, sp[2 * j + w]);
                }
            }
        }
        if (!ok) {  // drain: loads still landing in shared memory
            volatile int never = 0;
            for (int s = 0; s < NST && s < loaded; ++s) {
                ring.e = ring.e == 0 ? NST - 1 : ring.e - 1;
                if (ring.e == NST - 1) ring.ph ^= 1;
                mbar_wait(bar(FULL + ring.e), ring.ph, &never);
            }
        }
    } else if (warp == 3) {
        // ---------------- L2 prefetch of the next tile's first steps ----------------
        // Once the softmax warpgroups are half-way through tile lt, the K and V boxes of the first
        // PF_STEPS steps of tile lt+1 are prefetched into L2 (no shared memory, no completion
        // tracking). Those steps are the blocks both query blocks selected -- mostly the forced
        // current-chunk blocks, shared by all tiles of a head -- so a head change at a tile
        // boundary starts on L2 hits instead of every CTA waiting on HBM at once.
        constexpr int PF_STEPS = 32;
        for (int lt = 0; lt + 1 < nt; ++lt) {
            const int want = (lt << 16) | 1;
            const long long t0 = clock64();
            bool go = true;
            while (*progress < want) {
                if (*abort_flag || clock64() - t0 > kWaitLimitCycles) {
                    go = false;
                    break;
                }
                __nanosleep(256);
            }
            if (!go) break;
            const Tile tn = tiles[lt + 1];
            const int h = tn.tile / p.ntiles, nst = min(PF_STEPS, tn.n);
            for (int i = lane; i < 4 * nst; i += 32) {
                const uint2 st = steps[tn.first + i / 4];
                const int which = i & 3;   // K x, K y, V x, V y
                const int t0s = e_start((which & 1) ? st.y : st.x);
                const CUtensorMap *tm = which < 2 ? &tm_k : &tm_v;
                tma_prefetch_2d(tm, h * D, t0s);
                tma_prefetch_2d(tm, h * D + 64, t0s);
            }
        }
    } else if (warp == 1 || warp == 2) {
        // ---------------- MMA issuers: warp 1 for warpgroup 0, warp 2 for warpgroup 1 ----------------
        // tcgen05.mma blocks its issuing thread while the pipe holds an earlier MMA, so a single
        // issuer leaves the pipe idle for every instruction it spends between two operations.
        // With one issuer per warpgroup, one warp's waits overlap the other's MMAs. Everything
        // ordering the two streams is an explicit barrier: S_FREE (the shared S buffer), P_FULL
        // and PV_DONE (the shared P buffer, via the softmax), Q_FULL (the tile's queries).
        if (warp == 1) mma_issuer<0>(tmem, sRing, bar0, tiles, nt, abort_flag);
        else mma_issuer<1>(tmem, sRing, bar0, tiles, nt, abort_flag);
        // every MMA this warp issued has completed once DRAIN fires (two arrivals: both issuers)
        if (elect_one()) tc_commit(bar(DRAIN));
        __syncwarp();
        volatile int never = 0;
        mbar_wait(bar(DRAIN), 0, &never);
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

// Split mode: the rows of every split tile from its pieces. Grid (T, 16): CTA (t, y) takes rows
// [8y, 8y + 8) of tile t, one thread per (row, 4 dims), every piece's LSE and values loaded before
// any is used; CTAs of whole tiles return at once. Arithmetic of ss_lse_merge: L = max + log(sum
// w), w_p = exp(lse_p - max), out = sum w_p o_p / sum w; pieces without a token (lse -inf) take no
// part.
constexpr int MERGE_MAXP = MAXSPLIT_PIECES;
__global__ void __launch_bounds__(256) split_merge_kernel(const float *__restrict__ ws_o,
                                                          const float *__restrict__ ws_lse, int T, int G, int ntiles,
                                                          int H, int Lq, OutRows out, int out_fp32, float *lse) {
    const int t = blockIdx.x;
    const int ca = (int)(((long)t * G) / T), cb = (int)(((long)(t + 1) * G - 1) / T);
    if (ca == cb) return;                       // the whole tile is one CTA's: already written
    const int r = blockIdx.y * 8 + threadIdx.x / (D / 4), quad = threadIdx.x % (D / 4);
    const int h = t / ntiles, row = (t % ntiles) * 128 + r;
    if (row >= Lq) return;
    const int np = min(cb - ca + 1, MERGE_MAXP);
    float l[MERGE_MAXP];
    float4 v[MERGE_MAXP];
#pragma unroll
    for (int i = 0; i < MERGE_MAXP; ++i) {
        if (i < np) {
            const int slot = split_slot(ca + i, t, T, G);
            l[i] = ws_lse[(size_t)slot * 128 + r];
            v[i] = reinterpret_cast<const float4 *>(ws_o + ((size_t)slot * 128 + r) * D)[quad];
        }
    }
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < MERGE_MAXP; ++i)
        if (i < np) mx = fmaxf(mx, l[i]);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float wsum = 0.f;
    if (mx != -INFINITY) {
#pragma unroll
        for (int i = 0; i < MERGE_MAXP; ++i) {
            if (i < np && l[i] != -INFINITY) {
                const float w = __expf(l[i] - mx);
                acc.x = fmaf(w, v[i].x, acc.x);
                acc.y = fmaf(w, v[i].y, acc.y);
                acc.z = fmaf(w, v[i].z, acc.z);
                acc.w = fmaf(w, v[i].w, acc.w);
                wsum += w;
            }
        }
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    size_t base = ((size_t)row * out.heads + out.h0 + h) * D + quad * 4;
    int d_lo = 0;
    int d_hi = out.n;
    if (out.rows > 0) {   // owner mode (see OutRows)
        const int d = row / out.rows, rl = row - d * out.rows;
        base = (((size_t)out.slot * out.rows + rl) * out.heads + out.h0 + h) * D + quad * 4;
        d_lo = d;
        d_hi = d + 1;
        if (quad == 0) {
            const float l_row = wsum > 0.f ? mx + __logf(wsum) : -INFINITY;
            const size_t li = ((size_t)out.slot * out.heads + out.h0 + h) * out.rows + rl;
#pragma unroll
            for (int i = 0; i < SS_MAX_PEERS; ++i)
                if (i == d) out.lse[i][li] = l_row;
        }
    }
#pragma unroll
    for (int d = 0; d < SS_MAX_PEERS; ++d) {
        if (d >= d_hi) break;
        if (d < d_lo) continue;
        if (out_fp32) {
            reinterpret_cast<float4 *>(reinterpret_cast<float *>(out.p[d]) + base)[0] =
                make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
        } else {
            reinterpret_cast<uint2 *>(reinterpret_cast<__nv_bfloat16 *>(out.p[d]) + base)[0] =
                make_uint2(pack_bf16x2(acc.x * inv, acc.y * inv), pack_bf16x2(acc.z * inv, acc.w * inv));
        }
    }
    if (lse && quad == 0) lse[(size_t)h * Lq + row] = wsum > 0.f ? mx + __logf(wsum) : -INFINITY;
}

}  // namespace attn

// Steps of one tile: at most `sb_tile` sub-blocks, padded to an even number (>= 2) of steps.
static long attention_tile_steps(long sb_tile) { return std::max(2L, ((sb_tile + 3) & ~3L) / 2); }

static long attention_smem_for(int kb, int block, int n_ids, int tmax) {
    const int nwords = (kb + 31) / 32;
    const long sb_tile = (block == 64) ? std::min(2L * n_ids, (long)kb) : 2L * std::min(n_ids, kb);
    const long cap = tmax * attention_tile_steps(sb_tile);
    // alignment slack, fixed tables, ring, bitmaps, steps (8 B each)
    return 1024 + attn::OFF_RING + (long)attn::NST * attn::TILE_BYTES + 8L * tmax * nwords + 8L * cap;
}

int attention_smem_bytes(int Lk, int block, int n_ids, uint32_t *bytes) {
    const int kb = (Lk + block - 1) / block;
    const long total = attention_smem_for(kb, block, n_ids, 1);
    *bytes = (uint32_t)total;
    return total <= (long)attn::SMEM_LIMIT ? 0 : SS_ERR_SMEM;
}

static int g_attn_configured[SS_MAX_DEVICES] = {0};
static int g_num_sms[SS_MAX_DEVICES] = {0};
static std::mutex g_attn_mutex;

static void *g_attn_ctx[SS_MAX_DEVICES] = {nullptr};

// Per (device, context): the kernel's shared-memory attribute and the SM count. A new context on
// the device (after cudaDeviceReset) is configured again.
int attention_prepare(int device) {
    if (device < 0 || device >= SS_MAX_DEVICES) return SS_ERR_DEVICE;
    void *ctx = nullptr;
    int rc = current_context(&ctx);
    if (rc) return rc;
    std::lock_guard<std::mutex> lock(g_attn_mutex);
    if (g_attn_configured[device] && g_attn_ctx[device] == ctx) return 0;
    cudaError_t e = cudaFuncSetAttribute(attn::sparse_attention_kernel<1>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)attn::SMEM_LIMIT);
    if (e != cudaSuccess) return (int)e;
    e = cudaFuncSetAttribute(attn::sparse_attention_kernel<SS_MAX_PEERS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)attn::SMEM_LIMIT);
    if (e != cudaSuccess) return (int)e;
    int nsm = 0;
    e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess) return (int)e;
    g_num_sms[device] = nsm;
    g_attn_ctx[device] = ctx;
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

namespace ss {

// CTAs per tile at most, in split mode (the grid is min(#SMs, MAXSPLIT * T) CTAs).
constexpr int MAXSPLIT = 8;
static_assert(attn::MAXSPLIT_PIECES >= MAXSPLIT + 1, "pieces per tile");

// Measured on B200 (kernel alone): 156 tiles 77.8 -> 74.9 us and 222 tiles 144.9 -> 136.2 us with
// the split; at half a tile per SM or less every tile is cut in two or more equal pieces, config 4
// with 74 tiles 71.1 -> 52.3 us; in between a piece's fixed start-up, epilogue and merge cost more
// than the balance gained (111 tiles 71.9 -> 76.9 us), so those run whole.
static bool split_wanted(int T, int nsm) { return (T >= nsm && T < 2 * nsm) || 2 * T <= nsm; }
static int split_grid(int T, int nsm) { return std::min(nsm, MAXSPLIT * T); }
static size_t split_ws_bytes(int G) { return (size_t)2 * G * 128 * (attn::D + 1) * sizeof(float); }

// A ring geometry the kernels can follow for a window of Lk rows: the window's ring rows and the
// repeated sink rows fit the ring, and every physical row fits the 20-bit row field of a step.
int ring_check(const KvRing &r, int Lk) {
    if (r.C == 0) return r.S == 0 && r.head == 0 ? 0 : SS_ERR_SHAPE;
    if (r.S < 0 || r.C < 64 || r.head < 0 || r.head >= r.C) return SS_ERR_SHAPE;
    if ((int64_t)r.S + r.C + 64 >= (1 << 20) - 128) return SS_ERR_SHAPE;
    if (Lk > r.S && (int64_t)(Lk - r.S) + (r.S % 64) > r.C) return SS_ERR_SHAPE;
    return 0;
}

static int attention_launch(const void *q, const void *k, const void *v, const int32_t *ids, int H, int Lq, int Lk,
                            int block, int n_ids, float scale, void *out, int out_dtype, float *lse, int *status,
                            void *ws, size_t ws_bytes, cudaStream_t stream, KvRing ring = KvRing(),
                            const attn::OutRows *dst = nullptr) {
    if (!q || !k || !v || !ids || (!out && !dst)) return SS_ERR_POINTER;
    if (H <= 0 || Lq <= 0 || Lk <= 0 || n_ids <= 0 || (block != 64 && block != 128)) return SS_ERR_SHAPE;
    if (Lk >= (1 << 20) - 128 || (long)Lq * H * attn::D >= (1L << 31) || (long)Lk * H * attn::D >= (1L << 31))
        return SS_ERR_SHAPE;
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15u)
        return SS_ERR_POINTER;
    attn::OutRows rows;
    if (dst) {
        rows = *dst;
        if (rows.n < 1 || rows.n > SS_MAX_PEERS || rows.h0 < 0 || rows.heads < rows.h0 + H) return SS_ERR_SHAPE;
        if (rows.rows < 0 || (rows.rows > 0 && ((long)rows.rows * rows.n < Lq || rows.slot < 0 ||
                                                rows.slot >= rows.n)))
            return SS_ERR_SHAPE;
        if ((long)std::max(Lq, rows.n * rows.rows) * rows.heads * attn::D >= (1L << 31)) return SS_ERR_SHAPE;
    } else {
        rows.n = 1;
        rows.p[0] = out;
        rows.heads = H;
        rows.h0 = 0;
        rows.rows = 0;
        rows.slot = 0;
    }
    for (int d = 0; d < SS_MAX_PEERS; ++d) {
        if (d >= rows.n) {
            rows.p[d] = nullptr;
            rows.lse[d] = nullptr;
            continue;
        }
        if (!rows.p[d]) return SS_ERR_POINTER;
        if (reinterpret_cast<uintptr_t>(rows.p[d]) & 31u) return SS_ERR_POINTER;   // 32-byte row stores
        if (rows.rows > 0) {
            if (!rows.lse[d] || (reinterpret_cast<uintptr_t>(rows.lse[d]) & 3u)) return SS_ERR_POINTER;
        } else {
            rows.lse[d] = nullptr;
        }
    }
    if (out_dtype != 0 && out_dtype != 1) return SS_ERR_SHAPE;
    if (ring_check(ring, Lk)) return SS_ERR_SHAPE;
    if (ws && (reinterpret_cast<uintptr_t>(ws) & 255u)) return SS_ERR_POINTER;
    uint32_t smem1;
    int rc = attention_smem_bytes(Lk, block, n_ids, &smem1);
    if (rc) return rc;
    int device;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return (int)e;
    rc = attention_prepare(device);
    if (rc) return rc;

    attn::Params prm;
    prm.q = static_cast<const __nv_bfloat16 *>(q);
    prm.ids = ids;
    prm.out = rows;
    prm.lse = lse;
    prm.status = status;
    prm.H = H;
    prm.Lq = Lq;
    prm.Lk = Lk;
    prm.block = block;
    prm.n_ids = n_ids;
    prm.qb = (Lq + block - 1) / block;
    prm.kb = (Lk + block - 1) / block;
    prm.ntiles = (Lq + 127) / 128;
    prm.nwords = (prm.kb + 31) / 32;
    prm.T = prm.ntiles * H;
    prm.split = 0;
    prm.ws_o = prm.ws_lse = nullptr;
    prm.ring = ring;
    prm.own_n = 1;
    prm.own_r = 0;
    if (rows.rows > 0) {   // owner mode: the ids are the window's, this rank stores blocks j % n == slot
        prm.own_n = rows.n;
        prm.own_r = rows.slot;
    }
    const int nsm = g_num_sms[device] > 0 ? g_num_sms[device] : 148;
    const long sb_tile = (block == 64) ? std::min(2L * n_ids, (long)prm.kb) : 2L * std::min(n_ids, prm.kb);
    int G;
    if (ws && split_wanted(prm.T, nsm)) {
        // split mode: every CTA's units meet at most ceil(T/G) + 1 tiles; below one tile per SM
        // only where a piece keeps at least 8 steps of the longest list (short lists run whole)
        G = split_grid(prm.T, nsm);
        const int tmax = (prm.T + G - 1) / G + 1;
        const bool pieces_long = prm.T >= nsm || attention_tile_steps(sb_tile) * prm.T >= 8L * G;
        if (pieces_long && ws_bytes >= split_ws_bytes(G) &&
            attention_smem_for(prm.kb, block, n_ids, tmax) <= (long)attn::SMEM_LIMIT) {
            prm.split = 1;
            prm.tmax = tmax;
            prm.ws_o = static_cast<float *>(ws);
            prm.ws_lse = prm.ws_o + (size_t)2 * G * 128 * attn::D;
        }
    }
    if (!prm.split) {
        // one CTA per SM running ceil(T / G) tiles; fewer tiles per CTA (more CTAs) where the step
        // lists need the room
        G = std::max(std::min(prm.T, nsm), (prm.T + attn::MAXT - 1) / attn::MAXT);
        while (attention_smem_for(prm.kb, block, n_ids, (prm.T + G - 1) / G) > (long)attn::SMEM_LIMIT &&
               (prm.T + G - 1) / G > 1) {
            const int tmax = (prm.T + G - 1) / G;
            G = (prm.T + tmax - 2) / (tmax - 1);   // one tile fewer per CTA
        }
        prm.tmax = (prm.T + G - 1) / G;
    }
    prm.G = G;
    prm.step_cap = (int)(prm.tmax * attention_tile_steps(sb_tile));
    prm.out_fp32 = out_dtype;
    prm.scale_log2 = scale * 1.4426950408889634f;
    const long smem = attention_smem_for(prm.kb, block, n_ids, prm.tmax);
    if (smem > (long)attn::SMEM_LIMIT) return SS_ERR_SMEM;

    CUtensorMap tk, tv;
    const uint64_t row_bytes = (uint64_t)H * attn::D * 2;
    const uint64_t kv_rows = (uint64_t)ring.phys_rows(Lk);
    if (encode_tmap_2d_bf16(&tk, k, (uint64_t)H * attn::D, kv_rows, row_bytes, 64, 64)) return SS_ERR_DRIVER;
    if (encode_tmap_2d_bf16(&tv, v, (uint64_t)H * attn::D, kv_rows, row_bytes, 64, 64)) return SS_ERR_DRIVER;

    if (rows.n == 1)
        attn::sparse_attention_kernel<1><<<dim3((unsigned)G), attn::NTHREADS, (size_t)smem, stream>>>(tk, tv, prm);
    else
        attn::sparse_attention_kernel<SS_MAX_PEERS>
            <<<dim3((unsigned)G), attn::NTHREADS, (size_t)smem, stream>>>(tk, tv, prm);
    if (prm.split)
        attn::split_merge_kernel<<<dim3((unsigned)prm.T, 16), 256, 0, stream>>>(prm.ws_o, prm.ws_lse, prm.T, G,
                                                                                 prm.ntiles, H, Lq, rows, out_dtype, lse);
    return (int)cudaGetLastError();
}

}  // namespace ss

extern "C" int ss_attention(const void *q, const void *k, const void *v, const int32_t *ids, int H, int Lq, int Lk,
                            int block, int n_ids, float scale, void *out, int out_dtype, float *lse, int *status,
                            void *stream) {
    return ss::attention_launch(q, k, v, ids, H, Lq, Lk, block, n_ids, scale, out, out_dtype, lse, status, nullptr, 0,
                                static_cast<cudaStream_t>(stream));
}

extern "C" int ss_attention_workspace_bytes(int H, int Lq, size_t *bytes) {
    if (!bytes || H <= 0 || Lq <= 0) return SS_ERR_SHAPE;
    int device;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return (int)e;
    int rc = ss::attention_prepare(device);
    if (rc) return rc;
    const int nsm = ss::g_num_sms[device] > 0 ? ss::g_num_sms[device] : 148;
    const int T = (Lq + 127) / 128 * H;
    *bytes = ss::split_wanted(T, nsm) ? ss::split_ws_bytes(ss::split_grid(T, nsm)) : 0;
    return 0;
}

extern "C" int ss_attention_ws(const void *q, const void *k, const void *v, const int32_t *ids, int H, int Lq, int Lk,
                               int block, int n_ids, float scale, void *out, int out_dtype, float *lse, int *status,
                               void *workspace, size_t workspace_bytes, void *stream) {
    return ss::attention_launch(q, k, v, ids, H, Lq, Lk, block, n_ids, scale, out, out_dtype, lse, status, workspace,
                                workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" int ss_attention_ring(const void *q, const void *k, const void *v, const int32_t *ids, int H, int Lq,
                                 int Lk, int block, int n_ids, float scale, void *out, int out_dtype, float *lse,
                                 int *status, int ring_sink, int ring_cap, int ring_head, const int *ring_head_dev,
                                 void *workspace, size_t workspace_bytes, void *stream) {
    ss::KvRing ring;
    ring.S = ring_sink;
    ring.C = ring_cap;
    ring.head = ring_head;
    ring.head_dev = ring_head_dev;
    if (ring_cap <= 0) return SS_ERR_SHAPE;
    return ss::attention_launch(q, k, v, ids, H, Lq, Lk, block, n_ids, scale, out, out_dtype, lse, status, workspace,
                                workspace_bytes, static_cast<cudaStream_t>(stream), ring);
}

extern "C" int ss_attention_heads(const void *q, const void *k, const void *v, const int32_t *ids, int H, int Lq,
                                  int Lk, int block, int n_ids, float scale, void *const *outs, int P, int out_heads,
                                  int h0, int out_dtype, float *lse, int *status, int ring_sink, int ring_cap,
                                  int ring_head, const int *ring_head_dev, void *workspace, size_t workspace_bytes,
                                  void *stream) {
    if (!outs) return SS_ERR_POINTER;
    if (P < 1 || P > SS_MAX_PEERS) return SS_ERR_SHAPE;
    ss::KvRing ring;
    if (ring_cap > 0) {
        ring.S = ring_sink;
        ring.C = ring_cap;
        ring.head = ring_head;
        ring.head_dev = ring_head_dev;
    }
    ss::attn::OutRows rows;
    rows.n = P;
    rows.heads = out_heads;
    rows.h0 = h0;
    rows.rows = 0;
    rows.slot = 0;
    for (int d = 0; d < SS_MAX_PEERS; ++d) {
        rows.p[d] = d < P ? outs[d] : nullptr;
        rows.lse[d] = nullptr;
    }
    return ss::attention_launch(q, k, v, ids, H, Lq, Lk, block, n_ids, scale, nullptr, out_dtype, lse, status,
                                workspace, workspace_bytes, static_cast<cudaStream_t>(stream), ring, &rows);
}

extern "C" int ss_attention_kv_parts(const void *q, const void *k, const void *v, const int32_t *ids, int H, int Lq,
                                     int Lk, int block, int n_ids, float scale, void *const *o_parts,
                                     float *const *lse_parts, int P, int rows, int slot, int part_dtype,
                                     int *status, void *workspace, size_t workspace_bytes, void *stream) {
    if (!o_parts || !lse_parts) return SS_ERR_POINTER;
    if (P < 1 || P > SS_MAX_PEERS || rows <= 0) return SS_ERR_SHAPE;
    ss::attn::OutRows dst;
    dst.n = P;
    dst.heads = H;
    dst.h0 = 0;
    dst.rows = rows;
    dst.slot = slot;
    for (int d = 0; d < SS_MAX_PEERS; ++d) {
        dst.p[d] = d < P ? o_parts[d] : nullptr;
        dst.lse[d] = d < P ? lse_parts[d] : nullptr;
    }
    return ss::attention_launch(q, k, v, ids, H, Lq, Lk, block, n_ids, scale, nullptr, part_dtype, nullptr, status,
                                workspace, workspace_bytes, static_cast<cudaStream_t>(stream), ss::KvRing(), &dst);
}
