/*
 * ssparse_oracle.c -- CPU restatement of the routed sparse-attention router, TEST INFRASTRUCTURE.
 *
 * This file is the checker, never the product: only tests/, __graft_entry__.smoke() and the
 * CPU-baseline leg of bench.py load it. The CUDA library (streaming_sparse_b200/csrc) must
 * reproduce these results bit for bit; nothing in the package calls this code.
 *
 * Arithmetic contract (identical on the GPU):
 *   pooled[d]  = (((x_0[d] + x_1[d]) + x_2[d]) + ... ) / n     fp32 adds in token order, one
 *                                                              correctly rounded divide by the
 *                                                              number of valid tokens n
 *   proj[e]    = fmaf(pooled[127], W[127][e], ... fmaf(pooled[0], W[0][e], 0.0f))
 *   score[i,j] = fmaf(qh[i][R-1], kh[j][R-1], ... fmaf(qh[i][0], kh[j][0], 0.0f)),  -0 -> +0
 *   selection  = forced blocks  U  the `extra` unforced blocks with the largest key, where
 *                key = (order-preserving uint32 of the score) << 32 | (0xffffffff - block),
 *                so ties go to the lower block index; ids are written in ascending order.
 *
 * Reference behaviour restated (paths inside jurky123/streaming_sparse):
 *   - block pooling: prototype pooling segment() with one prototype reduces to the plain mean
 *     of the block's valid tokens (migration/unified_router/opt19/prototype.py:11-49, the
 *     t < N validity mask at :17,30); LightForcing-style mean pooling is the same reduction.
 *   - projection q @ basis, 128 -> 64 (migration/unified_router/opt8/projection.py:4-14;
 *     CPU form torch.bmm(q, basis) in migration/unified_router/fast_route.py:25-34).
 *   - block-score GEMM (migration/unified_router/opt16/route.py:34-47, fast_route.py:30).
 *   - integer-ordered fp32 keys for exact ordering (opt16/route.py:13-24 `_chosen`;
 *     local_experiments/video_runtime_v1/fixed_page_select.py:14-16) and the lower-index
 *     tie-break of the stable CPU select (streaming_sparse/v05/primitives.py:35-56). Unlike the
 *     raw bit order of fixed_page_select, -0 and +0 compare equal here, as in the stable
 *     float sort of v05 select.
 *   - forced set (sink and current-chunk blocks always kept, budget applied to the rest):
 *     local_experiments/video_runtime_v1/pipeline_graph.py:140-151.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* pooled/proj for nb blocks of `block` tokens over x[L][H][D] (fp32 copies of bf16 values). */
int oracle_pool_project(const float *x, int64_t row_stride, int L, int H, int D, int R,
                        int block, const float *W, float *pooled, float *proj) {
    int nb = (L + block - 1) / block;
    float *mean = (float *)malloc(sizeof(float) * (size_t)D);
    if (!mean) return -1;
    for (int h = 0; h < H; ++h) {
        for (int b = 0; b < nb; ++b) {
            int t0 = b * block;
            int n = L - t0 < block ? L - t0 : block;
            for (int d = 0; d < D; ++d) {
                float s = 0.0f;
                for (int t = 0; t < n; ++t) s = s + x[(int64_t)(t0 + t) * row_stride + h * D + d];
                mean[d] = s / (float)n;
                if (pooled) pooled[((int64_t)h * nb + b) * D + d] = mean[d];
            }
            for (int e = 0; e < R; ++e) {
                float acc = 0.0f;
                for (int d = 0; d < D; ++d) acc = fmaf(mean[d], W[((int64_t)h * D + d) * R + e], acc);
                proj[((int64_t)h * nb + b) * R + e] = acc;
            }
        }
    }
    free(mean);
    return 0;
}

/* S[h][i][j] = <qh[h][i], kh[h][j]>; returns the number of non-finite scores. */
int64_t oracle_scores(const float *qh, const float *kh, int H, int qb, int kb, int R, float *S) {
    int64_t bad = 0;
    for (int h = 0; h < H; ++h)
        for (int i = 0; i < qb; ++i)
            for (int j = 0; j < kb; ++j) {
                const float *a = qh + ((int64_t)h * qb + i) * R;
                const float *c = kh + ((int64_t)h * kb + j) * R;
                float acc = 0.0f;
                for (int e = 0; e < R; ++e) acc = fmaf(a[e], c[e], acc);
                if (acc == 0.0f) acc = 0.0f; /* canonicalise -0 */
                if (!isfinite(acc)) ++bad;
                S[((int64_t)h * qb + i) * kb + j] = acc;
            }
    return bad;
}

static uint32_t ordered_bits(float f) {
    uint32_t u;
    if (f == 0.0f) f = 0.0f;
    memcpy(&u, &f, 4);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

static int cmp_desc(const void *a, const void *b) {
    uint64_t x = *(const uint64_t *)a, y = *(const uint64_t *)b;
    return x < y ? 1 : (x > y ? -1 : 0);
}

/* Forced blocks: those overlapping [0, sink_tokens) or [Lk - Lq, Lk). */
int oracle_forced(int Lq, int Lk, int block, int sink_tokens, uint8_t *forced) {
    int kb = (Lk + block - 1) / block, count = 0;
    for (int j = 0; j < kb; ++j) {
        int64_t lo = (int64_t)j * block, hi = lo + block;
        if (hi > Lk) hi = Lk;
        int f = (lo < sink_tokens) || (hi > (int64_t)(Lk - Lq));
        forced[j] = (uint8_t)f;
        count += f;
    }
    return count;
}

/* Selection over S[H][qb][kb]: ids [H][qb][n_ids] ascending, mask [H][qb][kb] (optional). */
int oracle_select(const float *S, int H, int qb, int kb, const uint8_t *forced, int extra,
                  int32_t *ids, int n_ids, uint8_t *mask) {
    int nforced = 0;
    for (int j = 0; j < kb; ++j) nforced += forced[j] != 0;
    if (extra < 0 || extra > kb - nforced || n_ids != nforced + extra) return -1;
    uint64_t *keys = (uint64_t *)malloc(sizeof(uint64_t) * (size_t)(kb + 1));
    uint8_t *sel = (uint8_t *)malloc((size_t)kb + 1);
    if (!keys || !sel) { free(keys); free(sel); return -2; }
    for (int h = 0; h < H; ++h)
        for (int i = 0; i < qb; ++i) {
            const float *row = S + ((int64_t)h * qb + i) * kb;
            int m = 0;
            for (int j = 0; j < kb; ++j)
                if (!forced[j]) keys[m++] = ((uint64_t)ordered_bits(row[j]) << 32) | (uint64_t)(0xffffffffu - (uint32_t)j);
            qsort(keys, (size_t)m, sizeof(uint64_t), cmp_desc);
            for (int j = 0; j < kb; ++j) sel[j] = forced[j] ? 1 : 0;
            for (int r = 0; r < extra; ++r) sel[0xffffffffu - (uint32_t)(keys[r] & 0xffffffffu)] = 1;
            int32_t *out = ids + ((int64_t)h * qb + i) * n_ids;
            int c = 0;
            for (int j = 0; j < kb; ++j) {
                if (sel[j]) out[c++] = j;
                if (mask) mask[((int64_t)h * qb + i) * kb + j] = sel[j];
            }
        }
    free(keys);
    free(sel);
    return 0;
}
