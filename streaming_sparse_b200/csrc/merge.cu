// merge.cu -- log-sum-exp merge of P partial attention results.
//
//   L = logsumexp_p lse_p,   out = sum_p exp(lse_p - L) * o_p
// Reference: `merge` (local_experiments/video_runtime_v1/attention.py:40-45, two parts with
// logaddexp) and the split merge `_merge_restore` (migration/unified_router/opt21/attention.py:
// 7-15, base-2 weights). Used for KV-block sharding across GPUs (each rank attends over the
// blocks it owns, partial results are combined) and for any split of a block list.
// A row whose parts are all empty (every lse = -inf) produces zeros and L = -inf.
#include "common.cuh"

namespace ss {
namespace merge {

constexpr int D = 128;

// One thread per (row, head, 4 consecutive dims). For up to PMAX parts every part's LSE and
// float4 are loaded before any is used, so a thread has all of its loads in flight at once (a
// dependent loop over the parts kept one or two per thread in flight and left DRAM half idle);
// the parts are read once, so their loads are marked evict-first. PMAX = 0: any P, one part at a
// time. The arithmetic and its order are the same for every PMAX.
template <int PMAX>
__global__ void __launch_bounds__(256) lse_merge_kernel(const float *__restrict__ o, const float *__restrict__ lse,
                                                        int P, int H, int Lq, void *out, int out_fp32,
                                                        float *__restrict__ lse_out) {
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t total = (int64_t)Lq * H * (D / 4);
    if (gid >= total) return;
    const int quad = (int)(gid % (D / 4));
    const int64_t rh = gid / (D / 4);  // row * H + h
    const int h = (int)(rh % H);
    const int row = (int)(rh / H);
    const float *lp = lse + (int64_t)h * Lq + row;                          // part p at lp[p * H * Lq]
    const float4 *op = reinterpret_cast<const float4 *>(o + rh * D) + quad;  // part p at op[p * Lq * H * D / 4]
    const int64_t lstride = (int64_t)H * Lq, ostride = (int64_t)Lq * H * (D / 4);
    float mx = -INFINITY, wsum = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if constexpr (PMAX > 0) {
        float l[PMAX];
        float4 v[PMAX];
#pragma unroll
        for (int p = 0; p < PMAX; ++p) {
            if (p < P) {
                l[p] = __ldcs(lp + p * lstride);
                v[p] = __ldcs(op + p * ostride);
            }
        }
#pragma unroll
        for (int p = 0; p < PMAX; ++p)
            if (p < P) mx = fmaxf(mx, l[p]);
        if (mx != -INFINITY) {
#pragma unroll
            for (int p = 0; p < PMAX; ++p) {
                if (p < P) {
                    const float w = __expf(l[p] - mx);
                    acc.x = fmaf(w, v[p].x, acc.x);
                    acc.y = fmaf(w, v[p].y, acc.y);
                    acc.z = fmaf(w, v[p].z, acc.z);
                    acc.w = fmaf(w, v[p].w, acc.w);
                    wsum += w;
                }
            }
        }
    } else {
        for (int p = 0; p < P; ++p) mx = fmaxf(mx, lp[p * lstride]);
        if (mx != -INFINITY) {
            for (int p = 0; p < P; ++p) {
                const float w = __expf(lp[p * lstride] - mx);
                const float4 v = op[p * ostride];
                acc.x = fmaf(w, v.x, acc.x);
                acc.y = fmaf(w, v.y, acc.y);
                acc.z = fmaf(w, v.z, acc.z);
                acc.w = fmaf(w, v.w, acc.w);
                wsum += w;
            }
        }
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    acc.x *= inv;
    acc.y *= inv;
    acc.z *= inv;
    acc.w *= inv;
    const int64_t base = rh * D + quad * 4;
    if (out_fp32) {
        reinterpret_cast<float4 *>(reinterpret_cast<float *>(out) + base)[0] = acc;
    } else {
        uint2 pk = make_uint2(pack_bf16x2(acc.x, acc.y), pack_bf16x2(acc.z, acc.w));
        reinterpret_cast<uint2 *>(reinterpret_cast<__nv_bfloat16 *>(out) + base)[0] = pk;
    }
    if (lse_out && quad == 0) lse_out[(int64_t)h * Lq + row] = wsum > 0.f ? mx + __logf(wsum) : -INFINITY;
}

}  // namespace merge
}  // namespace ss

extern "C" int ss_lse_merge(const float *o_parts, const float *lse_parts, int P, int H, int Lq, void *out,
                            int out_dtype, float *lse_out, void *stream) {
    if (!o_parts || !lse_parts || !out) return SS_ERR_POINTER;
    if (P <= 0 || H <= 0 || Lq <= 0 || (out_dtype != 0 && out_dtype != 1)) return SS_ERR_SHAPE;
    if ((reinterpret_cast<uintptr_t>(o_parts) | reinterpret_cast<uintptr_t>(out)) & 15u) return SS_ERR_POINTER;
    const int64_t total = (int64_t)Lq * H * (ss::merge::D / 4);
    const unsigned blocks = (unsigned)((total + 255) / 256);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (P <= 2)
        ss::merge::lse_merge_kernel<2><<<blocks, 256, 0, st>>>(o_parts, lse_parts, P, H, Lq, out, out_dtype, lse_out);
    else if (P <= 4)
        ss::merge::lse_merge_kernel<4><<<blocks, 256, 0, st>>>(o_parts, lse_parts, P, H, Lq, out, out_dtype, lse_out);
    else if (P <= 8)
        ss::merge::lse_merge_kernel<8><<<blocks, 256, 0, st>>>(o_parts, lse_parts, P, H, Lq, out, out_dtype, lse_out);
    else
        ss::merge::lse_merge_kernel<0><<<blocks, 256, 0, st>>>(o_parts, lse_parts, P, H, Lq, out, out_dtype, lse_out);
    return (int)cudaGetLastError();
}
