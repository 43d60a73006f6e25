// dit.cu -- fused per-token kernels of the streaming DiT layer around the sparse attention.
//
// The rollout's self-attention layer feeds the routed attention from one q/k/v GEMM; what lies
// between the GEMMs is per-token, HBM-bound work that PyTorch runs as ~20 separate elementwise
// kernels per layer. Four kernels replace it, each one pass over its rows (16-byte vectors,
// one CTA per token row, fp32 math, bf16 out):
//
//   ss_qkv_norm_rope  q/k RMSNorm over the model width, the learned norm weight, 3-D RoPE, and
//                     the post-RoPE k plus v written straight into the KV-cache rows -- the
//                     reference's fused projection hook `project_cached_rotary`
//                     (wan/modules/causal_model.py:116-128, 241-246; its CUDA/Triton form in
//                     local_experiments/video_runtime_v1/rms_mean.py:38-72), which the plain
//                     path spells as norm_q/norm_k + causal_rope_apply + key_window.copy_
//                     (causal_model.py:110-114, 211-214, 239-243).
//   ss_adaln          LayerNorm (no affine) + per-frame modulation y * (1 + scale) + shift
//                     (causal_model.py:332, 344-345, 383) or LayerNorm with affine weight/bias
//                     (norm3, causal_model.py:285-287).
//   ss_rms_norm       WanRMSNorm of rows (the cross-attention query norm, model.py:70-86, 172).
//   ss_gate_residual  x += y * gate per frame (causal_model.py:337, 348-349), or x += y.
//
// Rounding follows the PyTorch expressions of the harness: RMSNorm's normalised value is
// rounded to bf16 before the weight multiply (WanRMSNorm: `_norm(x.float()).type_as(x) *
// weight`), LayerNorm's output is rounded to bf16 before modulation (`type_as(x)`), and each
// product and sum of the modulation, gate and rotation is rounded to fp32 separately (no FMA
// contraction), as the separate PyTorch kernels do.
#include <cuda_bf16.h>

#include "common.cuh"

namespace ss {
namespace dit {

constexpr int HD = 128;   // head dimension
constexpr int VEC = 8;    // bf16 per 16-byte vector

__device__ __forceinline__ void unpack8(const uint4 &v, float (&f)[VEC]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[2 * i] = __uint_as_float(w[i] << 16);
        f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
    const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(a));
    const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(b));
    return lo | (hi << 16);
}

__device__ __forceinline__ uint4 pack8(const float (&f)[VEC]) {
    return make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
}

__device__ __forceinline__ float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// sum of (a, b) over the CTA (blockDim.x a multiple of 32, at most 1024); every thread gets it
__device__ __forceinline__ float2 block_sum2(float a, float b, float2 *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        a += __shfl_xor_sync(0xffffffffu, a, o);
        b += __shfl_xor_sync(0xffffffffu, b, o);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();   // red may still be read by a previous call
    if (lane == 0) red[warp] = make_float2(a, b);
    __syncthreads();
    float2 s = make_float2(0.f, 0.f);
    for (int i = 0; i < nw; ++i) {   // the same order in every thread
        s.x += red[i].x;
        s.y += red[i].y;
    }
    return s;
}

// Where row r of the k/v output goes: row r (C = 0), or in a ring-buffer cache the physical row
// of window row t0 + r (the sink's rows in place, the rest at S + ((t - S + head) mod C) with
// head = (*head_dev + evicted) mod C, the head after this write's roll), written once more at
// S + C + that ring row when it is below 64 (the ring's mirrored rows).
struct RingRows {
    int S = 0, C = 0;
    int64_t t0 = 0;
    const int *head_dev = nullptr;
    int evicted = 0;
};

// One CTA per token row of width d = H * 128: q = rope(bf16(bf16(q * rq) * wq)), same for k,
// v copied; q to q_out, k and v to k_out / v_out (cache rows, placed by rr).
__global__ void __launch_bounds__(1024) qkv_norm_rope_kernel(
    const __nv_bfloat16 *__restrict__ qkv, int64_t ld, int d, const __nv_bfloat16 *__restrict__ wq,
    const __nv_bfloat16 *__restrict__ wk, float eps, const float *__restrict__ cos_t,
    const float *__restrict__ sin_t, __nv_bfloat16 *__restrict__ q_out, int64_t q_ld,
    __nv_bfloat16 *__restrict__ k_out, __nv_bfloat16 *__restrict__ v_out, int64_t kv_ld, RingRows rr, int c0,
    int c1) {
    __shared__ float2 red[32];
    const int64_t row = blockIdx.x;
    const int t = threadIdx.x;
    const bool active = t * VEC < d;
    const __nv_bfloat16 *src = qkv + row * ld;
    float q[VEC], k[VEC];
    uint4 vv = make_uint4(0, 0, 0, 0);
    float sq = 0.f, sk = 0.f;
    if (active) {
        unpack8(*reinterpret_cast<const uint4 *>(src + t * VEC), q);
        unpack8(*reinterpret_cast<const uint4 *>(src + d + t * VEC), k);
        vv = *reinterpret_cast<const uint4 *>(src + 2 * d + t * VEC);
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
            sq = __fadd_rn(sq, __fmul_rn(q[i], q[i]));
            sk = __fadd_rn(sk, __fmul_rn(k[i], k[i]));
        }
    }
    const float2 s = block_sum2(sq, sk, red);
    // the norm is over the whole row; only the columns [c0, c1) (whole heads) are written, at
    // column t * VEC - c0 of the outputs
    if (!active || t * VEC < c0 || t * VEC >= c1) return;
    const int oc = t * VEC - c0;
    const float rq = rsqrtf(__fadd_rn(__fdiv_rn(s.x, (float)d), eps));
    const float rk = rsqrtf(__fadd_rn(__fdiv_rn(s.y, (float)d), eps));
    float w_q[VEC], w_k[VEC];
    unpack8(*reinterpret_cast<const uint4 *>(wq + t * VEC), w_q);
    unpack8(*reinterpret_cast<const uint4 *>(wk + t * VEC), w_k);
    const int p0 = ((t * VEC) % HD) / 2;   // first rotation pair of this vector within its head
    const float *cr = cos_t + row * (HD / 2) + p0;
    const float *sr = sin_t + row * (HD / 2) + p0;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
        q[i] = round_bf16(__fmul_rn(round_bf16(__fmul_rn(q[i], rq)), w_q[i]));
        k[i] = round_bf16(__fmul_rn(round_bf16(__fmul_rn(k[i], rk)), w_k[i]));
    }
    float qo[VEC], ko[VEC];
#pragma unroll
    for (int j = 0; j < VEC / 2; ++j) {
        const float c = cr[j], sn = sr[j];
        qo[2 * j] = __fsub_rn(__fmul_rn(q[2 * j], c), __fmul_rn(q[2 * j + 1], sn));
        qo[2 * j + 1] = __fadd_rn(__fmul_rn(q[2 * j], sn), __fmul_rn(q[2 * j + 1], c));
        ko[2 * j] = __fsub_rn(__fmul_rn(k[2 * j], c), __fmul_rn(k[2 * j + 1], sn));
        ko[2 * j + 1] = __fadd_rn(__fmul_rn(k[2 * j], sn), __fmul_rn(k[2 * j + 1], c));
    }
    *reinterpret_cast<uint4 *>(q_out + row * q_ld + oc) = pack8(qo);
    int64_t krow = row, mrow = -1;
    if (rr.C) {
        const int64_t tw = rr.t0 + row;
        if (tw < rr.S) {
            krow = tw;
        } else {
            const int64_t head = ((int64_t)*rr.head_dev + rr.evicted) % rr.C;
            const int64_t pos = ((tw - rr.S + head) % rr.C + rr.C) % rr.C;
            krow = rr.S + pos;
            if (pos < 64) mrow = (int64_t)rr.S + rr.C + pos;
        }
    }
    const uint4 kk = pack8(ko);
    *reinterpret_cast<uint4 *>(k_out + krow * kv_ld + oc) = kk;
    *reinterpret_cast<uint4 *>(v_out + krow * kv_ld + oc) = vv;
    if (mrow >= 0) {
        *reinterpret_cast<uint4 *>(k_out + mrow * kv_ld + oc) = kk;
        *reinterpret_cast<uint4 *>(v_out + mrow * kv_ld + oc) = vv;
    }
}

// One CTA per token row of width d. LayerNorm (two passes over the registers: mean, then the
// mean of squared deviations), then either affine (weight, bias: bf16 vectors) or modulation
// with the row's frame f = row / frame_tokens: out = bf16(bf16(ln) * (1 + scale[f]) + shift[f]).
__global__ void __launch_bounds__(1024) adaln_kernel(const __nv_bfloat16 *__restrict__ x, int d, int frame_tokens,
                                                     const float *__restrict__ shift, const float *__restrict__ scale,
                                                     int64_t mod_ld, const __nv_bfloat16 *__restrict__ weight,
                                                     const __nv_bfloat16 *__restrict__ bias, float eps,
                                                     __nv_bfloat16 *__restrict__ out) {
    __shared__ float2 red[32];
    const int64_t row = blockIdx.x;
    const int t = threadIdx.x;
    const bool active = t * VEC < d;
    float v[VEC];
    float s = 0.f;
    if (active) {
        unpack8(*reinterpret_cast<const uint4 *>(x + row * d + t * VEC), v);
#pragma unroll
        for (int i = 0; i < VEC; ++i) s = __fadd_rn(s, v[i]);
    }
    const float mean = __fdiv_rn(block_sum2(s, 0.f, red).x, (float)d);
    float s2 = 0.f;
    if (active) {
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
            const float c = __fsub_rn(v[i], mean);
            s2 = __fadd_rn(s2, __fmul_rn(c, c));
        }
    }
    const float var = __fdiv_rn(block_sum2(s2, 0.f, red).x, (float)d);
    if (!active) return;
    const float rstd = rsqrtf(__fadd_rn(var, eps));
    float o[VEC];
    if (weight) {
        float w[VEC], b[VEC];
        unpack8(*reinterpret_cast<const uint4 *>(weight + t * VEC), w);
        unpack8(*reinterpret_cast<const uint4 *>(bias + t * VEC), b);
#pragma unroll
        for (int i = 0; i < VEC; ++i) o[i] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[i], mean), rstd), w[i]), b[i]);
    } else {
        const int64_t f = row / frame_tokens;
        const float4 *sh = reinterpret_cast<const float4 *>(shift + f * mod_ld + t * VEC);
        const float4 *sc = reinterpret_cast<const float4 *>(scale + f * mod_ld + t * VEC);
        const float4 a0 = sh[0], a1 = sh[1], c0 = sc[0], c1 = sc[1];
        const float shv[VEC] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const float scv[VEC] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
            const float y = round_bf16(__fmul_rn(__fsub_rn(v[i], mean), rstd));
            o[i] = __fadd_rn(__fmul_rn(y, __fadd_rn(1.f, scv[i])), shv[i]);
        }
    }
    *reinterpret_cast<uint4 *>(out + row * d + t * VEC) = pack8(o);
}

// x[r] = bf16(x[r] + bf16(y[r] * gate[f])) per 16-byte vector, f = r / frame_tokens (gate null:
// x[r] = bf16(x[r] + y[r])). x rows of width d contiguous; y rows at stride y_ld.
__global__ void __launch_bounds__(256) gate_residual_kernel(__nv_bfloat16 *__restrict__ x,
                                                            const __nv_bfloat16 *__restrict__ y, int64_t y_ld,
                                                            int64_t n, int d, int frame_tokens,
                                                            const float *__restrict__ gate, int64_t g_ld) {
    const int vpr = d / VEC;
    const int64_t total = n * vpr;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / vpr;
        const int c = (int)(i % vpr) * VEC;
        float xv[VEC], yv[VEC], o[VEC];
        unpack8(*reinterpret_cast<const uint4 *>(x + r * d + c), xv);
        unpack8(*reinterpret_cast<const uint4 *>(y + r * y_ld + c), yv);
        if (gate) {
            const float4 *g4 = reinterpret_cast<const float4 *>(gate + (r / frame_tokens) * g_ld + c);
            const float4 g0 = g4[0], g1 = g4[1];
            const float gv[VEC] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
            for (int j = 0; j < VEC; ++j) o[j] = __fadd_rn(xv[j], round_bf16(__fmul_rn(yv[j], gv[j])));
        } else {
#pragma unroll
            for (int j = 0; j < VEC; ++j) o[j] = __fadd_rn(xv[j], yv[j]);
        }
        *reinterpret_cast<uint4 *>(x + r * d + c) = pack8(o);
    }
}

// One CTA per token row: out = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * weight) (WanRMSNorm on
// rows of width d; the cross-attention query norm).
__global__ void __launch_bounds__(1024) rms_norm_kernel(const __nv_bfloat16 *__restrict__ x, int64_t x_ld, int d,
                                                        const __nv_bfloat16 *__restrict__ weight, float eps,
                                                        __nv_bfloat16 *__restrict__ out) {
    __shared__ float2 red[32];
    const int64_t row = blockIdx.x;
    const int t = threadIdx.x;
    const bool active = t * VEC < d;
    float v[VEC];
    float s = 0.f;
    if (active) {
        unpack8(*reinterpret_cast<const uint4 *>(x + row * x_ld + t * VEC), v);
#pragma unroll
        for (int i = 0; i < VEC; ++i) s = __fadd_rn(s, __fmul_rn(v[i], v[i]));
    }
    const float ss = block_sum2(s, 0.f, red).x;
    if (!active) return;
    const float r = rsqrtf(__fadd_rn(__fdiv_rn(ss, (float)d), eps));
    float w[VEC], o[VEC];
    unpack8(*reinterpret_cast<const uint4 *>(weight + t * VEC), w);
#pragma unroll
    for (int i = 0; i < VEC; ++i) o[i] = __fmul_rn(round_bf16(__fmul_rn(v[i], r)), w[i]);
    *reinterpret_cast<uint4 *>(out + row * d + t * VEC) = pack8(o);
}

// The same LayerNorm + modulation / affine with one warp per row, for rows of d = 256 * NV
// (lane l holds vectors l, l + 32, ...; butterfly reductions, no shared memory or block barrier).
template <int NV>
__global__ void __launch_bounds__(256) adaln_warp_kernel(const __nv_bfloat16 *__restrict__ x, int n, int frame_tokens,
                                                         const float *__restrict__ shift,
                                                         const float *__restrict__ scale, int64_t mod_ld,
                                                         const __nv_bfloat16 *__restrict__ weight,
                                                         const __nv_bfloat16 *__restrict__ bias, float eps,
                                                         __nv_bfloat16 *__restrict__ out) {
    constexpr int d = 256 * NV;
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= n) return;
    float v[NV][VEC];
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        unpack8(*reinterpret_cast<const uint4 *>(x + row * d + (k * 32 + lane) * VEC), v[k]);
#pragma unroll
        for (int i = 0; i < VEC; ++i) s = __fadd_rn(s, v[k][i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = __fdiv_rn(s, (float)d);
    float s2 = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k)
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
            const float c = __fsub_rn(v[k][i], mean);
            s2 = __fadd_rn(s2, __fmul_rn(c, c));
        }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    const float rstd = rsqrtf(__fadd_rn(__fdiv_rn(s2, (float)d), eps));
    const int64_t f = weight ? 0 : row / frame_tokens;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const int c0 = (k * 32 + lane) * VEC;
        float o[VEC];
        if (weight) {
            float w[VEC], b[VEC];
            unpack8(*reinterpret_cast<const uint4 *>(weight + c0), w);
            unpack8(*reinterpret_cast<const uint4 *>(bias + c0), b);
#pragma unroll
            for (int i = 0; i < VEC; ++i)
                o[i] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[k][i], mean), rstd), w[i]), b[i]);
        } else {
            const float4 *sh = reinterpret_cast<const float4 *>(shift + f * mod_ld + c0);
            const float4 *sc = reinterpret_cast<const float4 *>(scale + f * mod_ld + c0);
            const float4 a0 = sh[0], a1 = sh[1], g0 = sc[0], g1 = sc[1];
            const float shv[VEC] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float scv[VEC] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
            for (int i = 0; i < VEC; ++i) {
                const float y = round_bf16(__fmul_rn(__fsub_rn(v[k][i], mean), rstd));
                o[i] = __fadd_rn(__fmul_rn(y, __fadd_rn(1.f, scv[i])), shv[i]);
            }
        }
        *reinterpret_cast<uint4 *>(out + row * d + c0) = pack8(o);
    }
}

template <int NV>
static void launch_adaln_warp(const __nv_bfloat16 *x, int n, int frame_tokens, const float *shift, const float *scale,
                              int64_t mod_ld, const __nv_bfloat16 *w, const __nv_bfloat16 *b, float eps,
                              __nv_bfloat16 *out, cudaStream_t st) {
    adaln_warp_kernel<NV><<<(n + 7) / 8, 256, 0, st>>>(x, n, frame_tokens, shift, scale, mod_ld, w, b, eps, out);
}

static bool misaligned(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) != 0; }

static int row_threads(int d) { return ((d / VEC + 31) / 32) * 32; }

}  // namespace dit
}  // namespace ss

extern "C" int ss_qkv_norm_rope(const void *qkv, int64_t qkv_ld, int n, int H, const void *norm_q, const void *norm_k,
                                float eps, const float *cos_t, const float *sin_t, void *q_out, int64_t q_ld,
                                void *k_out, void *v_out, int64_t kv_ld, void *stream) {
    using namespace ss;
    if (!qkv || !norm_q || !norm_k || !cos_t || !sin_t || !q_out || !k_out || !v_out) return SS_ERR_POINTER;
    const int d = H * dit::HD;
    if (n < 0 || H <= 0 || d / dit::VEC > 1024 || qkv_ld < 3 * (int64_t)d || q_ld < d || kv_ld < d ||
        (qkv_ld % dit::VEC) || (q_ld % dit::VEC) || (kv_ld % dit::VEC))
        return SS_ERR_SHAPE;
    if (dit::misaligned(qkv) || dit::misaligned(norm_q) || dit::misaligned(norm_k) || dit::misaligned(q_out) ||
        dit::misaligned(k_out) || dit::misaligned(v_out) || dit::misaligned(cos_t) || dit::misaligned(sin_t))
        return SS_ERR_POINTER;
    if (n == 0) return 0;
    dit::qkv_norm_rope_kernel<<<n, dit::row_threads(d), 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16 *>(qkv), qkv_ld, d, static_cast<const __nv_bfloat16 *>(norm_q),
        static_cast<const __nv_bfloat16 *>(norm_k), eps, cos_t, sin_t, static_cast<__nv_bfloat16 *>(q_out), q_ld,
        static_cast<__nv_bfloat16 *>(k_out), static_cast<__nv_bfloat16 *>(v_out), kv_ld, dit::RingRows(), 0, d);
    return (int)cudaGetLastError();
}

extern "C" int ss_qkv_norm_rope_ring(const void *qkv, int64_t qkv_ld, int n, int H, const void *norm_q,
                                     const void *norm_k, float eps, const float *cos_t, const float *sin_t,
                                     void *q_out, int64_t q_ld, void *k_cache, void *v_cache, int64_t kv_ld,
                                     int ring_sink, int ring_cap, int64_t t0, const int *ring_head_dev, int evicted,
                                     void *stream) {
    using namespace ss;
    if (!qkv || !norm_q || !norm_k || !cos_t || !sin_t || !q_out || !k_cache || !v_cache || !ring_head_dev)
        return SS_ERR_POINTER;
    const int d = H * dit::HD;
    if (n < 0 || H <= 0 || d / dit::VEC > 1024 || qkv_ld < 3 * (int64_t)d || q_ld < d || kv_ld < d ||
        (qkv_ld % dit::VEC) || (q_ld % dit::VEC) || (kv_ld % dit::VEC))
        return SS_ERR_SHAPE;
    if (ring_sink < 0 || ring_cap < 64 || t0 < 0 || evicted < 0 || t0 + n > (int64_t)ring_sink + ring_cap)
        return SS_ERR_SHAPE;
    if (dit::misaligned(qkv) || dit::misaligned(norm_q) || dit::misaligned(norm_k) || dit::misaligned(q_out) ||
        dit::misaligned(k_cache) || dit::misaligned(v_cache) || dit::misaligned(cos_t) || dit::misaligned(sin_t))
        return SS_ERR_POINTER;
    if (n == 0) return 0;
    dit::RingRows rr;
    rr.S = ring_sink;
    rr.C = ring_cap;
    rr.t0 = t0;
    rr.head_dev = ring_head_dev;
    rr.evicted = evicted;
    dit::qkv_norm_rope_kernel<<<n, dit::row_threads(d), 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16 *>(qkv), qkv_ld, d, static_cast<const __nv_bfloat16 *>(norm_q),
        static_cast<const __nv_bfloat16 *>(norm_k), eps, cos_t, sin_t, static_cast<__nv_bfloat16 *>(q_out), q_ld,
        static_cast<__nv_bfloat16 *>(k_cache), static_cast<__nv_bfloat16 *>(v_cache), kv_ld, rr, 0, d);
    return (int)cudaGetLastError();
}

extern "C" int ss_qkv_norm_rope_heads(const void *qkv, int64_t qkv_ld, int n, int H, const void *norm_q,
                                      const void *norm_k, float eps, const float *cos_t, const float *sin_t, int h0,
                                      int nh, void *q_out, int64_t q_ld, void *k_out, void *v_out, int64_t kv_ld,
                                      int ring_sink, int ring_cap, int64_t t0, const int *ring_head_dev, int evicted,
                                      void *stream) {
    using namespace ss;
    if (!qkv || !norm_q || !norm_k || !cos_t || !sin_t || !q_out || !k_out || !v_out) return SS_ERR_POINTER;
    const int d = H * dit::HD;
    if (n < 0 || H <= 0 || d / dit::VEC > 1024 || h0 < 0 || nh <= 0 || h0 + nh > H || qkv_ld < 3 * (int64_t)d ||
        q_ld < (int64_t)nh * dit::HD || kv_ld < (int64_t)nh * dit::HD || (qkv_ld % dit::VEC) || (q_ld % dit::VEC) ||
        (kv_ld % dit::VEC))
        return SS_ERR_SHAPE;
    dit::RingRows rr;
    if (ring_cap > 0) {
        if (!ring_head_dev) return SS_ERR_POINTER;
        if (ring_sink < 0 || ring_cap < 64 || t0 < 0 || evicted < 0 || t0 + n > (int64_t)ring_sink + ring_cap)
            return SS_ERR_SHAPE;
        rr.S = ring_sink;
        rr.C = ring_cap;
        rr.t0 = t0;
        rr.head_dev = ring_head_dev;
        rr.evicted = evicted;
    }
    if (dit::misaligned(qkv) || dit::misaligned(norm_q) || dit::misaligned(norm_k) || dit::misaligned(q_out) ||
        dit::misaligned(k_out) || dit::misaligned(v_out) || dit::misaligned(cos_t) || dit::misaligned(sin_t))
        return SS_ERR_POINTER;
    if (n == 0) return 0;
    dit::qkv_norm_rope_kernel<<<n, dit::row_threads(d), 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16 *>(qkv), qkv_ld, d, static_cast<const __nv_bfloat16 *>(norm_q),
        static_cast<const __nv_bfloat16 *>(norm_k), eps, cos_t, sin_t, static_cast<__nv_bfloat16 *>(q_out), q_ld,
        static_cast<__nv_bfloat16 *>(k_out), static_cast<__nv_bfloat16 *>(v_out), kv_ld, rr, h0 * dit::HD,
        (h0 + nh) * dit::HD);
    return (int)cudaGetLastError();
}

extern "C" int ss_adaln(const void *x, int n, int d, int frame_tokens, const float *shift, const float *scale,
                        int64_t mod_ld, const void *weight, const void *bias, float eps, void *out, void *stream) {
    using namespace ss;
    if (!x || !out) return SS_ERR_POINTER;
    const bool affine = weight || bias, modulate = shift || scale;
    if (affine == modulate) return SS_ERR_SHAPE;   // exactly one of the two forms
    if (affine && (!weight || !bias)) return SS_ERR_POINTER;
    if (modulate && (!shift || !scale)) return SS_ERR_POINTER;
    if (n < 0 || d <= 0 || (d % dit::VEC) || d / dit::VEC > 1024 || (modulate && (frame_tokens <= 0 || mod_ld < d ||
                                                                                  (mod_ld % 4))))
        return SS_ERR_SHAPE;
    if (dit::misaligned(x) || dit::misaligned(out) || (affine && (dit::misaligned(weight) || dit::misaligned(bias))) ||
        (modulate && (dit::misaligned(shift) || dit::misaligned(scale))))
        return SS_ERR_POINTER;
    if (n == 0) return 0;
    {
        const auto *xb = static_cast<const __nv_bfloat16 *>(x);
        const auto *wb = static_cast<const __nv_bfloat16 *>(weight);
        const auto *bb = static_cast<const __nv_bfloat16 *>(bias);
        auto *ob = static_cast<__nv_bfloat16 *>(out);
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        bool warp_rows = true;   // rows of 256 * NV: one warp per row
        switch (d) {
            case 256: dit::launch_adaln_warp<1>(xb, n, frame_tokens, shift, scale, mod_ld, wb, bb, eps, ob, st); break;
            case 512: dit::launch_adaln_warp<2>(xb, n, frame_tokens, shift, scale, mod_ld, wb, bb, eps, ob, st); break;
            case 1024: dit::launch_adaln_warp<4>(xb, n, frame_tokens, shift, scale, mod_ld, wb, bb, eps, ob, st); break;
            case 1536: dit::launch_adaln_warp<6>(xb, n, frame_tokens, shift, scale, mod_ld, wb, bb, eps, ob, st); break;
            case 2048: dit::launch_adaln_warp<8>(xb, n, frame_tokens, shift, scale, mod_ld, wb, bb, eps, ob, st); break;
            default: warp_rows = false;
        }
        if (warp_rows) return (int)cudaGetLastError();
    }
    dit::adaln_kernel<<<n, dit::row_threads(d), 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16 *>(x), d, frame_tokens, shift, scale, mod_ld,
        static_cast<const __nv_bfloat16 *>(weight), static_cast<const __nv_bfloat16 *>(bias), eps,
        static_cast<__nv_bfloat16 *>(out));
    return (int)cudaGetLastError();
}

extern "C" int ss_rms_norm(const void *x, int64_t x_ld, int n, int d, const void *weight, float eps, void *out,
                           void *stream) {
    using namespace ss;
    if (!x || !weight || !out) return SS_ERR_POINTER;
    if (n < 0 || d <= 0 || (d % dit::VEC) || d / dit::VEC > 1024 || x_ld < d || (x_ld % dit::VEC)) return SS_ERR_SHAPE;
    if (dit::misaligned(x) || dit::misaligned(weight) || dit::misaligned(out)) return SS_ERR_POINTER;
    if (n == 0) return 0;
    dit::rms_norm_kernel<<<n, dit::row_threads(d), 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16 *>(x), x_ld, d, static_cast<const __nv_bfloat16 *>(weight), eps,
        static_cast<__nv_bfloat16 *>(out));
    return (int)cudaGetLastError();
}

extern "C" int ss_gate_residual(void *x, const void *y, int64_t y_ld, int n, int d, int frame_tokens,
                                const float *gate, int64_t gate_ld, void *stream) {
    using namespace ss;
    if (!x || !y) return SS_ERR_POINTER;
    if (n < 0 || d <= 0 || (d % dit::VEC) || y_ld < d || (y_ld % dit::VEC) ||
        (gate && (frame_tokens <= 0 || gate_ld < d || (gate_ld % 4))))
        return SS_ERR_SHAPE;
    if (dit::misaligned(x) || dit::misaligned(y) || (gate && dit::misaligned(gate))) return SS_ERR_POINTER;
    if (n == 0) return 0;
    int sms = 148, dev;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t total = (int64_t)n * (d / dit::VEC);
    const unsigned blocks = (unsigned)std::min<int64_t>((total + 255) / 256, (int64_t)sms * 8);
    dit::gate_residual_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<__nv_bfloat16 *>(x), static_cast<const __nv_bfloat16 *>(y), y_ld, n, d, frame_tokens, gate,
        gate_ld);
    return (int)cudaGetLastError();
}
