// cache.cu -- KV-cache append / evict for the streaming window.
//
// Semantics of the reference's CausalWanSelfAttention.forward (wan/modules/causal_model.py:
// 216-246): when a local window is in use and the new chunk would overflow the cache, the
// oldest non-sink tokens are evicted by shifting the rest of the window left onto the sink
// boundary, then the chunk is written at [local_end - n, local_end). The reference does the
// shift with a full `.clone()` of the rolled range; here it is a sequence of in-place 16-byte
// vector copies, each moving at most `evicted` rows, so no copy reads rows an earlier copy
// of the same call has already overwritten (stream order separates the copies). The chunk
// write is one 16-byte-vector copy kernel (the reference's sm_80 commit_tile,
// local_experiments/video_runtime_v1/csrc/fixed15_attention.cu:417-458, also writes with uint4).
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace ss {
namespace cache {

constexpr int D = 128;

// Copy n rows of `row_vec` uint4 each, for two tensors at once (K and V). A thread takes
// CP_UNROLL vectors of each tensor (grid-stride apart) and issues all of its loads before its
// stores, so 2 x CP_UNROLL 16-byte loads per thread are in flight; the sources are read once
// (evict-first), the destinations stay in L2 for the attention that reads them next. Source and
// destination ranges of one launch never overlap (the roll moves at most `evicted` rows a launch).
constexpr int CP_UNROLL = 4;

// Flat form: both sides are contiguous rows (stride == row_vec) and the copy has fewer than 2^31
// vectors, so vector i sits at offset i on both sides and 32-bit offsets from one base suffice.
__global__ void __launch_bounds__(256) copy_flat_kernel(const uint4 *__restrict__ src_k, const uint4 *__restrict__ src_v,
                                                        uint4 *__restrict__ dst_k, uint4 *__restrict__ dst_v,
                                                        int total) {
    const int stride = gridDim.x * blockDim.x;
    for (int i0 = blockIdx.x * blockDim.x + threadIdx.x; i0 < total; i0 += stride * CP_UNROLL) {
        uint4 a[CP_UNROLL], b[CP_UNROLL];
#pragma unroll
        for (int u = 0; u < CP_UNROLL; ++u) {
            const int i = i0 + u * stride;
            if (i < total) {
                a[u] = __ldcs(src_k + i);
                b[u] = __ldcs(src_v + i);
            }
        }
#pragma unroll
        for (int u = 0; u < CP_UNROLL; ++u) {
            const int i = i0 + u * stride;
            if (i < total) {
                dst_k[i] = a[u];
                dst_v[i] = b[u];
            }
        }
    }
}

// General form: rows of row_vec vectors at independent strides on the two sides.
__global__ void __launch_bounds__(256) copy_rows_kernel(const uint4 *__restrict__ src_k, const uint4 *__restrict__ src_v,
                                                        int64_t src_stride_vec, uint4 *__restrict__ dst_k,
                                                        uint4 *__restrict__ dst_v, int64_t dst_stride_vec,
                                                        int64_t n, int row_vec) {
    const int64_t total = n * row_vec;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < total; i0 += stride * CP_UNROLL) {
        uint4 a[CP_UNROLL], b[CP_UNROLL];
#pragma unroll
        for (int u = 0; u < CP_UNROLL; ++u) {
            const int64_t i = i0 + u * stride;
            if (i < total) {
                const int64_t s = (i / row_vec) * src_stride_vec + i % row_vec;
                a[u] = __ldcs(src_k + s);
                b[u] = __ldcs(src_v + s);
            }
        }
#pragma unroll
        for (int u = 0; u < CP_UNROLL; ++u) {
            const int64_t i = i0 + u * stride;
            if (i < total) {
                const int64_t d = (i / row_vec) * dst_stride_vec + i % row_vec;
                dst_k[d] = a[u];
                dst_v[d] = b[u];
            }
        }
    }
}

// Launch geometry of the copy kernels on one device: SM count and resident CTAs per SM of each
// form, queried once per device (a rolling append makes up to seven launches).
struct CopyGeometry {
    int sms = 0, per_sm_flat = 1, per_sm_rows = 1;
};
static CopyGeometry g_copy_geo[SS_MAX_DEVICES];
static std::mutex g_copy_mutex;

static int copy_geometry(CopyGeometry *out) {
    int dev;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= SS_MAX_DEVICES) return SS_ERR_DEVICE;
    std::lock_guard<std::mutex> lock(g_copy_mutex);
    CopyGeometry &g = g_copy_geo[dev];
    if (g.sms == 0) {
        int sms = 0, a = 0, b = 0;
        if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return (int)e;
        if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&a, copy_flat_kernel, 256, 0)) != cudaSuccess) return (int)e;
        if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, copy_rows_kernel, 256, 0)) != cudaSuccess) return (int)e;
        g.per_sm_flat = std::min(std::max(a, 1), 8);
        g.per_sm_rows = std::min(std::max(b, 1), 8);
        g.sms = std::max(sms, 1);
    }
    *out = g;
    return 0;
}

static int launch_copy(const void *sk, const void *sv, int64_t src_stride, void *dk, void *dv, int64_t dst_stride,
                       int64_t n, int H, cudaStream_t st) {
    if (n <= 0) return 0;
    const int row_vec = H * D / 8;  // uint4 = 8 bf16
    const int64_t total = n * row_vec;
    CopyGeometry geo;
    int rc = copy_geometry(&geo);
    if (rc) return rc;
    const int sms = geo.sms;
    const int64_t want = (total + 256 * CP_UNROLL - 1) / (256 * CP_UNROLL);
    // at most one wave of resident CTAs; the grid-stride loop covers the rest
    const bool flat = src_stride / 8 == row_vec && dst_stride / 8 == row_vec &&
                      total < ((int64_t)1 << 31) - (int64_t)sms * 8 * 256 * CP_UNROLL;
    const int per_sm = flat ? geo.per_sm_flat : geo.per_sm_rows;
    const unsigned blocks = (unsigned)std::min<int64_t>(want, (int64_t)sms * per_sm);
    if (flat)
        copy_flat_kernel<<<blocks, 256, 0, st>>>((const uint4 *)sk, (const uint4 *)sv, (uint4 *)dk, (uint4 *)dv,
                                                 (int)total);
    else
        copy_rows_kernel<<<blocks, 256, 0, st>>>((const uint4 *)sk, (const uint4 *)sv, src_stride / 8, (uint4 *)dk,
                                                (uint4 *)dv, dst_stride / 8, n, row_vec);
    return (int)cudaGetLastError();
}

// Rotation of the first `pairs` complex pairs of every (row, head) by phase[p] = (cos, sin), in
// float64 with separately rounded products and sums, then double -> float -> bf16 (round to
// nearest even each time), as the reference's float64 complex multiply and `.to(bfloat16)` do.
__global__ void __launch_bounds__(256) rope_shift_kernel(const uint32_t *__restrict__ src, int64_t src_ld2,
                                                         uint32_t *__restrict__ dst, int64_t dst_ld2, int64_t n, int H,
                                                         int pairs, const double *__restrict__ phase) {
    const int64_t total = n * H * pairs;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / ((int64_t)H * pairs);
        const int rem = (int)(i % ((int64_t)H * pairs));
        const int h = rem / pairs, p = rem % pairs;
        const uint32_t w = src[r * src_ld2 + h * (D / 2) + p];
        const double x = (double)__uint_as_float(w << 16), y = (double)__uint_as_float(w & 0xffff0000u);
        const double c = phase[2 * p], sn = phase[2 * p + 1];
        const double re = __dsub_rn(__dmul_rn(x, c), __dmul_rn(y, sn));
        const double im = __dadd_rn(__dmul_rn(x, sn), __dmul_rn(y, c));
        const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(__double2float_rn(re)));
        const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(__double2float_rn(im)));
        dst[r * dst_ld2 + h * (D / 2) + p] = lo | (hi << 16);
    }
}

// Write n rows (K and V, source rows `src_stride` elements apart) to ring rows [pos0, pos0 + n) mod C
// of a ring cache (ring row p at physical row S + p), and the rows that land on ring rows
// [0, 64) once more at S + C + p: at most three contiguous copies plus the mirrored part.
static int ring_write(const __nv_bfloat16 *sk, const __nv_bfloat16 *sv, int64_t src_stride, __nv_bfloat16 *kc,
                      __nv_bfloat16 *vc, int H, int S, int C, int64_t pos0, int64_t n, cudaStream_t st) {
    const int64_t row = (int64_t)H * D;
    int64_t done = 0;
    while (done < n) {
        const int64_t pos = (pos0 + done) % C;
        const int64_t m = std::min<int64_t>(n - done, C - pos);   // up to the ring's end
        int rc = launch_copy(sk + done * src_stride, sv + done * src_stride, src_stride, kc + (S + pos) * row,
                             vc + (S + pos) * row, row, m, H, st);
        if (rc) return rc;
        if (pos < 64) {   // the mirror of ring rows [0, 64)
            const int64_t mm = std::min<int64_t>(m, 64 - pos);
            rc = launch_copy(sk + done * src_stride, sv + done * src_stride, src_stride, kc + (S + C + pos) * row,
                             vc + (S + C + pos) * row, row, mm, H, st);
            if (rc) return rc;
        }
        done += m;
    }
    return 0;
}

// The sink's last S mod 64 rows repeated just before the ring's head (ring rows head - a .. head - 1).
static int ring_refresh_tail(__nv_bfloat16 *kc, __nv_bfloat16 *vc, int H, int S, int C, int head, cudaStream_t st) {
    const int a = S % 64;
    if (a == 0) return 0;
    const int64_t row = (int64_t)H * D;
    return ring_write(kc + (int64_t)(S - a) * row, vc + (int64_t)(S - a) * row, row, kc, vc, H, S, C,
                      ((int64_t)head - a + C) % C, a, st);
}

// The same writes with the ring's head in device memory (so that a captured CUDA graph places rows
// by the head at replay time): n rows (K and V, source rows src_stride_vec uint4 apart) go to ring
// rows (off + i + head') mod C, and once more to S + C + that row when it is below 64, where
// head' = (*head_dev + evicted) mod C is the head after this call's roll (evicted = 0 without one).
__global__ void __launch_bounds__(256) ring_rows_kernel(const uint4 *__restrict__ sk, const uint4 *__restrict__ sv,
                                                        int64_t src_stride_vec, uint4 *__restrict__ dk,
                                                        uint4 *__restrict__ dv, int S, int C, int64_t off, int n,
                                                        int row_vec, const int *head_dev, int evicted) {
    const int head = (int)(((int64_t)*head_dev + evicted) % C);
    const int64_t total = (int64_t)n * row_vec;
    for (int64_t x = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; x < total; x += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = x / row_vec, c = x % row_vec;
        const int64_t pos = ((off + i + head) % C + C) % C;
        const uint4 a = __ldcs(sk + i * src_stride_vec + c), b = __ldcs(sv + i * src_stride_vec + c);
        dk[(S + pos) * row_vec + c] = a;
        dv[(S + pos) * row_vec + c] = b;
        if (pos < 64) {
            dk[(S + C + pos) * row_vec + c] = a;
            dv[(S + C + pos) * row_vec + c] = b;
        }
    }
}

__global__ void ring_head_advance_kernel(int *head_dev, int evicted, int C) {
    *head_dev = (int)(((int64_t)*head_dev + evicted) % C);
}

static int ring_rows_launch(const __nv_bfloat16 *sk, const __nv_bfloat16 *sv, int64_t src_stride, __nv_bfloat16 *kc,
                            __nv_bfloat16 *vc, int H, int S, int C, int64_t off, int n, const int *head_dev,
                            int evicted, cudaStream_t st) {
    if (n <= 0) return 0;
    const int row_vec = H * D / 8;
    CopyGeometry geo;
    int rc = copy_geometry(&geo);
    if (rc) return rc;
    const int64_t total = (int64_t)n * row_vec;
    const unsigned blocks = (unsigned)std::min<int64_t>((total + 255) / 256, (int64_t)geo.sms * 8);
    ring_rows_kernel<<<blocks, 256, 0, st>>>((const uint4 *)sk, (const uint4 *)sv, src_stride / 8, (uint4 *)kc,
                                            (uint4 *)vc, S, C, off, n, row_vec, head_dev, evicted);
    return (int)cudaGetLastError();
}

}  // namespace cache
}  // namespace ss

extern "C" int ss_cache_rope_shift(const void *src, int64_t src_ld, void *dst, int64_t dst_ld, int n, int H, int pairs,
                                   const double *phase, void *stream) {
    using namespace ss;
    if (!src || !dst || !phase) return SS_ERR_POINTER;
    if (n < 0 || H <= 0 || pairs < 0 || pairs > cache::D / 2 || src_ld < (int64_t)H * cache::D ||
        dst_ld < (int64_t)H * cache::D || (src_ld % 2) || (dst_ld % 2))
        return SS_ERR_SHAPE;
    if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 3u ||
        (reinterpret_cast<uintptr_t>(phase) & 7u))
        return SS_ERR_POINTER;
    // rows the rotation leaves alone are still copied when dst is another buffer
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (src != dst && n > 0) {
        cudaError_t e = cudaMemcpy2DAsync(dst, (size_t)dst_ld * 2, src, (size_t)src_ld * 2, (size_t)H * cache::D * 2,
                                          (size_t)n, cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) return (int)e;
    }
    const int64_t total = (int64_t)n * H * pairs;
    if (total == 0) return 0;
    int sms = 148, dev;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const unsigned blocks = (unsigned)std::min<int64_t>((total + 255) / 256, (int64_t)sms * 8);
    cache::rope_shift_kernel<<<blocks, 256, 0, st>>>(static_cast<const uint32_t *>(src), src_ld / 2,
                                                     static_cast<uint32_t *>(dst), dst_ld / 2, n, H, pairs, phase);
    return (int)cudaGetLastError();
}

extern "C" int ss_cache_append(void *k_cache, void *v_cache, int cap, int H, const void *k_new, const void *v_new,
                               int64_t new_stride, int n_new, int local_attn, int64_t global_end, int64_t local_end,
                               int64_t current_start, int sink_tokens, int64_t *out_local_end, void *stream) {
    using namespace ss;
    if (!k_cache || !v_cache || !k_new || !v_new || !out_local_end) return SS_ERR_POINTER;
    if (cap <= 0 || H <= 0 || n_new <= 0 || n_new > cap || sink_tokens < 0 || global_end < 0 || local_end < 0 ||
        local_end > cap || current_start < 0)
        return SS_ERR_SHAPE;
    if (new_stride % 8 != 0 || new_stride < (int64_t)H * cache::D) return SS_ERR_SHAPE;
    if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) |
         reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new)) & 15u)
        return SS_ERR_POINTER;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t row = (int64_t)H * cache::D;  // elements per cache row
    const int64_t current_end = current_start + n_new;
    int64_t new_local_end;
    if (local_attn && current_end > global_end && n_new + local_end > cap) {
        const int64_t evicted = n_new + local_end - cap;
        const int64_t rolled = local_end - evicted - sink_tokens;
        if (rolled < 0) return SS_ERR_SHAPE;  // cache too small for the sink and the chunk
        __nv_bfloat16 *kc = static_cast<__nv_bfloat16 *>(k_cache);
        __nv_bfloat16 *vc = static_cast<__nv_bfloat16 *>(v_cache);
        for (int64_t done = 0; done < rolled; done += evicted) {
            const int64_t n = std::min<int64_t>(evicted, rolled - done);
            const int64_t src = sink_tokens + evicted + done, dst = sink_tokens + done;
            int rc = cache::launch_copy(kc + src * row, vc + src * row, row, kc + dst * row, vc + dst * row, row, n, H, st);
            if (rc) return rc;
        }
        new_local_end = local_end + current_end - global_end - evicted;
    } else {
        new_local_end = local_end + current_end - global_end;
    }
    const int64_t start = new_local_end - n_new;
    if (start < 0 || new_local_end > cap) return SS_ERR_SHAPE;
    int rc = cache::launch_copy(k_new, v_new, new_stride, static_cast<__nv_bfloat16 *>(k_cache) + start * row,
                                static_cast<__nv_bfloat16 *>(v_cache) + start * row, row, n_new, H, st);
    if (rc) return rc;
    *out_local_end = new_local_end;
    return 0;
}

extern "C" int ss_cache_append_ring(void *k_cache, void *v_cache, int cap, int H, const void *k_new,
                                    const void *v_new, int64_t new_stride, int n_new, int local_attn,
                                    int64_t global_end, int64_t local_end, int64_t current_start, int sink_tokens,
                                    int ring_cap, int ring_head, int *ring_head_dev, int64_t *out_local_end,
                                    int *out_ring_head, void *stream) {
    using namespace ss;
    if (!k_cache || !v_cache || !k_new || !v_new || !out_local_end || !out_ring_head) return SS_ERR_POINTER;
    if (cap <= 0 || H <= 0 || n_new <= 0 || n_new > cap || sink_tokens < 0 || sink_tokens > cap || global_end < 0 ||
        local_end < 0 || local_end > cap || current_start < 0)
        return SS_ERR_SHAPE;
    const int S = sink_tokens, C = ring_cap;
    if (C < 64 || (int64_t)C < (int64_t)cap - S + S % 64 || ring_head < 0 || ring_head >= C) return SS_ERR_SHAPE;
    if (new_stride % 8 != 0 || new_stride < (int64_t)H * cache::D) return SS_ERR_SHAPE;
    if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) |
         reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new)) & 15u)
        return SS_ERR_POINTER;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t row = (int64_t)H * cache::D;
    const int64_t current_end = current_start + n_new;
    int64_t new_local_end;
    int head = ring_head;
    int evicted_rows = 0;
    if (local_attn && current_end > global_end && n_new + local_end > cap) {
        // the roll: the window's rows after the sink move down by `evicted`, which in the ring is
        // only its head moving on by that many rows
        const int64_t evicted = n_new + local_end - cap;
        if (local_end - evicted - S < 0) return SS_ERR_SHAPE;   // cache too small for the sink and the chunk
        head = (int)(((int64_t)head + evicted) % C);
        evicted_rows = (int)evicted;
        new_local_end = local_end + current_end - global_end - evicted;
    } else {
        new_local_end = local_end + current_end - global_end;
    }
    const int64_t start = new_local_end - n_new;
    if (start < 0 || new_local_end > cap) return SS_ERR_SHAPE;
    __nv_bfloat16 *kc = static_cast<__nv_bfloat16 *>(k_cache), *vc = static_cast<__nv_bfloat16 *>(v_cache);
    const __nv_bfloat16 *kn = static_cast<const __nv_bfloat16 *>(k_new), *vn = static_cast<const __nv_bfloat16 *>(v_new);
    // chunk rows in the sink: their own rows; the rest: the ring from the window row's ring position
    const int64_t ns = std::max<int64_t>(0, std::min<int64_t>(S, new_local_end) - start);
    int rc = 0;
    if (ns > 0) rc = cache::launch_copy(kn, vn, new_stride, kc + start * row, vc + start * row, row, ns, H, st);
    if (rc) return rc;
    const int64_t t0 = start + ns;   // first window row of the chunk at or after S
    if (ring_head_dev) {
        // the head in device memory: rows placed by kernels that read it, then the head moved on
        if (n_new > ns) {
            rc = cache::ring_rows_launch(kn + ns * new_stride, vn + ns * new_stride, new_stride, kc, vc, H, S, C,
                                         t0 - S, (int)(n_new - ns), ring_head_dev, evicted_rows, st);
            if (rc) return rc;
        }
        const int a = S % 64;   // the sink's copy before the new head, after the chunk (it may hold sink rows)
        rc = cache::ring_rows_launch(kc + (int64_t)(S - a) * row, vc + (int64_t)(S - a) * row, row, kc, vc, H, S, C,
                                     -a, a, ring_head_dev, evicted_rows, st);
        if (rc) return rc;
        if (evicted_rows) {
            cache::ring_head_advance_kernel<<<1, 1, 0, st>>>(ring_head_dev, evicted_rows, C);
            if ((rc = (int)cudaGetLastError())) return rc;
        }
    } else {
        if (n_new > ns) {
            rc = cache::ring_write(kn + ns * new_stride, vn + ns * new_stride, new_stride, kc, vc, H, S, C,
                                   (t0 - S + head) % C, n_new - ns, st);
            if (rc) return rc;
        }
        rc = cache::ring_refresh_tail(kc, vc, H, S, C, head, st);   // after the chunk: it may hold the sink's rows
        if (rc) return rc;
    }
    *out_local_end = new_local_end;
    *out_ring_head = head;
    return 0;
}

extern "C" int ss_cache_ring_refresh(void *k_cache, void *v_cache, int H, int sink_tokens, int ring_cap, int ring_head,
                                     const int *ring_head_dev, void *stream) {
    using namespace ss;
    if (!k_cache || !v_cache) return SS_ERR_POINTER;
    if (H <= 0 || sink_tokens < 0 || ring_cap < 64 || ring_head < 0 || ring_head >= ring_cap) return SS_ERR_SHAPE;
    if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15u) return SS_ERR_POINTER;
    __nv_bfloat16 *kc = static_cast<__nv_bfloat16 *>(k_cache), *vc = static_cast<__nv_bfloat16 *>(v_cache);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (ring_head_dev) {
        const int a = sink_tokens % 64;
        const int64_t row = (int64_t)H * cache::D;
        return cache::ring_rows_launch(kc + (int64_t)(sink_tokens - a) * row, vc + (int64_t)(sink_tokens - a) * row,
                                       row, kc, vc, H, sink_tokens, ring_cap, -a, a, ring_head_dev, 0, st);
    }
    return cache::ring_refresh_tail(kc, vc, H, sink_tokens, ring_cap, ring_head, st);
}

extern "C" int ss_cache_ring_commit(void *k_cache, void *v_cache, int H, int sink_tokens, int ring_cap,
                                    int *ring_head_dev, int evicted, int refresh, void *stream) {
    using namespace ss;
    if (!k_cache || !v_cache || !ring_head_dev) return SS_ERR_POINTER;
    if (H <= 0 || sink_tokens < 0 || ring_cap < 64 || evicted < 0) return SS_ERR_SHAPE;
    if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15u) return SS_ERR_POINTER;
    __nv_bfloat16 *kc = static_cast<__nv_bfloat16 *>(k_cache), *vc = static_cast<__nv_bfloat16 *>(v_cache);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int rc = 0;
    if (refresh || evicted) {   // the sink's copy before the head after this write
        const int a = sink_tokens % 64;
        const int64_t row = (int64_t)H * cache::D;
        rc = cache::ring_rows_launch(kc + (int64_t)(sink_tokens - a) * row, vc + (int64_t)(sink_tokens - a) * row, row,
                                     kc, vc, H, sink_tokens, ring_cap, -a, a, ring_head_dev, evicted, st);
        if (rc) return rc;
    }
    if (evicted) {
        cache::ring_head_advance_kernel<<<1, 1, 0, st>>>(ring_head_dev, evicted, ring_cap);
        rc = (int)cudaGetLastError();
    }
    return rc;
}
