// peer.cu -- the cross-GPU step of KV-block sharding, over peer memory (NVLink / NVSwitch).
//
// With the KV window split block-cyclically over the GPUs of a node, every rank attends over the
// blocks it owns and holds a partial result (o_r, lse_r) for every query row. The partials are
// combined by log-sum-exp, the arithmetic of `merge` (local_experiments/video_runtime_v1/
// attention.py:40-45) and of the split merge `_merge_restore` (migration/unified_router/opt21/
// attention.py:7-15). Here the exchange and the merge are one kernel: each rank reads the other
// ranks' partials straight from their memory (peer loads through buffers the ranks opened to
// each other with CUDA IPC) and writes the merged rows, so the partials cross NVLink once and
// there is no separate collective or weighting pass.
//
//   ss_ipc_handle / ss_ipc_open / ss_ipc_close  export a caller-allocated device buffer to the
//       other ranks of the node and map theirs (no allocation by the library)
//   ss_peer_barrier      every rank posts an epoch into each peer's flag array, then waits
//       (bounded) until every peer has posted it into its own: after it, the partials the peers
//       wrote before their barrier are visible
//   ss_lse_merge_peers   merged rows [row0, row1) from P partials given as P peer pointers
//   ss_lse_merge_gather  the same merge, each merged row stored into several ranks' outputs: after
//       ss_attention_kv_parts left every rank's partial rows with the rank that owns them (the
//       reduce-scatter, inside the attention's epilogue), each rank merges its own rows from its
//       own memory and stores them into every rank's output (the all-gather, inside the merge)
#include <string.h>

#include <mutex>

#include "common.cuh"

namespace ss {
namespace peer {

constexpr int D = 128;

struct Parts {
    const void *o[SS_MAX_PEERS];
    const float *lse[SS_MAX_PEERS];
};
struct Flags {
    int *f[SS_MAX_PEERS];
};
struct Outs {
    void *p[SS_MAX_PEERS];
    int n;
};
// The wait a merge makes before it reads the partials (counter == nullptr: none): the flags and
// epoch of ss_peer_barrier, the epoch already advanced and posted by post_kernel.
struct Sync {
    Flags fl;
    int rank;
    int *counter;
    int *status;
};

__device__ __forceinline__ void st_release_sys(int *p, int v) {
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int *p) {
    int v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// fl.f[i] for a per-thread i, selected without indexing the parameter array (no local copy).
__device__ __forceinline__ int *flag_of(const Flags &fl, int i) {
    int *f = nullptr;
#pragma unroll
    for (int j = 0; j < SS_MAX_PEERS; ++j)
        if (j == i) f = fl.f[j];
    return f;
}

// One warp. The epoch is this rank's counter + 1 (the counter lives in device memory and is
// advanced here, so a captured and replayed barrier still posts a new epoch each time). Lane
// p < P posts the epoch into slot `rank` of peer p's flags, then waits until slot p of this
// rank's flags holds it (or a later one). Every wait is bounded: after ~2 s the kernel sets
// SS_DEV_TIMEOUT in *status and returns.
__global__ void __launch_bounds__(32) barrier_kernel(const __grid_constant__ Flags fl, int rank, int P, int *counter,
                                                     int *status) {
    const int p = threadIdx.x;
    const int epoch = *counter + 1;
    __syncwarp();
    if (p == 0) *counter = epoch;
    if (p < P) {
        __threadfence_system();                  // this rank's earlier writes before the post
        st_release_sys(flag_of(fl, p) + rank, epoch);
        const int *mine = flag_of(fl, rank) + p;
        const long long t0 = clock64();
        bool ok = true;
        while (ld_acquire_sys(mine) - epoch < 0) {
            if (clock64() - t0 > kWaitLimitCycles) {
                ok = false;
                break;
            }
            __nanosleep(64);
        }
        if (!ok) report(status, SS_DEV_TIMEOUT);
    }
}

// The first half of barrier_kernel: lane p < P posts the advanced epoch into slot `rank` of peer
// p's flags; the wait is left to the kernel that follows (merge_peers_kernel with a Sync).
__global__ void __launch_bounds__(32) post_kernel(const __grid_constant__ Flags fl, int rank, int P, int *counter) {
    const int p = threadIdx.x;
    const int epoch = *counter + 1;
    __syncwarp();
    if (p == 0) *counter = epoch;
    if (p < P) {
        __threadfence_system();                  // this rank's earlier writes before the post
        st_release_sys(flag_of(fl, p) + rank, epoch);
    }
}

// Eight consecutive values of a part (element offset 8*idx8) as two float4, one 16-byte load
// (bf16) or two (fp32), read through L2: peer data crosses NVLink in whole 16-byte pieces.
__device__ __forceinline__ void load8(const void *base, int64_t idx8, bool bf16, float4 &a, float4 &b) {
    if (bf16) {
        const uint4 u = __ldcg(reinterpret_cast<const uint4 *>(base) + idx8);
        a = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                        __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
        b = make_float4(__uint_as_float(u.z << 16), __uint_as_float(u.z & 0xffff0000u),
                        __uint_as_float(u.w << 16), __uint_as_float(u.w & 0xffff0000u));
    } else {
        a = __ldcg(reinterpret_cast<const float4 *>(base) + 2 * idx8);
        b = __ldcg(reinterpret_cast<const float4 *>(base) + 2 * idx8 + 1);
    }
}

__device__ __forceinline__ void fma4(float w, const float4 &v, float4 &acc) {
    acc.x = fmaf(w, v.x, acc.x);
    acc.y = fmaf(w, v.y, acc.y);
    acc.z = fmaf(w, v.z, acc.z);
    acc.w = fmaf(w, v.w, acc.w);
}

// One thread per (row, head, 8 dims) of rows [row0, row1). Every part's LSE and values are loaded
// before any is used (all of a thread's peer loads in flight at once); arithmetic and order are
// those of ss_lse_merge: L = max + log(sum w), w_p = exp(lse_p - max), out = sum w_p o_p / sum w.
// The merged row is stored into every out.p[d] (d < out.n), this GPU's or a peer's.
// With sync.counter, every CTA first waits, bounded, until every rank has posted the epoch this
// rank's post_kernel posted (only local loads: the flags live in this rank's memory).
template <int PMAX>
__global__ void __launch_bounds__(256) merge_peers_kernel(Parts parts, int P, int part_bf16, int H, int Lq, int row0,
                                                          int row1, Outs out, int out_fp32, float *lse_out, Sync sync) {
    if (sync.counter) {
        if (threadIdx.x < 32) {
            const int p = threadIdx.x;
            const int epoch = *sync.counter;
            if (p < P) {
                const int *mine = flag_of(sync.fl, sync.rank) + p;
                const long long t0 = clock64();
                bool ok = true;
                while (ld_acquire_sys(mine) - epoch < 0) {
                    if (clock64() - t0 > kWaitLimitCycles) {
                        ok = false;
                        break;
                    }
                    __nanosleep(32);
                }
                if (!ok) report(sync.status, SS_DEV_TIMEOUT);
            }
            __syncwarp();
        }
        __syncthreads();
    }
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t total = (int64_t)(row1 - row0) * H * (D / 8);
    if (gid >= total) return;
    const int oct = (int)(gid % (D / 8));
    const int64_t rh = (int64_t)row0 * H + gid / (D / 8);   // row * H + h
    const int h = (int)(rh % H);
    const int row = (int)(rh / H);
    const int64_t idx8 = rh * (D / 8) + oct;
    float l[PMAX];
    float4 va[PMAX], vb[PMAX];
#pragma unroll
    for (int p = 0; p < PMAX; ++p) {
        if (p < P) {
            l[p] = __ldcg(parts.lse[p] + (int64_t)h * Lq + row);
            load8(parts.o[p], idx8, part_bf16 != 0, va[p], vb[p]);
        }
    }
    float mx = -INFINITY, wsum = 0.f;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
#pragma unroll
    for (int p = 0; p < PMAX; ++p)
        if (p < P) mx = fmaxf(mx, l[p]);
    if (mx != -INFINITY) {
#pragma unroll
        for (int p = 0; p < PMAX; ++p) {
            if (p < P) {
                const float w = __expf(l[p] - mx);
                fma4(w, va[p], a);
                fma4(w, vb[p], b);
                wsum += w;
            }
        }
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    const float r[8] = {a.x * inv, a.y * inv, a.z * inv, a.w * inv, b.x * inv, b.y * inv, b.z * inv, b.w * inv};
    const int64_t base = rh * D + oct * 8;
    const uint4 packed = make_uint4(pack_bf16x2(r[0], r[1]), pack_bf16x2(r[2], r[3]), pack_bf16x2(r[4], r[5]),
                                    pack_bf16x2(r[6], r[7]));
#pragma unroll
    for (int d = 0; d < SS_MAX_PEERS; ++d) {
        if (d >= out.n) break;
        if (out_fp32) {
            float4 *dst = reinterpret_cast<float4 *>(reinterpret_cast<float *>(out.p[d]) + base);
            dst[0] = make_float4(r[0], r[1], r[2], r[3]);
            dst[1] = make_float4(r[4], r[5], r[6], r[7]);
        } else {
            reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(out.p[d]) + base)[0] = packed;
        }
    }
    if (lse_out && oct == 0) lse_out[(int64_t)h * Lq + row] = wsum > 0.f ? mx + __logf(wsum) : -INFINITY;
}

using AddressRangeFn = CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr);

static AddressRangeFn address_range_fn() {
    static AddressRangeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<AddressRangeFn>(p);
    });
    return fn;
}

}  // namespace peer
}  // namespace ss

extern "C" int ss_ipc_handle(const void *ptr, void *handle, size_t *offset) {
    using namespace ss;
    if (!ptr || !handle || !offset) return SS_ERR_POINTER;
    peer::AddressRangeFn fn = peer::address_range_fn();
    if (!fn) return SS_ERR_DRIVER;
    CUdeviceptr base = 0;
    size_t size = 0;
    if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return SS_ERR_DRIVER;
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
    if (e != cudaSuccess) return (int)e;
    static_assert(sizeof(cudaIpcMemHandle_t) == SS_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof(h));
    *offset = (size_t)(reinterpret_cast<uintptr_t>(ptr) - (uintptr_t)base);
    return 0;
}

extern "C" int ss_ipc_open(const void *handle, size_t offset, void **ptr) {
    if (!handle || !ptr) return SS_ERR_POINTER;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void *base = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return (int)e;
    *ptr = static_cast<uint8_t *>(base) + offset;
    return 0;
}

extern "C" int ss_ipc_close(void *ptr, size_t offset) {
    if (!ptr) return SS_ERR_POINTER;
    return (int)cudaIpcCloseMemHandle(static_cast<uint8_t *>(ptr) - offset);
}

extern "C" int ss_peer_barrier(int *const *flags, int rank, int P, int *epoch, int *status, void *stream) {
    using namespace ss;
    if (!flags || !epoch) return SS_ERR_POINTER;
    if (P <= 0 || P > SS_MAX_PEERS || rank < 0 || rank >= P) return SS_ERR_SHAPE;
    peer::Flags fl;
    for (int p = 0; p < SS_MAX_PEERS; ++p) fl.f[p] = p < P ? flags[p] : nullptr;
    for (int p = 0; p < P; ++p)
        if (!fl.f[p] || (reinterpret_cast<uintptr_t>(fl.f[p]) & 3u)) return SS_ERR_POINTER;
    peer::barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(fl, rank, P, epoch, status);
    return (int)cudaGetLastError();
}

static int merge_launch(const void *const *o_parts, const float *const *lse_parts, int P, int part_dtype, int H,
                        int Lq, int row0, int row1, const void *const *outs, int n_out, int out_dtype,
                        float *lse_out, void *stream, int *const *flags = nullptr, int rank = 0,
                        int *epoch = nullptr, int *status = nullptr) {
    using namespace ss;
    if (!o_parts || !lse_parts || !outs) return SS_ERR_POINTER;
    if (n_out < 1 || n_out > SS_MAX_PEERS) return SS_ERR_SHAPE;
    peer::Sync sync;
    sync.counter = nullptr;
    sync.rank = rank;
    sync.status = status;
    for (int p = 0; p < SS_MAX_PEERS; ++p) sync.fl.f[p] = nullptr;
    if (flags) {
        if (!epoch || (reinterpret_cast<uintptr_t>(epoch) & 3u)) return SS_ERR_POINTER;
        if (P > SS_MAX_PEERS || rank < 0 || rank >= P) return SS_ERR_SHAPE;
        for (int p = 0; p < P; ++p) {
            sync.fl.f[p] = flags[p];
            if (!flags[p] || (reinterpret_cast<uintptr_t>(flags[p]) & 3u)) return SS_ERR_POINTER;
        }
        sync.counter = epoch;
    }
    if (P <= 0 || P > SS_MAX_PEERS || H <= 0 || Lq <= 0 || row0 < 0 || row1 < row0 || row1 > Lq ||
        (part_dtype != 0 && part_dtype != 1) || (out_dtype != 0 && out_dtype != 1))
        return SS_ERR_SHAPE;
    peer::Parts parts;
    for (int p = 0; p < SS_MAX_PEERS; ++p) {
        parts.o[p] = p < P ? o_parts[p] : nullptr;
        parts.lse[p] = p < P ? lse_parts[p] : nullptr;
    }
    for (int p = 0; p < P; ++p) {
        if (!parts.o[p] || !parts.lse[p]) return SS_ERR_POINTER;
        if ((reinterpret_cast<uintptr_t>(parts.o[p]) & 15u) ||
            (reinterpret_cast<uintptr_t>(parts.lse[p]) & 3u))
            return SS_ERR_POINTER;
    }
    peer::Outs out;
    for (int d = 0; d < SS_MAX_PEERS; ++d) {
        out.p[d] = d < n_out ? const_cast<void *>(outs[d]) : nullptr;
        if (d < n_out && (!out.p[d] || (reinterpret_cast<uintptr_t>(out.p[d]) & 15u))) return SS_ERR_POINTER;
    }
    out.n = n_out;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (row1 == row0) {
        // no rows to merge: the barrier alone
        if (sync.counter) peer::barrier_kernel<<<1, 32, 0, st>>>(sync.fl, rank, P, epoch, status);
        return (int)cudaGetLastError();
    }
    if (sync.counter) {
        peer::post_kernel<<<1, 32, 0, st>>>(sync.fl, rank, P, epoch);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return (int)e;
    }
    const int64_t total = (int64_t)(row1 - row0) * H * (peer::D / 8);
    const unsigned blocks = (unsigned)((total + 255) / 256);
    const int bf = part_dtype == 0;
    if (P <= 2)
        peer::merge_peers_kernel<2><<<blocks, 256, 0, st>>>(parts, P, bf, H, Lq, row0, row1, out, out_dtype, lse_out,
                                                              sync);
    else if (P <= 4)
        peer::merge_peers_kernel<4><<<blocks, 256, 0, st>>>(parts, P, bf, H, Lq, row0, row1, out, out_dtype, lse_out,
                                                              sync);
    else
        peer::merge_peers_kernel<8><<<blocks, 256, 0, st>>>(parts, P, bf, H, Lq, row0, row1, out, out_dtype, lse_out,
                                                              sync);
    return (int)cudaGetLastError();
}

extern "C" int ss_lse_merge_peers(const void *const *o_parts, const float *const *lse_parts, int P, int part_dtype,
                                  int H, int Lq, int row0, int row1, void *out, int out_dtype, float *lse_out,
                                  void *stream) {
    if (!out) return SS_ERR_POINTER;
    const void *outs[1] = {out};
    return merge_launch(o_parts, lse_parts, P, part_dtype, H, Lq, row0, row1, outs, 1, out_dtype, lse_out, stream);
}

extern "C" int ss_lse_merge_gather(const void *const *o_parts, const float *const *lse_parts, int P, int part_dtype,
                                   int H, int Lq, int row0, int row1, void *const *outs, int n_out, int out_dtype,
                                   int *const *flags, int rank, int *epoch, int *status, void *stream) {
    if (!outs) return SS_ERR_POINTER;
    return merge_launch(o_parts, lse_parts, P, part_dtype, H, Lq, row0, row1, outs, n_out, out_dtype, nullptr,
                        stream, flags, rank, epoch, status);
}
