// common.cuh -- sm_100a primitives shared by the libssparse kernels: mbarriers with bounded
// waits, TMA tile loads, tcgen05 (TMEM alloc / MMA / commit / ld / st) and descriptor builders.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/ssparse.h"

namespace ss {

// ---------------------------------------------------------------------------------------------
// status reporting
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void report(int *status, int bits) {
    if (status) atomicOr(status, bits);
}

// ---------------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
                 ::"r"(bar), "r"(bytes) : "memory");
}

// With SS_MBAR_SUSPEND_NS > 0, a thread whose phase has not completed is suspended in try_wait
// until the phase completes or about that many nanoseconds pass. Off by default: on B200 the
// attention kernel measured slower with a suspend hint (1 us to 500 us) than with plain polling.
#ifndef SS_MBAR_SUSPEND_NS
#define SS_MBAR_SUSPEND_NS 0
#endif
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
#if SS_MBAR_SUSPEND_NS > 0
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(bar), "r"(parity), "n"(SS_MBAR_SUSPEND_NS) : "memory");
#else
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
#endif
    return ok != 0;
}

// Every wait in these kernels is bounded: after `kWaitLimitCycles` SM clocks (about 2 s), or once
// another thread of the CTA has given up (signalled through *abort), the wait returns false,
// the caller reports SS_DEV_TIMEOUT and unwinds. A healthy wait completes in microseconds.
constexpr long long kWaitLimitCycles = 4000000000ll;

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 0u) {
            if (*abort) return false;
            if (clock64() - t0 > kWaitLimitCycles) {
                *abort = 1;
                return false;
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------
// TMA (no multicast anywhere in this library)
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// Brings the box at {x, y} of a tensor map into L2 (no shared memory, no completion tracking).
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap *map, int x, int y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y)
                 : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------------------------
// tcgen05
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
// D[tmem] (+)= A[smem] * B[smem], kind::f16 (bf16 inputs, fp32 accumulate)
__device__ __forceinline__ void mma_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float *v) {
    uint32_t *r = reinterpret_cast<uint32_t *>(v);
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
// tcgen05.ld writes its destination registers asynchronously: they hold the loaded values only
// after tcgen05.wait::ld. The compiler does not know that, and may read those registers -- or
// spill them to local memory -- anywhere after the load instruction. Call this on every 32-register
// block loaded by tmem_ld32, after tmem_wait_ld(): it claims to rewrite the registers, so no use of
// them can be placed before it (asm volatile statements keep their order).
__device__ __forceinline__ void tmem_ld_fence32(float *v) {
    uint32_t *r = reinterpret_cast<uint32_t *>(v);
    asm volatile(""
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31]));
}

// tcgen05.st reads its source registers asynchronously, until tcgen05.wait::st; the compiler
// does not know that and may reuse (or reload from a spill slot into) those registers right
// after the store instruction. Call this on every 32-register block stored by tmem_st32, after
// tmem_wait_st(): it reads the registers, so they keep their values until the wait is past.
__device__ __forceinline__ void tmem_st_fence32(const float *v) {
    const uint32_t *r = reinterpret_cast<const uint32_t *>(v);
    asm volatile("" ::"r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
                 "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
                 "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
                 "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float *v) {
    const uint32_t *r = reinterpret_cast<const uint32_t *>(v);
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
          "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
          "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// Shared-memory matrix descriptor (tcgen05 format: version 1, 128-byte swizzle).
//   K-major operand  : rows of 128 B (64 bf16 of K), 8-row swizzle atoms 1024 B apart (SBO).
//   MN-major operand : rows of 128 B (64 bf16 of M/N) per K index, 8 K-rows per atom (SBO),
//                      consecutive 64-wide M/N chunks LBO bytes apart.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((addr & 0x3FFFFu) >> 4);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= 1ull << 46;  // descriptor version for sm_100
    d |= 2ull << 61;  // SWIZZLE_128B
    return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B and fp32 D.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, bool a_mn_major, bool b_mn_major) {
    return (1u << 4)                         // D format: f32
           | (1u << 7)                       // A format: bf16
           | (1u << 10)                      // B format: bf16
           | ((a_mn_major ? 1u : 0u) << 15)  // A major
           | ((b_mn_major ? 1u : 0u) << 16)  // B major
           | ((uint32_t)(N >> 3) << 17)      // N / 8
           | ((uint32_t)(M >> 4) << 24);     // M / 16
}

// One lane of a converged warp (elect.sync). Warp-specialised roles run their loops on the
// whole, converged warp and issue single-thread instructions (tcgen05.mma, tcgen05.commit, TMA)
// from the elected lane: issued from a lone diverged lane, each tcgen05.mma costs ~139 cycles
// of issue time whatever its size (measured on B200), versus its math time when converged.
__device__ __forceinline__ bool elect_one() {
    uint32_t pred;
    asm volatile("{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}" : "=r"(pred));
    return pred != 0;
}

// ---------------------------------------------------------------------------------------------
// misc math
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

// ---------------------------------------------------------------------------------------------
// KV ring: where a window row lives in a ring-buffer cache
// ---------------------------------------------------------------------------------------------
// A ring cache keeps the window's first S (sink) rows at physical rows [0, S) and the rest in a
// ring of C rows at [S, S + C): window row t >= S sits at S + ((t - S + head) mod C). Two copies
// make every 64-row sub-block of the window (rows [64s, 64s + 64)) one contiguous physical range,
// so K/V still load as one box per sub-block:
//   - rows [S + C, S + C + 64) repeat ring rows [0, 64) (a sub-block that runs past the ring's end);
//   - when S is not a multiple of 64, the sink's last S mod 64 rows are repeated just before the
//     ring's head, at ring rows head - S mod 64 .. head - 1 (the sub-block that starts in the sink).
// C = 0 means a plain contiguous window (physical row = window row).
struct KvRing {
    int S = 0, C = 0, head = 0;
    const int *head_dev = nullptr;   // when set, the head is read from device memory (graph replays)
    // this ring with the head from device memory when it lives there
    __device__ __forceinline__ KvRing resolved() const {
        KvRing r = *this;
        if (head_dev) r.head = *head_dev;
        return r;
    }
    // physical row of the first row of the 64-row sub-block starting at window row t0 (t0 % 64 == 0)
    __host__ __device__ __forceinline__ int sub_row(int t0) const {
        if (C == 0 || t0 + 64 <= S) return t0;
        int x = (t0 - S + head) % C;
        if (x < 0) x += C;
        return S + x;
    }
    // physical rows the cache needs for a window of `rows` rows
    __host__ __device__ __forceinline__ int64_t phys_rows(int64_t rows) const {
        return C == 0 ? rows : (int64_t)S + C + 64;
    }
};

}  // namespace ss

// host helpers (defined in capi.cu)
namespace ss {
int encode_tmap_2d_bf16(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer,
                        uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer);
int encode_tmap_2d_bf16_rows(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer,
                             uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer);
int current_context(void **ctx);
int ring_check(const KvRing &ring, int Lk);   // attention_sm100.cu: a geometry the kernels can follow
}
