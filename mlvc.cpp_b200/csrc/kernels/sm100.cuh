// sm_100a device primitives used by the tensor-core kernels: mbarriers with
// bounded waits, TMA tile loads, tcgen05 (TMEM alloc, UMMA issue, commit,
// TMEM->register loads) and the shared-memory matrix descriptors.
//
// Every wait in this file is bounded by wall-clock time (%globaltimer).  When a
// wait runs out it records an error code in the module-wide status word, sets
// the CTA-local abort flag and returns false, so the calling role winds down
// instead of spinning; the host reads the status word after each run.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "params.h"

// Module-wide error status (0 = ok).  Read by the host through
// cuModuleGetGlobal("mlvc_b200_status") after every synchronising call.
extern "C" __device__ unsigned int mlvc_b200_status;
// Limit of every bounded wait in nanoseconds (module-wide, kWaitLimitNs
// unless the host's wait-expiry test shortens it for one launch).
extern "C" __device__ unsigned long long mlvc_b200_wait_limit_ns;

namespace mlvc_b200 {

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s
// Status bit of a Gather whose index is outside the table (the wait-timeout
// bits of the tensor-core kernels are 0x1 .. 0x80).
constexpr unsigned int kStatusGatherIndex = 0x100u;

__device__ __forceinline__ unsigned long long globaltimer_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool elect_one()
{
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "elect.sync _|P, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, P;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

// ------------------------------------------------- programmatic launch
// With programmatic stream serialisation the next kernel in the stream may
// start while this one runs; it must call pdl_wait() before touching memory
// that earlier kernels read or write (it returns once they have completed and
// their writes are visible).  Without a programmatic dependency both are
// no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// ---------------------------------------------------------------- mbarrier
// Rounds a pointer into dynamic shared memory up to 1024 bytes by pointer
// arithmetic on the shared array itself, so that the compiler keeps knowing
// the address space of everything derived from it (shared-memory loads and
// stores instead of generic ones).
__device__ __forceinline__ uint8_t* align_smem_1024(uint8_t* smem)
{
    return smem + ((1024u - (smem_u32(smem) & 1023u)) & 1023u);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, P;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: while the phase is incomplete the thread
// may be suspended (woken when the phase completes, at the latest after
// hint_ns) instead of returning at once, so waiting warps stop taking issue
// slots from the single-thread producer and MMA roles on their sub-partition.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity, uint32_t hint_ns)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, P;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Suspend-time hint of the bounded wait's loop: the abort flag and the time
// limit are still checked at least this often.
constexpr uint32_t kWaitSuspendNs = 100000;  // 100 us

// Bounded wait on `bar` completing the phase with the given parity.  Returns
// false (after recording `code`) when the CTA is aborting or the wait ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          unsigned int code)
{
    if (mbar_try_wait(bar, parity))
        return true;
    const unsigned long long start = globaltimer_ns();
    const unsigned long long limit = mlvc_b200_wait_limit_ns;
    while (true) {
        // Plain polling: a suspend-time hint here (mbar_try_wait_suspend)
        // measured no gain at 1920x1088 and 2 % slower on the 8-block stack.
        if (mbar_try_wait(bar, parity))
            return true;
        if (*abort_flag)
            return false;
        if (globaltimer_ns() - start > limit) {
            *abort_flag = 1;
            atomicOr(&mlvc_b200_status, code);
            return false;
        }
    }
}

// ------------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map)
{
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

// TMA bulk-tensor stores (shared -> global), tracked per thread in bulk groups.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y)
{
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(src)), "r"(x), "r"(y)
                 : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int x, int y, int z)
{
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
                 : "memory");
}

__device__ __forceinline__ void tma_store_5d(const CUtensorMap* map, const void* src, int c0, int c1, int c2, int c3,
                                             int c4)
{
    asm volatile("cp.async.bulk.tensor.5d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5, %6}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
                 : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Wait until at most N committed groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read()
{
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until every committed group has completed (writes performed).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Makes this thread's generic-proxy shared-memory writes visible to the async
// proxy (TMA) before a bulk copy reads them.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D(tmem) (+)= A(smem desc) * B(smem desc)^T, kind::f16 (FP16 inputs, FP32 accumulate).
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives once on `bar` when all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void umma_commit(uint64_t* bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 lanes x 32 bit, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16])
{
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i)
        v[i] = __uint_as_float(r[i]);
}

// Issue-only variants: several loads may be in flight before one
// tmem_wait_ld() (the destination registers are undefined until then).
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t (&r)[16])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor (tcgen05 format): start address, leading
// and stride byte offsets in 16-byte units, version 1 at bits 46-47, layout
// type at bits 61-63 (0 = no swizzle / interleaved core matrices, 2 = 128-byte
// swizzle).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes, uint32_t layout)
{
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= 1ull << 46;
    d |= static_cast<uint64_t>(layout & 7u) << 61;
    return d;
}

// Instruction descriptor for kind::f16: FP16 A and B (K-major), FP32 accumulator.
__host__ __device__ constexpr uint32_t idesc_f16_f32(uint32_t m, uint32_t n)
{
    return (1u << 4)            // D format F32
           | (0u << 7)          // A format F16
           | (0u << 10)         // B format F16
           | ((n >> 3) << 17)   // N / 8
           | ((m >> 4) << 24);  // M / 16
}

// ------------------------------------------------------------ FP16 helpers
__device__ __forceinline__ float round_h(float v) { return __half2float(__float2half_rn(v)); }

__device__ __forceinline__ uint32_t pack_h2(float a, float b)
{
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// a_lo = fma(x_lo, w_lo, a_lo), a_hi = fma(x_hi, w_hi, a_hi) on the two FP16
// halves of x2 and w2 with FP32 accumulators (sm_100 mixed-precision
// fma.rn.f32.f16).  A product of two FP16 values is exact in FP32, so each
// result equals fmaf(float(x), float(w), a) bit for bit, without the two
// FP16 -> FP32 conversions (a slow pipe) that fmaf would need.
__device__ __forceinline__ void fma_h2(float& a_lo, float& a_hi, uint32_t x2, uint32_t w2)
{
    asm("{\n\t.reg .b16 xl, xh, wl, wh;\n\t"
        "mov.b32 {xl, xh}, %2;\n\t"
        "mov.b32 {wl, wh}, %3;\n\t"
        "fma.rn.f32.f16 %0, xl, wl, %0;\n\t"
        "fma.rn.f32.f16 %1, xh, wh, %1;\n\t}"
        : "+f"(a_lo), "+f"(a_hi)
        : "r"(x2), "r"(w2));
}

__device__ __forceinline__ void unpack_h2(uint32_t u, float& a, float& b)
{
    __half2 h = *reinterpret_cast<__half2*>(&u);
    float2 f = __half22float2(h);
    a = f.x;
    b = f.y;
}

}  // namespace mlvc_b200
