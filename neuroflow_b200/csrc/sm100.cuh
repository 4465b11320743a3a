// sm100.cuh -- thin inline-PTX layer for Blackwell (sm_100a): shared-memory
// mbarriers, TMA bulk-tensor copies, tcgen05 MMA/TMEM, and the UMMA descriptors.
//
// Every spin-wait in this file is bounded (2 s of %globaltimer): a wait that exceeds
// its budget returns false, the caller raises the CTA's abort flag so that the kernel can tear down (release
// TMEM, drain its own copies) and report an error code to the host instead of
// hanging the GPU.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace nfx {

// Error codes written to the device error word (see nfx_errors in nfx_abi.cpp).
enum : unsigned {
    kErrWaitTmaFull = 1u << 0,
    kErrWaitSlotFree = 1u << 1,
    kErrWaitAccFull = 1u << 2,
    kErrWaitAccFree = 1u << 3,
    kErrWaitDrain = 1u << 4,
};

// A wait gives up after this many nanoseconds of the global timer.
constexpr uint64_t kWaitNs = 2000000000ull;

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "elect.sync _|P, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, P;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, P;\n\t}"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    return ok != 0;
}

// Non-blocking test of a phase (mbarrier.test_wait: never suspends the thread).
__device__ __forceinline__ bool mbar_test_addr(uint32_t addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, P;\n\t}"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    return ok != 0;
}

// One try of a bounded wait.  try_wait may suspend the thread until the phase completes,
// so a wait with a budget below the default tests without suspending instead: then the
// budget, not the phase, decides when the wait ends.
__device__ __forceinline__ bool mbar_try_budget(uint32_t addr, uint32_t parity, uint64_t budget_ns) {
    if (budget_ns >= kWaitNs) return mbar_try_wait(addr, parity);
    return mbar_test_addr(addr, parity);
}

// The budget has run out.  Budgets below kTimerGrainNs are finer than the global
// timer's update interval, so they count as spent at the first retry.
constexpr uint64_t kTimerGrainNs = 1000;
__device__ __forceinline__ bool budget_spent(uint64_t t0, uint64_t budget_ns) {
    return budget_ns < kTimerGrainNs || global_ns() - t0 > budget_ns;
}

// Non-blocking test: true when the phase with the given parity has completed.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, P;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity to complete, polling.  Gives up
// early when another warp of the CTA has raised `abort`.  For waits on a kernel's
// critical path (an epilogue waiting for its accumulator): the warp resumes as soon
// as the phase completes.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          uint64_t budget_ns = kWaitNs) {
    const uint32_t addr = smem_u32(bar);
    if (mbar_try_budget(addr, parity, budget_ns)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_budget(addr, parity, budget_ns)) return true;
        if ((i & 63u) == 1u) {
            if (*abort) return false;
            if (budget_spent(t0, budget_ns)) return false;
        }
    }
}

// The same wait with exponential back-off (__nanosleep from `min_ns` up to `max_ns`)
// between tries (the abort flag and the time budget are checked every 8 tries): a waiting warp takes almost no issue slots from the warps doing the
// arithmetic, at the price of resuming up to `max_ns` late.  For producers that run
// stages ahead and for the single-thread MMA issuer.
__device__ __forceinline__ bool mbar_wait_backoff(uint64_t* bar, uint32_t parity, volatile int* abort,
                                                  uint32_t max_ns, uint32_t min_ns = 32,
                                                  uint64_t budget_ns = kWaitNs) {
    const uint32_t addr = smem_u32(bar);
    if (mbar_try_budget(addr, parity, budget_ns)) return true;
    const uint64_t t0 = global_ns();
    uint32_t ns = min_ns;
    for (uint32_t i = 1;; ++i) {
        __nanosleep(ns);
        if (mbar_try_budget(addr, parity, budget_ns)) return true;
        ns = ns * 2 < max_ns ? ns * 2 : max_ns;
        if ((i & 7u) == 1u) {
            if (*abort) return false;
            if (budget_spent(t0, budget_ns)) return false;
        }
    }
}

// Wait for this CTA's own asynchronous work (a TMA load it issued, the completion of
// an MMA commit) before teardown.  Such work completes by itself, so the wait ignores
// the abort flag; it is still bounded by the default budget.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity) {
    const uint32_t addr = smem_u32(bar);
    if (mbar_try_wait(addr, parity)) return true;
    const uint64_t t0 = global_ns();
    uint32_t ns = 32;
    for (;;) {
        __nanosleep(ns);
        if (mbar_try_wait(addr, parity)) return true;
        ns = ns * 2 < 1024u ? ns * 2 : 1024u;
        if (global_ns() - t0 > kWaitNs) return false;
    }
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialization may start while the previous kernel in the stream still runs; it
// touches only its own shared memory, TMEM and read-only tables until grid_dep_wait(),
// which returns once the previous grid has completed and its memory is visible (at
// once when there is no such dependency).  grid_dep_launch() lets the next kernel
// launch early; its CTAs are placed as this kernel's CTAs leave the SMs.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void grid_dep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dep_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor) -- loads without multicast only.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x,
                                             int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(x), "r"(y), "r"(smem_u32(src))
        : "memory");
}

__device__ __forceinline__ void tma_store_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void tma_store_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void tma_store_wait_all() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Generic-proxy writes to shared memory become visible to the async proxy (TMA store).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, commit, loads, fences
// ---------------------------------------------------------------------------
// Whole warp.  Writes the TMEM base address to *dst_smem.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, int8 x int8 -> int32.  One thread issues.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(
            d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
        : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, tf32 x tf32 -> fp32.  One thread issues.
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(
            d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
        : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, f16 x f16 -> fp32 (both f16: the instruction
// descriptor of idesc_f16).  One thread issues.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(
            d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
        : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, FP8 x FP8 -> fp32 (formats in the instruction
// descriptor; both E4M3 here).  One thread issues.
__device__ __forceinline__ void mma_f8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(
            d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
        : "memory");
}

// Arrive on `bar` once all previously issued tcgen05 ops of this thread complete.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t gets lane (base lane + t).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t (&r)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld1(uint32_t taddr, uint32_t& r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
}

// ---------------------------------------------------------------------------
// UMMA shared-memory descriptors (K-major, swizzled) and instruction descriptors
// ---------------------------------------------------------------------------
// Swizzle modes: rows of 32/64/128 bytes; the 16-byte chunk index inside a row is
// XOR-ed with address bits [7, 7+log2(rows_per_128B...)) -- the same pattern TMA
// writes with CU_TENSOR_MAP_SWIZZLE_{32,64,128}B.
enum class Swz : int { B32 = 32, B64 = 64, B128 = 128 };

__host__ __device__ constexpr uint32_t swz_layout_type(int row_bytes) {
    return row_bytes == 128 ? 2u : (row_bytes == 64 ? 4u : 6u);
}

// Byte offset (inside a 1024-byte aligned region) of logical byte `o` of a K-major
// tile whose rows are `row_bytes` wide.
__host__ __device__ constexpr uint32_t swz_offset(uint32_t o, int row_bytes) {
    const uint32_t mask = row_bytes == 128 ? 7u : (row_bytes == 64 ? 3u : 1u);
    return o ^ (((o >> 7) & mask) << 4);
}

// K-major, swizzled: LBO unused (1), SBO = 8 rows * row_bytes.
__device__ __forceinline__ uint64_t umma_desc(uint32_t smem_addr, int row_bytes) {
    const uint64_t start = (smem_addr >> 4) & 0x3FFFu;
    const uint64_t lbo = 1;
    const uint64_t sbo = ((8u * row_bytes) >> 4) & 0x3FFFu;
    return start | (lbo << 16) | (sbo << 32) | (1ull << 46) |
           (static_cast<uint64_t>(swz_layout_type(row_bytes)) << 61);
}

// kind::i8, signed A and B, int32 D, both K-major, M = 128.
__host__ __device__ constexpr uint32_t idesc_i8(int n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(128 >> 4) << 24);
}

// kind::f8f6f4 with E4M3 A and B (format code 0), fp32 D, both K-major, M = 128
// (set bit 15 for an MN-major A).
__host__ __device__ constexpr uint32_t idesc_e4m3(int n) {
    return (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(128 >> 4) << 24);
}

// MN-major operand, 64-byte swizzle: atoms of 8 K rows x 64 bytes of M, `lbo` bytes
// between M atoms, `sbo` bytes between groups of 8 K rows.
__device__ __forceinline__ uint64_t umma_desc_mn_sw64(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
    return static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu) |
           (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) |
           (static_cast<uint64_t>(4u) << 61);
}

// x rounded to nearest (ties away) at tf32 precision (10 stored mantissa bits), as the
// fp32 bit pattern the tensor core reads.
__device__ __forceinline__ float tf32_rna(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// kind::f16 with f16 A and B (format code 0 for both), fp32 D, both K-major, M = 128.
__host__ __device__ constexpr uint32_t idesc_f16(int n) {
    return (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(128 >> 4) << 24);
}

// kind::tf32, fp32 D, both K-major, M = 128.
__host__ __device__ constexpr uint32_t idesc_tf32(int n) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(128 >> 4) << 24);
}

}  // namespace nfx
