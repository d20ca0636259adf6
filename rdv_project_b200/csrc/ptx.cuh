// Thin inline-PTX layer for sm_100a: mbarriers (with bounded waits), bulk
// (TMA 1-D) copies, proxy fences and the tcgen05 family (TMEM alloc, UMMA
// issue/commit, TMEM loads). Every wait in this file is bounded: on expiry it
// raises the CTA-wide abort flag and records a status bit in global memory,
// so a scheduling bug surfaces as an error code instead of a hung GPU.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

namespace rdvb {

// Status bits written to the device status word (rdvb_device_status()).
enum : uint32_t {
    kStatusTimeoutXFull = 1u << 0,
    kStatusTimeoutXEmpty = 1u << 1,
    kStatusTimeoutAFull = 1u << 2,
    kStatusTimeoutAccFull = 1u << 3,
    kStatusTimeoutWFull = 1u << 4,
    kStatusTimeoutWEmpty = 1u << 5,
    kStatusTimeoutDrain = 1u << 6,
    kStatusTimeoutOther = 1u << 7,
};

// Device status word: OR of the kStatus* bits raised by any kernel of this
// library since the host last cleared it (rdvb_device_status). This library
// is a single translation unit, so the definition lives here.
__device__ uint32_t g_status;

// A bounded wait gives up after this many nanoseconds (%globaltimer).
#ifndef RDVB_WAIT_LIMIT_NS
#define RDVB_WAIT_LIMIT_NS 2000000000ull
#endif

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Same, but the thread may sleep up to `hint_ns` (it resumes as soon as the
// phase completes), so a waiting warp does not take issue slots from the
// warps sharing its scheduler.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Non-blocking test of the phase with the given parity.
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Suspend-time hint of the bounded waits below (nanoseconds).
#ifndef RDVB_SLEEP_HINT_NS
#define RDVB_SLEEP_HINT_NS 500000u
#endif
#ifndef RDVB_SPIN_TRIES
#define RDVB_SPIN_TRIES 0
#endif

// Waits for the phase with the given parity to complete. Returns false (and
// raises *abort) if the CTA was aborted or the wait ran past the limit.
// Each try sleeps up to RDVB_SLEEP_HINT_NS, so the abort flag and the time
// limit are still checked regularly.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile uint32_t* abort,
                                          uint32_t* status, uint32_t code) {
#pragma unroll 1
    for (int i = 0; i < RDVB_SPIN_TRIES; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    if (mbar_try_wait_sleep(bar, parity, RDVB_SLEEP_HINT_NS)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        if (mbar_try_wait_sleep(bar, parity, RDVB_SLEEP_HINT_NS)) return true;
        if (*abort) return false;
        if (global_timer_ns() - t0 > RDVB_WAIT_LIMIT_NS) {
            *abort = 1u;
            atomicOr(status, code);
            return false;
        }
    }
}

// Warp-wide bounded wait: lane 0 waits on the barrier, the outcome is
// broadcast and the warp re-converges (__syncwarp orders lane 0's acquire
// before the other lanes' later accesses). One waiting thread per warp
// instead of 32 keeps the barrier traffic off the shared-memory pipe the
// tensor core reads its operands through. Call with all 32 lanes.
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, volatile uint32_t* abort,
                                               uint32_t* status, uint32_t code) {
    bool ok = true;
    if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort, status, code);
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    __syncwarp();
    return ok;
}

// Drain wait used on the abort path: ignores the abort flag, keeps its own
// time limit.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity) {
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait_sleep(bar, parity, 500000u)) {
        if (global_timer_ns() - t0 > RDVB_WAIT_LIMIT_NS) {
            atomicOr(&g_status, kStatusTimeoutDrain);
            return;
        }
    }
}

// ------------------------------------------------------- bulk async copies
// Global -> shared 1-D bulk copy (TMA engine), completion counted on `bar`
// in bytes. dst/src 16-byte aligned, bytes a multiple of 16. No multicast.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

// Global -> shared tiled 4-D tensor copy (TMA) of the box at coordinates
// (c0 innermost .. c3) of `tmap` (a kernel-parameter tensor map), completion
// counted on `bar` in bytes (the whole box; out-of-range elements are
// zero-filled). c0 * element size must be a multiple of 16 bytes; the other
// coordinates may be negative or past the end. No multicast.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void* tmap, int c0, int c1, int c2, int c3,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
        "%5}], [%6];" ::"r"(dst),
        "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
        : "memory");
}

// Shared -> global 1-D bulk copy, tracked by the issuing thread's bulk group.
__device__ __forceinline__ void bulk_s2g(void* dst, uint32_t src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all_read() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Generic-proxy shared-memory writes -> visible to the async proxy (UMMA/TMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ------------------------------------------------------------------ tcgen05
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

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (f16 or bf16 inputs,
// f32 accumulate), issued by one thread; only a tcgen05.commit from that same
// thread tracks it (a commit from another lane arrives at once). The MMA
// reads shared memory and TMEM written by other threads and by bulk copies,
// so it carries a "memory" clobber: no load or store of the issuing thread
// moves across it, whatever the surrounding code.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Same with the A operand read from tensor memory (M=128 rows = lanes, 16-bit
// elements packed two per 32-bit column: one K=16 step spans 8 columns).
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive once on `bar` when every previously issued tcgen05 op of this
// thread has completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns; thread i gets lane (base + i).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
// The registers of a tcgen05.ld hold the data only after tcgen05.wait::ld,
// but the compiler sees them defined at the load, and a wait with only a
// "memory" clobber does not stop it from scheduling arithmetic on them
// before the wait (register uses are not memory accesses). So the only wait
// offered here redefines the loaded registers (and reg_barrier, placed
// after it, those of a second load waited on by the same instruction): no
// use of them can move above the wait.
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15])
                 :
                 : "memory");
}
__device__ __forceinline__ void reg_barrier(uint32_t (&r)[16]) {
    asm volatile(""
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15])
                 :
                 : "memory");
}

// 32 lanes x 8 consecutive 32-bit columns; thread i writes lane (base + i).
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]), "r"(r[1]),
        "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// UMMA shared-memory matrix descriptor for a K-major operand in the
// canonical 128-byte-swizzled layout: rows of 128 bytes (64 x 16-bit
// elements), 8-row core groups 1024 bytes apart (SBO), 16-byte chunks
// XOR-swizzled with (row % 8). Start address must sit inside a
// 1024-byte-aligned atom; advancing K by 16 elements adds 32 bytes.
// Bit layout (sm_100 descriptor): [0,14) addr>>4, [16,30) LBO>>4,
// [32,46) SBO>>4, [46,48) version=1, [49,52) base offset=0, [61,64) layout
// (2 = SWIZZLE_128B).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;             // LBO (unused for swizzled K-major) = 16 B
    d |= static_cast<uint64_t>(1024u >> 4) << 32;     // SBO = 1024 B
    d |= static_cast<uint64_t>(1u) << 46;             // descriptor version (sm_100)
    d |= static_cast<uint64_t>(2u) << 61;             // SWIZZLE_128B
    return d;
}

// Descriptor for a K-major operand with no swizzle ("interleaved" core
// matrices): 8 rows x 16 bytes per core matrix stored contiguously, the two
// 8-element K halves of a K=16 slice 128 bytes apart (LBO), 8-row groups 256
// bytes apart (SBO). Element (row, k), k < 16, sits at
// (row/8)*256 + (k/8)*128 + (row%8)*16 + (k%8)*2.
__device__ __forceinline__ uint64_t umma_desc_k16_plain(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(128u >> 4) << 16;      // LBO
    d |= static_cast<uint64_t>(256u >> 4) << 32;      // SBO
    d |= static_cast<uint64_t>(1u) << 46;             // version
    return d;                                         // layout 0 = no swizzle
}

__host__ __device__ __forceinline__ uint32_t k16_plain_offset(uint32_t row, uint32_t k) {
    return (row >> 3) * 256u + (k >> 3) * 128u + (row & 7u) * 16u + (k & 7u) * 2u;
}

// Instruction descriptor, kind::f16: D f32, A/B f16 (0) or bf16 (1), both
// K-major, M = 128, N = n (multiple of 16, 16..256).
__host__ __device__ constexpr uint32_t umma_idesc_f16(uint32_t n, uint32_t ab_bf16) {
    return (1u << 4)                    // D format f32
           | (ab_bf16 << 7)             // A format
           | (ab_bf16 << 10)            // B format
           | ((n >> 3) << 17)           // N >> 3
           | ((128u >> 4) << 24);       // M >> 4
}

// Byte offset of element (row, k) inside a K-major SW128 block whose rows
// are `rows` long in the row dimension (rows multiple of 8): 64-element
// K atoms are stored one after another, each rows*128 bytes.
__host__ __device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t k, uint32_t rows) {
    const uint32_t atom = k >> 6;
    const uint32_t kk = k & 63u;
    const uint32_t chunk = (kk >> 3) ^ (row & 7u);
    return atom * rows * 128u + row * 128u + chunk * 16u + (kk & 7u) * 2u;
}

// ------------------------------------------------------- packed conversions
// {lo, hi} -> f16x2 / bf16x2, round to nearest even, optional ReLU clamp.
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}
__device__ __forceinline__ uint32_t pack_f16x2_relu(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.relu.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}
__device__ __forceinline__ uint32_t pack_bf16x2_relu(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.relu.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// (a0 + b0, a1 + b1) in one packed fp32 instruction (sm_100).
__device__ __forceinline__ void add_f32x2(float& a0, float& a1, float b0, float b1) {
    uint64_t pa, pb, pd;
    asm("mov.b64 %0, {%1, %2};" : "=l"(pa) : "f"(a0), "f"(a1));
    asm("mov.b64 %0, {%1, %2};" : "=l"(pb) : "f"(b0), "f"(b1));
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(pd) : "l"(pa), "l"(pb));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a0), "=f"(a1) : "l"(pd));
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
                 : "memory");
}

}  // namespace rdvb
