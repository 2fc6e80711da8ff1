// Thin inline-PTX wrappers for sm_100a: mbarriers, bulk/tensor async copies,
// tcgen05 (TMEM allocation, loads, MMA, commit), programmatic dependent
// launch and L2-level exchange between CTAs. Every wait is bounded: after the limit it raises a device flag and
// returns false so the kernel can drain and exit instead of hanging.
#pragma once
#include <cuda.h>
#include <cstdint>

namespace zs {

// Bit 0: a pipeline wait gave up (see zipserv_device_flags()). All device
// code is compiled as one translation unit (zipserv_cuda.cu), so this is the
// library's single copy.
static __device__ unsigned int g_device_flags = 0;

namespace ptx {

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
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Same test, but a thread whose phase is not complete yet is suspended until
// it completes or about `hint_ns` pass, instead of returning at once: waiting
// warps then stop taking issue slots from the warps that do the work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity,
                                                    uint32_t hint_ns) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity), "r"(hint_ns)
        : "memory");
    return done != 0;
}

// Wait for the phase with the given parity to complete, suspended between
// tests. Gives up after about two seconds, sets g_device_flags bit 0 and
// returns false.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = global_timer_ns();
    do {
        if (mbar_try_wait_sleep(bar, parity, 1000000u)) return true;
    } while (global_timer_ns() - start < 2000000000ull);
    atomicOr(&g_device_flags, 1u);
    return false;
}

// Named barrier `id` (1..15; 0 is __syncthreads) over `threads` threads,
// whole warps.
__device__ __forceinline__ void named_barrier_sync(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Programmatic dependent launch: let the next kernel in the stream begin
// launching, and wait until every kernel this one depends on has completed
// and its memory is visible (a no-op when launched without the attribute).
__device__ __forceinline__ void launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void wait_prerequisites() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Global FP32 x4 store / load that bypass L1 (partial tiles exchanged
// between CTAs through L2).
__device__ __forceinline__ void stg_cg_f4(float* p, float4 v) {
    asm volatile("st.global.cg.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y),
                 "f"(v.z), "f"(v.w)
                 : "memory");
}
// Volatile (relaxed, system scope) 16-byte store and load of two 64-bit
// words, for data exchanged with other GPUs without fences: each naturally
// aligned 64-bit element is written and read whole, so a word that carries
// its own flag is either entirely old or entirely new.
__device__ __forceinline__ void st_volatile_v2u64(uint64_t* p, uint64_t a, uint64_t b) {
    asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void ld_volatile_v2u64(const uint64_t* p, uint64_t& a, uint64_t& b) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ float4 ldg_cg_f4(const float* p) {
    float4 v;
    asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}

// Bounded wait until the global word at `p` (written by other CTAs with
// release semantics) reaches `value`: acquire loads, gives up after
// `limit_ns` and returns false. With `flag` set, giving up also raises
// g_device_flags bit 0 (a wait that must not expire); without it the caller
// has a fallback for the case.
__device__ __forceinline__ bool wait_global_geq(const uint32_t* p, uint32_t value,
                                                uint64_t limit_ns = 2000000000ull,
                                                bool flag = true) {
    uint64_t start = 0;
    for (uint32_t i = 0; i < (1u << 30); ++i) {
        uint32_t v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
        if (v >= value) return true;
        if ((i & 15) == 15) {
            const uint64_t now = global_timer_ns();
            if (!start) start = now;
            else if (now - start > limit_ns) break;
            __nanosleep(64);
        }
    }
    if (flag) atomicOr(&g_device_flags, 1u);
    return false;
}
// System-scope release store and bounded acquire wait for equality (flags
// exchanged with other GPUs over NVLink). The wait gives up after limit_ns,
// raises g_device_flags bit 0 and returns false.
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ bool wait_global_eq_sys(const uint32_t* p, uint32_t value,
                                                   uint64_t limit_ns) {
    uint64_t start = 0;
    for (uint32_t i = 0; i < (1u << 30); ++i) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
        if (v == value) return true;
        if ((i & 15) == 15) {
            const uint64_t now = global_timer_ns();
            if (!start) start = now;
            else if (now - start > limit_ns) break;
            __nanosleep(64);
        }
    }
    atomicOr(&g_device_flags, 1u);
    return false;
}
// Acquire-release increment of a global counter; returns the prior value.
__device__ __forceinline__ uint32_t atom_acq_rel_add(uint32_t* p, uint32_t v) {
    uint32_t prior;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;"
                 : "=r"(prior)
                 : "l"(p), "r"(v)
                 : "memory");
    return prior;
}
// Release increment of a global counter (orders this thread's earlier writes
// before the increment for any CTA that acquires the counter).
__device__ __forceinline__ void red_release_add(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// ------------------------------------------------------------- async copies
// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
// dst and src 16-byte aligned, bytes a positive multiple of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(policy)
        : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// 2-D tiled tensor load (no multicast), completing on `bar`.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar), "l"(policy)
        : "memory");
}
// 3-D tiled tensor load (no multicast), completing on `bar`.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            int z, uint32_t bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar), "l"(policy)
        : "memory");
}
// 4-D tiled tensor load (no multicast), completing on `bar`.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            int z, int w, uint32_t bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(bar),
        "l"(policy)
        : "memory");
}
// Bitmap planes of a slot: one 4-D load when one map spans the three planes,
// else one 3-D load per plane map (plane b lands at dst + b * plane_stride).
__device__ __forceinline__ void load_planes(uint32_t dst, uint32_t plane_stride,
                                            const CUtensorMap* maps, int count, int x, int y,
                                            uint32_t bar, uint64_t policy, int lane) {
    if (count == 1) {
        if (lane == 0) tma_load_4d(dst, &maps[0], 0, x, y, 0, bar, policy);
    } else if (lane < 3) {
        tma_load_3d(dst + uint32_t(lane) * plane_stride, &maps[lane], 0, x, y, bar, policy);
    }
}
// 2-D tiled tensor store from this CTA's shared memory.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int x, int y, uint32_t src) {
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(x), "r"(y), "r"(src)
        : "memory");
}
__device__ __forceinline__ void bulk_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until at most N committed bulk groups are still reading shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ------------------------------------------------------------------ tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     dst_smem),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
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
__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
          "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (BF16 inputs, FP32
// accumulate), issued by one elected lane of a converged warp: every lane
// computes the (warp-uniform) descriptors, so they stay in uniform registers
// and the issue needs no per-lane register transfers.
__device__ __forceinline__ void mma_bf16_ss_elect(uint32_t d_tmem, uint64_t a_desc,
                                                  uint64_t b_desc, uint32_t idesc,
                                                  uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// One K slice of 64: four K = 16 MMAs (the first overwrites the accumulator
// unless `accumulate`) and a commit to `bar`, all from one elected lane of a
// converged warp. Descriptors are passed as their 32-bit halves: stepping
// 16 K elements adds AK to A's start-address field (16-byte units; 2 for a
// 128-byte-swizzled operand, 2 * LBO / 16 without swizzle) and 2 to B's
// (128-byte swizzled), which never carries out of the field for
// shared-memory addresses.
template <int AK>
__device__ __forceinline__ void mma_bf16_slice_elect(uint32_t d_tmem, uint32_t a_lo, uint32_t a_hi,
                                                     uint32_t b_lo, uint32_t b_hi, uint32_t idesc,
                                                     uint32_t accumulate, uint32_t bar) {
    asm volatile(
        "{\n\t.reg .pred e, p, q;\n\t"
        ".reg .b32 al, bl;\n\t"
        ".reg .b64 ad, bd;\n\t"
        "setp.ne.b32 p, %7, 0;\n\t"
        "setp.eq.b32 q, %7, %7;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "mov.b64 ad, {%1, %2};\n\t"
        "mov.b64 bd, {%3, %4};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], ad, bd, %5, p;\n\t"
        "add.u32 al, %1, %8;\n\t"
        "add.u32 bl, %3, 2;\n\t"
        "mov.b64 ad, {al, %2};\n\t"
        "mov.b64 bd, {bl, %4};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], ad, bd, %5, q;\n\t"
        "add.u32 al, %1, %9;\n\t"
        "add.u32 bl, %3, 4;\n\t"
        "mov.b64 ad, {al, %2};\n\t"
        "mov.b64 bd, {bl, %4};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], ad, bd, %5, q;\n\t"
        "add.u32 al, %1, %10;\n\t"
        "add.u32 bl, %3, 6;\n\t"
        "mov.b64 ad, {al, %2};\n\t"
        "mov.b64 bd, {bl, %4};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], ad, bd, %5, q;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%6];\n\t}" ::"r"(
            d_tmem),
        "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(bar), "r"(accumulate),
        "n"(AK), "n"(2 * AK), "n"(3 * AK)
        : "memory");
}
// Commit from one elected lane of a converged warp (see mma_bf16_ss_elect).
__device__ __forceinline__ void mma_commit_elect(uint32_t bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}"
        ::"r"(bar)
        : "memory");
}

// Instruction descriptor: BF16 x BF16 -> FP32, both operands K-major,
// M = 128, N = n (multiple of 16, 16..256).
__host__ __device__ constexpr uint32_t idesc_bf16_m128(uint32_t n) {
    return (1u << 4)            // D format F32
           | (1u << 7)          // A format BF16
           | (1u << 10)         // B format BF16
           | ((n >> 3) << 17)   // N / 8
           | ((128u >> 4) << 24);  // M / 16
}

// Shared-memory matrix descriptor for a K-major operand without swizzle:
// 8-row x 16-byte core matrices (rows 16 bytes apart), `lbo` bytes apart
// along K and `sbo` bytes apart along M / N.
__device__ __forceinline__ uint64_t smem_desc_kmajor(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return uint64_t((addr & 0x3FFFF) >> 4) | (uint64_t(lbo >> 4) << 16)  // LBO: K direction
           | (uint64_t(sbo >> 4) << 32)                                  // SBO: M direction
           | (uint64_t(1) << 46);                                        // version; no swizzle
}

// Shared-memory matrix descriptor for a K-major operand stored in the
// 128-byte-swizzled layout TMA writes for a 64-element (128 B) BF16 box
// width: 8-row x 128 B atoms, atoms 1024 B apart.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
    return uint64_t((addr & 0x3FFFF) >> 4) | (uint64_t(1) << 16)  // LBO (unused when swizzled)
           | (uint64_t(1024 >> 4) << 32)                            // SBO
           | (uint64_t(1) << 46)                                    // descriptor version
           | (uint64_t(2) << 61);                                   // SWIZZLE_128B
}


// ------------------------------------------------------------ shared memory
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds16(uint32_t a) {
    uint16_t v;
    asm volatile("ld.shared.b16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts8(uint32_t a, uint32_t v) {
    asm volatile("st.shared.b8 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ void sts16(uint32_t a, uint32_t v) {
    asm volatile("st.shared.b16 [%0], %1;" ::"r"(a), "h"(uint16_t(v)) : "memory");
}
__device__ __forceinline__ void sts32(uint32_t a, uint32_t v) {
    asm volatile("st.shared.b32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ void sts64(uint32_t a, int2 v) {
    asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(a), "r"(v.x), "r"(v.y) : "memory");
}
__device__ __forceinline__ void sts128(uint32_t a, uint4 v) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}

// Non-volatile shared loads: the compiler may schedule them freely, so their
// address must be data-dependent on whatever wait guards the data (see
// launder()).
__device__ __forceinline__ uint32_t lds_s32(uint32_t a) {
    uint32_t v;
    asm("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ int2 lds_s64(uint32_t a) {
    int2 v;
    asm("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds_u64(uint32_t a) {
    uint2 v;
    asm("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds_s128(uint32_t a) {
    uint4 v;
    asm("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds_u8(uint32_t a) {
    uint32_t v;
    asm("ld.shared.u8 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t a) {
    uint16_t v;
    asm("ld.shared.b16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
// Make `v` opaque to the compiler at this point in program order, so values
// (addresses) derived from it cannot be computed - and loads through them
// cannot be hoisted - above the preceding volatile asm (e.g. a barrier wait).
__device__ __forceinline__ uint32_t launder(uint32_t v) {
    asm volatile("" : "+r"(v));
    return v;
}

// Integer multiply-adds on the FMA pipe. Callers pass multipliers held in
// registers (see RowDecoder::k*), so the compiler cannot turn them into
// shifts or LEAs on the (busier) integer ALU pipe.
__device__ __forceinline__ uint32_t mad_lo(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t mul_hi(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.hi.u32 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint2 lds_v64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    return __byte_perm(a, b, sel);
}

}  // namespace ptx
}  // namespace zs
