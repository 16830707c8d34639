// ptx.cuh — thin inline-PTX wrappers for the sm_100a features the attention kernels use:
// mbarriers (with bounded waits), TMA tensor loads (no multicast anywhere), tcgen05 TMEM allocation,
// tcgen05.mma (kind::f16, one CTA), tcgen05.ld/st and the tcgen05 ordering fences.
//
// Every wait in this library is bounded: mbar_wait() gives up after a wall-clock limit (globaltimer)
// and returns false, so a kernel whose producer never arrives reports an error instead of hanging the
// GPU. Callers turn a false into a status-word flag and unwind.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>

namespace b200 {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
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
// Same, but the thread may sleep until the phase completes or suspend_ns elapse (whichever comes
// first), instead of returning at once: waiting warps then stop competing for issue slots.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity,
                                                    uint32_t suspend_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(suspend_ns)
        : "memory");
    return ok != 0;
}
// Waits for the phase with the given parity to complete. Returns false if it has not completed
// after timeout_ns of wall-clock time (the caller records the error and unwinds). Each try sleeps
// at most 100 us, so the timeout is checked at least that often.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint64_t timeout_ns) {
    const uint32_t a = smem_u32(bar);
    if (mbar_try_wait(a, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait_sleep(a, parity, 100000u)) return true;
        if (globaltimer_ns() - t0 > timeout_ns) return false;
    }
}

// Non-blocking test of a phase.
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
// Same contract as mbar_wait, for a single thread on a latency-critical chain (a pipeline whose
// stages land just in time): it polls with test_wait instead of letting the thread be suspended,
// so it resumes within a few cycles of the phase completing. The wall clock is read every 256
// polls; the bound is the same.
__device__ __forceinline__ bool mbar_wait_spin(uint64_t *bar, uint32_t parity, uint64_t timeout_ns) {
    const uint32_t a = smem_u32(bar);
    if (mbar_test_wait(a, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        for (int i = 0; i < 256; ++i)
            if (mbar_test_wait(a, parity)) return true;
        if (globaltimer_ns() - t0 > timeout_ns) return false;
    }
}

// Makes generic-proxy writes to shared memory (e.g. P tiles written by threads) visible to the
// async proxy (TMA, tcgen05.mma operands).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- TMA (tensor, no multicast)
// 3-D tiled load of one box into shared memory; completion is signalled as transaction bytes on bar.
// The innermost coordinate c0 must be a multiple of 8 (16-bit elements): the callers only pass
// multiples of 64.
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}
// 2-D tiled load of one box (no multicast); the innermost coordinate c0 is a multiple of 64 halves
// at every call site.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int c0,
                                            int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}
// Contiguous bulk copy global -> shared (no tensor map, no multicast). dst, src and bytes must be
// multiples of 16; completion is signalled as transaction bytes on bar.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// Prefetch of `bytes` contiguous bytes into L2 (16-byte aligned address and size; no shared memory, no
// completion to wait for).
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(src)),
                 "r"(bytes)
                 : "memory");
}
// Prefetch of one 3-D box into L2 (no shared memory, no completion to wait for). It only warms L2,
// which is coherent for the whole GPU, so it may run before a grid dependency wait: a later load still
// returns what the producing kernel wrote.
__device__ __forceinline__ void tma_prefetch_l2_3d(const CUtensorMap *map, int c0, int c1, int c2) {
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// 3-D tiled TMA store shared -> global (this GPU's memory only), tracked by the issuing thread's
// bulk async-group. Box rows outside the tensor map's extent are not written. The smem writes it
// reads must be made visible to the async proxy first (fence_proxy_async_smem by each writer).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, const void *src, int c0, int c1,
                                             int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until this thread's committed bulk stores have finished READING shared memory (the source
// may be overwritten); the global writes may still be in flight.
__device__ __forceinline__ void bulk_wait_group_read0() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Waits until this thread's committed bulk stores are complete (global writes performed).
__device__ __forceinline__ void bulk_wait_group0() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05: TMEM
// Warp-collective. Writes the TMEM base address of ncols columns (power of two >= 32) to *dst.
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst)),
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
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives row (lane base + t),
// columns [taddr.col, taddr.col + 32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32"
        " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15,"
        " %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
// Same shape, 16 columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32"
        " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
// 32 lanes x 64 consecutive 32-bit columns in one instruction: thread t receives row (lane base + t),
// columns [taddr.col, taddr.col + 64) as r[c / 32][c % 32].
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&r)[2][32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x64.b32"
        " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];"
        : "=r"(r[0][0]), "=r"(r[0][1]), "=r"(r[0][2]), "=r"(r[0][3]), "=r"(r[0][4]), "=r"(r[0][5]),
          "=r"(r[0][6]), "=r"(r[0][7]), "=r"(r[0][8]), "=r"(r[0][9]), "=r"(r[0][10]), "=r"(r[0][11]),
          "=r"(r[0][12]), "=r"(r[0][13]), "=r"(r[0][14]), "=r"(r[0][15]), "=r"(r[0][16]), "=r"(r[0][17]),
          "=r"(r[0][18]), "=r"(r[0][19]), "=r"(r[0][20]), "=r"(r[0][21]), "=r"(r[0][22]), "=r"(r[0][23]),
          "=r"(r[0][24]), "=r"(r[0][25]), "=r"(r[0][26]), "=r"(r[0][27]), "=r"(r[0][28]), "=r"(r[0][29]),
          "=r"(r[0][30]), "=r"(r[0][31]), "=r"(r[1][0]), "=r"(r[1][1]), "=r"(r[1][2]), "=r"(r[1][3]),
          "=r"(r[1][4]), "=r"(r[1][5]), "=r"(r[1][6]), "=r"(r[1][7]), "=r"(r[1][8]), "=r"(r[1][9]),
          "=r"(r[1][10]), "=r"(r[1][11]), "=r"(r[1][12]), "=r"(r[1][13]), "=r"(r[1][14]), "=r"(r[1][15]),
          "=r"(r[1][16]), "=r"(r[1][17]), "=r"(r[1][18]), "=r"(r[1][19]), "=r"(r[1][20]), "=r"(r[1][21]),
          "=r"(r[1][22]), "=r"(r[1][23]), "=r"(r[1][24]), "=r"(r[1][25]), "=r"(r[1][26]), "=r"(r[1][27]),
          "=r"(r[1][28]), "=r"(r[1][29]), "=r"(r[1][30]), "=r"(r[1][31])
        : "r"(taddr));
}
// 32 lanes x 64 consecutive 32-bit columns in one instruction (r[c / 16][c % 16] -> column c).
__device__ __forceinline__ void tmem_st64(uint32_t taddr, const uint32_t (&r)[4][16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x64.b32"
        " [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63, %64};"
        :: "r"(taddr),
        "r"(r[0][0]), "r"(r[0][1]), "r"(r[0][2]), "r"(r[0][3]), "r"(r[0][4]), "r"(r[0][5]),
        "r"(r[0][6]), "r"(r[0][7]), "r"(r[0][8]), "r"(r[0][9]), "r"(r[0][10]), "r"(r[0][11]),
        "r"(r[0][12]), "r"(r[0][13]), "r"(r[0][14]), "r"(r[0][15]), "r"(r[1][0]), "r"(r[1][1]),
        "r"(r[1][2]), "r"(r[1][3]), "r"(r[1][4]), "r"(r[1][5]), "r"(r[1][6]), "r"(r[1][7]),
        "r"(r[1][8]), "r"(r[1][9]), "r"(r[1][10]), "r"(r[1][11]), "r"(r[1][12]), "r"(r[1][13]),
        "r"(r[1][14]), "r"(r[1][15]), "r"(r[2][0]), "r"(r[2][1]), "r"(r[2][2]), "r"(r[2][3]),
        "r"(r[2][4]), "r"(r[2][5]), "r"(r[2][6]), "r"(r[2][7]), "r"(r[2][8]), "r"(r[2][9]),
        "r"(r[2][10]), "r"(r[2][11]), "r"(r[2][12]), "r"(r[2][13]), "r"(r[2][14]), "r"(r[2][15]),
        "r"(r[3][0]), "r"(r[3][1]), "r"(r[3][2]), "r"(r[3][3]), "r"(r[3][4]), "r"(r[3][5]),
        "r"(r[3][6]), "r"(r[3][7]), "r"(r[3][8]), "r"(r[3][9]), "r"(r[3][10]), "r"(r[3][11]),
        "r"(r[3][12]), "r"(r[3][13]), "r"(r[3][14]), "r"(r[3][15])
        : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32"
        " [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16,"
        " %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
            taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
        "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
        "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32"
        " [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(
            taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15])
        : "memory");
}

// ---------------------------------------------------------------- tcgen05: MMA
// Shared-memory matrix descriptor, 128-byte swizzle (the layout TMA writes with
// CU_TENSOR_MAP_SWIZZLE_128B for 128-byte rows). Fields: start address >> 4 in bits [0,14), leading
// byte offset >> 4 in [16,30), stride byte offset >> 4 in [32,46), descriptor version 1 at bit 46,
// layout type 2 (SWIZZLE_128B) in bits [61,64). Base offset 0: every tile starts 1024-byte aligned.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}

// Instruction descriptor for kind::f16 with fp16 A and B and fp32 accumulation:
// D format F32 (bits [4,6) = 1), A/B format F16 (0), A major bit 15, B major bit 16 (0 = K-major,
// 1 = MN-major), N >> 3 in bits [17,23), M >> 4 in bits [24,29).
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N, int a_mn_major,
                                                     int b_mn_major) {
    return (1u << 4) | (static_cast<uint32_t>(a_mn_major) << 15) |
           (static_cast<uint32_t>(b_mn_major) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread. accumulate = 0 overwrites D.
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]^T: A (M x 16 fp16, K-major) is read from TMEM, lane m = row m,
// 8 consecutive 32-bit columns holding the 16 halves as packed pairs (even element in the low half).
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Same two MMAs with the shared-memory descriptors passed as (lo, hi) words: callers keep the high
// words fixed and advance only the low word (start address), so issuing an MMA costs a 32-bit add
// rather than a full descriptor build. accumulate must be an immediate 0 or 1 after unrolling.
__device__ __forceinline__ void umma_f16_ss_lohi(uint32_t d_tmem, uint32_t a_lo, uint32_t a_hi,
                                                 uint32_t b_lo, uint32_t b_hi, uint32_t idesc,
                                                 uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t.reg .b64 da, db;\n\t"
        "mov.b64 da, {%1, %2};\n\t"
        "mov.b64 db, {%3, %4};\n\t"
        "setp.ne.b32 p, %6, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %5, p;\n\t}" ::"r"(d_tmem),
        "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_f16_ts_lohi(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo,
                                                 uint32_t b_hi, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t.reg .b64 db;\n\t"
        "mov.b64 db, {%2, %3};\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], db, %4, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrives once on bar when every tcgen05.mma previously issued by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// ---------------------------------------------------------------- thread-block clusters
// Rank of this CTA in its cluster (0 for a launch without clusters).
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Hardware barrier over every thread of every CTA in the cluster; release/acquire order the
// shared-memory writes before it with the distributed shared-memory reads after it. Executed by all
// threads of each CTA, like __syncthreads.
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
                 "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The two halves of cluster_sync_all, for a barrier whose wait comes long after the arrival. The
// arrival is relaxed: a thread whose earlier shared-memory writes peers must see after their wait
// issues fence_cluster() first (mbarrier initialisation is published by fence_mbar_init).
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void fence_cluster() {
    asm volatile("fence.acq_rel.cluster;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Remote 16-byte store into another CTA's shared memory (cluster address) that signals its bytes
// on an mbarrier in that CTA (cluster address): the receiver waits on its own barrier, the sender
// never waits.
__device__ __forceinline__ void st_async_v4(uint32_t cluster_saddr, float4 v, uint32_t cluster_bar) {
    asm volatile(
        "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
            cluster_saddr),
        "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(cluster_bar)
        : "memory");
}
__device__ __forceinline__ void st_async_v2(uint32_t cluster_saddr, float a, float b, uint32_t cluster_bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(
                     cluster_saddr),
                 "f"(a), "f"(b), "r"(cluster_bar)
                 : "memory");
}
// Address of the same shared-memory location in the CTA of cluster rank `rank`.
__device__ __forceinline__ uint32_t dsmem_addr(uint32_t local_saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_saddr), "r"(rank));
    return r;
}
// Loads from this CTA's shared memory by shared-window address.
__device__ __forceinline__ float4 lds_v4(uint32_t saddr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(saddr)
                 : "memory");
    return v;
}
__device__ __forceinline__ float2 lds_v2(uint32_t saddr) {
    float2 v;
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(saddr) : "memory");
    return v;
}

// One lane of the (fully converged) warp is elected: true there, false on the other 31. Code that
// runs on the whole warp and lets only the elected lane issue keeps its operands warp-uniform.
__device__ __forceinline__ bool elect_one() {
    uint32_t e;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "elect.sync _|p, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(e));
    return e != 0;
}

// ---------------------------------------------------------------- per-warpgroup register budget
// Executed by all 128 threads of a warpgroup: lowers / raises the registers each of its threads may
// use. Raises wait until other warpgroups of the CTA have released enough, so a split must add up to
// what the CTA was launched with.
template <uint32_t N>
__device__ __forceinline__ void reg_dealloc() {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void reg_alloc() {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

// ---------------------------------------------------------------- programmatic dependent launch
// Waits until the grids this one depends on (launched with programmatic stream serialization) have
// completed and their memory is visible; a no-op for an ordinary launch.
__device__ __forceinline__ void grid_dependency_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
// Lets the dependent grid start launching (its CTAs still wait in grid_dependency_wait for this
// grid's completion before reading what it writes).
__device__ __forceinline__ void grid_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- math
// Hardware base-2 exponential (MUFU.EX2), flush-to-zero; ex2(-inf) = +0.
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// acc + (float)half_k(packed) with the sm_100 mixed-precision add (one instruction, no convert).
__device__ __forceinline__ float add_f16lo_f32(uint32_t packed, float acc) {
    float r;
    asm("{\n\t.reg .f16 lo, hi;\n\tmov.b32 {lo, hi}, %1;\n\tadd.f32.f16 %0, lo, %2;\n\t}"
        : "=f"(r)
        : "r"(packed), "f"(acc));
    return r;
}
__device__ __forceinline__ float add_f16hi_f32(uint32_t packed, float acc) {
    float r;
    asm("{\n\t.reg .f16 lo, hi;\n\tmov.b32 {lo, hi}, %1;\n\tadd.f32.f16 %0, hi, %2;\n\t}"
        : "=f"(r)
        : "r"(packed), "f"(acc));
    return r;
}

// Two fp32 lanes in one instruction (sm_100 packed fp32): (x, y) as one 64-bit register pair.
__device__ __forceinline__ uint64_t pair_f32(float x, float y) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(x), "f"(y));
    return r;
}
// (ax * b.x + c.x, ay * b.y + c.y)
__device__ __forceinline__ void fma2_f32(float &dx, float &dy, float ax, float ay, uint64_t b, uint64_t c) {
    asm("{\n\t.reg .b64 a, d;\n\tmov.b64 a, {%2, %3};\n\tfma.rn.f32x2 d, a, %4, %5;\n\tmov.b64 {%0, %1}, d;\n\t}"
        : "=f"(dx), "=f"(dy)
        : "f"(ax), "f"(ay), "l"(b), "l"(c));
}

// max(a, b, c) in one instruction (sm_100 three-input max).
__device__ __forceinline__ float max3f(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

}  // namespace b200
