// Inline-PTX building blocks for the sm_100a HGEMM kernels: mbarriers with
// bounded waits, TMA tile loads, tcgen05 (TMEM allocation, MMA, commit,
// TMEM -> register loads), UMMA shared-memory / instruction descriptors and
// thread-block-cluster helpers.
//
// These replace the SM80 wrappers the reference kernels are built on
// (ldmatrix / mma.sync in csrc/common/layout.cuh:35-88 and cp.async in
// csrc/common/async_copy.cuh:14-54 of the reference). Every TMA load here
// brings one CTA's own operand tile into that CTA's shared memory.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace hgemm {

// ---------------------------------------------------------------- basics ---

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t warp_index() {
    return __shfl_sync(0xffffffffu, threadIdx.x / 32, 0);
}

// ------------------------------------------------------------- mbarriers ---

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

// Makes barrier initialisation visible to the async proxy (TMA, tcgen05) and
// to the other CTAs of the cluster.
__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Error codes a kernel writes into its status word. They mirror the C-ABI's
// HGEMM_SM100_ERR_* values.
enum : int {
    kStatusOk = 0,
    kStatusPipelineTimeout = 5,
};

// Wait-state shared by the warps of one CTA. A wait that runs past its time
// limit raises `abort`; every other wait in the CTA sees the flag and gives up
// too, so that all roles reach the teardown in bounded time.
struct WaitCtl {
    volatile int* abort;      // shared-memory flag
    int* status;              // device status word (may be null)
    uint64_t timeout_ns;
};

__device__ __forceinline__ void raise_abort(const WaitCtl& w, int code) {
    *w.abort = 1;
    if (w.status != nullptr) atomicCAS(w.status, 0, code);
}

// Bounded wait on an mbarrier phase. Returns false when the limit ran out or
// when another role of this CTA already gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, const WaitCtl& w) {
    const uint32_t a = smem_addr(bar);
    if (mbar_try_wait(a, parity)) return true;
    const uint64_t start = global_timer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(a, parity)) return true;
        if ((i & 31u) == 0) {
            if (*w.abort) return false;
            if (global_timer_ns() - start > w.timeout_ns) {
                raise_abort(w, kStatusPipelineTimeout);
                return false;
            }
        }
    }
}

// Wait used on teardown paths only: bounded, never raises the abort flag.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
    const uint32_t a = smem_addr(bar);
    const uint64_t start = global_timer_ns();
    while (!mbar_try_wait(a, parity)) {
        if (global_timer_ns() - start > limit_ns) return false;
    }
    return true;
}

// ------------------------------------------------------------------- TMA ---

__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled bulk-tensor load global -> this CTA's shared memory; completion is
// reported as transaction bytes on `bar`. `x` is the innermost coordinate.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];"
        ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)),
          "r"(x), "r"(y)
        : "memory");
}

// Untiled bulk copy global -> this CTA's shared memory (addresses 16-byte
// aligned, size a multiple of 16); completion as transaction bytes on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// 2-D tiled TMA store this CTA's shared memory -> global (out-of-range parts
// of the box are not written). Tracked by the issuing thread's bulk groups.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int32_t x, int32_t y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(src)), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until at most N of this thread's bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Waits until all of this thread's bulk groups have completed.
__device__ __forceinline__ void bulk_wait_group_all() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (tcgen05 / TMA) reads of the same memory.
__device__ __forceinline__ void fence_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Orders this thread's generic-proxy and async-proxy (bulk copy) accesses to
// global memory.
__device__ __forceinline__ void fence_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Untiled bulk copy this CTA's shared memory -> global (addresses 16-byte
// aligned, size a multiple of 16), tracked by the bulk async-group.
__device__ __forceinline__ void bulk_store(void* dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
                 ::"l"(reinterpret_cast<uint64_t>(dst)), "r"(smem_addr(src)), "r"(bytes)
                 : "memory");
}

// Programmatic dependent launch. launch_dependents lets the next grid of
// the stream be scheduled before this one ends; wait blocks until the grids
// this one depends on have completed and their memory is visible (a no-op
// for a launch without that dependency).
__device__ __forceinline__ void grid_dependents_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void grid_dependency_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Barrier among the 128 threads of warps 0-3 (named barrier 1).
__device__ __forceinline__ void epilogue_bar_sync() {
    asm volatile("bar.sync 1, 128;" ::: "memory");
}

// --------------------------------------------------------------- tcgen05 ---

// Allocates `ncols` TMEM columns (power of two, 32..512); must be executed by
// one whole warp. The TMEM address is written to `*slot` in shared memory.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_addr(slot)), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]; FP16 inputs, FP32 accumulation.
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives (once) on `bar` when every tcgen05 operation this thread issued so
// far has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives
// lane (taddr.lane + t), columns taddr.col .. taddr.col + 31.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
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

// 32 lanes x 16 columns (used when the accumulator is only 16 columns wide).
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

// ----------------------------------------------------------- descriptors ---

// Shared-memory matrix descriptor (tcgen05 "matrix descriptor"):
//   bits  0-13 start address >> 4      bits 16-29 leading byte offset >> 4
//   bits 32-45 stride byte offset >> 4 bits 46-47 version (1 on sm_100)
//   bits 49-51 base offset (0: atoms are 1024-byte aligned)
//   bits 61-63 layout: 2 = 128-byte swizzle
// For a K-major operand in 128-byte swizzle the tile is rows of 128 bytes
// (64 halves of K), 8-row groups 1024 bytes apart: SBO = 1024, LBO unused.
// For an MN-major operand the tile is K-rows of 128 bytes (64 halves of M/N)
// in 8-row, 1024-byte groups (SBO) and 64-wide M/N chunks LBO bytes apart.
__device__ __forceinline__ uint64_t make_smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(2) << 61;
    return d;
}

// Instruction descriptor for kind::f16 with FP16 A/B and FP32 accumulation.
//   bits 4-5 D format (1 = F32)   bits 7-9 / 10-12 A / B format (0 = F16)
//   bit 15 A major (1 = MN)       bit 16 B major (1 = MN)
//   bits 17-22 N >> 3             bits 24-28 M >> 4
__host__ __device__ constexpr uint32_t make_idesc_f16(int m, int n, bool a_mn_major, bool b_mn_major) {
    return (1u << 4) | (static_cast<uint32_t>(a_mn_major) << 15) |
           (static_cast<uint32_t>(b_mn_major) << 16) |
           (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// Byte offset of the 16-byte chunk `chunk` (0..7) of row `row` inside a
// 128-byte-swizzled tile whose base is 1024-byte aligned (the layout TMA
// writes for CU_TENSOR_MAP_SWIZZLE_128B).
__device__ __forceinline__ uint32_t swz128(uint32_t row, uint32_t byte_in_row) {
    return row * 128u + ((((byte_in_row >> 4) ^ (row & 7u)) << 4) | (byte_in_row & 15u));
}

// ------------------------------------------------- CTA-pair (cta_group::2) ---
// A pair of CTAs (cluster of 2) shares one MMA: the even CTA issues
// tcgen05.mma.cta_group::2 with M = 256, reading rows 0-127 of A and columns
// 0..N/2-1 of B from its own shared memory and the rest from the odd CTA's
// shared memory at the same offsets; each CTA's TMEM receives its 128 rows.

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_addr(slot)), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_mma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrives once on the mbarrier at shared::cluster address `bar` (this CTA's
// or the peer's) when this thread's prior cta_group::2 MMAs have completed.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(bar) : "memory");
}

// One commit that arrives once on the mbarrier at the same shared-memory
// offset `bar` in both CTAs of the pair (CTA mask 0b11) when this thread's
// prior cta_group::2 MMAs have completed. Replaces a commit per CTA: each
// commit costs the MMA-issuing thread time between MMA batches (measured: one
// commit per stage instead of two made the 256x256 pair kernel 3-4 % faster).
__device__ __forceinline__ void tc_commit_pair_both(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
                 ::"r"(bar), "h"(static_cast<uint16_t>(0x3)) : "memory");
}

// 2-D tiled TMA load into this CTA's shared memory whose transaction bytes
// complete on `bar`, an mbarrier of either CTA of the pair (shared::cluster
// address). Used so that both CTAs' tiles complete on the MMA CTA's barrier.
// Only this CTA's own tile is written.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar,
                                                 int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];"
        ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

// Sleeps about `ns` nanoseconds (teardown after an aborted pipeline only).
__device__ __forceinline__ void settle_ns(uint64_t ns) {
    const uint64_t start = global_timer_ns();
    while (global_timer_ns() - start < ns) __nanosleep(1000);
}

// Arrive on an mbarrier of another CTA of the cluster (release, cluster scope).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait with cluster-scope acquire (the barrier is completed by
// arrivals or commits from the other CTA of the pair).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, const WaitCtl& w) {
    const uint32_t a = smem_addr(bar);
    if (mbar_try_wait_cluster(a, parity)) return true;
    const uint64_t start = global_timer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait_cluster(a, parity)) return true;
        if ((i & 31u) == 0) {
            if (*w.abort) return false;
            if (global_timer_ns() - start > w.timeout_ns) {
                raise_abort(w, kStatusPipelineTimeout);
                return false;
            }
        }
    }
}

// --------------------------------------------------------------- cluster ---

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
                 "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}

// Stores to the shared memory of another CTA of the cluster (shared::cluster
// address from map_to_rank); they complete asynchronously and become visible
// to that CTA after a cluster barrier.
__device__ __forceinline__ void st_dsmem_f4(uint32_t addr, float a, float b, float c, float d) {
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
                 : "memory");
}
__device__ __forceinline__ void st_dsmem_f32(uint32_t addr, float a) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(a) : "memory");
}

// ----------------------------------------------------------- conversions ---

__device__ __forceinline__ uint32_t pack_half2(uint32_t lo_bits, uint32_t hi_bits) {
    __half2 h = __floats2half2_rn(__uint_as_float(lo_bits), __uint_as_float(hi_bits));
    return *reinterpret_cast<uint32_t*>(&h);
}

}  // namespace hgemm
