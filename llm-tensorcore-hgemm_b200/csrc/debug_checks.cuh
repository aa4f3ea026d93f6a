// Bounds checks of the debug build (-DHGEMM_DEBUG, libhgemm_sm100_debug.so).
//
// The TMA paths are bounds-checked by the hardware (a tensor map clips every
// box to the matrix). The paths that compute global addresses themselves are
// checked here before each access: the generic (no-TMA) tile loader, the
// operand-staging copy and the epilogue's register stores. A failed check
// skips the access and records the first failure (source line and two
// indices) in a device record that hgemm_sm100_debug_read() returns; it also
// sets HGEMM_SM100_ERR_DEBUG_BOUNDS in the launch's status word where the
// kernel has one. Nothing traps. Release builds compile every check to `true`.
//
// The predicates are host/device functions so that the host library can
// expose them (hgemm_sm100_debug_check_*) for tests on the CPU.
#pragma once

#include <cstdint>

namespace hgemm {

// Row-major matrix of `rows` x `cols` elements of `esize` bytes with a pitch of
// `ld` elements at address `base`.
struct Extent {
    uintptr_t base;
    long long rows, cols, ld;
    int esize;
};

// True when the 16-byte-aligned vector at `vec` holds at least one element of
// the matrix: such a load stays inside the 16-byte blocks (and so the pages)
// that the matrix's own elements occupy. The generic loader's contract.
__host__ __device__ inline bool vec_touches_matrix(uintptr_t vec, const Extent& x) {
    if (vec % 16 != 0 || x.rows <= 0 || x.cols <= 0 || x.esize <= 0) return false;
    const long long lo = static_cast<long long>(vec) - static_cast<long long>(x.base);
    // Elements whose first byte lies in [vec, vec + 16).
    long long e0 = lo >= 0 ? (lo + x.esize - 1) / x.esize : 0;
    const long long e1 = (lo + 15) >= 0 ? (lo + 15) / x.esize : -1;
    for (long long e = e0; e <= e1; ++e) {
        const long long r = e / x.ld, c = e % x.ld;
        if (r < x.rows && c < x.cols) return true;
    }
    return false;
}

// True when the `count` consecutive elements at `ptr` are all elements of the
// matrix (one row, columns inside it). Every checked store and element load.
__host__ __device__ inline bool span_in_matrix(uintptr_t ptr, long long count, const Extent& x) {
    if (count <= 0 || x.esize <= 0 || ptr < x.base) return false;
    const long long off = static_cast<long long>(ptr - x.base);
    if (off % x.esize != 0) return false;
    const long long e = off / x.esize;
    const long long r = e / x.ld, c = e % x.ld;
    return r < x.rows && c + count <= x.cols;
}

#ifdef HGEMM_DEBUG
struct DebugRecord {
    int line;              // source line of the first failed check (0: none)
    long long index0, index1;
};
__device__ DebugRecord g_debug_record;

__device__ __noinline__ bool debug_fail(int line, long long i0, long long i1, int* status) {
    if (atomicCAS(&g_debug_record.line, 0, line) == 0) {
        g_debug_record.index0 = i0;
        g_debug_record.index1 = i1;
    }
    if (status != nullptr) atomicCAS(status, 0, 9 /* HGEMM_SM100_ERR_DEBUG_BOUNDS */);
    return false;
}
// `cond` or, when it fails, record the failure and give false (skip the access).
#define HG_DEBUG_OK(cond, i0, i1, status) \
    ((cond) ? true : ::hgemm::debug_fail(__LINE__, static_cast<long long>(i0), static_cast<long long>(i1), (status)))
#else
#define HG_DEBUG_OK(cond, i0, i1, status) true
#endif

}  // namespace hgemm
