// sm_100a HGEMM kernels: C[M,N] = A[M,K] @ B[K,N], FP16 in, FP32 accumulate
// in TMEM, FP16 out, all row-major, alpha = 1, beta = 0.
//
// They replace the reference's kernel family (csrc/v1..v6 of the reference;
// its best, mma_async_kernel in csrc/v6_mma_async.cu:226-403, is a two-stage
// cp.async + mma.sync pipeline). Four kernel templates cover every shape:
//
//  * hgemm_persistent_kernel: one CTA per SM walks 128 x BN output tiles in
//    grouped raster order. Warp 4 streams A/B tiles with TMA into a STAGES-deep
//    shared-memory ring (full/empty mbarriers), one thread of warp 5 issues
//    tcgen05.mma into one of two TMEM accumulators, warps 0-3 drain the other
//    accumulator (tcgen05.ld -> FP16 -> global) while the next tile's MMAs run.
//
//  * hgemm_pair_kernel: the same persistent scheme on clusters of two CTAs
//    whose even CTA issues tcgen05.mma.cta_group::2 over both CTAs' tiles.
//
//  * hgemm_streamk_kernel: persistent whole-tile waves, then the remaining
//    tiles' K blocks cut into equal ranges per CTA, partial tiles combined in
//    a fixed order through the caller's workspace.
//
//  * hgemm_tile_kernel: one output tile per CTA, optionally split over K across
//    the CTAs of a thread-block cluster whose FP32 partials are summed in a
//    fixed order (through the workspace, or distributed shared memory when
//    the caller gives none).
//    kSwap computes C^T = B^T A^T so that a few activation rows (decode) sit
//    on the MMA's N side while 128 weight columns fill the MMA's M side.
//    kTma = false replaces TMA with loads by warps 0-3 (aligned 16-byte
//    vectors shifted into place, elements outside the matrix zero) for
//    operands whose strides or base addresses TMA cannot describe (the role
//    the reference gives its v5 scalar fallback, csrc/v6_mma_async.cu:428-437).
//
// Operand tiles in shared memory use the 128-byte swizzle that TMA writes:
//  * the K-major tile ("Kmaj", from a row-major [rows x K] matrix) holds rows
//    of 64 halves of K, 128 bytes each;
//  * the MN-major tile ("MNmaj", from a row-major [K x cols] matrix) holds
//    64-wide column chunks, each 64 K-rows of 128 bytes (8 KiB per chunk).
// Every mbarrier wait is bounded; when one runs out the CTA records
// HGEMM_SM100_ERR_PIPELINE_TIMEOUT in the status word, all roles give up,
// in-flight copies and MMAs are drained (also bounded) and TMEM is freed.
#pragma once

#include "debug_checks.cuh"
#include "sm100_ptx.cuh"

namespace hgemm {

constexpr int kBlockK = 64;            // K per pipeline stage (one 128-byte swizzle row)
constexpr int kMmaM = 128;             // UMMA M (rows of the accumulator = TMEM lanes)
constexpr int kThreads = 192;          // warps 0-3 epilogue, 4 TMA producer, 5 MMA issuer
constexpr uint32_t kChunkBytes = 64u * 128u;  // one 64-wide MN-major chunk of a stage
constexpr uint64_t kDrainLimitNs = 200ull * 1000ull * 1000ull;

__host__ __device__ constexpr uint32_t cmax(uint32_t a, uint32_t b) { return a > b ? a : b; }
__host__ __device__ constexpr uint32_t tmem_cols_for(uint32_t n) {
    return n <= 32 ? 32 : (n <= 64 ? 64 : (n <= 128 ? 128 : (n <= 256 ? 256 : 512)));
}

// Rounds the dynamic shared-memory window up to the 1024-byte alignment the
// 128-byte swizzle atoms need.
__device__ __forceinline__ uint8_t* align_1024(uint8_t* p) {
    const uint32_t a = smem_addr(p);
    return p + (((a + 1023u) & ~1023u) - a);
}

struct GemmParams {
    const __half* a;       // [M, lda]
    const __half* b;       // [K, ldb]
    void* c;               // [M, ldc], FP16 (or FP32 when out_f32)
    int m, n, k;
    long long lda, ldb, ldc;
    int vec_ok;            // C base 16-byte aligned and ldc % 8 == 0
    int tma_store;         // persistent/pair kernels: store C tiles with TMA (FP16, vec_ok)
    int out_f32;           // store FP32 instead of FP16 (tensor-parallel partials)
    int group_m;           // persistent kernel: M-tiles per raster group
    int inject;            // test-only: arm the first stage with 16 extra bytes
    int* status;
    unsigned long long timeout_ns;
    // Stream-K (hgemm_streamk_kernel only): FP32 partial tiles and their
    // readiness flags in the caller's workspace, one slot per CTA.
    float* partials;
    unsigned long long* flags;
    unsigned long long epoch;  // this launch's flag value (never 0)
    int streamk;               // 1: stream-K k-ranges, 0: whole tiles
    // Fused epilogue (kEpi* bits; 0 = plain store). Applied once, by whoever
    // stores the final FP32 sum of an output element: split-K and stream-K
    // partials stay raw.
    int epi;
    int epi_vec;               // bias and residual 16-byte aligned, ldr % 8 == 0
    const __half* bias;        // [n] (kEpiBias), indexed by accumulator column
    const __half* residual;    // [m, ldr] (kEpiResidual)
    long long ldr;
    // Row scatter of an FP32 partial (tensor-parallel down-projection): with
    // sc_ranks > 0, output row i goes to slot sc_rank of the receive buffer of
    // rank q = i / sc_rows, sc_dest[q] (a peer GPU's memory for q != sc_rank),
    // at row i - q * sc_rows of that slot.
    int sc_ranks, sc_rank, sc_rows;
    int sc_bulk;               // rows leave through cp.async.bulk (persistent and pair kernels)
    long long sc_ld;
    float* sc_dest[8];
};

// Epilogue bits. With kEpiSiluMul the accumulator columns come in (gate, up)
// pairs 2j, 2j + 1 and output column j = silu(gate) * up: C is [m, n / 2].
constexpr int kEpiBias = 1;
constexpr int kEpiResidual = 2;
constexpr int kEpiSiluMul = 4;

// Debug builds: the `count` consecutive output elements at `ptr` (output
// row `row`, column `col`) lie inside C. Scatter destinations (peer buffers)
// are not checked. Release builds: always true.
__device__ __forceinline__ bool c_span_ok(const GemmParams& p, const void* ptr, long long count, int row, int col) {
#ifdef HGEMM_DEBUG
    if (p.sc_ranks > 0) return true;
    const Extent x{reinterpret_cast<uintptr_t>(p.c), p.m, (p.epi & kEpiSiluMul) ? p.n / 2 : p.n, p.ldc,
                   p.out_f32 ? 4 : 2};
    return HG_DEBUG_OK(span_in_matrix(reinterpret_cast<uintptr_t>(ptr), count, x), row, col, p.status);
#else
    (void)p; (void)ptr; (void)count; (void)row; (void)col;
    return true;
#endif
}

// Start of FP32 output row `row` (< m): C, or its scatter destination.
__device__ __forceinline__ float* f32_row(const GemmParams& p, int row) {
    if (p.sc_ranks > 0) {
        const int q = row / p.sc_rows;
        return p.sc_dest[q] + (static_cast<long long>(p.sc_rank) * p.sc_rows + (row - q * p.sc_rows)) * p.sc_ld;
    }
    return static_cast<float*>(p.c) + static_cast<long long>(row) * p.ldc;
}

// ------------------------------------------------------------ epilogue ----

// silu(g) * u = g / (1 + e^-g) * u in FP32 (for g -> -inf the quotient goes to
// -0, as the limit does).
__device__ __forceinline__ float silu_mul(float g, float u) { return __fdividef(g, 1.f + __expf(-g)) * u; }

// Swapped tiles hold the (gate, up) columns of one output column in lanes
// 2i (gate) and 2i + 1 (up), rows j in registers. For the row pair (j, j + 1)
// held as (v0, v1), one exchange gives the even lane (gate, up) of row j and
// the odd lane (gate, up) of row j + 1. Called by all 32 lanes together.
__device__ __forceinline__ void silu_pair(uint32_t v0, uint32_t v1, int odd, float& g, float& u) {
    const float send = __uint_as_float(odd ? v0 : v1);
    const float recv = __shfl_xor_sync(0xffffffffu, send, 1);
    g = odd ? recv : __uint_as_float(v0);
    u = odd ? __uint_as_float(v1) : recv;
}

// Adds kCnt FP16 values src[0 .. kCnt) (only the first `avail` when not
// `vec`) to the FP32 bit patterns v. With `vec`, src is aligned to
// 2 * kCnt bytes (16 at most): one 8-byte load for kCnt = 4, 16-byte loads
// for multiples of 8.
template <int kCnt>
__device__ __forceinline__ void add_halves(const __half* src, bool vec, int avail, uint32_t* v) {
    static_assert(kCnt == 4 || kCnt % 8 == 0, "segment of 4 or a multiple of 8 columns");
    if (vec) {
        if constexpr (kCnt == 4) {
            const uint2 q = __ldg(reinterpret_cast<const uint2*>(src));
            const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&q.x));
            const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&q.y));
            v[0] = __float_as_uint(__uint_as_float(v[0]) + f0.x);
            v[1] = __float_as_uint(__uint_as_float(v[1]) + f0.y);
            v[2] = __float_as_uint(__uint_as_float(v[2]) + f1.x);
            v[3] = __float_as_uint(__uint_as_float(v[3]) + f1.y);
        } else {
#pragma unroll
            for (int i = 0; i < kCnt; i += 8) {
                const uint4 q = __ldg(reinterpret_cast<const uint4*>(src + i));
                const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
                    v[i + 2 * j] = __float_as_uint(__uint_as_float(v[i + 2 * j]) + f.x);
                    v[i + 2 * j + 1] = __float_as_uint(__uint_as_float(v[i + 2 * j + 1]) + f.y);
                }
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < kCnt; ++i)
            if (i < avail) v[i] = __float_as_uint(__uint_as_float(v[i]) + __half2float(src[i]));
    }
}

// Bias and residual terms of kCnt consecutive accumulator columns col0 .. of
// output row `row`, added in place (no-op without those epilogue bits).
template <int kCnt>
__device__ __forceinline__ void epi_add_row(const GemmParams& p, int row, int col0, uint32_t* v) {
    if ((p.epi & (kEpiBias | kEpiResidual)) == 0 || col0 >= p.n) return;
    const bool vec = p.epi_vec && col0 + kCnt <= p.n;
    if (p.epi & kEpiBias) add_halves<kCnt>(p.bias + col0, vec, p.n - col0, v);
    if ((p.epi & kEpiResidual) && row < p.m)
        add_halves<kCnt>(p.residual + static_cast<long long>(row) * p.ldr + col0, vec, p.n - col0, v);
}

// Swapped tiles: one accumulator row = output column `col`, kCnt accumulator
// columns = output rows row0 .. row0 + kCnt - 1.
template <int kCnt>
__device__ __forceinline__ void epi_add_col(const GemmParams& p, int col, int row0, uint32_t* v) {
    if ((p.epi & (kEpiBias | kEpiResidual)) == 0 || col >= p.n) return;
    const float bias = (p.epi & kEpiBias) ? __half2float(p.bias[col]) : 0.f;
#pragma unroll
    for (int j = 0; j < kCnt; ++j) {
        float x = __uint_as_float(v[j]) + bias;
        if ((p.epi & kEpiResidual) && row0 + j < p.m)
            x += __half2float(p.residual[static_cast<long long>(row0 + j) * p.ldr + col]);
        v[j] = __float_as_uint(x);
    }
}

// Stores `cnt` (16 or 32) consecutive accumulator columns of one output row.
template <int kCnt>
__device__ __forceinline__ void store_row_segment(const GemmParams& p, int row, int col0,
                                                  const uint32_t* vin) {
    if (row >= p.m) return;
    uint32_t v[kCnt];
#pragma unroll
    for (int i = 0; i < kCnt; ++i) v[i] = vin[i];
    epi_add_row<kCnt>(p, row, col0, v);
    if (p.epi & kEpiSiluMul) {
        // col0 is a multiple of 16: output columns col0 / 2 .. (8-aligned).
        __half* crow = static_cast<__half*>(p.c) + static_cast<long long>(row) * p.ldc + (col0 >> 1);
        if (p.vec_ok && col0 + kCnt <= p.n) {
#pragma unroll
            for (int i = 0; i < kCnt; i += 16) {
                uint4 q;
                q.x = pack_half2(__float_as_uint(silu_mul(__uint_as_float(v[i + 0]), __uint_as_float(v[i + 1]))),
                                 __float_as_uint(silu_mul(__uint_as_float(v[i + 2]), __uint_as_float(v[i + 3]))));
                q.y = pack_half2(__float_as_uint(silu_mul(__uint_as_float(v[i + 4]), __uint_as_float(v[i + 5]))),
                                 __float_as_uint(silu_mul(__uint_as_float(v[i + 6]), __uint_as_float(v[i + 7]))));
                q.z = pack_half2(__float_as_uint(silu_mul(__uint_as_float(v[i + 8]), __uint_as_float(v[i + 9]))),
                                 __float_as_uint(silu_mul(__uint_as_float(v[i + 10]), __uint_as_float(v[i + 11]))));
                q.w = pack_half2(__float_as_uint(silu_mul(__uint_as_float(v[i + 12]), __uint_as_float(v[i + 13]))),
                                 __float_as_uint(silu_mul(__uint_as_float(v[i + 14]), __uint_as_float(v[i + 15]))));
                if (c_span_ok(p, crow + (i >> 1), 8, row, (col0 + i) >> 1))
                    *reinterpret_cast<uint4*>(crow + (i >> 1)) = q;
            }
        } else {
#pragma unroll
            for (int i = 0; i < kCnt; i += 2)
                if (col0 + i < p.n && c_span_ok(p, crow + (i >> 1), 1, row, (col0 + i) >> 1))
                    crow[i >> 1] = __float2half_rn(silu_mul(__uint_as_float(v[i]), __uint_as_float(v[i + 1])));
        }
        return;
    }
    if (p.out_f32) {
        float* crow = f32_row(p, row);
        if (p.vec_ok && col0 + kCnt <= p.n) {
#pragma unroll
            for (int i = 0; i < kCnt; i += 4)
                if (c_span_ok(p, crow + col0 + i, 4, row, col0 + i))
                    *reinterpret_cast<uint4*>(crow + col0 + i) = make_uint4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        } else {
#pragma unroll
            for (int i = 0; i < kCnt; ++i)
                if (col0 + i < p.n && c_span_ok(p, crow + col0 + i, 1, row, col0 + i)) crow[col0 + i] = __uint_as_float(v[i]);
        }
        return;
    }
    __half* crow = static_cast<__half*>(p.c) + static_cast<long long>(row) * p.ldc;
    if (p.vec_ok && col0 + kCnt <= p.n) {
#pragma unroll
        for (int i = 0; i < kCnt; i += 8) {
            uint4 q;
            q.x = pack_half2(v[i + 0], v[i + 1]);
            q.y = pack_half2(v[i + 2], v[i + 3]);
            q.z = pack_half2(v[i + 4], v[i + 5]);
            q.w = pack_half2(v[i + 6], v[i + 7]);
            if (c_span_ok(p, crow + col0 + i, 8, row, col0 + i)) *reinterpret_cast<uint4*>(crow + col0 + i) = q;
        }
    } else {
#pragma unroll
        for (int i = 0; i < kCnt; ++i)
            if (col0 + i < p.n && c_span_ok(p, crow + col0 + i, 1, row, col0 + i))
                crow[col0 + i] = __float2half_rn(__uint_as_float(v[i]));
    }
}

// FP32 rows of a row scatter through shared memory: the warp's 32 x 32 block
// (lane l = row row0 + l, v = its columns col0 .. col0 + 31) is transposed
// through `box` (4 KB, element (r, c) at r * 32 + (c ^ r): conflict-free both
// ways) so that each store instruction writes 32 consecutive floats of one
// row: whole 128-byte lines for the stores that cross NVLink, instead of 32
// rows' 16-byte pieces. All 32 lanes call it together.
__device__ __forceinline__ void store_block_f32(const GemmParams& p, float* box, uint32_t lane, const uint32_t* v,
                                                int row0, int col0) {
    __syncwarp();
#pragma unroll
    for (int c = 0; c < 32; ++c) box[lane * 32u + (static_cast<uint32_t>(c) ^ lane)] = __uint_as_float(v[c]);
    __syncwarp();
    const int col = col0 + static_cast<int>(lane);
#pragma unroll 4
    for (int r = 0; r < 32; ++r) {
        const int row = row0 + r;
        if (row < p.m && col < p.n) f32_row(p, row)[col] = box[r * 32 + static_cast<int>(lane ^ static_cast<uint32_t>(r))];
    }
    __syncwarp();
}

// The same block through the bulk-copy engine: each lane stages its row
// (128 bytes, row-major) in one of the warp's two 4 KB buffers and hands it to
// cp.async.bulk (shared -> global; the row's owner may be a peer GPU), so the
// rows leave the SM as asynchronous bulk transfers rather than LSU stores.
// A buffer is rewritten only after the copies that read it two blocks ago have
// read it (each lane commits one bulk group per block). Needs 16-byte-aligned
// destination rows and n % 4 == 0 (p.sc_bulk).
__device__ __forceinline__ void store_block_f32_bulk(const GemmParams& p, uint8_t* bufs, uint32_t& buf,
                                                     uint32_t lane, const uint32_t* v, int row0, int col0) {
    float* row_buf = reinterpret_cast<float*>(bufs + buf * 4096u) + lane * 32u;
    bulk_wait_group_read<1>();
#pragma unroll
    for (int c = 0; c < 32; c += 4)
        *reinterpret_cast<uint4*>(row_buf + c) = make_uint4(v[c], v[c + 1], v[c + 2], v[c + 3]);
    fence_async_shared();
    const int row = row0 + static_cast<int>(lane);
    const int cols = min(32, p.n - col0);
    if (row < p.m && cols > 0) bulk_store(f32_row(p, row) + col0, row_buf, static_cast<uint32_t>(cols) * 4u);
    bulk_commit_group();
    buf ^= 1u;
}

// Swapped tiles: accumulator row = output column `col`, accumulator columns =
// output rows row0 .. row0 + cnt - 1. Called by all 32 lanes of a warp
// together, lane l holding column col0 + l for a 32-aligned col0.
template <int kCnt>
__device__ __forceinline__ void store_col_segment(const GemmParams& p, int col, int row0,
                                                  const uint32_t* vin) {
    uint32_t v[kCnt];
#pragma unroll
    for (int j = 0; j < kCnt; ++j) v[j] = vin[j];
    epi_add_col<kCnt>(p, col, row0, v);
    if (p.epi & kEpiSiluMul) {
        // The (gate, up) pair of output column col / 2 sits in lanes 2i, 2i + 1;
        // of each two output rows the even lane finishes the first, the odd
        // lane the second.
        const int odd = col & 1;
#pragma unroll
        for (int j = 0; j < kCnt; j += 2) {
            float g, u;
            silu_pair(v[j], v[j + 1], odd, g, u);
            const int row = row0 + j + odd;
            __half* dst = static_cast<__half*>(p.c) + static_cast<long long>(row) * p.ldc + (col >> 1);
            if (col < p.n && row < p.m && c_span_ok(p, dst, 1, row, col >> 1)) *dst = __float2half_rn(silu_mul(g, u));
        }
        return;
    }
    if (col >= p.n) return;
#pragma unroll
    for (int j = 0; j < kCnt; ++j) {
        const int row = row0 + j;
        if (row < p.m) {
            if (p.out_f32) {
                float* dst = f32_row(p, row) + col;
                if (c_span_ok(p, dst, 1, row, col)) *dst = __uint_as_float(v[j]);
            } else {
                __half* dst = static_cast<__half*>(p.c) + static_cast<long long>(row) * p.ldc + col;
                if (c_span_ok(p, dst, 1, row, col)) *dst = __float2half_rn(__uint_as_float(v[j]));
            }
        }
    }
}

// Bias + residual terms of output (row, col .. col + 3) as FP32 (zero
// without those epilogue bits or outside C); col a multiple of 4.
__device__ __forceinline__ float4 epi_terms_quad(const GemmParams& p, int row, int col) {
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    epi_add_row<4>(p, row, col, w);
    return make_float4(__uint_as_float(w[0]), __uint_as_float(w[1]), __uint_as_float(w[2]), __uint_as_float(w[3]));
}

// Stores 4 consecutive output columns of one row from an FP32 quad (col a
// multiple of 4). With `terms_added` the caller has added the bias and
// residual terms already (epi_terms_quad).
__device__ __forceinline__ void store_quad(const GemmParams& p, int row, int col, float4 v,
                                           bool terms_added = false) {
    if (row >= p.m || col >= p.n) return;
    if (p.epi) {
        if (!terms_added) {
            const float4 t = epi_terms_quad(p, row, col);
            v.x += t.x; v.y += t.y; v.z += t.z; v.w += t.w;
        }
        if (p.epi & kEpiSiluMul) {
            __half* c = static_cast<__half*>(p.c) + static_cast<long long>(row) * p.ldc + (col >> 1);
            const float h0 = silu_mul(v.x, v.y), h1 = silu_mul(v.z, v.w);
            if (p.vec_ok && col + 4 <= p.n) {
                if (c_span_ok(p, c, 2, row, col >> 1)) *reinterpret_cast<__half2*>(c) = __floats2half2_rn(h0, h1);
            } else {
                if (c_span_ok(p, c, 1, row, col >> 1)) c[0] = __float2half_rn(h0);
                if (col + 2 < p.n && c_span_ok(p, c + 1, 1, row, (col >> 1) + 1)) c[1] = __float2half_rn(h1);
            }
            return;
        }
    }
    const long long off = static_cast<long long>(row) * p.ldc + col;
    if (p.out_f32) {
        float* c = f32_row(p, row) + col;
        if (p.vec_ok && col + 4 <= p.n) {
            if (c_span_ok(p, c, 4, row, col)) *reinterpret_cast<float4*>(c) = v;
        } else {
            const int cnt = min(4, p.n - col);
            if (c_span_ok(p, c, cnt, row, col)) {
                c[0] = v.x;
                if (col + 1 < p.n) c[1] = v.y;
                if (col + 2 < p.n) c[2] = v.z;
                if (col + 3 < p.n) c[3] = v.w;
            }
        }
        return;
    }
    __half* c = static_cast<__half*>(p.c) + off;
    if (p.vec_ok && col + 4 <= p.n) {
        uint2 q;
        q.x = pack_half2(__float_as_uint(v.x), __float_as_uint(v.y));
        q.y = pack_half2(__float_as_uint(v.z), __float_as_uint(v.w));
        if (c_span_ok(p, c, 4, row, col)) *reinterpret_cast<uint2*>(c) = q;
    } else if (c_span_ok(p, c, min(4, p.n - col), row, col)) {
        c[0] = __float2half_rn(v.x);
        if (col + 1 < p.n) c[1] = __float2half_rn(v.y);
        if (col + 2 < p.n) c[2] = __float2half_rn(v.z);
        if (col + 3 < p.n) c[3] = __float2half_rn(v.w);
    }
}

// TMA-store epilogue: converts 64 accumulator columns of this warp's 32 rows
// (lane = row) to FP16 in a 128-byte-swizzled 32 x 64 shared-memory box and
// lane 0 stores the box with TMA at output (x = col0, y = row0). `buf`
// alternates between two boxes per warp; before a box is rewritten, the
// store that read it two boxes ago must have finished reading.
__device__ __forceinline__ void store_box_tma(const CUtensorMap* map, uint8_t* box, uint32_t lane,
                                              const uint32_t* v0, const uint32_t* v1, int col0, int row0) {
    if (lane == 0) bulk_wait_group_read<1>();
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t* v = j < 4 ? v0 + 8 * j : v1 + 8 * (j - 4);
        uint4 q;
        q.x = pack_half2(v[0], v[1]);
        q.y = pack_half2(v[2], v[3]);
        q.z = pack_half2(v[4], v[5]);
        q.w = pack_half2(v[6], v[7]);
        *reinterpret_cast<uint4*>(box + lane * 128u + ((static_cast<uint32_t>(j) ^ (lane & 7u)) << 4)) = q;
    }
    fence_async_shared();
    __syncwarp();
    if (lane == 0) {
        tma_store_2d(map, box, col0, row0);
        bulk_commit_group();
    }
}

// Swapped-tile epilogue box: kRows output rows (accumulator columns) x 32
// output columns (the warp's 32 accumulator rows); lane l holds column
// n0 + l, v[j] for row m0 + j. Staged densely ([row][32] halves, 64-byte
// rows, unswizzled map) and written by one TMA store (which clips at the
// matrix edges). Double-buffered per warp like store_box_tma.
// With `silu` (the SwiGLU epilogue) lanes 2i, 2i + 1 hold a (gate, up) pair:
// the box is kRows x 16 output columns starting at n0 / 2.
template <int kRows>
__device__ __forceinline__ void store_box_tma_t(const CUtensorMap* map, uint8_t* box, uint32_t lane,
                                                const uint32_t* v, int n0, int m0, bool silu = false) {
    if (lane == 0) bulk_wait_group_read<1>();
    __syncwarp();
    __half* h = reinterpret_cast<__half*>(box);
    if (silu) {
        const int odd = static_cast<int>(lane & 1u);
#pragma unroll
        for (int j = 0; j < kRows; j += 2) {
            float g, u;
            silu_pair(v[j], v[j + 1], odd, g, u);
            h[(j + odd) * 16 + (lane >> 1)] = __float2half_rn(silu_mul(g, u));
        }
    } else {
#pragma unroll
        for (int j = 0; j < kRows; ++j) h[j * 32 + lane] = __float2half_rn(__uint_as_float(v[j]));
    }
    fence_async_shared();
    __syncwarp();
    if (lane == 0) {
        tma_store_2d(map, box, silu ? n0 / 2 : n0, m0);
        bulk_commit_group();
    }
}

// ------------------------------------------------- generic tile loaders ----
//
// Operands TMA cannot describe (a base that is not 16-byte aligned, a pitch
// that is not a multiple of 8 halves) reach the generic tile kernel with only
// their element (2-byte) alignment. Its loader threads move 8-element pieces
// (one 16-byte unit of the swizzled tile): each piece's bytes lie in at most
// two 16-byte-aligned vectors, which are loaded whole and shifted into place.
// A vector is loaded only when it holds an element of the operand, so no load
// reaches outside the 16-byte blocks - and so the pages - that the operand's
// own elements occupy; elements outside the matrix read as zero.

struct Piece8 {
    uint4 v0, v1;   // the aligned vector holding the first element, and the next one
    uint32_t off;   // byte offset of the first element inside v0 (even)
    int nv;         // elements of the piece inside the matrix (<= 0: none)
};

// `ext` is the operand (debug builds check that each loaded vector holds one
// of its elements; `i0`, `i1` are the piece's row and column for the record).
__device__ __forceinline__ Piece8 fetch_piece8(const __half* x, int nv, const Extent& ext, int i0, int i1,
                                               int* status) {
    Piece8 r;
    r.v0 = make_uint4(0u, 0u, 0u, 0u);
    r.v1 = r.v0;
    const uintptr_t a = reinterpret_cast<uintptr_t>(x);
    r.off = static_cast<uint32_t>(a & 15u);
    r.nv = nv;
    const uint4* v = reinterpret_cast<const uint4*>(a - r.off);
    (void)ext; (void)i0; (void)i1; (void)status;
    if (nv > 0 && HG_DEBUG_OK(vec_touches_matrix(reinterpret_cast<uintptr_t>(v), ext), i0, i1, status))
        r.v0 = __ldg(v);
    // v1 starts at element (16 - off) / 2 of the piece.
    if (r.off != 0u && nv > static_cast<int>((16u - r.off) >> 1) &&
        HG_DEBUG_OK(vec_touches_matrix(reinterpret_cast<uintptr_t>(v + 1), ext), i0, i1, status))
        r.v1 = __ldg(v + 1);
    return r;
}

// The piece's 8 elements as one 16-byte unit (little-endian halves), missing
// elements zero.
__device__ __forceinline__ uint4 assemble_piece8(const Piece8& r) {
    const uint32_t w[8] = {r.v0.x, r.v0.y, r.v0.z, r.v0.w, r.v1.x, r.v1.y, r.v1.z, r.v1.w};
    const uint32_t q = r.off >> 2;               // first word holding a wanted half
    const bool odd_half = (r.off & 2u) != 0u;    // it starts in that word's upper half
    uint32_t s[5];
#pragma unroll
    for (int i = 0; i < 5; ++i) s[i] = q == 0 ? w[i] : q == 1 ? w[i + 1] : q == 2 ? w[i + 2] : w[i + 3];
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t v = odd_half ? __funnelshift_r(s[i], s[i + 1], 16) : s[i];
        const uint32_t keep = (2 * i + 1 < r.nv) ? 0xffffffffu : (2 * i < r.nv) ? 0x0000ffffu : 0u;
        o[i] = v & keep;
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// One stage of the generic tile kernel, by 128 cooperating threads: the
// K-major tile (rows r0 .. r0 + kKRows - 1 of A, K range k0 .. k0 + 63) and the
// MN-major tile (K rows k0 .. k0 + 63 of B, columns c0 .. c0 + kMNCols - 1), in
// the 128-byte-swizzled layout TMA would write. All of a thread's loads are
// issued before its shared-memory stores.
template <int kKRows, int kMNCols>
__device__ __forceinline__ void load_stage_generic(uint8_t* s_k, uint8_t* s_mn, const GemmParams& p, int r0,
                                                   int c0, int k0, int tid) {
    constexpr int kKPieces = kKRows * 8 / 128;          // pieces per thread
    constexpr int kPerRow = kMNCols / 8;
    constexpr int kMNPieces = 64 * kPerRow / 128;
    static_assert(kKRows * 8 % 128 == 0 && 64 * kPerRow % 128 == 0, "whole pieces per thread");
    Piece8 pk[kKPieces], pm[kMNPieces];
    const Extent ext_a{reinterpret_cast<uintptr_t>(p.a), p.m, p.k, p.lda, 2};
    const Extent ext_b{reinterpret_cast<uintptr_t>(p.b), p.k, p.n, p.ldb, 2};
#pragma unroll
    for (int j = 0; j < kKPieces; ++j) {
        const int idx = tid + 128 * j;
        const int gr = r0 + (idx >> 3), gk = k0 + 8 * (idx & 7);
        const int nv = gr < p.m ? min(p.k - gk, 8) : 0;
        pk[j] = fetch_piece8(p.a + static_cast<long long>(gr) * p.lda + gk, nv, ext_a, gr, gk, p.status);
    }
#pragma unroll
    for (int j = 0; j < kMNPieces; ++j) {
        const int idx = tid + 128 * j;
        const int gk = k0 + idx / kPerRow, gc = c0 + 8 * (idx % kPerRow);
        const int nv = gk < p.k ? min(p.n - gc, 8) : 0;
        pm[j] = fetch_piece8(p.b + static_cast<long long>(gk) * p.ldb + gc, nv, ext_b, gk, gc, p.status);
    }
#pragma unroll
    for (int j = 0; j < kKPieces; ++j) {
        const int idx = tid + 128 * j;
        *reinterpret_cast<uint4*>(s_k + swz128(idx >> 3, (idx & 7) * 16)) = assemble_piece8(pk[j]);
    }
#pragma unroll
    for (int j = 0; j < kMNPieces; ++j) {
        const int idx = tid + 128 * j;
        const int kk = idx / kPerRow, c = 8 * (idx % kPerRow);
        *reinterpret_cast<uint4*>(s_mn + (c >> 6) * kChunkBytes + swz128(kk, (c & 63) * 2)) = assemble_piece8(pm[j]);
    }
}

// ---------------------------------------------------- operand staging ----

// Copies a row-major FP16 [rows x cols] matrix between row pitches. Grid y
// walks rows, grid x and the threads walk 8-element column chunks, so a warp
// covers 256 consecutive elements of one row on both sides (coalesced).
// kDstAligned: the destination base is 16-byte aligned and its pitch a
// multiple of 8, so each thread writes one 16-byte vector (zero-filling the
// row padding); otherwise the destination is written element by element and
// the source (then the aligned side) read as one 16-byte vector.
template <bool kDstAligned>
__global__ void __launch_bounds__(256)
copy_rows_kernel(const __half* __restrict__ src, long long ld_src, __half* __restrict__ dst,
                 long long ld_dst, long long rows, long long cols) {
    const long long col_step = static_cast<long long>(gridDim.x) * blockDim.x * 8;
    // Debug builds: reads stay inside the source rows (the aligned source of
    // a copy-back is the padded staging buffer, its whole pitch owned), writes
    // inside the destination rows (likewise).
    const Extent xs{reinterpret_cast<uintptr_t>(src), rows, kDstAligned ? cols : ld_src, ld_src, 2};
    const Extent xd{reinterpret_cast<uintptr_t>(dst), rows, kDstAligned ? ld_dst : cols, ld_dst, 2};
    (void)xs; (void)xd;
    for (long long r = blockIdx.y; r < rows; r += gridDim.y) {
        const __half* srow = src + r * ld_src;
        __half* drow = dst + r * ld_dst;
        for (long long c = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 8; c < cols;
             c += col_step) {
            __align__(16) __half v[8];
            if constexpr (kDstAligned) {
                if (!HG_DEBUG_OK(span_in_matrix(reinterpret_cast<uintptr_t>(srow + c), min(8LL, cols - c), xs) &&
                                     span_in_matrix(reinterpret_cast<uintptr_t>(drow + c), 8, xd),
                                 r, c, nullptr))
                    continue;
                if (c + 8 <= cols) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) v[j] = __ldg(srow + c + j);
                } else {
#pragma unroll
                    for (int j = 0; j < 8; ++j) v[j] = (c + j < cols) ? __ldg(srow + c + j) : __float2half_rn(0.f);
                }
                *reinterpret_cast<uint4*>(drow + c) = *reinterpret_cast<const uint4*>(v);
            } else {
                if (!HG_DEBUG_OK(span_in_matrix(reinterpret_cast<uintptr_t>(srow + c), 8, xs) &&
                                     span_in_matrix(reinterpret_cast<uintptr_t>(drow + c), min(8LL, cols - c), xd),
                                 r, c, nullptr))
                    continue;
                *reinterpret_cast<uint4*>(v) = __ldg(reinterpret_cast<const uint4*>(srow + c));
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    if (c + j < cols) drow[c + j] = v[j];
            }
        }
    }
}

// ---------------------------------------------------------- descriptors ----

__device__ __forceinline__ uint64_t kmaj_desc(uint32_t tile, int kk) {
    return make_smem_desc(tile + kk * 32u, 16u, 1024u);
}
__device__ __forceinline__ uint64_t mnmaj_desc(uint32_t tile, int kk) {
    return make_smem_desc(tile + kk * 2048u, kChunkBytes, 1024u);
}

// Waits for the last armed phase of every used stage's full barrier, so that
// no TMA write into this CTA's shared memory is still in flight at exit.
// A producer that owns every kStep-th stage from `which` on (kStages a
// multiple of kStep) and armed `issued` loads in order drains its own stages.
// Owner side of the tensor-parallel row scatter: out[j][c] = FP16 of the FP32
// sum of slots[s][j][c] over s = 0 .. ranks - 1, added in that order (one
// rounding), written to every destination of `outs` (with the peers' copies
// of these rows among them, an all-gather). Grid-stride over rows x column
// groups; kVec: cols, ld_slots and ld_out multiples of 4 with 16- / 8-byte-
// aligned bases, one float4 per slot per step. Streaming loads: the slots are
// read once.
// Up to 8 FP16 destinations of one reduction (this GPU's output and its
// peers' copies of the same rows).
struct SlotOutputs {
    __half* ptr[8];
    int count;
};

template <bool kVec>
__global__ void __launch_bounds__(256) reduce_slots_kernel(const float* __restrict__ slots, int ranks,
                                                           long long rows, long long cols, long long ld_slots,
                                                           SlotOutputs outs, long long ld_out) {
    const long long slot_stride = rows * ld_slots;
    const long long per_row = kVec ? cols / 4 : cols;
    const long long total = rows * per_row;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long r = i / per_row;
        const long long c = (i - r * per_row) * (kVec ? 4 : 1);
        const float* src = slots + r * ld_slots + c;
        if constexpr (kVec) {
            float4 acc = __ldcs(reinterpret_cast<const float4*>(src));
            for (int s = 1; s < ranks; ++s) {
                const float4 x = __ldcs(reinterpret_cast<const float4*>(src + s * slot_stride));
                acc.x += x.x; acc.y += x.y; acc.z += x.z; acc.w += x.w;
            }
            uint2 q;
            q.x = pack_half2(__float_as_uint(acc.x), __float_as_uint(acc.y));
            q.y = pack_half2(__float_as_uint(acc.z), __float_as_uint(acc.w));
            for (int o = 0; o < outs.count; ++o) *reinterpret_cast<uint2*>(outs.ptr[o] + r * ld_out + c) = q;
        } else {
            float acc = __ldcs(src);
            for (int s = 1; s < ranks; ++s) acc += __ldcs(src + s * slot_stride);
            const __half h = __float2half_rn(acc);
            for (int o = 0; o < outs.count; ++o) outs.ptr[o][r * ld_out + c] = h;
        }
    }
}

template <int kStages, int kStep = 1>
__device__ __forceinline__ void drain_tma(uint64_t* full, uint32_t issued, uint32_t which = 0) {
    constexpr uint32_t kOwn = kStages / kStep;
    const uint32_t used = issued < kOwn ? issued : kOwn;
    for (uint32_t t = 0; t < used; ++t) {
        const uint32_t arms = issued / kOwn + (t < issued % kOwn ? 1u : 0u);
        mbar_wait_drain(&full[which + kStep * t], (arms - 1u) & 1u, kDrainLimitNs);
    }
}

// ========================================================== tile kernel ====

template <int kBNm, bool kSwap, bool kTma, int kStages>
struct TileCfg {
    static constexpr int kKRows = kSwap ? kBNm : kMmaM;     // rows of the K-major tile
    static constexpr int kMNCols = kSwap ? kMmaM : kBNm;    // cols of the MN-major tile
    // Two TMA producers and two MMA issuers with an accumulator each for
    // tiles of at most 128 columns fed by TMA (see the kernel); one of each
    // otherwise. Each producer owns the stages of one parity.
    static constexpr bool kDual = kTma && kBNm <= 128;
    // K per stage. A stage holds kKB / 64 K-major atoms of kKRows x 64
    // halves, and per 64-column MN-major chunk kKB rows. (128-deep stages -
    // 8 MMAs per barrier hand-off - measured no faster than 64-deep ones
    // with twice the ring depth once the tile runs two producers and two
    // issuers.)
    static constexpr int kKB = 64;
    static constexpr uint32_t kKAtomBytes = kKRows * 128u;
    static constexpr uint32_t kMNChunkBytes = kKB * 128u;
    static constexpr uint32_t kKBytes = kKAtomBytes * (kKB / 64);
    static constexpr uint32_t kMNBytes = (kMNCols / 64) * kMNChunkBytes;
    static constexpr uint32_t kStageBytes = kKBytes + kMNBytes;
    // Split-K receive buffer (FP32): accumulator rows are divided among the
    // CTAs of the cluster in whole quads of 4 rows (rank r owns rows from
    // 4 * (r * 32 / split)); CTA o receives, from every rank s, the rows it
    // owns: [s][local row][kBNm + 4] or, swapped, [s][col][local row] (the
    // output's contiguous dimension contiguous, quads 16-byte aligned). Rows
    // per rank <= 4 * ceil(32 / split); over split 2..16,
    // split * 4 * ceil(32 / split) <= 180. The buffer reuses the stage ring
    // once every CTA's MMAs are done.
    static constexpr uint32_t kRecvBytes = kSwap ? 180u * kBNm * 4u : 180u * (kBNm + 4) * 4u;
    static constexpr uint32_t kRecvOff = 0u;
    // Workspace exchange: one FP32 tile per CTA, staged in the stage ring.
    static constexpr uint32_t kSlotFloats = kSwap ? 128u * kBNm : 128u * (kBNm + 4);
    static_assert(kSlotFloats * 4u <= kStages * kStageBytes, "staging fits the stage ring");
    static_assert(kSwap || kStages * kStageBytes >= 4u * 8192u, "TMA-store boxes fit the stage ring");
    static constexpr uint32_t kDataBytes = cmax(kStages * kStageBytes, kRecvBytes);
    static constexpr uint32_t kBarBytes = 256;
    static constexpr uint32_t kSmemBytes = kDataBytes + kBarBytes + 1024;
    static_assert(!kDual || kStages % 2 == 0, "dual producers own alternate stages");
    static constexpr uint32_t kTmemCols = tmem_cols_for(kDual ? 2 * kBNm : kBNm);
    static constexpr uint32_t kIdesc = make_idesc_f16(kMmaM, kBNm, kSwap, !kSwap);
    static constexpr int kChunk = kBNm >= 32 ? 32 : 16;     // columns per tcgen05.ld
    static_assert(kKRows % 8 == 0, "K-major tile rows must fill 8-row swizzle atoms");
    static_assert(kMNCols % 64 == 0, "MN-major tile must be whole 64-wide chunks");
    static_assert(kBNm % 16 == 0 && kBNm >= 16 && kBNm <= 256, "UMMA N for M=128");
    static_assert(2 * kStages + 4 <= 30, "barrier area");
    static_assert(kSmemBytes <= 232448, "shared memory");
};

// Loads kCnt accumulator columns at TMEM address t (the warp's lane base
// included); with `two`, adds the second accumulator at t + off. Warp-uniform.
template <int kCnt>
__device__ __forceinline__ void tmem_ld_acc(uint32_t t, uint32_t off, bool two, uint32_t (&v)[kCnt]) {
    if constexpr (kCnt == 32) {
        tmem_ld_32x32b_x32(t, v);
    } else {
        tmem_ld_32x32b_x16(t, v);
    }
    if (two) {
        uint32_t w[kCnt];
        if constexpr (kCnt == 32) {
            tmem_ld_32x32b_x32(t + off, w);
        } else {
            tmem_ld_32x32b_x16(t + off, w);
        }
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < kCnt; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) + __uint_as_float(w[j]));
    } else {
        tmem_wait_ld();
    }
}

// Split-K reduction of the rows this CTA owns (first .. first + nrows - 1 of
// the accumulator tile) from the receive buffer, summed over ranks
// 0..split-1 in order, stored to C. Receive layouts: [rank][local row][kBNm
// + 4] floats, rank stride nrows_max rows; swapped [rank][col][local row],
// rank stride kBNm * nrows_max, column stride sw_stride. All threads of the
// CTA take part.
template <int kBNm, bool kSwap>
__device__ __forceinline__ void reduce_owned_rows(const GemmParams& p, const float* recv, int split, int nrows,
                                                  int nrows_max, int sw_stride, int first, int acc_row0,
                                                  int acc_col0) {
    // kU independent items per thread per step (loads of all of them are in
    // flight together); out-of-range item slots load item 0 and store nothing.
    constexpr int kU = 4;
    const int rank_stride = kSwap ? kBNm * nrows_max : nrows_max * (kBNm + 4);
    // Fast store path: FP16, 16-byte-aligned rows, tile inside C.
    const int rows_total = kSwap ? p.n : p.m;
    const int cols_total = kSwap ? p.m : p.n;
    const bool has_terms = (p.epi & (kEpiBias | kEpiResidual)) != 0;
    const bool fast = !p.out_f32 && !p.epi && p.vec_ok && acc_row0 + first + nrows <= rows_total && acc_col0 + kBNm <= cols_total;
    const int quads = nrows >> 2;                         // nrows is a multiple of 4
    const int total = kSwap ? kBNm * quads : nrows * (kBNm / 4);
    for (int base = threadIdx.x; base < total; base += kU * kThreads) {
        float4 acc[kU];
        int off[kU], row[kU], col[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int it = base + u * kThreads < total ? base + u * kThreads : 0;
            if constexpr (kSwap) {
                // (output row m = accumulator column, 4 consecutive n)
                const int m = it / quads, lq = (it - m * quads) * 4;
                off[u] = m * sw_stride + lq;
                row[u] = acc_col0 + m;
                col[u] = acc_row0 + first + lq;
            } else {
                constexpr int kQ = kBNm / 4;
                const int lr = it / kQ, cq = (it - lr * kQ) * 4;
                off[u] = lr * (kBNm + 4) + cq;
                row[u] = acc_row0 + first + lr;
                col[u] = acc_col0 + cq;
            }
            acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        // Bias / residual terms, loaded together with the partials (their
        // latency overlaps the partial loads instead of following the sum).
        float4 terms[kU];
        if (has_terms) {
#pragma unroll
            for (int u = 0; u < kU; ++u) terms[u] = epi_terms_quad(p, row[u], col[u]);
        }
        for (int s = 0; s < split; ++s) {
            const float* rs = recv + s * rank_stride;
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const float4 x = *reinterpret_cast<const float4*>(rs + off[u]);
                acc[u].x += x.x; acc[u].y += x.y; acc[u].z += x.z; acc[u].w += x.w;
            }
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            if (base + u * kThreads >= total) break;
            if (fast) {
                uint2 q;
                q.x = pack_half2(__float_as_uint(acc[u].x), __float_as_uint(acc[u].y));
                q.y = pack_half2(__float_as_uint(acc[u].z), __float_as_uint(acc[u].w));
                *reinterpret_cast<uint2*>(static_cast<__half*>(p.c) + static_cast<long long>(row[u]) * p.ldc +
                                          col[u]) = q;
            } else {
                if (has_terms) {
                    acc[u].x += terms[u].x; acc[u].y += terms[u].y; acc[u].z += terms[u].z; acc[u].w += terms[u].w;
                }
                store_quad(p, row[u], col[u], acc[u], true);
            }
        }
    }
}

// Grid: x = 128-row accumulator tiles (M tiles, or N tiles when swapped),
// y = kBNm-wide accumulator column tiles, z = K splits (== cluster size).
template <int kBNm, bool kSwap, bool kTma, int kStages>
__global__ void __launch_bounds__(kThreads, 1)
hgemm_tile_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_mn,
                  const __grid_constant__ CUtensorMap tm_c, const GemmParams p) {
    using Cfg = TileCfg<kBNm, kSwap, kTma, kStages>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align_1024(smem_raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kDataBytes);
    uint64_t* empty = full + kStages;
    uint64_t* tfull = empty + kStages;
    uint64_t* drain = tfull + 1;           // [2], one per MMA issuer
    uint64_t* xfer = drain + 2;            // split-K partial rows landed (workspace exchange)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xfer + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const uint32_t warp = warp_index();
    const uint32_t lane = threadIdx.x & 31u;

    if (warp == 4 && lane == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], kTma ? 1u : 128u);
            mbar_init(&empty[s], 1u);
        }
        mbar_init(tfull, Cfg::kDual ? 2u : 1u);
        mbar_init(&drain[0], 1u);
        mbar_init(&drain[1], 1u);
        mbar_init(xfer, 1u);
        *abort_flag = 0;
        mbar_init_fence();
        if (kTma) {
            tma_prefetch_map(&tm_k);
            tma_prefetch_map(&tm_mn);
        }
    }
    if (warp == 5) {
        tmem_alloc(tmem_slot, Cfg::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem_base = *tmem_slot;
    // The set-up above touches only this CTA's shared memory and TMEM, so it
    // may overlap the previous kernel of the stream; global memory is only
    // touched after that kernel has completed.
    grid_dependents_launch();
    grid_dependency_wait();
    const WaitCtl wc{abort_flag, p.status, p.timeout_ns};

    const int acc_row0 = blockIdx.x * kMmaM;   // accumulator rows (M, or N when swapped)
    const int acc_col0 = blockIdx.y * kBNm;    // accumulator cols (N, or M when swapped)
    const int k_rows0 = kSwap ? acc_col0 : acc_row0;   // first A row of the K-major tile
    const int mn_cols0 = kSwap ? acc_row0 : acc_col0;  // first B column of the MN-major tile
    const int nkb = (p.k + Cfg::kKB - 1) / Cfg::kKB;   // K blocks of this kernel
    const int split = gridDim.z;
    const int kb0 = static_cast<int>(blockIdx.z) * nkb / split;
    const int kb1 = (static_cast<int>(blockIdx.z) + 1) * nkb / split;

    // --------------------------------------------------------- producers --
    // A producer thread's barrier waits and copy issues take a few hundred
    // cycles per K block; with narrow tiles that is more than the MMAs, so
    // kDual tiles use two producers: lane 0 of warp 4 loads the even K blocks
    // (even stages), lane 0 of warp 2 (idle until the epilogue) the odd ones.
    if (kTma) {
        if (lane == 0 && (warp == 4 || (Cfg::kDual && warp == 2))) {
            const int which = warp == 4 ? 0 : 1;
            constexpr int kStep = Cfg::kDual ? 2 : 1;
            uint32_t issued = 0;
            bool ok = true;
            for (int kb = kb0 + which; kb < kb1; kb += kStep) {
                const int i = kb - kb0;
                const uint32_t stage = static_cast<uint32_t>(i % kStages);
                const uint32_t phase = static_cast<uint32_t>(i / kStages) & 1u;
                if (!mbar_wait(&empty[stage], phase ^ 1u, wc)) { ok = false; break; }
                uint8_t* s_k = smem + stage * Cfg::kStageBytes;
                uint8_t* s_mn = s_k + Cfg::kKBytes;
                const uint32_t extra = (p.inject && kb == kb0) ? 16u : 0u;
                mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes + extra);
#pragma unroll
                for (int h = 0; h < Cfg::kKB / 64; ++h) {
                    const int k0 = kb * Cfg::kKB + 64 * h;
                    tma_load_2d(s_k + h * Cfg::kKAtomBytes, &tm_k, &full[stage], k0, k_rows0);
#pragma unroll
                    for (int j = 0; j < Cfg::kMNCols / 64; ++j)
                        tma_load_2d(s_mn + j * Cfg::kMNChunkBytes + h * kChunkBytes, &tm_mn, &full[stage],
                                    mn_cols0 + 64 * j, k0);
                }
                ++issued;
            }
            if (!ok || *abort_flag) drain_tma<kStages, kStep>(full, issued, static_cast<uint32_t>(which));
        }
    } else if (warp < 4) {
        const int tid = threadIdx.x;
        uint32_t stage = 0, phase = 0;
        for (int kb = kb0; kb < kb1; ++kb) {
            if (!mbar_wait(&empty[stage], phase ^ 1u, wc)) break;
            uint8_t* s_k = smem + stage * Cfg::kStageBytes;
            uint8_t* s_mn = s_k + Cfg::kKBytes;
            load_stage_generic<Cfg::kKRows, Cfg::kMNCols>(s_k, s_mn, p, k_rows0, mn_cols0, kb * kBlockK, tid);
            fence_async_shared();
            mbar_arrive(&full[stage]);
            if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
    }

    // ------------------------------------------------------ MMA issuers --
    // One thread issues a K block's MMAs and commits the block's stage. An
    // issuer's barrier wait leaves the tensor pipe idle for a few hundred
    // cycles, which the 64-cycle MMAs of a narrow tile cannot cover, so tiles
    // of at most 128 columns use two issuers: lane 0 of warp 5 takes the even
    // K blocks into accumulator 0, lane 0 of warp 3 (idle until the epilogue)
    // the odd ones into accumulator 1, and each fills the other's gaps. The
    // epilogue adds the two accumulators (fixed order: deterministic).
    if (lane == 0 && (warp == 5 || (Cfg::kDual && warp == 3))) {
        const int which = warp == 5 ? 0 : 1;
        constexpr int kStep = Cfg::kDual ? 2 : 1;
        const uint32_t d = tmem_base + static_cast<uint32_t>(which * kBNm);
        bool ok = true, first = true;
        for (int kb = kb0 + which; kb < kb1; kb += kStep) {
            const int i = kb - kb0;
            const uint32_t stage = static_cast<uint32_t>(i % kStages);
            const uint32_t phase = static_cast<uint32_t>(i / kStages) & 1u;
            if (!mbar_wait(&full[stage], phase, wc)) { ok = false; break; }
            tc_fence_after_sync();
            const uint32_t s_k = smem_addr(smem + stage * Cfg::kStageBytes);
            const uint32_t s_mn = s_k + Cfg::kKBytes;
#pragma unroll
            for (int kk = 0; kk < Cfg::kKB / 16; ++kk) {
                const uint64_t dk = make_smem_desc(s_k + (kk >> 2) * Cfg::kKAtomBytes + (kk & 3) * 32u, 16u, 1024u);
                const uint64_t dmn = make_smem_desc(s_mn + kk * 2048u, Cfg::kMNChunkBytes, 1024u);
                tc_mma_f16(d, kSwap ? dmn : dk, kSwap ? dk : dmn, Cfg::kIdesc, (!first || kk > 0) ? 1u : 0u);
            }
            first = false;
            tc_commit(&empty[stage]);
        }
        if (ok) {
            tc_commit(tfull);
        } else {
            tc_commit(&drain[which]);
            mbar_wait_drain(&drain[which], 0, kDrainLimitNs);
        }
    }
    __syncwarp();
    // Accumulator 1 holds data only when its issuer had a K block.
    const bool two = Cfg::kDual && kb1 - kb0 >= 2;

    // --------------------------------------------------------- epilogue --
    // Without a split the accumulator goes to C: through per-warp shared-memory
    // boxes and TMA stores when C allows it (p.tma_store), else with direct
    // stores. With a K split the accumulator rows are divided among the CTAs
    // of the cluster in whole quads (rank r owns rows from 4 * (r * 32 / split));
    // each CTA sums its rows over ranks 0..split-1 in rank order
    // (deterministic) and stores them. The partial tiles travel
    //  * through the caller's workspace when there is one (p.partials): each
    //    CTA stages its FP32 tile in shared memory, grouped by owning rank,
    //    copies it to its workspace slot with one bulk copy and, after a
    //    cluster barrier, bulk-loads the rows it owns from every rank's slot;
    //  * else through distributed shared memory: every CTA pushes each row
    //    into the receive buffer of its owner with remote stores, and one
    //    cluster barrier makes them visible.
    // The stage ring is idle once tfull has completed (every MMA has read its
    // operands), so boxes, staging and receive buffers reuse it.
    const bool split_k = split > 1;
    const bool via_l2 = split_k && p.partials != nullptr;
    const uint32_t rank = cluster_ctarank();
    const int nrows_max = 4 * ((32 + split - 1) / split);   // rows owned per rank, bound
    const int first = 4 * (static_cast<int>(rank) * 32 / split);          // multiple of 4
    const int nrows = 4 * ((static_cast<int>(rank) + 1) * 32 / split) - first;
    // Swapped receive layout [rank][col][local row]: column stride.
    const int sw_stride = via_l2 ? nrows : nrows_max;
    volatile int* xchg_go = abort_flag + 1;   // workspace exchange proceeds
    bool ok = false;
    if (warp < 4) {
        // Warp-uniform: tcgen05.ld below is .sync.aligned.
        ok = __all_sync(0xffffffffu, mbar_wait(tfull, 0, wc));
        tc_fence_after_sync();
    }
    // Push receive buffers inside the stage ring: every CTA's MMAs must be
    // done (its tfull observed above) before anyone writes into it.
    if (split_k && !via_l2) cluster_sync();
    if (warp < 4) {
        if (ok) {
            const int r = warp * 32 + lane;   // accumulator row = TMEM lane
            const uint32_t t_row = tmem_base + ((warp * 32u) << 16);
            const int owner = ((r >> 2) * split + split - 1) >> 5;
            const int o_first = 4 * (owner * 32 / split);
            const int lr = r - o_first;
            if (!split_k && p.tma_store) {
                uint8_t* boxes = smem + warp * 8192u;
                uint32_t buf = 0;
                if constexpr (kSwap) {
#pragma unroll 1
                    for (int c = 0; c < kBNm; c += Cfg::kChunk) {
                        uint32_t v[Cfg::kChunk];
                        tmem_ld_acc<Cfg::kChunk>(t_row + c, kBNm, two, v);
                        epi_add_col<Cfg::kChunk>(p, acc_row0 + r, acc_col0 + c, v);
                        store_box_tma_t<Cfg::kChunk>(&tm_c, boxes + buf * 2048u, lane, v,
                                                     acc_row0 + static_cast<int>(warp) * 32, acc_col0 + c,
                                                     (p.epi & kEpiSiluMul) != 0);
                        buf ^= 1u;
                    }
                } else {
#pragma unroll 1
                    for (int c = 0; c < kBNm; c += 64) {
                        uint32_t v0[32], v1[32];
                        tmem_ld_acc<32>(t_row + c, kBNm, two, v0);
                        tmem_ld_acc<32>(t_row + c + 32, kBNm, two, v1);
                        epi_add_row<32>(p, acc_row0 + r, acc_col0 + c, v0);
                        epi_add_row<32>(p, acc_row0 + r, acc_col0 + c + 32, v1);
                        store_box_tma(&tm_c, boxes + buf * 4096u, lane, v0, v1, acc_col0 + c,
                                      acc_row0 + static_cast<int>(warp) * 32);
                        buf ^= 1u;
                    }
                }
                if (lane == 0) bulk_wait_group_all();
            } else {
                float* stage_f = reinterpret_cast<float*>(smem);
                const uint32_t recv = map_to_rank(smem_addr(smem + Cfg::kRecvOff), owner);
                const int o_rows = 4 * ((owner + 1) * 32 / split) - o_first;
#pragma unroll 1
                for (int c = 0; c < kBNm; c += Cfg::kChunk) {
                    uint32_t v[Cfg::kChunk];
                    tmem_ld_acc<Cfg::kChunk>(t_row + c, kBNm, two, v);
                    if (via_l2) {
                        if constexpr (kSwap) {
                            // Owner blocks [col][local row], block o at kBNm * o_first.
                            float* dst = stage_f + kBNm * o_first + lr;
#pragma unroll
                            for (int j = 0; j < Cfg::kChunk; ++j)
                                dst[(c + j) * o_rows] = __uint_as_float(v[j]);
                        } else {
                            // Rows of kBNm + 4 floats (owner blocks are row ranges).
                            float* dst = stage_f + r * (kBNm + 4) + c;
#pragma unroll
                            for (int j = 0; j < Cfg::kChunk; j += 4)
                                *reinterpret_cast<uint4*>(dst + j) = make_uint4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                        }
                    } else if (split_k) {
                        if constexpr (kSwap) {
#pragma unroll
                            for (int j = 0; j < Cfg::kChunk; ++j)
                                st_dsmem_f32(recv + ((rank * kBNm + c + j) * sw_stride + lr) * 4u,
                                             __uint_as_float(v[j]));
                        } else {
                            const uint32_t row_off = (rank * nrows_max + lr) * (kBNm + 4);
#pragma unroll
                            for (int j = 0; j < Cfg::kChunk; j += 4)
                                st_dsmem_f4(recv + (row_off + c + j) * 4u, __uint_as_float(v[j]),
                                            __uint_as_float(v[j + 1]), __uint_as_float(v[j + 2]),
                                            __uint_as_float(v[j + 3]));
                        }
                    } else if constexpr (kSwap) {
                        store_col_segment<Cfg::kChunk>(p, acc_row0 + r, acc_col0 + c, v);
                    } else {
                        store_row_segment<Cfg::kChunk>(p, acc_row0 + r, acc_col0 + c, v);
                    }
                }
                if (via_l2) {
                    fence_async_shared();   // staging -> bulk copy (async proxy)
                    if constexpr (!kSwap) {
                        // This warp's 32 staged rows are contiguous: store them now.
                        __syncwarp();
                        if (lane == 0) {
                            const size_t slot = blockIdx.x + static_cast<size_t>(gridDim.x) *
                                                                 (blockIdx.y + static_cast<size_t>(gridDim.y) * rank);
                            const uint32_t off = warp * 32u * (kBNm + 4);
                            bulk_store(p.partials + slot * Cfg::kSlotFloats + off, stage_f + off,
                                       32u * (kBNm + 4) * 4u);
                            bulk_commit_group();
                            bulk_wait_group_all();
                            fence_async_global();
                        }
                    }
                }
            }
        }
        tc_fence_before_sync();
    }

    if (via_l2) {
        // Slot of CTA (x, y, z): x + gridDim.x * (y + gridDim.y * z); the
        // cluster spans z, so rank s of this cluster is z = s.
        const size_t slot0 = blockIdx.x + static_cast<size_t>(gridDim.x) * blockIdx.y;
        const size_t zstride = static_cast<size_t>(gridDim.x) * gridDim.y;
        if constexpr (kSwap) {
            // Owner-grouped staging spans all warps' rows: one bulk copy.
            if (warp < 4) epilogue_bar_sync();
            if (threadIdx.x == 0 && *abort_flag == 0) {
                bulk_store(p.partials + (slot0 + zstride * rank) * Cfg::kSlotFloats, smem,
                           Cfg::kSlotFloats * 4u);
                bulk_commit_group();
                bulk_wait_group_all();
                fence_async_global();
            }
        }
        // A pipeline that gave up leaves its slot unwritten: skip the loads
        // (the status word already records the failure).
        if (threadIdx.x == 0) *xchg_go = *abort_flag == 0;
        __syncwarp();
        cluster_sync();   // every slot of the cluster written (release / acquire)
        const bool go = *xchg_go != 0;
        float* recv = reinterpret_cast<float*>(smem + Cfg::kRecvOff);
        if (go && threadIdx.x == 0) {
            fence_async_global();
            const uint32_t row_floats = kSwap ? kBNm : kBNm + 4;   // floats per owned row
            const uint32_t bytes = static_cast<uint32_t>(nrows) * row_floats * 4u;
            mbar_arrive_expect_tx(xfer, bytes * static_cast<uint32_t>(split));
            for (int s2 = 0; s2 < split; ++s2) {
                const float* src = p.partials + (slot0 + zstride * s2) * Cfg::kSlotFloats +
                                   static_cast<size_t>(first) * row_floats;
                bulk_load(recv + static_cast<size_t>(s2) * nrows_max * row_floats, src, bytes, xfer);
            }
        }
        // Every thread of the CTA reduces; the wait is bounded like any other.
        ok = go && mbar_wait(xfer, 0, wc);
        // After a timeout, the issuing thread lets its copies land (bounded).
        if (go && !ok && threadIdx.x == 0) mbar_wait_drain(xfer, 0, kDrainLimitNs);
        if (ok) reduce_owned_rows<kBNm, kSwap>(p, recv, split, nrows, nrows_max, sw_stride, first, acc_row0, acc_col0);
    } else if (split_k) {
        cluster_sync();
        const float* recv = reinterpret_cast<const float*>(smem + Cfg::kRecvOff);
        reduce_owned_rows<kBNm, kSwap>(p, recv, split, nrows, nrows_max, sw_stride, first, acc_row0, acc_col0);
    }

    if (p.sc_ranks > 0) __threadfence_system();   // peer stores of a scatter, before the grid ends
    __syncthreads();
    if (warp == 5) {
        tc_fence_after_sync();
        tmem_dealloc(tmem_base, Cfg::kTmemCols);
    }
}

// ==================================================== persistent kernel ====

template <int kBN, int kStages>
struct PersistCfg {
    static constexpr uint32_t kABytes = kMmaM * 128u;        // 128 x 64 halves
    static constexpr uint32_t kBBytes = kBN * 128u;          // 64 x kBN halves
    static constexpr uint32_t kStageBytes = kABytes + kBBytes;
    static constexpr uint32_t kEpiBytes = 4u * 2u * 4096u;   // 4 warps x 2 boxes of 32 x 64 halves
    static constexpr uint32_t kDataBytes = kStages * kStageBytes + kEpiBytes;
    static constexpr uint32_t kBarBytes = 256;
    static constexpr uint32_t kSmemBytes = kDataBytes + kBarBytes + 1024;
    static constexpr uint32_t kTmemCols = tmem_cols_for(2 * kBN);
    static constexpr uint32_t kIdesc = make_idesc_f16(kMmaM, kBN, false, true);
    static_assert(kBN % 64 == 0 && kBN <= 256, "tile width");
    static_assert(2 * kStages + 5 <= 30, "barrier area");
    static_assert(kSmemBytes <= 232448, "shared memory");
};

// `rot` rotates the M-tile order (a bijection on the tiles).
__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int group_m,
                                            int& tm, int& tn, int rot = 0) {
    const int width = group_m * tiles_n;
    const int g = t / width;
    const int first_m = g * group_m;
    const int gsz = min(tiles_m - first_m, group_m);
    const int in = t - g * width;
    tm = first_m + in % gsz;
    if (rot != 0) tm = (tm + rot) % tiles_m;
    tn = in / gsz;
}

// Inverse of tile_coords without rotation: the raster index of tile (tm, tn).
__device__ __forceinline__ int tile_index(int tm, int tn, int tiles_m, int tiles_n, int group_m) {
    const int g = tm / group_m;
    const int first_m = g * group_m;
    const int gsz = min(tiles_m - first_m, group_m);
    return g * group_m * tiles_n + tn * gsz + (tm - first_m);
}

// M-tile rotation of a row scatter: rank r starts on the rows of rank r + 1,
// so that at any time each owner receives from about one peer instead of
// all of them writing into the same owner's buffer (NVLink incast).
__device__ __forceinline__ int scatter_rotation(const GemmParams& p, int tile_rows, int tiles_m) {
    if (p.sc_ranks <= 1) return 0;
    return static_cast<int>((static_cast<long long>(p.sc_rank + 1) * p.sc_rows / tile_rows) % tiles_m);
}

template <int kBN, int kStages>
__global__ void __launch_bounds__(kThreads, 1)
hgemm_persistent_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                        const __grid_constant__ CUtensorMap tm_c, const GemmParams p) {
    using Cfg = PersistCfg<kBN, kStages>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align_1024(smem_raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kDataBytes);
    uint64_t* empty = full + kStages;
    uint64_t* tfull = empty + kStages;      // [2]
    uint64_t* tempty = tfull + 2;           // [2]
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const uint32_t warp = warp_index();
    const uint32_t lane = threadIdx.x & 31u;

    if (warp == 4 && lane == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1u);
            mbar_init(&empty[s], 1u);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1u);
            mbar_init(&tempty[i], 128u);
        }
        mbar_init(drain, 1u);
        *abort_flag = 0;
        mbar_init_fence();
        tma_prefetch_map(&tm_a);
        tma_prefetch_map(&tm_b);
    }
    if (warp == 5) {
        tmem_alloc(tmem_slot, Cfg::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem_base = *tmem_slot;
    // The set-up above touches only this CTA's shared memory and TMEM, so it
    // may overlap the previous kernel of the stream; global memory is only
    // touched after that kernel has completed.
    grid_dependents_launch();
    grid_dependency_wait();
    const WaitCtl wc{abort_flag, p.status, p.timeout_ns};

    const int tiles_m = (p.m + kMmaM - 1) / kMmaM;
    const int m_rot = scatter_rotation(p, kMmaM, tiles_m);
    const int tiles_n = (p.n + kBN - 1) / kBN;
    const int num_tiles = tiles_m * tiles_n;
    const int nkb = (p.k + kBlockK - 1) / kBlockK;

    if (warp == 4) {
        if (lane == 0) {
            uint32_t stage = 0, phase = 0, issued = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                int tm, tn;
                tile_coords(t, tiles_m, tiles_n, p.group_m, tm, tn, m_rot);
                for (int kb = 0; kb < nkb; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, wc)) { ok = false; break; }
                    uint8_t* s_a = smem + stage * Cfg::kStageBytes;
                    uint8_t* s_b = s_a + Cfg::kABytes;
                    const uint32_t extra = (p.inject && issued == 0) ? 16u : 0u;
                    mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes + extra);
                    tma_load_2d(s_a, &tm_a, &full[stage], kb * kBlockK, tm * kMmaM);
#pragma unroll
                    for (int j = 0; j < kBN / 64; ++j)
                        tma_load_2d(s_b + j * kChunkBytes, &tm_b, &full[stage], tn * kBN + 64 * j,
                                    kb * kBlockK);
                    ++issued;
                    if (++stage == kStages) { stage = 0; phase ^= 1u; }
                }
            }
            if (!ok || *abort_flag) drain_tma<kStages>(full, issued);
        }
    } else if (warp == 5) {
        if (lane == 0) {
            uint32_t stage = 0, phase = 0, iter = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++iter) {
                const uint32_t acc = iter & 1u, acc_phase = (iter >> 1) & 1u;
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, wc)) { ok = false; break; }
                tc_fence_after_sync();
                const uint32_t d = tmem_base + acc * kBN;
                for (int kb = 0; kb < nkb; ++kb) {
                    if (!mbar_wait(&full[stage], phase, wc)) { ok = false; break; }
                    tc_fence_after_sync();
                    const uint32_t s_a = smem_addr(smem + stage * Cfg::kStageBytes);
                    const uint32_t s_b = s_a + Cfg::kABytes;
#pragma unroll
                    for (int kk = 0; kk < kBlockK / 16; ++kk)
                        tc_mma_f16(d, kmaj_desc(s_a, kk), mnmaj_desc(s_b, kk), Cfg::kIdesc,
                                   (kb > 0 || kk > 0) ? 1u : 0u);
                    tc_commit(&empty[stage]);
                    if (++stage == kStages) { stage = 0; phase ^= 1u; }
                }
                if (ok) tc_commit(&tfull[acc]);
            }
            if (!ok) {
                tc_commit(drain);
                mbar_wait_drain(drain, 0, kDrainLimitNs);
            }
        }
    } else {
        // Epilogue warps 0-3: warp w owns TMEM lanes 32w .. 32w + 31.
        const uint32_t t_lane = (warp * 32u) << 16;
        uint8_t* boxes = smem + kStages * Cfg::kStageBytes + warp * 8192u;
        uint32_t buf = 0, iter = 0;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++iter) {
            const uint32_t acc = iter & 1u, acc_phase = (iter >> 1) & 1u;
            if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase, wc))) break;
            tc_fence_after_sync();
            int tm, tn;
            tile_coords(t, tiles_m, tiles_n, p.group_m, tm, tn, m_rot);
            const int row = tm * kMmaM + warp * 32 + lane;
            const uint32_t t_acc = tmem_base + t_lane + acc * kBN;
            if (p.tma_store) {
#pragma unroll 1
                for (int c = 0; c < kBN; c += 64) {
                    uint32_t v0[32], v1[32];
                    tmem_ld_32x32b_x32(t_acc + c, v0);
                    tmem_ld_32x32b_x32(t_acc + c + 32, v1);
                    tmem_wait_ld();
                    epi_add_row<32>(p, row, tn * kBN + c, v0);
                    epi_add_row<32>(p, row, tn * kBN + c + 32, v1);
                    store_box_tma(&tm_c, boxes + buf * 4096u, lane, v0, v1, tn * kBN + c,
                                  tm * kMmaM + warp * 32);
                    buf ^= 1u;
                }
            } else {
#pragma unroll 1
                for (int c = 0; c < kBN; c += 32) {
                    uint32_t v[32];
                    tmem_ld_32x32b_x32(t_acc + c, v);
                    tmem_wait_ld();
                    if (p.sc_bulk)
                        store_block_f32_bulk(p, boxes, buf, lane, v, tm * kMmaM + warp * 32, tn * kBN + c);
                    else if (p.sc_ranks > 0)
                        store_block_f32(p, reinterpret_cast<float*>(boxes), lane, v, tm * kMmaM + warp * 32, tn * kBN + c);
                    else
                        store_row_segment<32>(p, row, tn * kBN + c, v);
                }
            }
            tc_fence_before_sync();
            mbar_arrive(&tempty[acc]);
        }
        if (p.tma_store && lane == 0) bulk_wait_group_all();
        if (p.sc_bulk) bulk_wait_group_all();     // every lane's row copies have landed
    }

    __syncwarp();
    if (p.sc_ranks > 0) __threadfence_system();   // peer stores of a scatter, before the grid ends
    tc_fence_before_sync();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after_sync();
        tmem_dealloc(tmem_base, Cfg::kTmemCols);
    }
}

// ============================================== CTA-pair persistent kernel ====
//
// kTileM x kTileN output tiles (kTileM = 256 or 128, kTileN = 256 or 128) per
// cluster of two CTAs (cta_group::2). CTA r of the pair TMA-loads the r-th
// kTileM/2 rows of the A tile and the r-th kTileN/2 columns of the B tile
// into its own shared memory; the even CTA's single MMA thread issues
// M=kTileM, N=kTileN MMAs that read both CTAs' tiles, and each CTA's TMEM
// receives the accumulator of its own kTileM/2 rows (two buffers). With
// 128 rows per CTA, row i sits in TMEM lane i. With 64 rows per CTA the
// accumulator is folded: lanes 0-63 hold rows 0-63 of columns 0 .. kTileN/2-1
// and lanes 64-127 the same rows of columns kTileN/2 .. kTileN-1, in
// kTileN/2 TMEM columns. 64-row tiles halve the A bytes each SM's tensor
// core reads per MMA (the per-MMA cost at N <= 256 is set by A rows), so
// they keep full efficiency at half the M granularity.
// Both CTAs' loads complete their bytes on the even CTA's "stage full"
// barrier (armed once with both CTAs' bytes); the MMA thread commits "stage
// empty" and "accumulator full" to the barriers of both CTAs with one
// multicast commit each; one lane per
// epilogue warp of either CTA arrives on the even CTA's "accumulator empty".
// Pairs step through the tiles in waves (pair g takes tiles g, g + G, ...);
// odd waves walk K from the last block down, so that a tile starts on the
// A rows / B columns the previous wave's tiles in the same raster group
// read last, while they are still in L2 (at 8192^3: 1.06 -> 0.93 GB read
// from DRAM per launch). The MMA side only counts K blocks, so the order
// changes nothing but the FP32 summation order of a tile. The direction is
// that of the output tile's wave in the unrotated raster, so a row-scatter
// launch (rows rotated per rank) sums every tile exactly as a plain launch.

template <int kTileMT, int kTileNT, int kStages>
struct PairCfg {
    static constexpr int kTileM = kTileMT, kTileN = kTileNT;   // pair tile
    static constexpr int kRows = kTileM / 2;                   // A rows (output rows) per CTA
    static constexpr int kHalfN = kTileN / 2;                  // B columns each CTA loads
    static constexpr bool kFolded = kRows == 64;               // 64-row accumulator layout
    static constexpr uint32_t kAccCols = kFolded ? kTileN / 2 : kTileN;   // TMEM columns per buffer
    static constexpr uint32_t kABytes = kRows * 128u;           // kRows rows x 64 halves
    static constexpr uint32_t kBBytes = kHalfN * 128u;          // 64 k-rows x kHalfN halves
    static constexpr uint32_t kStageBytes = kABytes + kBBytes;
    static constexpr uint32_t kEpiBytes = 4u * 2u * 4096u;   // 4 warps x 2 boxes of 32 x 64 halves
    static constexpr uint32_t kDataBytes = kStages * kStageBytes + kEpiBytes;
    static constexpr uint32_t kBarBytes = 256;
    static constexpr uint32_t kSmemBytes = kDataBytes + kBarBytes + 1024;
    static constexpr uint32_t kTmemCols = tmem_cols_for(2 * kAccCols);   // 2 accumulators
    static constexpr uint32_t kIdesc = make_idesc_f16(kTileM, kTileN, false, true);
    static_assert(kTileN == 128 || kTileN == 256, "pair tile width");
    static_assert(kTileM == 128 || kTileM == 256, "pair tile height");
    static_assert(2 * kStages + 5 <= 30, "barrier area");
    static_assert(kSmemBytes <= 232448, "shared memory");
};

template <int kTileMT, int kTileNT, int kStages>
__global__ void __launch_bounds__(kThreads, 1)
hgemm_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                  const __grid_constant__ CUtensorMap tm_c, const GemmParams p) {
    using Cfg = PairCfg<kTileMT, kTileNT, kStages>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align_1024(smem_raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kDataBytes);   // even CTA
    uint64_t* empty = full + kStages;
    uint64_t* tfull = empty + kStages;      // [2]
    uint64_t* tempty = tfull + 2;           // [2], even CTA
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const uint32_t warp = warp_index();
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t rank = cluster_ctarank();   // 0 = MMA CTA, 1 = peer
    const bool leader = rank == 0;

    if (warp == 4 && lane == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1u);
            mbar_init(&empty[s], 1u);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1u);
            mbar_init(&tempty[i], 8u);     // one lane of each epilogue warp, both CTAs
        }
        mbar_init(drain, 1u);
        *abort_flag = 0;
        mbar_init_fence();
        tma_prefetch_map(&tm_a);
        tma_prefetch_map(&tm_b);
    }
    if (warp == 5) {
        tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before_sync();
    cluster_sync();                       // both CTAs' barriers exist before any remote op
    tc_fence_after_sync();
    const uint32_t tmem_base = *tmem_slot;
    // The set-up above touches only this CTA's shared memory and TMEM, so it
    // may overlap the previous kernel of the stream; global memory is only
    // touched after that kernel has completed.
    grid_dependents_launch();
    grid_dependency_wait();
    const WaitCtl wc{abort_flag, p.status, p.timeout_ns};

    const int tiles_m = (p.m + Cfg::kTileM - 1) / Cfg::kTileM;
    const int m_rot = scatter_rotation(p, Cfg::kTileM, tiles_m);
    const int tiles_n = (p.n + Cfg::kTileN - 1) / Cfg::kTileN;
    const int num_tiles = tiles_m * tiles_n;
    const int nkb = (p.k + kBlockK - 1) / kBlockK;
    const int pair = blockIdx.x >> 1;
    const int npairs = gridDim.x >> 1;

    if (warp == 4) {
        if (lane == 0) {
            uint32_t stage = 0, phase = 0, issued = 0;
            bool ok = true;
            for (int t = pair; t < num_tiles && ok; t += npairs) {
                int tm, tn;
                tile_coords(t, tiles_m, tiles_n, p.group_m, tm, tn, m_rot);
                const int row0 = tm * Cfg::kTileM + static_cast<int>(rank) * Cfg::kRows;
                const int col0 = tn * Cfg::kTileN + static_cast<int>(rank) * Cfg::kHalfN;
                const int t_out = m_rot != 0 ? tile_index(tm, tn, tiles_m, tiles_n, p.group_m) : t;
                const bool backwards = ((t_out / npairs) & 1) != 0;
                for (int kq = 0; kq < nkb; ++kq) {
                    const int kb = backwards ? nkb - 1 - kq : kq;
                    if (!mbar_wait_cluster(&empty[stage], phase ^ 1u, wc)) { ok = false; break; }
                    uint8_t* s_a = smem + stage * Cfg::kStageBytes;
                    uint8_t* s_b = s_a + Cfg::kABytes;
                    const uint32_t bar = map_to_rank(smem_addr(&full[stage]), 0);
                    if (leader) {
                        const uint32_t extra = (p.inject && issued == 0) ? 16u : 0u;
                        mbar_arrive_expect_tx(&full[stage], 2u * Cfg::kStageBytes + extra);
                    }
                    tma_load_2d_pair(s_a, &tm_a, bar, kb * kBlockK, row0);
#pragma unroll
                    for (int j = 0; j < Cfg::kHalfN / 64; ++j)
                        tma_load_2d_pair(s_b + j * kChunkBytes, &tm_b, bar, col0 + 64 * j, kb * kBlockK);
                    ++issued;
                    if (++stage == kStages) { stage = 0; phase ^= 1u; }
                }
            }
            if (leader && (!ok || *abort_flag)) drain_tma<kStages>(full, issued);
        }
    } else if (warp == 5) {
        if (lane == 0 && leader) {
            uint32_t stage = 0, phase = 0, iter = 0;
            bool ok = true;
            for (int t = pair; t < num_tiles && ok; t += npairs, ++iter) {
                const uint32_t acc = iter & 1u, acc_phase = (iter >> 1) & 1u;
                if (!mbar_wait_cluster(&tempty[acc], acc_phase ^ 1u, wc)) { ok = false; break; }
                tc_fence_after_sync();
                const uint32_t d = tmem_base + acc * Cfg::kAccCols;
                for (int kb = 0; kb < nkb; ++kb) {
                    if (!mbar_wait(&full[stage], phase, wc)) { ok = false; break; }
                    tc_fence_after_sync();
                    const uint32_t s_a = smem_addr(smem + stage * Cfg::kStageBytes);
                    const uint32_t s_b = s_a + Cfg::kABytes;
#pragma unroll
                    for (int kk = 0; kk < kBlockK / 16; ++kk)
                        tc_mma_f16_pair(d, kmaj_desc(s_a, kk), mnmaj_desc(s_b, kk), Cfg::kIdesc,
                                        (kb > 0 || kk > 0) ? 1u : 0u);
                    tc_commit_pair_both(smem_addr(&empty[stage]));
                    if (++stage == kStages) { stage = 0; phase ^= 1u; }
                }
                if (ok) {
                    tc_commit_pair_both(smem_addr(&tfull[acc]));
                }
            }
            if (!ok) {
                tc_commit_pair(smem_addr(drain));
                mbar_wait_drain(drain, 0, kDrainLimitNs);
            }
        }
    } else {
        const uint32_t t_lane = (warp * 32u) << 16;
        const uint32_t tempty_leader0 = map_to_rank(smem_addr(&tempty[0]), 0);
        const uint32_t tempty_leader1 = map_to_rank(smem_addr(&tempty[1]), 0);
        uint8_t* boxes = smem + kStages * Cfg::kStageBytes + warp * 8192u;
        uint32_t buf = 0, iter = 0;
        for (int t = pair; t < num_tiles; t += npairs, ++iter) {
            const uint32_t acc = iter & 1u, acc_phase = (iter >> 1) & 1u;
            if (!__all_sync(0xffffffffu, mbar_wait_cluster(&tfull[acc], acc_phase, wc))) break;
            tc_fence_after_sync();
            int tm, tn;
            tile_coords(t, tiles_m, tiles_n, p.group_m, tm, tn, m_rot);
            // Warp w: its 32 TMEM lanes are rows row0 .. row0 + 31 of columns
            // col0 .. col0 + kAccCols - 1 (folded layout: warps 2, 3 hold the
            // right half of the columns of the rows of warps 0, 1).
            const int wrow = Cfg::kFolded ? static_cast<int>(warp & 1u) * 32 : static_cast<int>(warp) * 32;
            const int row0 = tm * Cfg::kTileM + static_cast<int>(rank) * Cfg::kRows + wrow;
            const int col0 = tn * Cfg::kTileN + (Cfg::kFolded ? static_cast<int>(warp >> 1) * (Cfg::kTileN / 2) : 0);
            const uint32_t t_acc = tmem_base + t_lane + acc * Cfg::kAccCols;
            if (p.tma_store) {
#pragma unroll 1
                for (int c = 0; c < static_cast<int>(Cfg::kAccCols); c += 64) {
                    uint32_t v0[32], v1[32];
                    tmem_ld_32x32b_x32(t_acc + c, v0);
                    tmem_ld_32x32b_x32(t_acc + c + 32, v1);
                    tmem_wait_ld();
                    epi_add_row<32>(p, row0 + static_cast<int>(lane), col0 + c, v0);
                    epi_add_row<32>(p, row0 + static_cast<int>(lane), col0 + c + 32, v1);
                    store_box_tma(&tm_c, boxes + buf * 4096u, lane, v0, v1, col0 + c, row0);
                    buf ^= 1u;
                }
            } else {
#pragma unroll 1
                for (int c = 0; c < static_cast<int>(Cfg::kAccCols); c += 32) {
                    uint32_t v[32];
                    tmem_ld_32x32b_x32(t_acc + c, v);
                    tmem_wait_ld();
                    if (p.sc_bulk)
                        store_block_f32_bulk(p, boxes, buf, lane, v, row0, col0 + c);
                    else if (p.sc_ranks > 0)
                        store_block_f32(p, reinterpret_cast<float*>(boxes), lane, v, row0, col0 + c);
                    else
                        store_row_segment<32>(p, row0 + static_cast<int>(lane), col0 + c, v);
                }
            }
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc ? tempty_leader1 : tempty_leader0);
        }
        if (p.tma_store && lane == 0) bulk_wait_group_all();
        if (p.sc_bulk) bulk_wait_group_all();     // every lane's row copies have landed
    }

    __syncwarp();
    // An aborted pipeline may leave the peer's copies in flight towards the
    // even CTA's barrier; give them time to land before either CTA exits.
    if (*abort_flag) settle_ns(2000000ull);
    if (p.sc_ranks > 0) __threadfence_system();   // peer stores of a scatter, before the grid ends
    tc_fence_before_sync();
    cluster_sync();                       // no CTA leaves while its pair may still touch it
    if (warp == 5) {
        tc_fence_after_sync();
        tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
    }
}

// ================================================ stream-K persistent kernel ====
//
// One CTA per SM over (tile, 64-deep K block) work. The first T - n_sk tiles
// are processed whole, in waves (CTA g takes tiles g, g + G, ...), which keeps
// concurrently processed tiles adjacent in raster order (L2 reuse). The last
// n_sk tiles' K blocks are cut into G equal contiguous ranges, one per CTA,
// so every SM ends at the same time whatever T is (n_sk = 0: whole tiles
// only). The host picks n_sk so that each range spans at least one tile:
// a tile is then shared by at most two CTAs. The CTA owning a split tile's
// last K block finishes it: it adds the FP32 partial that lower-numbered CTAs
// left in their workspace slots (fixed order - deterministic) and stores C.
// Each CTA processes its range backwards, so the partial it owes is computed
// first and the tile it finishes last. Finishers only wait for lower-numbered
// CTAs; the launch is cooperative, so all CTAs are resident. A slot's flag
// holds the launch's epoch while its partial is valid; the finisher resets it
// to 0 after use (safe under CUDA-graph replay). All waits are bounded.
//
// Partial slots are stored as float4 columns-major-by-quad ([quad][row]),
// so that both the producer's stores and the finisher's reads are
// coalesced; the finisher pulls a slot into the (then idle) stage buffers
// with one bulk copy.
//
// kSwap as in hgemm_tile_kernel (accumulator rows = output columns).

struct Seg {
    int tile, kb0, kb1;   // K blocks [kb0, kb1) of tile
};

// Segments of one CTA, in processing order. Every role iterates identically.
struct SegIter {
    long long start, pe;     // stream-K part: remaining range [start, pe) of K-block positions
    int next_tile, G, T_dp, KB;
    __device__ SegIter(int g, int G_, int T, int KB_, int n_sk) : G(G_), T_dp(T - n_sk), KB(KB_) {
        const long long base = static_cast<long long>(T - n_sk) * KB_;
        const long long W = static_cast<long long>(n_sk) * KB_;
        start = base + W * g / G_;
        pe = base + W * (g + 1) / G_;
        next_tile = g;
    }
    __device__ bool next(Seg& s) {
        if (next_tile < T_dp) {
            s.tile = next_tile;
            s.kb0 = 0;
            s.kb1 = KB;
            next_tile += G;
            return true;
        }
        if (pe <= start) return false;
        const int tile = static_cast<int>((pe - 1) / KB);
        const long long t0 = static_cast<long long>(tile) * KB;
        const long long ps = start > t0 ? start : t0;
        s.tile = tile;
        s.kb0 = static_cast<int>(ps - t0);
        s.kb1 = static_cast<int>(pe - t0);
        pe = ps;
        return true;
    }
};

// CTA whose stream-K range contains K-block position `pos` (relative to the
// start of the stream-K part, W positions in total).
__device__ __forceinline__ int sk_owner(long long pos, int G, long long W) {
    int g = static_cast<int>(pos * G / W);
    while (g + 1 < G && W * (g + 1) / G <= pos) ++g;
    while (g > 0 && W * g / G > pos) --g;
    return g;
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

template <int kBNm, bool kSwap, int kStages>
struct StreamKCfg {
    static constexpr int kKRows = kSwap ? kBNm : kMmaM;
    static constexpr int kMNCols = kSwap ? kMmaM : kBNm;
    static constexpr uint32_t kKBytes = kKRows * 128u;
    static constexpr uint32_t kMNBytes = kMNCols * 128u;
    static constexpr uint32_t kStageBytes = kKBytes + kMNBytes;
    // TMA-store boxes, two per epilogue warp: 32 x 64 halves, or (swapped)
    // kChunk x 32 halves.
    static constexpr uint32_t kEpiBytes = kSwap ? 4u * 2u * 2048u : 4u * 2u * 4096u;
    static constexpr uint32_t kDataBytes = kStages * kStageBytes + kEpiBytes;
    static constexpr uint32_t kBarBytes = 256;
    static constexpr uint32_t kSmemBytes = kDataBytes + kBarBytes + 1024;
    static constexpr uint32_t kAccCols = tmem_cols_for(kBNm);       // one accumulator
    static constexpr uint32_t kTmemCols = tmem_cols_for(2 * kAccCols);
    static constexpr uint32_t kIdesc = make_idesc_f16(kMmaM, kBNm, kSwap, !kSwap);
    static constexpr int kChunk = kBNm >= 32 ? 32 : 16;
    static constexpr uint32_t kSlotBytes = static_cast<uint32_t>(kMmaM) * kBNm * 4u;
    static_assert(kKRows % 8 == 0 && kMNCols % 64 == 0, "tile shape");
    static_assert(kBNm % 16 == 0 && kBNm >= 16 && kBNm <= 256, "UMMA N for M=128");
    static_assert(2 * kStages + 9 <= 31, "barrier area");
    static_assert(kSlotBytes <= kStages * kStageBytes, "a partial slot must fit the stage buffers");
    static_assert(kSmemBytes <= 232448, "shared memory");
};

template <int kBNm, bool kSwap, int kStages>
__global__ void __launch_bounds__(kThreads, 1)
hgemm_streamk_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_mn,
                     const __grid_constant__ CUtensorMap tm_c, const GemmParams p) {
    (void)tm_c;
    using Cfg = StreamKCfg<kBNm, kSwap, kStages>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align_1024(smem_raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kDataBytes);
    uint64_t* empty = full + kStages;
    uint64_t* tfull = empty + kStages;      // [2]
    uint64_t* tempty = tfull + 2;           // [2]
    uint64_t* drain = tempty + 2;
    uint64_t* published = drain + 1;        // 128 epilogue threads wrote the partial
    uint64_t* consumed = published + 1;     // 128 epilogue threads read the partial
    uint64_t* landed = consumed + 1;        // a producer's slot arrived in shared memory
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(landed + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const uint32_t warp = warp_index();
    const uint32_t lane = threadIdx.x & 31u;

    if (warp == 4 && lane == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1u);
            mbar_init(&empty[s], 1u);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1u);
            mbar_init(&tempty[i], 128u);
        }
        mbar_init(drain, 1u);
        mbar_init(published, 128u);   // a CTA produces <= 1 partial and finishes <= 1 tile,
        mbar_init(consumed, 128u);    // so these are used at most once per launch ...
        mbar_init(landed, 1u);        // ... and this once per producer slot read
        *abort_flag = 0;
        mbar_init_fence();
        tma_prefetch_map(&tm_k);
        tma_prefetch_map(&tm_mn);
    }
    if (warp == 5) {
        tmem_alloc(tmem_slot, Cfg::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem_base = *tmem_slot;
    // The set-up above touches only this CTA's shared memory and TMEM, so it
    // may overlap the previous kernel of the stream; global memory is only
    // touched after that kernel has completed.
    grid_dependents_launch();
    grid_dependency_wait();
    const WaitCtl wc{abort_flag, p.status, p.timeout_ns};

    // Accumulator tiles: rows = M (N when swapped) in 128s, cols = kBNm wide.
    const int rows_total = kSwap ? p.n : p.m;
    const int cols_total = kSwap ? p.m : p.n;
    const int tiles_r = (rows_total + kMmaM - 1) / kMmaM;
    const int m_rot = kSwap ? 0 : scatter_rotation(p, kMmaM, tiles_r);
    const int tiles_c = (cols_total + kBNm - 1) / kBNm;
    const int T = tiles_r * tiles_c;
    const int KB = (p.k + kBlockK - 1) / kBlockK;
    const int G = gridDim.x;
    const int g = blockIdx.x;
    const int n_sk = p.streamk;

    if (warp == 4) {
        if (lane == 0) {
            uint32_t stage = 0, phase = 0, issued = 0;
            bool ok = true;
            SegIter it(g, G, T, KB, n_sk);
            Seg sg;
            while (ok && it.next(sg)) {
                int tr, tc;
                tile_coords(sg.tile, tiles_r, tiles_c, p.group_m, tr, tc, m_rot);
                const int k_rows0 = kSwap ? tc * kBNm : tr * kMmaM;
                const int mn_cols0 = kSwap ? tr * kMmaM : tc * kBNm;
                for (int kb = sg.kb0; kb < sg.kb1; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, wc)) { ok = false; break; }
                    uint8_t* s_k = smem + stage * Cfg::kStageBytes;
                    uint8_t* s_mn = s_k + Cfg::kKBytes;
                    const uint32_t extra = (p.inject && issued == 0) ? 16u : 0u;
                    mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes + extra);
                    tma_load_2d(s_k, &tm_k, &full[stage], kb * kBlockK, k_rows0);
#pragma unroll
                    for (int j = 0; j < Cfg::kMNCols / 64; ++j)
                        tma_load_2d(s_mn + j * kChunkBytes, &tm_mn, &full[stage], mn_cols0 + 64 * j,
                                    kb * kBlockK);
                    ++issued;
                    if (++stage == kStages) { stage = 0; phase ^= 1u; }
                }
            }
            if (!ok || *abort_flag) drain_tma<kStages>(full, issued);
        }
    } else if (warp == 5) {
        if (lane == 0) {
            uint32_t stage = 0, phase = 0, iter = 0;
            bool ok = true;
            SegIter it(g, G, T, KB, n_sk);
            Seg sg;
            while (ok && it.next(sg)) {
                const uint32_t acc = iter & 1u, acc_phase = (iter >> 1) & 1u;
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, wc)) { ok = false; break; }
                tc_fence_after_sync();
                const uint32_t d = tmem_base + acc * Cfg::kAccCols;
                for (int kb = sg.kb0; kb < sg.kb1; ++kb) {
                    if (!mbar_wait(&full[stage], phase, wc)) { ok = false; break; }
                    tc_fence_after_sync();
                    const uint32_t s_k = smem_addr(smem + stage * Cfg::kStageBytes);
                    const uint32_t s_mn = s_k + Cfg::kKBytes;
#pragma unroll
                    for (int kk = 0; kk < kBlockK / 16; ++kk) {
                        const uint64_t dk = kmaj_desc(s_k, kk);
                        const uint64_t dmn = mnmaj_desc(s_mn, kk);
                        tc_mma_f16(d, kSwap ? dmn : dk, kSwap ? dk : dmn, Cfg::kIdesc,
                                   (kb > sg.kb0 || kk > 0) ? 1u : 0u);
                    }
                    tc_commit(&empty[stage]);
                    if (++stage == kStages) { stage = 0; phase ^= 1u; }
                }
                if (ok) tc_commit(&tfull[acc]);
                ++iter;
            }
            if (!ok) {
                tc_commit(drain);
                mbar_wait_drain(drain, 0, kDrainLimitNs);
            }
        }
    } else {
        const uint32_t t_lane = (warp * 32u) << 16;
        const int r = warp * 32 + lane;                 // accumulator row (TMEM lane)
        const long long W_sk = static_cast<long long>(n_sk) * KB;
        const long long base_sk = static_cast<long long>(T - n_sk) * KB;
        uint32_t iter = 0, epi_buf = 0;
        SegIter it(g, G, T, KB, n_sk);
        Seg sg;
        while (it.next(sg)) {
            const uint32_t acc = iter & 1u, acc_phase = (iter >> 1) & 1u;
            ++iter;
            if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase, wc))) break;
            tc_fence_after_sync();
            int tr, tc;
            tile_coords(sg.tile, tiles_r, tiles_c, p.group_m, tr, tc, m_rot);
            const uint32_t t_acc = tmem_base + t_lane + acc * Cfg::kAccCols;
            const bool produce = sg.kb1 < KB;                 // partial owed to a later CTA
            const bool finish = !produce && sg.kb0 > 0;       // adds earlier CTAs' partials
            int p_lo = g;
            if (finish) {
                p_lo = sk_owner(static_cast<long long>(sg.tile) * KB - base_sk, G, W_sk);
                // Wait (bounded) until every earlier CTA's partial of this tile is published.
                bool ready = true;
                for (int q = p_lo; q < g && ready; ++q) {
                    const uint64_t t0 = global_timer_ns();
                    while (ld_acquire_u64(p.flags + q) != p.epoch) {
                        if (*abort_flag || global_timer_ns() - t0 > p.timeout_ns) {
                            raise_abort(wc, kStatusPipelineTimeout);
                            ready = false;
                            break;
                        }
                    }
                }
                if (!__all_sync(0xffffffffu, ready)) {
                    tc_fence_before_sync();
                    mbar_arrive(&tempty[acc]);
                    break;
                }
            }
            // The finisher segment is this CTA's last: the stage buffers are idle
            // (its MMAs completed). With a single producer (what the host plans)
            // its slot is pulled there with bulk copies; with several, slots
            // are read from global memory. Either way the sum is
            // (slot p_lo + ... + slot g-1) + own, in that order.
            const float4* staged = reinterpret_cast<const float4*>(smem);
            const float4* slots = reinterpret_cast<const float4*>(p.partials);
            constexpr size_t kSlotQuads = Cfg::kSlotBytes / 16;
            float4* my_slot = reinterpret_cast<float4*>(p.partials) + static_cast<size_t>(g) * kSlotQuads;
            const bool one_producer = finish && p_lo == g - 1;
            bool ok_tile = true;
            if (one_producer) {
                if (r == 0) {
                    mbar_arrive_expect_tx(landed, Cfg::kSlotBytes);
                    const uint8_t* src = reinterpret_cast<const uint8_t*>(slots + static_cast<size_t>(p_lo) * kSlotQuads);
                    for (uint32_t off = 0; off < Cfg::kSlotBytes; off += 32768u) {
                        const uint32_t n = Cfg::kSlotBytes - off < 32768u ? Cfg::kSlotBytes - off : 32768u;
                        bulk_load(smem + off, src + off, n, landed);
                    }
                }
                ok_tile = __all_sync(0xffffffffu, mbar_wait(landed, 0, wc));
            }
            if (ok_tile && !kSwap && p.tma_store && !produce) {
                // Whole or finished tile: 64-column boxes through shared memory.
                uint8_t* boxes = smem + kStages * Cfg::kStageBytes + warp * 8192u;
#pragma unroll 1
                for (int c = 0; c < kBNm; c += 64) {
                    uint32_t v0[32], v1[32];
                    tmem_ld_32x32b_x32(t_acc + c, v0);
                    tmem_ld_32x32b_x32(t_acc + c + 32, v1);
                    if (finish) {
                        // The 16 partial quads of this row's 64 columns, loaded
                        // together (overlapping the TMEM loads), then added.
                        float4 part[16];
                        const size_t q0 = static_cast<size_t>(c / 4) * kMmaM + r;
                        if (one_producer) {
#pragma unroll
                            for (int q = 0; q < 16; ++q) part[q] = staged[q0 + static_cast<size_t>(q) * kMmaM];
                        } else {
#pragma unroll
                            for (int q = 0; q < 16; ++q)
                                part[q] = __ldcg(slots + static_cast<size_t>(p_lo) * kSlotQuads + q0 + static_cast<size_t>(q) * kMmaM);
                            for (int s2 = p_lo + 1; s2 < g; ++s2) {
#pragma unroll
                                for (int q = 0; q < 16; ++q) {
                                    const float4 x = __ldcg(slots + static_cast<size_t>(s2) * kSlotQuads + q0 + static_cast<size_t>(q) * kMmaM);
                                    part[q].x += x.x; part[q].y += x.y; part[q].z += x.z; part[q].w += x.w;
                                }
                            }
                        }
                        tmem_wait_ld();
#pragma unroll
                        for (int q = 0; q < 16; ++q) {
                            uint32_t* v = q < 8 ? v0 + 4 * q : v1 + 4 * (q - 8);
                            v[0] = __float_as_uint(part[q].x + __uint_as_float(v[0]));
                            v[1] = __float_as_uint(part[q].y + __uint_as_float(v[1]));
                            v[2] = __float_as_uint(part[q].z + __uint_as_float(v[2]));
                            v[3] = __float_as_uint(part[q].w + __uint_as_float(v[3]));
                        }
                    } else {
                        tmem_wait_ld();
                    }
                    epi_add_row<32>(p, tr * kMmaM + r, tc * kBNm + c, v0);
                    epi_add_row<32>(p, tr * kMmaM + r, tc * kBNm + c + 32, v1);
                    store_box_tma(&tm_c, boxes + epi_buf * 4096u, lane, v0, v1, tc * kBNm + c,
                                  tr * kMmaM + warp * 32);
                    epi_buf ^= 1u;
                }
            } else if (ok_tile) {
#pragma unroll 1
                for (int c = 0; c < kBNm; c += Cfg::kChunk) {
                    uint32_t v[Cfg::kChunk];
                    if constexpr (Cfg::kChunk == 32) {
                        tmem_ld_32x32b_x32(t_acc + c, v);
                    } else {
                        tmem_ld_32x32b_x16(t_acc + c, v);
                    }
                    tmem_wait_ld();
                    if (produce) {
#pragma unroll
                        for (int j = 0; j < Cfg::kChunk; j += 4)
                            my_slot[((c + j) / 4) * kMmaM + r] = make_float4(
                                __uint_as_float(v[j]), __uint_as_float(v[j + 1]), __uint_as_float(v[j + 2]),
                                __uint_as_float(v[j + 3]));
                        continue;
                    }
                    if (finish) {
#pragma unroll
                        for (int j = 0; j < Cfg::kChunk; j += 4) {
                            const size_t qi = static_cast<size_t>((c + j) / 4) * kMmaM + r;
                            float4 sum;
                            if (one_producer) {
                                sum = staged[qi];
                            } else {
                                sum = __ldcg(slots + static_cast<size_t>(p_lo) * kSlotQuads + qi);
                                for (int q = p_lo + 1; q < g; ++q) {
                                    const float4 x = __ldcg(slots + static_cast<size_t>(q) * kSlotQuads + qi);
                                    sum.x += x.x; sum.y += x.y; sum.z += x.z; sum.w += x.w;
                                }
                            }
                            v[j] = __float_as_uint(sum.x + __uint_as_float(v[j]));
                            v[j + 1] = __float_as_uint(sum.y + __uint_as_float(v[j + 1]));
                            v[j + 2] = __float_as_uint(sum.z + __uint_as_float(v[j + 2]));
                            v[j + 3] = __float_as_uint(sum.w + __uint_as_float(v[j + 3]));
                        }
                    }
                    if constexpr (kSwap) {
                        if (p.tma_store) {
                            epi_add_col<Cfg::kChunk>(p, tr * kMmaM + r, tc * kBNm + c, v);
                            store_box_tma_t<Cfg::kChunk>(&tm_c, smem + kStages * Cfg::kStageBytes + warp * 4096u + epi_buf * 2048u,
                                                         lane, v, tr * kMmaM + static_cast<int>(warp) * 32, tc * kBNm + c,
                                                         (p.epi & kEpiSiluMul) != 0);
                            epi_buf ^= 1u;
                        } else {
                            store_col_segment<Cfg::kChunk>(p, tr * kMmaM + r, tc * kBNm + c, v);
                        }
                    } else {
                        if constexpr (Cfg::kChunk == 32) {
                            if (p.sc_ranks > 0) {
                                store_block_f32(p, reinterpret_cast<float*>(smem + kStages * Cfg::kStageBytes + warp * 8192u),
                                                lane, v, tr * kMmaM + static_cast<int>(warp) * 32, tc * kBNm + c);
                                continue;
                            }
                        }
                        store_row_segment<Cfg::kChunk>(p, tr * kMmaM + r, tc * kBNm + c, v);
                    }
                }
            }
            tc_fence_before_sync();
            mbar_arrive(&tempty[acc]);
            if (!ok_tile) break;
            if (produce) {
                // Publish this CTA's partial: each thread fences its stores at
                // GPU scope and arrives; thread 0 waits (bounded) for all 128
                // and then release-stores the flag.
                __threadfence();
                mbar_arrive(published);
                if (r == 0 && mbar_wait(published, 0, wc)) st_release_u64(p.flags + g, p.epoch);
            } else if (finish) {
                // Once all 128 threads have read the partial, reset its flag so
                // that a replay of this launch waits for a fresh one.
                mbar_arrive(consumed);
                if (r == 0 && mbar_wait(consumed, 0, wc))
                    for (int q = p_lo; q < g; ++q) p.flags[q] = 0ull;
            }
        }
        if (p.tma_store && lane == 0) bulk_wait_group_all();
    }

    __syncwarp();
    if (p.sc_ranks > 0) __threadfence_system();   // peer stores of a scatter, before the grid ends
    tc_fence_before_sync();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after_sync();
        tmem_dealloc(tmem_base, Cfg::kTmemCols);
    }
}

// ======================================== stream-K CTA-pair kernel (256x256) ====
//
// The CTA-pair kernel's 256 x 256 tiles with the stream-K work split of
// hgemm_streamk_kernel: pair g of G processes whole tiles g, g + G, ... in
// waves, then its equal share of the K blocks of the last (T mod G) + G tiles
// (each share at least one tile long, so a tile has at most two owners). A
// share that does not end a tile leaves its FP32 partial in the workspace:
// each CTA of the pair its own 128 rows, in slot 2 g + rank, published with
// flag 2 g + rank; the pair owning a tile's last K block adds the partials of
// the lower-numbered pairs in pair order (deterministic) to its own and
// stores C. Slots are [quad][row] float4 columns as in hgemm_streamk_kernel,
// flags hold the launch's epoch while valid and are reset by the finisher.
// All waits are bounded; the host sizes the grid so that every pair is
// resident at once.

template <int kStages>
__global__ void __launch_bounds__(kThreads, 1)
hgemm_pair_streamk_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                          const __grid_constant__ CUtensorMap tm_c, const GemmParams p) {
    using Cfg = PairCfg<256, 256, kStages>;
    constexpr uint32_t kSlotBytes = 128u * 256u * 4u;   // one CTA's FP32 half of a pair tile
    static_assert(kSlotBytes <= kStages * Cfg::kStageBytes, "a partial slot fits the stage ring");
    static_assert(2 * kStages + 9 <= 31, "barrier area");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align_1024(smem_raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kDataBytes);   // even CTA
    uint64_t* empty = full + kStages;
    uint64_t* tfull = empty + kStages;      // [2]
    uint64_t* tempty = tfull + 2;           // [2], even CTA
    uint64_t* drain = tempty + 2;
    uint64_t* published = drain + 1;        // 128 epilogue threads wrote this CTA's partial
    uint64_t* consumed = published + 1;     // 128 epilogue threads read the producers' partials
    uint64_t* landed = consumed + 1;        // a producer's slot arrived in shared memory
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(landed + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const uint32_t warp = warp_index();
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t rank = cluster_ctarank();   // 0 = MMA CTA, 1 = peer
    const bool leader = rank == 0;

    if (warp == 4 && lane == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1u);
            mbar_init(&empty[s], 1u);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1u);
            mbar_init(&tempty[i], 8u);     // one lane of each epilogue warp, both CTAs
        }
        mbar_init(drain, 1u);
        mbar_init(published, 128u);       // a CTA produces <= 1 partial and finishes <= 1 tile
        mbar_init(consumed, 128u);
        mbar_init(landed, 1u);
        *abort_flag = 0;
        mbar_init_fence();
        tma_prefetch_map(&tm_a);
        tma_prefetch_map(&tm_b);
    }
    if (warp == 5) {
        tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before_sync();
    cluster_sync();                       // both CTAs' barriers exist before any remote op
    tc_fence_after_sync();
    const uint32_t tmem_base = *tmem_slot;
    grid_dependents_launch();
    grid_dependency_wait();
    const WaitCtl wc{abort_flag, p.status, p.timeout_ns};

    const int tiles_m = (p.m + 255) / 256;
    const int tiles_n = (p.n + 255) / 256;
    const int T = tiles_m * tiles_n;
    const int KB = (p.k + kBlockK - 1) / kBlockK;
    const int G = gridDim.x >> 1;
    const int g = blockIdx.x >> 1;
    const int n_sk = p.streamk;

    if (warp == 4) {
        if (lane == 0) {
            uint32_t stage = 0, phase = 0, issued = 0;
            bool ok = true;
            SegIter it(g, G, T, KB, n_sk);
            Seg sg;
            while (ok && it.next(sg)) {
                int tm, tn;
                tile_coords(sg.tile, tiles_m, tiles_n, p.group_m, tm, tn);
                const int row0 = tm * 256 + static_cast<int>(rank) * Cfg::kRows;
                const int col0 = tn * 256 + static_cast<int>(rank) * Cfg::kHalfN;
                // Whole tiles walk K backwards on odd waves, as in hgemm_pair_kernel.
                const bool backwards = sg.tile < T - n_sk && ((sg.tile / G) & 1) != 0;
                for (int kq = sg.kb0; kq < sg.kb1; ++kq) {
                    const int kb = backwards ? sg.kb0 + sg.kb1 - 1 - kq : kq;
                    if (!mbar_wait_cluster(&empty[stage], phase ^ 1u, wc)) { ok = false; break; }
                    uint8_t* s_a = smem + stage * Cfg::kStageBytes;
                    uint8_t* s_b = s_a + Cfg::kABytes;
                    const uint32_t bar = map_to_rank(smem_addr(&full[stage]), 0);
                    if (leader) {
                        const uint32_t extra = (p.inject && issued == 0) ? 16u : 0u;
                        mbar_arrive_expect_tx(&full[stage], 2u * Cfg::kStageBytes + extra);
                    }
                    tma_load_2d_pair(s_a, &tm_a, bar, kb * kBlockK, row0);
#pragma unroll
                    for (int j = 0; j < Cfg::kHalfN / 64; ++j)
                        tma_load_2d_pair(s_b + j * kChunkBytes, &tm_b, bar, col0 + 64 * j, kb * kBlockK);
                    ++issued;
                    if (++stage == kStages) { stage = 0; phase ^= 1u; }
                }
            }
            if (leader && (!ok || *abort_flag)) drain_tma<kStages>(full, issued);
        }
    } else if (warp == 5) {
        if (lane == 0 && leader) {
            uint32_t stage = 0, phase = 0, iter = 0;
            bool ok = true;
            SegIter it(g, G, T, KB, n_sk);
            Seg sg;
            while (ok && it.next(sg)) {
                const uint32_t acc = iter & 1u, acc_phase = (iter >> 1) & 1u;
                if (!mbar_wait_cluster(&tempty[acc], acc_phase ^ 1u, wc)) { ok = false; break; }
                tc_fence_after_sync();
                const uint32_t d = tmem_base + acc * Cfg::kAccCols;
                for (int kb = sg.kb0; kb < sg.kb1; ++kb) {
                    if (!mbar_wait(&full[stage], phase, wc)) { ok = false; break; }
                    tc_fence_after_sync();
                    const uint32_t s_a = smem_addr(smem + stage * Cfg::kStageBytes);
                    const uint32_t s_b = s_a + Cfg::kABytes;
#pragma unroll
                    for (int kk = 0; kk < kBlockK / 16; ++kk)
                        tc_mma_f16_pair(d, kmaj_desc(s_a, kk), mnmaj_desc(s_b, kk), Cfg::kIdesc,
                                        (kb > sg.kb0 || kk > 0) ? 1u : 0u);
                    tc_commit_pair_both(smem_addr(&empty[stage]));
                    if (++stage == kStages) { stage = 0; phase ^= 1u; }
                }
                if (ok) tc_commit_pair_both(smem_addr(&tfull[acc]));
                ++iter;
            }
            if (!ok) {
                tc_commit_pair(smem_addr(drain));
                mbar_wait_drain(drain, 0, kDrainLimitNs);
            }
        }
    } else if (warp < 4) {
        const uint32_t t_lane = (warp * 32u) << 16;
        const int r = warp * 32 + lane;                 // accumulator row of this CTA (TMEM lane)
        const uint32_t tempty_leader0 = map_to_rank(smem_addr(&tempty[0]), 0);
        const uint32_t tempty_leader1 = map_to_rank(smem_addr(&tempty[1]), 0);
        const long long W_sk = static_cast<long long>(n_sk) * KB;
        const long long base_sk = static_cast<long long>(T - n_sk) * KB;
        const int slot = 2 * g + static_cast<int>(rank);
        uint32_t iter = 0, epi_buf = 0;
        SegIter it(g, G, T, KB, n_sk);
        Seg sg;
        while (it.next(sg)) {
            const uint32_t acc = iter & 1u, acc_phase = (iter >> 1) & 1u;
            ++iter;
            if (!__all_sync(0xffffffffu, mbar_wait_cluster(&tfull[acc], acc_phase, wc))) break;
            tc_fence_after_sync();
            int tm, tn;
            tile_coords(sg.tile, tiles_m, tiles_n, p.group_m, tm, tn);
            const int row_base = tm * 256 + static_cast<int>(rank) * Cfg::kRows;
            const uint32_t t_acc = tmem_base + t_lane + acc * Cfg::kAccCols;
            const bool produce = sg.kb1 < KB;                 // partial owed to a later pair
            const bool finish = !produce && sg.kb0 > 0;       // adds earlier pairs' partials
            int p_lo = g;
            if (finish) {
                p_lo = sk_owner(static_cast<long long>(sg.tile) * KB - base_sk, G, W_sk);
                bool ready = true;
                for (int q = p_lo; q < g && ready; ++q) {
                    const uint64_t t0 = global_timer_ns();
                    while (ld_acquire_u64(p.flags + 2 * q + rank) != p.epoch) {
                        if (*abort_flag || global_timer_ns() - t0 > p.timeout_ns) {
                            raise_abort(wc, kStatusPipelineTimeout);
                            ready = false;
                            break;
                        }
                    }
                }
                if (!__all_sync(0xffffffffu, ready)) {
                    tc_fence_before_sync();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(acc ? tempty_leader1 : tempty_leader0);
                    break;
                }
            }
            // The finisher segment is this pair's last: the stage ring is idle
            // (every MMA completed), so a single producer's slot is pulled into
            // it with bulk copies; with several producers slots are read from
            // global memory. The sum is (slot p_lo + ... + slot g - 1) + own.
            const float4* staged = reinterpret_cast<const float4*>(smem);
            const float4* slots = reinterpret_cast<const float4*>(p.partials);
            constexpr size_t kSlotQuads = kSlotBytes / 16;
            float4* my_slot = reinterpret_cast<float4*>(p.partials) + static_cast<size_t>(slot) * kSlotQuads;
            const bool one_producer = finish && p_lo == g - 1;
            bool ok_tile = true;
            if (one_producer) {
                if (r == 0) {
                    mbar_arrive_expect_tx(landed, kSlotBytes);
                    const uint8_t* src = reinterpret_cast<const uint8_t*>(
                        slots + static_cast<size_t>(2 * p_lo + static_cast<int>(rank)) * kSlotQuads);
                    for (uint32_t off = 0; off < kSlotBytes; off += 32768u)
                        bulk_load(smem + off, src + off, 32768u, landed);
                }
                ok_tile = __all_sync(0xffffffffu, mbar_wait(landed, 0, wc));
            }
            if (ok_tile && p.tma_store && !produce) {
                uint8_t* boxes = smem + kStages * Cfg::kStageBytes + warp * 8192u;
#pragma unroll 1
                for (int c = 0; c < 256; c += 64) {
                    uint32_t v0[32], v1[32];
                    tmem_ld_32x32b_x32(t_acc + c, v0);
                    tmem_ld_32x32b_x32(t_acc + c + 32, v1);
                    if (finish) {
                        float4 part[16];
                        const size_t q0 = static_cast<size_t>(c / 4) * 128u + r;
                        if (one_producer) {
#pragma unroll
                            for (int q = 0; q < 16; ++q) part[q] = staged[q0 + static_cast<size_t>(q) * 128u];
                        } else {
#pragma unroll
                            for (int q = 0; q < 16; ++q)
                                part[q] = __ldcg(slots + static_cast<size_t>(2 * p_lo + static_cast<int>(rank)) * kSlotQuads +
                                                 q0 + static_cast<size_t>(q) * 128u);
                            for (int s2 = p_lo + 1; s2 < g; ++s2) {
#pragma unroll
                                for (int q = 0; q < 16; ++q) {
                                    const float4 x = __ldcg(slots + static_cast<size_t>(2 * s2 + static_cast<int>(rank)) *
                                                                        kSlotQuads + q0 + static_cast<size_t>(q) * 128u);
                                    part[q].x += x.x; part[q].y += x.y; part[q].z += x.z; part[q].w += x.w;
                                }
                            }
                        }
                        tmem_wait_ld();
#pragma unroll
                        for (int q = 0; q < 16; ++q) {
                            uint32_t* v = q < 8 ? v0 + 4 * q : v1 + 4 * (q - 8);
                            v[0] = __float_as_uint(part[q].x + __uint_as_float(v[0]));
                            v[1] = __float_as_uint(part[q].y + __uint_as_float(v[1]));
                            v[2] = __float_as_uint(part[q].z + __uint_as_float(v[2]));
                            v[3] = __float_as_uint(part[q].w + __uint_as_float(v[3]));
                        }
                    } else {
                        tmem_wait_ld();
                    }
                    epi_add_row<32>(p, row_base + r, tn * 256 + c, v0);
                    epi_add_row<32>(p, row_base + r, tn * 256 + c + 32, v1);
                    store_box_tma(&tm_c, boxes + epi_buf * 4096u, lane, v0, v1, tn * 256 + c,
                                  row_base + static_cast<int>(warp) * 32);
                    epi_buf ^= 1u;
                }
            } else if (ok_tile) {
#pragma unroll 1
                for (int c = 0; c < 256; c += 32) {
                    uint32_t v[32];
                    tmem_ld_32x32b_x32(t_acc + c, v);
                    tmem_wait_ld();
                    if (produce) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4)
                            my_slot[((c + j) / 4) * 128 + r] = make_float4(
                                __uint_as_float(v[j]), __uint_as_float(v[j + 1]), __uint_as_float(v[j + 2]),
                                __uint_as_float(v[j + 3]));
                        continue;
                    }
                    if (finish) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4) {
                            const size_t qi = static_cast<size_t>((c + j) / 4) * 128u + r;
                            float4 sum;
                            if (one_producer) {
                                sum = staged[qi];
                            } else {
                                sum = __ldcg(slots + static_cast<size_t>(2 * p_lo + static_cast<int>(rank)) * kSlotQuads + qi);
                                for (int q = p_lo + 1; q < g; ++q) {
                                    const float4 x = __ldcg(slots + static_cast<size_t>(2 * q + static_cast<int>(rank)) *
                                                                        kSlotQuads + qi);
                                    sum.x += x.x; sum.y += x.y; sum.z += x.z; sum.w += x.w;
                                }
                            }
                            v[j] = __float_as_uint(sum.x + __uint_as_float(v[j]));
                            v[j + 1] = __float_as_uint(sum.y + __uint_as_float(v[j + 1]));
                            v[j + 2] = __float_as_uint(sum.z + __uint_as_float(v[j + 2]));
                            v[j + 3] = __float_as_uint(sum.w + __uint_as_float(v[j + 3]));
                        }
                    }
                    store_row_segment<32>(p, row_base + r, tn * 256 + c, v);
                }
            }
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc ? tempty_leader1 : tempty_leader0);
            if (!ok_tile) break;
            if (produce) {
                __threadfence();
                mbar_arrive(published);
                if (r == 0 && mbar_wait(published, 0, wc)) st_release_u64(p.flags + slot, p.epoch);
            } else if (finish) {
                mbar_arrive(consumed);
                if (r == 0 && mbar_wait(consumed, 0, wc))
                    for (int q = p_lo; q < g; ++q) p.flags[2 * q + rank] = 0ull;
            }
        }
        if (p.tma_store && lane == 0) bulk_wait_group_all();
    }

    __syncwarp();
    if (*abort_flag) settle_ns(2000000ull);
    tc_fence_before_sync();
    cluster_sync();                       // no CTA leaves while its pair may still touch it
    if (warp == 5) {
        tc_fence_after_sync();
        tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
    }
}

}  // namespace hgemm
