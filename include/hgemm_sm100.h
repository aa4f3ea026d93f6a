/*
 * hgemm_sm100.h - C ABI of the B200 (sm_100a) FP16 HGEMM library.
 *
 *   C[M,N] = A[M,K] @ B[K,N]   FP16 inputs, FP32 accumulation, FP16 output,
 *                              row-major, alpha = 1, beta = 0.
 *
 * This is the boundary between host code (the llm_hgemm pybind11 module, or
 * any other FFI) and the hand-written sm_100a kernels. It takes plain device
 * pointers, sizes and a stream; no C++ exceptions and no torch types cross it.
 *
 * It replaces the reference's torch-typed launcher layer:
 *   - csrc/kernels.h:6-78 and csrc/references/reference.h:13-29
 *     (`void launch_X(const Tensor& a, const Tensor& b, Tensor& out,
 *      cudaStream_t)`, one per backend)                -> hgemm_sm100_run
 *   - csrc/dispatch.cpp:30-32 (`auto` -> backend) and :58-95 (name -> launcher
 *     chain)                       -> hgemm_sm100_config_from_name / _resolve
 *   - csrc/dispatch.cpp:104-128 (`backend_info`)  -> hgemm_sm100_workspace_bytes,
 *                                                    hgemm_sm100_workspace_size
 *   - csrc/dispatch.cpp:99-101 (`has_cutlass`)    -> no counterpart (always 0)
 * Input validation with the reference's messages (csrc/contract.cpp:3-22)
 * stays in the host module; this layer re-checks sizes, strides and
 * alignment and reports violations as status codes.
 *
 * Threading: every entry point is thread-safe. Launches are asynchronous on
 * the given stream; nothing synchronises the host.
 */
#ifndef HGEMM_SM100_H_
#define HGEMM_SM100_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes (return value of every int-returning entry point). */
enum {
    HGEMM_SM100_OK = 0,
    HGEMM_SM100_ERR_INVALID_ARGUMENT = 1,  /* null pointer, size <= 0, ld < row */
    HGEMM_SM100_ERR_UNKNOWN_CONFIG = 2,    /* config id out of range            */
    HGEMM_SM100_ERR_UNSUPPORTED_DEVICE = 3,/* current device is not sm_100      */
    HGEMM_SM100_ERR_LAUNCH = 4,            /* CUDA launch / attribute failure   */
    HGEMM_SM100_ERR_PIPELINE_TIMEOUT = 5,  /* a kernel wait ran out (status word)*/
    HGEMM_SM100_ERR_TENSOR_MAP = 6,        /* cuTensorMapEncodeTiled failed     */
    HGEMM_SM100_ERR_CUDA = 7,              /* other CUDA runtime error          */
    HGEMM_SM100_ERR_SCRATCH_LIMIT = 8,     /* needs more scratch than the static
                                              buffer of hgemm_sm100_run_static_scratch */
    HGEMM_SM100_ERR_DEBUG_BOUNDS = 9       /* debug build: a device bounds check
                                              failed (status word)               */
};

/* Kernel configurations. Every name is also accepted by
 * hgemm_sm100_config_from_name (the `implementation=` strings of llm_hgemm). */
enum {
    HGEMM_SM100_CFG_AUTO = 0,              /* "auto": shape heuristic           */
    HGEMM_SM100_CFG_PERSISTENT_128x256 = 1,/* "tc_persistent_128x256"           */
    HGEMM_SM100_CFG_PERSISTENT_128x128 = 2,/* "tc_persistent_128x128"           */
    HGEMM_SM100_CFG_SPLITK_128x128 = 3,    /* "tc_splitk_128x128": cluster split-K */
    HGEMM_SM100_CFG_SWAPAB = 4,            /* "tc_swapab": C^T = B^T A^T, M <= 256 */
    HGEMM_SM100_CFG_GENERIC_128x128 = 5,   /* "tc_generic_128x128": no TMA       */
    HGEMM_SM100_CFG_PAIR_256x256 = 6,      /* "tc_pair_256x256": CTA pair,
                                              cta_group::2, persistent          */
    HGEMM_SM100_CFG_SPLITK_128x256 = 7,    /* "tc_splitk_128x256": cluster split-K */
    HGEMM_SM100_CFG_STREAMK_128x256 = 8,   /* "tc_streamk_128x256": persistent,
                                              stream-K ranges (workspace)       */
    HGEMM_SM100_CFG_STREAMK_SWAPAB = 9,    /* "tc_streamk_swapab": the same with
                                              C^T = B^T A^T, M <= 128           */
    HGEMM_SM100_CFG_PAIR_256x128 = 10,     /* "tc_pair_256x128": CTA pair, 256 x 128
                                              tiles (one wave for mid-size M)   */
    HGEMM_SM100_CFG_PAIR_128x256 = 11,     /* "tc_pair_128x256": CTA pair, 128 x 256
                                              tiles, 64 rows per CTA            */
    HGEMM_SM100_CFG_PAIR_128x128 = 12,     /* "tc_pair_128x128": CTA pair, 128 x 128
                                              tiles, 64 rows per CTA            */
    HGEMM_SM100_CFG_STREAMK_PAIR_256x256 = 13, /* "tc_streamk_pair_256x256": CTA-pair
                                              256 x 256 tiles in waves, the last
                                              partial wave's K blocks spread over
                                              all pairs (workspace)              */
    HGEMM_SM100_CFG_COUNT = 14
};

/* Flags. */
enum {
    HGEMM_SM100_FLAG_OUT_F32 = 1,          /* C is FP32 (tensor-parallel partials) */
    HGEMM_SM100_FLAG_TEST_INJECT_TX = 2    /* test only: arm one stage with 16 bytes
                                              more than TMA delivers, so that the
                                              pipeline wait runs out */
};

/* Fused epilogue (HgemmSm100Args.epilogue, a bit set; 0 = C = A @ B). Every
 * term is added to the FP32 accumulator and the result rounded to FP16 once,
 * by the CTA that stores the final sum (split-K and stream-K partials stay
 * raw). Not combinable with HGEMM_SM100_FLAG_OUT_F32. The reference accepts
 * only epilogue "none" (csrc/dispatch.cpp:52); these extend that argument. */
enum {
    HGEMM_SM100_EPI_BIAS = 1,      /* + bias[j], FP16 [n]                         */
    HGEMM_SM100_EPI_RESIDUAL = 2,  /* + residual[i, j], FP16 [m x ldr] (ldr >= n); it
                                      may be C itself (ldr == ldc): each element
                                      is read before it is written              */
    HGEMM_SM100_EPI_SILU_MUL = 4   /* SwiGLU: B's columns hold (gate, up) pairs
                                      2j, 2j + 1 and C[i, j] = silu(g) * u with
                                      g, u the FP32 sums of those columns (after
                                      the bias); n even, C is [m x n/2]
                                      (ldc >= n/2); not with EPI_RESIDUAL       */
};

typedef struct HgemmSm100Args {
    const void* a;       /* FP16 [m x lda], row-major, device memory          */
    const void* b;       /* FP16 [k x ldb], row-major                         */
    void* c;             /* FP16 (or FP32 with FLAG_OUT_F32) [m x ldc]        */
    int64_t m, n, k;     /* > 0, each < 2^31                                   */
    int64_t lda, ldb, ldc;  /* leading dimensions in elements (>= k, n, n;
                               ldc >= n/2 with EPI_SILU_MUL)                 */
    int32_t config;      /* HGEMM_SM100_CFG_*                                 */
    int32_t split_k;     /* 0 = choose; else K splits (1..16), split configs  */
    int32_t flags;       /* HGEMM_SM100_FLAG_*                                */
    int32_t* status;     /* optional device int32 the kernel sets on a pipeline
                            timeout; NULL = the library's own status word     */
    uint64_t timeout_ns; /* per-wait limit inside the kernel; 0 = 2 s          */
    void* workspace;     /* optional device scratch for staging operands that
                            TMA cannot describe (see hgemm_sm100_workspace_size);
                            NULL = no staging                                 */
    uint64_t workspace_bytes;
    int32_t epilogue;    /* HGEMM_SM100_EPI_* bits; 0 = plain C = A @ B       */
    int32_t reserved;    /* 0                                                 */
    const void* bias;    /* FP16 [n], device memory, with EPI_BIAS            */
    const void* residual;/* FP16 [m x ldr], device memory, with EPI_RESIDUAL  */
    int64_t ldr;         /* residual leading dimension in elements            */
} HgemmSm100Args;

/* Launches C = A @ B on `stream` (a cudaStream_t; NULL = legacy default) on
 * the current device. TMA needs 16-byte-aligned bases and leading dimensions
 * that are multiples of 8 halves. For operands that break this (ragged
 * shapes such as N = 8193, or offset views):
 *   - with a workspace of at least hgemm_sm100_workspace_size(args) bytes,
 *     the offending operands are first copied (stream-ordered) into aligned,
 *     padded staging buffers in the workspace, the TMA kernels run on those,
 *     and a staged C is copied back;
 *   - without one, the generic (no-TMA) configuration runs, as the
 *     reference's v6 kernels fall back to v5 (csrc/v6_mma_async.cu:428-437).
 * Returns HGEMM_SM100_OK or an error; device-side pipeline timeouts are
 * reported through the status word. */
int hgemm_sm100_run(const HgemmSm100Args* args, void* stream);

/* The configuration and K split that hgemm_sm100_run would launch for
 * `args` (after `auto` resolution and the alignment fallback). */
int hgemm_sm100_resolve(const HgemmSm100Args* args, int32_t* config_out, int32_t* split_out);

/* Name <-> id of a configuration; unknown names give -1, unknown ids NULL. */
int32_t hgemm_sm100_config_from_name(const char* name);
const char* hgemm_sm100_config_name(int32_t config);
int32_t hgemm_sm100_num_configs(void);

/* Global-memory workspace a configuration uses for an (m, n, k) problem with
 * aligned operands on the current device (HGEMM_SM100_CFG_AUTO is resolved to
 * the configuration it picks first): the stream-K configurations' per-CTA
 * slots and flags, or the split-K tile configurations' partial-tile exchange
 * (at the split the library chooses); 0 otherwise. Counterpart of
 * backend_info()["workspace_bytes"] (reference csrc/dispatch.cpp:104-128). */
size_t hgemm_sm100_workspace_bytes(int32_t config, int64_t m, int64_t n, int64_t k);

/* Workspace bytes hgemm_sm100_run needs for `args`: staging buffers for
 * operands that TMA cannot describe, plus, when the call resolves to a
 * stream-K configuration, one FP32 partial-tile slot and one flag per CTA,
 * or, for a split-K tile configuration, one FP32 partial tile per CTA
 * (exchanged through L2; without it the partials go through distributed
 * shared memory). 0 when none applies. Queries the current device (cached);
 * launches nothing. No state is kept between calls: any workspace of this
 * size works, whatever it contains. */
size_t hgemm_sm100_workspace_size(const HgemmSm100Args* args);

/* Runs C = A @ B like hgemm_sm100_run, but takes no workspace and allocates
 * nothing: the scratch that the stream-K kernels need (one FP32 partial-tile
 * slot and one flag per CTA) comes from a static device buffer of
 * HGEMM_SM100_STATIC_SCRATCH_BYTES inside this library, which every GPU that
 * loads the library holds until the process exits.
 * No counterpart in the reference. It exists for callers that cannot
 * allocate device memory when they call a GEMM: a plugin or FFI host handed
 * only input/output pointers and a stream, a runtime that plans all of its
 * memory ahead of time, or code that must not call cudaMalloc (which can
 * synchronise the device) on its hot path.
 * - config: HGEMM_SM100_CFG_AUTO (stream-K; swap-AB for m <= 128) or one of
 *   the two stream-K configurations; anything else -> ERR_UNKNOWN_CONFIG.
 *   With AUTO, a problem whose 128x256 split tail would need more scratch
 *   than the buffer runs whole tiles on the persistent kernel instead, which
 *   needs none.
 * - A and B must satisfy the TMA rules (16-byte-aligned bases, lda and ldb
 *   multiples of 8); otherwise ERR_INVALID_ARGUMENT (staging would need
 *   scratch of the operands' size).
 * - An explicit stream-K configuration whose scratch exceeds the static
 *   buffer is rejected with HGEMM_SM100_ERR_SCRATCH_LIMIT and nothing is
 *   launched (the swap-AB configuration, m <= 128, always fits; a 128x256
 *   stream-K split tail does not on a 148-SM GPU).
 * - The first call of any entry point of this library on a device looks up
 *   the buffer's device address (cudaGetSymbolAddress) with that device
 *   current; make that first call before any stream capture.
 * - Every call shares the one buffer and it keeps the last call's contents;
 *   nothing in it needs clearing (each launch's flags carry a fresh value that
 *   stale contents never equal). Calls that overlap on the GPU (for example
 *   on two streams) race on it: serialise them. */
#define HGEMM_SM100_STATIC_SCRATCH_BYTES (16u * 1024u * 1024u)
int hgemm_sm100_run_static_scratch(const HgemmSm100Args* args, void* stream);

/* ------------------------------------------- tensor-parallel row scatter --
 * The row-parallel (K-split) GEMM of a tensor-parallel layer produces one FP32
 * partial C per GPU, and the layer's output is their sum. No counterpart in
 * the reference (single-GPU); this replaces "FP32 GEMM, then NCCL
 * reduce-scatter": the GEMM's epilogue writes each output row straight into
 * the receive buffer of the GPU that owns the row (stores to peer memory over
 * NVLink, issued tile by tile while the next tiles compute), and each owner
 * then sums its slots (hgemm_sm100_reduce_slots). */
#define HGEMM_SM100_MAX_RANKS 8

typedef struct HgemmSm100Scatter {
    int32_t ranks;          /* 1 .. HGEMM_SM100_MAX_RANKS                        */
    int32_t rank;           /* this GPU's rank                                   */
    int64_t rows_per_rank;  /* m == ranks * rows_per_rank; rank q owns rows
                               [q * rows_per_rank, (q + 1) * rows_per_rank)      */
    int64_t ld_dest;        /* row pitch of every receive buffer, floats (>= n)  */
    void* dest[HGEMM_SM100_MAX_RANKS];
                            /* receive buffer of each rank as mapped in this
                               process (dest[rank] local, the others peer
                               mappings, see hgemm_sm100_ipc_open): FP32
                               [ranks][rows_per_rank][ld_dest], slot s written
                               by rank s                                         */
} HgemmSm100Scatter;

/* hgemm_sm100_run with the row scatter: args->flags must include
 * HGEMM_SM100_FLAG_OUT_F32 and args->epilogue must be 0; args->c / ldc are
 * not written (pass any valid pointer and ldc >= n). Output row i (of m)
 * goes to dest[q] + ((rank * rows_per_rank) + i - q * rows_per_rank) * ld_dest,
 * q = i / rows_per_rank. The kernel waits for no other GPU: the caller orders
 * every owner's reduction after all ranks' GEMMs (a collective on the stream,
 * for example), and a receive buffer is not rewritten before its owner has
 * reduced it (double-buffer across steps). */
int hgemm_sm100_run_scatter(const HgemmSm100Args* args, const HgemmSm100Scatter* scatter, void* stream);

/* out[j, c] = FP16(sum of slots[s][j][c] over s = 0 .. ranks-1, added in that
 * order in FP32, one rounding), j < rows, c < cols. slots: FP32
 * [ranks][rows][ld_slots], out: FP16 [rows][ld_out], device memory. */
int hgemm_sm100_reduce_slots(const void* slots, int32_t ranks, int64_t rows, int64_t cols, int64_t ld_slots,
                             void* out, int64_t ld_out, void* stream);

/* hgemm_sm100_reduce_slots writing the same FP16 rows to n_outs (1 .. 8)
 * destinations outs[i] (each [rows][ld_out]): with the peers' copies of the
 * owned rows among them (peer mappings), the all-gather that completes an
 * all-reduce. The caller orders the peers' reads after it (a collective on
 * the stream) and their earlier reads of those rows before it. */
int hgemm_sm100_reduce_slots_gather(const void* slots, int32_t ranks, int64_t rows, int64_t cols, int64_t ld_slots,
                                    void* const* outs, int32_t n_outs, int64_t ld_out, void* stream);

/* Device memory on the current device whose CUDA IPC handle maps exactly this
 * range in another process of the node (a whole cudaMalloc allocation). */
int hgemm_sm100_alloc_shared(uint64_t bytes, void** ptr_out);
int hgemm_sm100_free_shared(void* ptr);
/* 64-byte IPC handle of an hgemm_sm100_alloc_shared pointer; mapping of a
 * peer's handle in this process (peer access enabled), and its release. */
int hgemm_sm100_ipc_handle(const void* ptr, void* handle_out);
int hgemm_sm100_ipc_open(const void* handle, void** ptr_out);
int hgemm_sm100_ipc_close(void* ptr);

/* Human-readable text of a status code. */
const char* hgemm_sm100_status_string(int status);

/* Reads (and with clear != 0 resets) the library's own device status word of
 * the current device. Synchronises the device; for tests and debugging. */
int hgemm_sm100_read_status(int32_t* value, int clear);

/* ------------------------------------------------------------ debug build --
 * The same library compiled with -DHGEMM_DEBUG (libhgemm_sm100_debug.so,
 * `python build.py --debug`) checks, before every global access whose address
 * the kernels compute themselves (the generic no-TMA tile loader, the operand
 * staging copy, the epilogue's register stores), that it stays inside its
 * matrix. A failed check skips the access, records the first failure and sets
 * HGEMM_SM100_ERR_DEBUG_BOUNDS in the status word; nothing traps. The
 * reference has no such switch: its kernels are checked by sanitizer runs only.
 *
 * hgemm_sm100_debug_build: 1 in a debug build, else 0.
 * hgemm_sm100_debug_read: the first recorded failure of the current device
 * (source line, or 0 when none, and two indices of the access: row and
 * column); synchronises the device; clear != 0 resets the record. In a
 * release build it reports line 0.
 * hgemm_sm100_debug_vec_touches / _span_in: the checks themselves, on the
 * host, for tests. A row-major matrix of rows x cols elements of esize bytes,
 * pitch ld elements, at address base: vec_touches is 1 when the 16-byte-aligned
 * vector at `vec` holds at least one of its elements (the generic loader's
 * rule), span_in is 1 when the `count` consecutive elements at `ptr` are
 * elements of one of its rows. */
int hgemm_sm100_debug_build(void);
int hgemm_sm100_debug_read(int32_t* line, int64_t* index0, int64_t* index1, int clear);
int hgemm_sm100_debug_vec_touches(uint64_t vec, uint64_t base, int64_t rows, int64_t cols, int64_t ld,
                                  int32_t esize);
int hgemm_sm100_debug_span_in(uint64_t ptr, int64_t count, uint64_t base, int64_t rows, int64_t cols,
                              int64_t ld, int32_t esize);

#ifdef __cplusplus
}
#endif

#endif /* HGEMM_SM100_H_ */
