"""ctypes binding of the C ABI in include/hgemm_sm100.h.

This is the binding a non-torch host (or any FFI user) writes against
``libhgemm_sm100.so``; the tests use it to call the kernels through the C
boundary directly. ``load()`` only opens the library (no GPU needed).
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libhgemm_sm100.so"
# The same library built with -DHGEMM_DEBUG (device-side bounds checks).
DEBUG_LIB_PATH = Path(__file__).resolve().parent / "libhgemm_sm100_debug.so"

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_UNKNOWN_CONFIG = 2
ERR_UNSUPPORTED_DEVICE = 3
ERR_LAUNCH = 4
ERR_PIPELINE_TIMEOUT = 5
ERR_TENSOR_MAP = 6
ERR_CUDA = 7
ERR_SCRATCH_LIMIT = 8
ERR_DEBUG_BOUNDS = 9
STATIC_SCRATCH_BYTES = 16 * 1024 * 1024

CFG_AUTO = 0
CFG_PERSISTENT_128x256 = 1
CFG_PERSISTENT_128x128 = 2
CFG_SPLITK_128x128 = 3
CFG_SWAPAB = 4
CFG_GENERIC_128x128 = 5
CFG_PAIR_256x256 = 6
CFG_SPLITK_128x256 = 7
CFG_STREAMK_128x256 = 8
CFG_STREAMK_SWAPAB = 9
CFG_PAIR_256x128 = 10
CFG_PAIR_128x256 = 11
CFG_PAIR_128x128 = 12
CFG_STREAMK_PAIR_256x256 = 13

FLAG_OUT_F32 = 1
FLAG_TEST_INJECT_TX = 2

# Fused-epilogue bits (HGEMM_SM100_EPI_*).
EPI_BIAS = 1
EPI_RESIDUAL = 2
EPI_SILU_MUL = 4


class HgemmSm100Args(ctypes.Structure):
    _fields_ = [
        ("a", ctypes.c_void_p),
        ("b", ctypes.c_void_p),
        ("c", ctypes.c_void_p),
        ("m", ctypes.c_int64),
        ("n", ctypes.c_int64),
        ("k", ctypes.c_int64),
        ("lda", ctypes.c_int64),
        ("ldb", ctypes.c_int64),
        ("ldc", ctypes.c_int64),
        ("config", ctypes.c_int32),
        ("split_k", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("status", ctypes.c_void_p),
        ("timeout_ns", ctypes.c_uint64),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_uint64),
        ("epilogue", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("bias", ctypes.c_void_p),
        ("residual", ctypes.c_void_p),
        ("ldr", ctypes.c_int64),
    ]


MAX_RANKS = 8


class HgemmSm100Scatter(ctypes.Structure):
    """Mirror of ``HgemmSm100Scatter`` (tensor-parallel row scatter)."""
    _fields_ = [
        ("ranks", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("rows_per_rank", ctypes.c_int64),
        ("ld_dest", ctypes.c_int64),
        ("dest", ctypes.c_void_p * MAX_RANKS),
    ]


_libs: dict[bool, ctypes.CDLL] = {}


def load(debug: bool = False) -> ctypes.CDLL:
    """The kernel library (``debug``: its -DHGEMM_DEBUG build)."""
    if debug not in _libs:
        lib = ctypes.CDLL(str(DEBUG_LIB_PATH if debug else LIB_PATH))
        lib.hgemm_sm100_run.argtypes = [ctypes.POINTER(HgemmSm100Args), ctypes.c_void_p]
        lib.hgemm_sm100_run.restype = ctypes.c_int
        lib.hgemm_sm100_resolve.argtypes = [ctypes.POINTER(HgemmSm100Args),
                                            ctypes.POINTER(ctypes.c_int32),
                                            ctypes.POINTER(ctypes.c_int32)]
        lib.hgemm_sm100_resolve.restype = ctypes.c_int
        lib.hgemm_sm100_config_from_name.argtypes = [ctypes.c_char_p]
        lib.hgemm_sm100_config_from_name.restype = ctypes.c_int32
        lib.hgemm_sm100_config_name.argtypes = [ctypes.c_int32]
        lib.hgemm_sm100_config_name.restype = ctypes.c_char_p
        lib.hgemm_sm100_num_configs.argtypes = []
        lib.hgemm_sm100_num_configs.restype = ctypes.c_int32
        lib.hgemm_sm100_workspace_bytes.argtypes = [ctypes.c_int32, ctypes.c_int64,
                                                    ctypes.c_int64, ctypes.c_int64]
        lib.hgemm_sm100_workspace_bytes.restype = ctypes.c_size_t
        lib.hgemm_sm100_run_static_scratch.argtypes = [ctypes.POINTER(HgemmSm100Args), ctypes.c_void_p]
        lib.hgemm_sm100_run_static_scratch.restype = ctypes.c_int
        lib.hgemm_sm100_workspace_size.argtypes = [ctypes.POINTER(HgemmSm100Args)]
        lib.hgemm_sm100_workspace_size.restype = ctypes.c_size_t
        lib.hgemm_sm100_status_string.argtypes = [ctypes.c_int]
        lib.hgemm_sm100_status_string.restype = ctypes.c_char_p
        lib.hgemm_sm100_read_status.argtypes = [ctypes.POINTER(ctypes.c_int32), ctypes.c_int]
        lib.hgemm_sm100_read_status.restype = ctypes.c_int
        lib.hgemm_sm100_run_scatter.argtypes = [ctypes.POINTER(HgemmSm100Args),
                                                ctypes.POINTER(HgemmSm100Scatter), ctypes.c_void_p]
        lib.hgemm_sm100_run_scatter.restype = ctypes.c_int
        lib.hgemm_sm100_reduce_slots.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
                                                 ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
                                                 ctypes.c_int64, ctypes.c_void_p]
        lib.hgemm_sm100_reduce_slots.restype = ctypes.c_int
        lib.hgemm_sm100_reduce_slots_gather.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
                                                        ctypes.c_int64, ctypes.c_int64,
                                                        ctypes.POINTER(ctypes.c_void_p), ctypes.c_int32,
                                                        ctypes.c_int64, ctypes.c_void_p]
        lib.hgemm_sm100_reduce_slots_gather.restype = ctypes.c_int
        lib.hgemm_sm100_alloc_shared.argtypes = [ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p)]
        lib.hgemm_sm100_alloc_shared.restype = ctypes.c_int
        lib.hgemm_sm100_free_shared.argtypes = [ctypes.c_void_p]
        lib.hgemm_sm100_free_shared.restype = ctypes.c_int
        lib.hgemm_sm100_ipc_handle.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        lib.hgemm_sm100_ipc_handle.restype = ctypes.c_int
        lib.hgemm_sm100_ipc_open.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]
        lib.hgemm_sm100_ipc_open.restype = ctypes.c_int
        lib.hgemm_sm100_ipc_close.argtypes = [ctypes.c_void_p]
        lib.hgemm_sm100_ipc_close.restype = ctypes.c_int
        lib.hgemm_sm100_debug_build.argtypes = []
        lib.hgemm_sm100_debug_build.restype = ctypes.c_int
        lib.hgemm_sm100_debug_read.argtypes = [ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int64),
                                               ctypes.POINTER(ctypes.c_int64), ctypes.c_int]
        lib.hgemm_sm100_debug_read.restype = ctypes.c_int
        lib.hgemm_sm100_debug_vec_touches.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int64,
                                                      ctypes.c_int64, ctypes.c_int64, ctypes.c_int32]
        lib.hgemm_sm100_debug_vec_touches.restype = ctypes.c_int
        lib.hgemm_sm100_debug_span_in.argtypes = [ctypes.c_uint64, ctypes.c_int64, ctypes.c_uint64, ctypes.c_int64,
                                                  ctypes.c_int64, ctypes.c_int64, ctypes.c_int32]
        lib.hgemm_sm100_debug_span_in.restype = ctypes.c_int
        _libs[debug] = lib
    return _libs[debug]


def make_args(a_ptr: int, b_ptr: int, c_ptr: int, m: int, n: int, k: int, *,
              lda: int | None = None, ldb: int | None = None, ldc: int | None = None,
              config: int = CFG_AUTO, split_k: int = 0, flags: int = 0,
              status_ptr: int | None = None, timeout_ns: int = 0,
              workspace_ptr: int | None = None, workspace_bytes: int = 0,
              epilogue: int = 0, bias_ptr: int | None = None, residual_ptr: int | None = None,
              ldr: int | None = None) -> HgemmSm100Args:
    if ldc is None:
        ldc = n // 2 if epilogue & EPI_SILU_MUL else n
    return HgemmSm100Args(a_ptr, b_ptr, c_ptr, m, n, k,
                          k if lda is None else lda, n if ldb is None else ldb,
                          ldc, config, split_k, flags,
                          status_ptr, timeout_ns, workspace_ptr, workspace_bytes,
                          epilogue, 0, bias_ptr, residual_ptr, n if ldr is None else ldr)


def run(args: HgemmSm100Args, stream: int = 0, debug: bool = False) -> int:
    return load(debug).hgemm_sm100_run(ctypes.byref(args), ctypes.c_void_p(stream))


def run_static_scratch(args: HgemmSm100Args, stream: int = 0) -> int:
    """hgemm_sm100_run_static_scratch: no workspace, nothing allocated."""
    return load().hgemm_sm100_run_static_scratch(ctypes.byref(args), ctypes.c_void_p(stream))


def resolve(args: HgemmSm100Args, debug: bool = False) -> tuple[int, int, int]:
    cfg, split = ctypes.c_int32(0), ctypes.c_int32(0)
    rc = load(debug).hgemm_sm100_resolve(ctypes.byref(args), ctypes.byref(cfg), ctypes.byref(split))
    return rc, cfg.value, split.value


def workspace_size(args: HgemmSm100Args, debug: bool = False) -> int:
    return load(debug).hgemm_sm100_workspace_size(ctypes.byref(args))


def status_string(code: int) -> str:
    return load().hgemm_sm100_status_string(code).decode()


def read_status(clear: bool = True, debug: bool = False) -> tuple[int, int]:
    v = ctypes.c_int32(0)
    rc = load(debug).hgemm_sm100_read_status(ctypes.byref(v), 1 if clear else 0)
    return rc, v.value


def debug_read(clear: bool = True, debug: bool = True) -> tuple[int, int, int, int]:
    """(rc, line, index0, index1) of the first failed bounds check recorded by
    the debug build (line 0: none)."""
    line, i0, i1 = ctypes.c_int32(0), ctypes.c_int64(0), ctypes.c_int64(0)
    rc = load(debug).hgemm_sm100_debug_read(ctypes.byref(line), ctypes.byref(i0), ctypes.byref(i1),
                                            1 if clear else 0)
    return rc, line.value, i0.value, i1.value


def debug_vec_touches(vec: int, base: int, rows: int, cols: int, ld: int, esize: int = 2) -> bool:
    return bool(load().hgemm_sm100_debug_vec_touches(vec, base, rows, cols, ld, esize))


def debug_span_in(ptr: int, count: int, base: int, rows: int, cols: int, ld: int, esize: int = 2) -> bool:
    return bool(load().hgemm_sm100_debug_span_in(ptr, count, base, rows, cols, ld, esize))


# ------------------------------------------- tensor-parallel row scatter --

def make_scatter(ranks: int, rank: int, rows_per_rank: int, ld_dest: int, dest: list[int]) -> HgemmSm100Scatter:
    if len(dest) != ranks or ranks > MAX_RANKS:
        raise ValueError("one destination per rank, at most 8 ranks")
    arr = (ctypes.c_void_p * MAX_RANKS)(*dest, *([None] * (MAX_RANKS - ranks)))
    return HgemmSm100Scatter(ranks, rank, rows_per_rank, ld_dest, arr)


def run_scatter(args: HgemmSm100Args, scatter: HgemmSm100Scatter, stream: int = 0) -> int:
    return load().hgemm_sm100_run_scatter(ctypes.byref(args), ctypes.byref(scatter), ctypes.c_void_p(stream))


def reduce_slots(slots_ptr: int, ranks: int, rows: int, cols: int, ld_slots: int, out_ptr: int, ld_out: int,
                 stream: int = 0) -> int:
    return load().hgemm_sm100_reduce_slots(slots_ptr, ranks, rows, cols, ld_slots, out_ptr, ld_out,
                                           ctypes.c_void_p(stream))


def reduce_slots_gather(slots_ptr: int, ranks: int, rows: int, cols: int, ld_slots: int, out_ptrs: list[int],
                        ld_out: int, stream: int = 0) -> int:
    outs = (ctypes.c_void_p * len(out_ptrs))(*out_ptrs)
    return load().hgemm_sm100_reduce_slots_gather(slots_ptr, ranks, rows, cols, ld_slots, outs, len(out_ptrs),
                                                  ld_out, ctypes.c_void_p(stream))


class DeviceArray:
    """A device buffer of this library (e.g. hgemm_sm100_alloc_shared) seen
    through the CUDA array interface, so that ``torch.as_tensor`` wraps it
    without a copy. The buffer must outlive the tensor."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 2, "strides": None}


def _checked(rc: int, what: str) -> None:
    if rc != OK:
        raise RuntimeError(f"{what} failed: {status_string(rc)}")


def alloc_shared(nbytes: int) -> int:
    p = ctypes.c_void_p()
    _checked(load().hgemm_sm100_alloc_shared(nbytes, ctypes.byref(p)), "hgemm_sm100_alloc_shared")
    return p.value


def free_shared(ptr: int) -> None:
    _checked(load().hgemm_sm100_free_shared(ptr), "hgemm_sm100_free_shared")


def ipc_handle(ptr: int) -> bytes:
    buf = ctypes.create_string_buffer(64)
    _checked(load().hgemm_sm100_ipc_handle(ptr, buf), "hgemm_sm100_ipc_handle")
    return buf.raw


def ipc_open(handle: bytes) -> int:
    if len(handle) != 64:
        raise ValueError("IPC handles are 64 bytes")
    p = ctypes.c_void_p()
    _checked(load().hgemm_sm100_ipc_open(handle, ctypes.byref(p)), "hgemm_sm100_ipc_open")
    return p.value


def ipc_close(ptr: int) -> None:
    _checked(load().hgemm_sm100_ipc_close(ptr), "hgemm_sm100_ipc_close")
