"""In-tree build of the llm_hgemm native libraries (sm_100a only).

Produces, next to the Python sources in ``llm_hgemm/``:

* ``libhgemm_sm100.so`` - the hand-written tcgen05/TMA kernels and the C ABI of
  ``include/hgemm_sm100.h`` (nvcc, ``-gencode arch=compute_100a,code=sm_100a``,
  static CUDA runtime, no torch);
* ``libhgemm_sm100_debug.so`` - the same with ``-DHGEMM_DEBUG`` (device-side
  bounds checks that record a failure instead of trapping), for tests;
* ``_C<EXT_SUFFIX>`` - the pybind11/torch host module (contract checks, name
  dispatch, current-stream launch) linked against ``libhgemm_sm100.so``;
* ``_comparators<EXT_SUFFIX>`` - benchmark-only cuBLASLt comparator (never in
  the ``hgemm`` dispatch path).

Counterpart of the reference's ``setup.py`` (CUDAExtension with
``-gencode=arch=compute_86,code=sm_86``, setup.py:12-45), built in place so the
shared objects travel with the source tree. Rebuilds only what is stale.

Usage: ``python build.py [--force]``.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
OUT_DIR = PKG_ROOT / "llm_hgemm"
INCLUDE = REPO_ROOT / "include"
BUILD_DIR = PKG_ROOT / "_build"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")

KERNEL_LIB = OUT_DIR / "libhgemm_sm100.so"
# The same sources with -DHGEMM_DEBUG: device-side bounds checks that record
# a failure instead of trapping (include/hgemm_sm100.h, debug build).
DEBUG_LIB = OUT_DIR / "libhgemm_sm100_debug.so"
KERNEL_SOURCES = [CSRC / "hgemm_sm100.cu"]
KERNEL_DEPS = KERNEL_SOURCES + [CSRC / "hgemm_kernels.cuh", CSRC / "sm100_ptx.cuh", CSRC / "debug_checks.cuh",
                                INCLUDE / "hgemm_sm100.h"]
HOST_SOURCES = [CSRC / "host" / "bindings.cpp", CSRC / "host" / "contract.cpp",
                CSRC / "host" / "dispatch.cpp"]
HOST_DEPS = HOST_SOURCES + [CSRC / "host" / "hgemm.h", INCLUDE / "hgemm_sm100.h"]
COMPARATOR_SOURCES = [CSRC / "comparators" / "cublaslt_comparator.cpp"]


def ext_suffix() -> str:
    return sysconfig.get_config_var("EXT_SUFFIX") or ".so"


def host_module() -> Path:
    return OUT_DIR / f"_C{ext_suffix()}"


def comparator_module() -> Path:
    return OUT_DIR / f"_comparators{ext_suffix()}"


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.exists() and d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + proc.stdout + proc.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} ... {cmd[-1]}")


def build_kernel_lib(force: bool = False, debug: bool = False) -> Path:
    target = DEBUG_LIB if debug else KERNEL_LIB
    if not force and not _stale(target, KERNEL_DEPS):
        return target
    BUILD_DIR.mkdir(exist_ok=True)
    cmd = [NVCC, *ARCH_FLAGS, "-O3", "-std=c++17", "-lineinfo", "-Xptxas", "-v",
           "-Xcompiler", "-fPIC", "-shared", "-cudart", "static",
           *(["-DHGEMM_DEBUG"] if debug else []),
           f"-I{INCLUDE}", f"-I{CSRC}", *map(str, KERNEL_SOURCES),
           "-o", str(target)]
    _run(cmd)
    return target


def _torch_flags() -> tuple[list[str], list[str]]:
    import torch
    from torch.utils import cpp_extension

    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cflags = ["-O3", "-std=c++17", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
              "-DTORCH_API_INCLUDE_EXTENSION_H", "-DTORCH_EXTENSION_NAME=_C",
              f"-I{sysconfig.get_paths()['include']}", f"-I{CUDA_HOME / 'include'}",
              f"-I{INCLUDE}"]
    cflags += [f"-I{p}" for p in cpp_extension.include_paths()]
    lib_dirs = cpp_extension.library_paths()
    ldflags = [f"-L{p}" for p in lib_dirs] + [f"-Wl,-rpath,{p}" for p in lib_dirs]
    ldflags += ["-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda"]
    return cflags, ldflags


def _compile_objects(sources: list[Path], cflags: list[str], tag: str) -> list[Path]:
    BUILD_DIR.mkdir(exist_ok=True)
    objs = [BUILD_DIR / f"{tag}_{s.stem}.o" for s in sources]
    with ThreadPoolExecutor(max_workers=len(sources)) as pool:
        list(pool.map(lambda so: _run(["g++", *cflags, "-c", str(so[0]), "-o", str(so[1])]),
                      zip(sources, objs)))
    return objs


def build_host_module(force: bool = False) -> Path:
    target = host_module()
    if not force and not _stale(target, HOST_DEPS + [KERNEL_LIB]):
        return target
    cflags, ldflags = _torch_flags()
    objs = _compile_objects(HOST_SOURCES, cflags + [f"-I{CSRC / 'host'}"], "host")
    _run(["g++", "-shared", *map(str, objs), "-o", str(target), f"-L{OUT_DIR}", "-lhgemm_sm100",
          "-Wl,-rpath,$ORIGIN", *ldflags])
    return target


def build_comparator_module(force: bool = False) -> Path | None:
    target = comparator_module()
    if not all(s.exists() for s in COMPARATOR_SOURCES):
        return None
    if not force and not _stale(target, COMPARATOR_SOURCES):
        return target
    cflags, ldflags = _torch_flags()
    cflags = [f if f != "-DTORCH_EXTENSION_NAME=_C" else "-DTORCH_EXTENSION_NAME=_comparators"
              for f in cflags]
    objs = _compile_objects(COMPARATOR_SOURCES, cflags, "cmp")
    _run(["g++", "-shared", *map(str, objs), "-o", str(target),
          f"-L{CUDA_HOME / 'lib64'}", "-lcublasLt", "-lcudart", *ldflags])
    return target


def build(force: bool = False, debug: bool = True) -> None:
    if shutil.which(NVCC) is None and not Path(NVCC).exists():
        raise RuntimeError(f"nvcc not found at {NVCC}")
    with ThreadPoolExecutor(max_workers=2) as pool:
        jobs = [pool.submit(build_kernel_lib, force)]
        if debug:
            jobs.append(pool.submit(build_kernel_lib, force, True))
        for j in jobs:
            j.result()
    build_host_module(force)
    build_comparator_module(force)


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--force", action="store_true", help="rebuild everything")
    parser.add_argument("--no-debug", action="store_true", help="skip the -DHGEMM_DEBUG kernel library")
    args = parser.parse_args()
    build(args.force, debug=not args.no_debug)
    print(f"built {KERNEL_LIB.name}, {'' if args.no_debug else DEBUG_LIB.name + ', '}{host_module().name}")


if __name__ == "__main__":
    main()
