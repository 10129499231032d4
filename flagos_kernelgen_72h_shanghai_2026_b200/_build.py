"""In-tree build of libfarq.so and libdsa_topk.so (the sm_100a kernels behind
the C ABIs in include/farq.h and include/dsa_topk.h).

The library is compiled with nvcc directly (no torch headers): it exports only
plain-C entry points, so the Python host binds it with ctypes. The built file
lives next to this module so it travels with the source tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
INCLUDE_DIR = REPO_DIR / "include"
CSRC_DIR = PKG_DIR / "csrc"
SOURCES = [CSRC_DIR / "farq.cu", *sorted(CSRC_DIR.glob("farq_inst_*.cu")),
           *sorted(CSRC_DIR.glob("farq_ar_inst_*.cu")), CSRC_DIR / "farq_noalloc.cu"]
HEADERS = [INCLUDE_DIR / "farq.h", CSRC_DIR / "farq_kernel.cuh", CSRC_DIR / "farq_ar_kernel.cuh"]
LIB_PATH = PKG_DIR / "libfarq.so"

TOPK_SOURCES = [CSRC_DIR / "dsa_topk.cu"]
TOPK_HEADERS = [INCLUDE_DIR / "dsa_topk.h", CSRC_DIR / "dsa_topk_kernel.cuh"]
TOPK_LIB_PATH = PKG_DIR / "libdsa_topk.so"

OBJ_DIR = PKG_DIR / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [*ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-O3"]
LINK_FLAGS = [*ARCH, "-shared", "-Xcompiler", "-fPIC"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: cannot build libfarq.so")
    return cand


def _stale(lib: Path, deps: list[Path]) -> bool:
    if not lib.exists():
        return True
    t = lib.stat().st_mtime
    return any(p.stat().st_mtime > t for p in deps)


def is_stale() -> bool:
    return _stale(LIB_PATH, SOURCES + HEADERS)


def is_topk_stale() -> bool:
    return _stale(TOPK_LIB_PATH, TOPK_SOURCES + TOPK_HEADERS)


def _run(cmd: list[str], verbose: bool) -> str:
    if verbose:
        print(" ".join(cmd))
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    return res.stderr


def build_lib(force: bool = False, verbose: bool = False) -> Path:
    """Compile libfarq.so for sm_100a if it is missing or older than its sources."""
    if not force and not is_stale():
        return LIB_PATH
    return _compile(SOURCES, LIB_PATH, verbose)


def build_topk_lib(force: bool = False, verbose: bool = False) -> Path:
    """Compile libdsa_topk.so for sm_100a if it is missing or older than its sources."""
    if not force and not is_topk_stale():
        return TOPK_LIB_PATH
    return _compile(TOPK_SOURCES, TOPK_LIB_PATH, verbose)


FAST_SOURCE = CSRC_DIR / "farq_fast.cpp"


def fast_ext_path() -> Path:
    import sysconfig
    return PKG_DIR / ("_farq_fast" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_fast_ext(force: bool = False, verbose: bool = False) -> Path:
    """Compile the C++ launch path of the Python operators (_farq_fast, a
    torch extension module linked against libfarq.so and libdsa_topk.so)
    with g++, in-tree, if it is missing or older than its sources."""
    out = fast_ext_path()
    deps = [FAST_SOURCE, INCLUDE_DIR / "farq.h", INCLUDE_DIR / "dsa_topk.h", LIB_PATH, TOPK_LIB_PATH]
    if not force and not _stale(out, deps):
        return out
    import sysconfig

    import torch
    from torch.utils import cpp_extension

    cuda_home = os.path.dirname(os.path.dirname(_nvcc()))
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-w",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_farq_fast",
           "-DTORCH_API_INCLUDE_EXTENSION_H",
           *[f"-I{p}" for p in cpp_extension.include_paths()],
           f"-I{sysconfig.get_paths()['include']}", f"-I{cuda_home}/include", f"-I{INCLUDE_DIR}",
           str(FAST_SOURCE), "-o", str(out) + ".tmp",
           *[f"-L{p}" for p in cpp_extension.library_paths()],
           "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
           f"-L{PKG_DIR}", "-lfarq", "-ldsa_topk",
           "-Wl,-rpath,$ORIGIN", *[f"-Wl,-rpath,{p}" for p in cpp_extension.library_paths()]]
    _run(cmd, verbose)
    os.replace(str(out) + ".tmp", out)
    return out


def build_all(force: bool = False, verbose: bool = False) -> list[Path]:
    libs = [build_lib(force, verbose), build_topk_lib(force, verbose)]
    return libs + [build_fast_ext(force, verbose)]


def _compile(sources: list[Path], lib_path: Path, verbose: bool) -> Path:
    """Each translation unit is compiled to an object in parallel (the kernel
    instantiations dominate), then linked into one shared library."""
    from concurrent.futures import ThreadPoolExecutor

    nvcc = _nvcc()
    OBJ_DIR.mkdir(exist_ok=True)
    flags = [*NVCC_FLAGS, f"-I{INCLUDE_DIR}", f"-I{CSRC_DIR}"]
    if verbose:
        flags.append("-Xptxas=-v")
    jobs = []
    for src in sources:
        # the tensor-parallel tables are compiled once per WMAX (1, 2, 4, 8)
        variants = ([(f"_w{w}", [f"-DFARQ_AR_WMAX={w}"]) for w in (1, 2, 4, 8)]
                    if src.name.startswith("farq_ar_inst_") else [("", [])])
        for suffix, defs in variants:
            obj = OBJ_DIR / (src.stem + suffix + ".o")
            jobs.append(([nvcc, *flags, *defs, "-c", "-o", str(obj), str(src)], obj))
    with ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 1)) as ex:
        logs = list(ex.map(lambda j: _run(j[0], verbose), jobs))
    if verbose:
        for log in logs:
            if log:
                print(log)
    tmp = lib_path.with_suffix(".so.tmp")
    _run([nvcc, *LINK_FLAGS, "-o", str(tmp), *(str(o) for _, o in jobs)], verbose)
    os.replace(tmp, lib_path)
    return lib_path


if __name__ == "__main__":
    import sys
    print(build_all(force="--force" in sys.argv, verbose="-v" in sys.argv))
