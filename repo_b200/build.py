"""Build the sm_100a CUDA library ``repo_b200/lib/libcubicsplat_b200.so``.

Each ``csrc/*.cu`` is compiled by nvcc for ``compute_100a``/``sm_100a`` (no
other architecture is built) and linked into one shared library with the C ABI
declared in ``include/cubicsplat_b200.h``.  The library is built in-tree so that
it travels with the repository.  ``-fmad=false`` keeps every floating-point
expression in its written order (the kernels write their fused multiply-adds
out explicitly).
"""
from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB_DIR = os.path.join(HERE, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libcubicsplat_b200.so")
OBJ_DIR = os.path.join(HERE, "_build")
HEADERS = [os.path.join(ROOT, "include", "cubicsplat_b200.h"), os.path.join(CSRC, "cs_common.cuh")]


def nvcc_path() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found (set NVCC or add /usr/local/cuda/bin to PATH)")
    return cand


NVCC_FLAGS = [
    "-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo",
    "-fmad=false", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include"),
]


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, verbose_ptxas=False):
    obj = os.path.join(OBJ_DIR, os.path.basename(src) + ".o")
    if not _stale(obj, [src] + HEADERS) and not verbose_ptxas:
        return obj, ""
    cmd = [nvcc_path(), *NVCC_FLAGS, "-c", src, "-o", obj]
    if verbose_ptxas:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}")
    return obj, r.stderr


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    os.makedirs(LIB_DIR, exist_ok=True)
    os.makedirs(OBJ_DIR, exist_ok=True)
    srcs = sources()
    if force:
        for s in srcs:
            o = os.path.join(OBJ_DIR, os.path.basename(s) + ".o")
            if os.path.exists(o):
                os.remove(o)
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose_ptxas), srcs))
    objs = [o for o, _ in results]
    if verbose_ptxas:
        for (o, log), s in zip(results, srcs):
            print(f"== {os.path.basename(s)}\n{log}")
    if force or _stale(LIB_PATH, objs):
        cmd = [nvcc_path(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a",
               "-cudart", "static", *objs, "-o", LIB_PATH]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
    return LIB_PATH


EXT_SRC = os.path.join(CSRC, "torch_api.cpp")
EXT_PATH = os.path.join(LIB_DIR, "_cs_torch.so")


def cuda_include() -> str:
    return os.path.join(os.path.dirname(os.path.dirname(nvcc_path())), "include")


def build_torch_ext(force: bool = False) -> str:
    """Compile the torch binding (``csrc/torch_api.cpp``, host C++ only) into
    ``lib/_cs_torch.so``, linked against the C-ABI library beside it."""
    import sysconfig

    import torch
    import torch.utils.cpp_extension as ce
    deps = [EXT_SRC, HEADERS[0], LIB_PATH]
    if not force and not _stale(EXT_PATH, deps):
        return EXT_PATH
    torch_lib = ce.library_paths()[0]
    cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-shared", "-fPIC",
           "-fvisibility=hidden",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch.compiled_with_cxx11_abi())}",
           "-DTORCH_EXTENSION_NAME=_cs_torch", "-DTORCH_API_INCLUDE_EXTENSION_H"]
    for inc in ce.include_paths() + [sysconfig.get_paths()["include"],
                                     os.path.join(ROOT, "include"), cuda_include()]:
        cmd += ["-isystem" if inc != os.path.join(ROOT, "include") else "-I", inc]
    cmd += [EXT_SRC, "-o", EXT_PATH, "-L", torch_lib, "-lc10", "-lc10_cuda", "-ltorch",
            "-ltorch_cpu", "-ltorch_python", "-L", LIB_DIR, "-l:libcubicsplat_b200.so",
            "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"torch binding build failed:\n{r.stderr}")
    return EXT_PATH


def build_all(force: bool = False, verbose_ptxas: bool = False) -> str:
    path = build(force=force, verbose_ptxas=verbose_ptxas)
    build_torch_ext(force=force)
    return path


if __name__ == "__main__":
    print(build_all(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv))
