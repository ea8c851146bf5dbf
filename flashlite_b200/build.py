"""In-tree build of the flashlite_b200 native code.

Produces, next to this file:
  libflashlite_b200.so   the C-ABI library (all CUDA kernels, sm_100a only)
  _C<EXT_SUFFIX>         the torch binding (pybind11), linked against the above

Both are plain nvcc / g++ invocations (no JIT cache, no setuptools), so the
built files sit in the source tree and travel with it. Rebuilds only what is
older than its sources. Run: ``python -m flashlite_b200.build``.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
BUILD = PKG / "_build"

CUDA_SOURCES = ["fl_api.cu", "fl_flash2.cu", "fl_flash2_sk.cu", "fl_flash2_bwd.cu", "fl_naive.cu",
                "fl_noalloc.cu", "fl_selftest.cu"]
HEADERS = ["fl_ptx.cuh", "fl_internal.h", "fl_flash2_common.cuh"]
LIB = PKG / "libflashlite_b200.so"
EXT = PKG / ("_C" + sysconfig.get_config_var("EXT_SUFFIX"))

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
    "-Xptxas", "-v", "--expt-relaxed-constexpr",
]


def _cuda_home() -> Path:
    for cand in (os.environ.get("CUDA_HOME"), "/usr/local/cuda"):
        if cand and (Path(cand) / "bin" / "nvcc").exists():
            return Path(cand)
    nvcc = shutil.which("nvcc")
    if nvcc:
        return Path(nvcc).resolve().parent.parent
    raise RuntimeError("nvcc not found: set CUDA_HOME")


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def _run(cmd, log: Path | None = None) -> str:
    r = subprocess.run(cmd, capture_output=True, text=True)
    out = r.stdout + r.stderr
    if log is not None:
        log.write_text(" ".join(map(str, cmd)) + "\n" + out)
    if r.returncode != 0:
        raise RuntimeError(f"build command failed ({r.returncode}):\n{' '.join(map(str, cmd))}\n{out}")
    return out


def build_library(verbose: bool = False) -> Path:
    """Compile every CUDA source for sm_100a and link libflashlite_b200.so."""
    nvcc = str(_cuda_home() / "bin" / "nvcc")
    BUILD.mkdir(exist_ok=True)
    hdrs = [CSRC / h for h in HEADERS] + [INCLUDE / "flashlite_b200.h"]
    jobs = []
    for src in CUDA_SOURCES:
        obj = BUILD / (src + ".o")
        if _stale(obj, [CSRC / src] + hdrs + [Path(__file__)]):
            jobs.append((CSRC / src, obj))

    def compile_one(job):
        src, obj = job
        return _run([nvcc, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)],
                    BUILD / (src.name + ".log"))

    if jobs:
        with ThreadPoolExecutor(max_workers=len(jobs)) as ex:
            for out in ex.map(compile_one, jobs):
                if verbose:
                    print(out)
    objs = [BUILD / (s + ".o") for s in CUDA_SOURCES]
    if _stale(LIB, objs):
        _run([nvcc, *ARCH_FLAGS, "-shared", "-o", str(LIB), *map(str, objs)],
             BUILD / "link.log")
    return LIB


def build_binding(verbose: bool = False) -> Path:
    """Compile the torch binding (flash_attn.cpp) against libflashlite_b200.so."""
    import torch
    from torch.utils import cpp_extension as ce

    src = CSRC / "flash_attn.cpp"
    if not _stale(EXT, [src, INCLUDE / "flashlite_b200.h", LIB, Path(__file__)]):
        return EXT
    cxx = os.environ.get("CXX", "g++")
    incs = ce.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"]]
    libdirs = ce.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = [cxx, "-O2", "-std=c++17", "-shared", "-fPIC", "-w",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_C",
           "-DTORCH_API_INCLUDE_EXTENSION_H",
           *[f"-I{p}" for p in incs], str(src), "-o", str(EXT),
           *[f"-L{p}" for p in libdirs], f"-L{PKG}",
           "-lflashlite_b200", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
           "-ltorch_python", "-lcudart",
           "-Wl,-rpath,$ORIGIN"]
    out = _run(cmd, BUILD / "binding.log")
    if verbose:
        print(out)
    return EXT


def build(verbose: bool = False) -> None:
    build_library(verbose)
    build_binding(verbose)


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print(f"built {LIB.name} and {EXT.name}")
