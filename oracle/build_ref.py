"""Build the reference's own extension into oracle/_ref/ (checker only).

TEST INFRASTRUCTURE. Compiles thebigblender/FlashLite's sources where they
lie (csrc/flash_attn.cpp, csrc/kernel_naive.cu, csrc/kernel_flash2.cu; they
are read in place, never copied) into a Python extension module named
``flash_attn_wmma``, written to ``oracle/_ref/``. The nvcc flags are the
reference's own (setup.py:39-48) except the architecture, which is sm_100a
instead of sm_86 so the binary runs on a B200. The reference's own build
system (setup.py / CMake) is not run.

Used by GPU tests to compare against the reference kernels on the same
inputs, and by ``bench.py --impl reference`` to time them beside the CPU
baseline. Needs the reference tree, so it only runs in the build container;
the built .so travels to GPU boxes with the repository snapshot.

The reference root comes from the command line or the FLASHLITE_REFERENCE
environment variable; ``build_if_available`` also looks for a ``reference``
directory beside this repository's own directory.

Run: python -m oracle.build_ref  [reference_root]
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT_DIR = HERE / "_ref"
MODULE = "flash_attn_wmma"
EXT = OUT_DIR / (MODULE + sysconfig.get_config_var("EXT_SUFFIX"))

# setup.py:39-48 of the reference, with -arch retargeted to sm_100a
REF_NVCC_FLAGS = [
    "-O3", "-gencode", "arch=compute_100a,code=sm_100a", "--use_fast_math", "-std=c++17",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_HALF2_OPERATORS__",
]


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"reference build failed:\n{' '.join(cmd)}\n{r.stdout}{r.stderr}")


def reference_root() -> Path | None:
    """The reference tree: $FLASHLITE_REFERENCE, else ``../reference`` next to
    this repository; None when neither holds the reference's sources."""
    env = os.environ.get("FLASHLITE_REFERENCE")
    for cand in ([Path(env)] if env else []) + [HERE.parent.parent / "reference"]:
        if (cand / "csrc" / "kernel_flash2.cu").exists():
            return cand
    return None


def build(ref_root: Path) -> Path:
    import torch
    from torch.utils import cpp_extension as ce

    csrc = ref_root / "csrc"
    srcs = [csrc / "flash_attn.cpp", csrc / "kernel_naive.cu", csrc / "kernel_flash2.cu"]
    for s in srcs:
        if not s.exists():
            raise FileNotFoundError(s)
    OUT_DIR.mkdir(exist_ok=True)
    tmp = OUT_DIR / "obj"
    tmp.mkdir(exist_ok=True)
    incs = ce.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"], str(csrc / "includes")]
    defs = [f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
            f"-DTORCH_EXTENSION_NAME={MODULE}", "-DTORCH_API_INCLUDE_EXTENSION_H"]
    nvcc = "/usr/local/cuda/bin/nvcc" if Path("/usr/local/cuda/bin/nvcc").exists() else "nvcc"
    objs = []
    procs = []
    for s in srcs:
        obj = tmp / (s.name + ".o")
        objs.append(obj)
        if s.suffix == ".cu":
            cmd = [nvcc, *REF_NVCC_FLAGS, "-Xcompiler", "-fPIC", "-w", *defs,
                   *[f"-I{p}" for p in incs], "-c", str(s), "-o", str(obj)]
        else:
            cmd = ["g++", "-O3", "-std=c++17", "-fPIC", "-w", *defs, *[f"-I{p}" for p in incs],
                   "-c", str(s), "-o", str(obj)]
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    for cmd, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            raise RuntimeError(f"reference build failed:\n{' '.join(cmd)}\n{out}")
    libdirs = ce.library_paths(device_type="cuda")
    _run(["g++", "-shared", "-o", str(EXT), *map(str, objs), *[f"-L{p}" for p in libdirs],
          "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-ltorch_cuda",
          "-lcudart"])
    return EXT


def build_if_available() -> Path | None:
    """Build when the reference tree is present and the module is missing."""
    if EXT.exists():
        return EXT
    root = reference_root()
    if root is None:
        return None
    try:
        return build(root)
    except Exception as exc:  # the checker is optional; the product build is not
        print(f"oracle/_ref not built: {exc}", file=sys.stderr)
        return None


def load():
    """Import the built reference module under its own name, or return None."""
    import importlib.util

    import torch  # noqa: F401

    if not EXT.exists():
        return None
    spec = importlib.util.spec_from_file_location(MODULE, EXT)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    root = Path(sys.argv[1]) if len(sys.argv) > 1 else reference_root()
    if root is None:
        sys.exit("reference tree not found: pass its path or set FLASHLITE_REFERENCE")
    print("built", build(root))
