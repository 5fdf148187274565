"""Build libasu_b200.so (all CUDA kernels + the C ABI) in-tree for sm_100a with nvcc, and
libasu_torch.so (the C++ torch registration of the single-request resolver op) with g++.

    python -m asu_ascend_b200.build          # or build() then build_torch_binding()

Objects go to asu_ascend_b200/_build/, the libraries to asu_ascend_b200/.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libasu_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-cudart", "shared", "-Xcompiler", "-fPIC", "-Xptxas", "-v",
         f"-I{ROOT / 'include'}"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists() and shutil.which(cand) is None:
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libasu_b200.so")
    return cand


def _compile(src: Path) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    deps = [src, *CSRC.glob("*.cuh"), ROOT / "include" / "asu_b200.h"]
    if obj.exists() and obj.stat().st_mtime >= max(d.stat().st_mtime for d in deps):
        return obj, ""
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj, res.stderr


def build(verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    with ThreadPoolExecutor(max_workers=min(8, len(sources))) as ex:
        results = list(ex.map(_compile, sources))
    objs = [o for o, _ in results]
    if verbose:
        for _, log in results:
            if log:
                print(log, file=sys.stderr)
    if not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        # One CUDA runtime per process: link the shared libcudart so that, loaded after torch, the
        # library binds to the runtime torch already loaded (same soname) and shares its state.
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "shared", "-Xcompiler", "-fPIC",
               "-Xlinker", "-rpath,/usr/local/cuda/lib64", *map(str, objs), "-o", str(tmp)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


TORCH_LIB = PKG / "libasu_torch.so"


def build_torch_binding() -> Path:
    """libasu_torch.so: the C++ torch registration of the single-request resolver op
    (csrc/torch_binding.cpp), linked against libasu_b200.so and the installed torch."""
    import torch
    from torch.utils import cpp_extension as ce

    src = CSRC / "torch_binding.cpp"
    deps = [src, ROOT / "include" / "asu_b200.h", LIB]
    if TORCH_LIB.exists() and TORCH_LIB.stat().st_mtime >= max(d.stat().st_mtime for d in deps):
        return TORCH_LIB
    incs = ce.include_paths(device_type="cuda")
    libdirs = ce.library_paths(device_type="cuda")
    # the system g++ (the compiler torch is built with): a toolchain that links its own copy of
    # libstdc++ into the library would run a second set of locale facets next to the process's
    # and crash on the first formatted number
    cxx = shutil.which("g++", path="/usr/bin:/bin") or shutil.which("g++") or "g++"
    tmp = TORCH_LIB.with_suffix(".so.tmp")
    cmd = [cxx, "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
           *(f"-I{i}" for i in incs), f"-I{ROOT / 'include'}", str(src), "-o", str(tmp),
           *(f"-L{d}" for d in libdirs), f"-L{PKG}", "-lasu_b200", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
           "-ltorch_cuda", "-Wl,-rpath,$ORIGIN", *(f"-Wl,-rpath,{d}" for d in libdirs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"torch binding build failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, TORCH_LIB)
    return TORCH_LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
    print(build_torch_binding())
