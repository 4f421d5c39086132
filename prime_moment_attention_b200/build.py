"""Build libpma.so (the C-ABI library of include/pma.h) in place with nvcc for sm_100a, and
_pma_torch.so, the torch.ops.pma operators over that C ABI (csrc/torch_ops.cpp, g++ against the
installed PyTorch).

    python -m prime_moment_attention_b200.build        # or build() from Python

Objects go to _build/ under the package; the shared libraries land next to this
file, where the package loads them from.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libpma.so")
TORCH_LIB = os.path.join(HERE, "_pma_torch.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-Xptxas", "-v"]


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(OUT, os.path.basename(src) + ".o")
    deps = glob.glob(os.path.join(CSRC, "*.cuh")) + [os.path.join(HERE, "..", "include", "pma.h"), src]
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(d) for d in deps):
        return obj
    cmd = [_nvcc(), *ARCH, *FLAGS, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}")
    if verbose:
        with open(obj + ".ptxas.txt", "w") as f:
            f.write(r.stderr)
    return obj


def build_torch_ops(verbose: bool = True) -> str:
    """_pma_torch.so: csrc/torch_ops.cpp compiled against the installed PyTorch, linked to libpma.so
    (found next to it at run time through an $ORIGIN rpath)."""
    import torch
    import torch.utils.cpp_extension as ce
    src = os.path.join(CSRC, "torch_ops.cpp")
    deps = [src, os.path.join(HERE, "..", "include", "pma.h"), LIB]
    if os.path.exists(TORCH_LIB) and os.path.getmtime(TORCH_LIB) >= max(os.path.getmtime(d) for d in deps):
        return TORCH_LIB
    cuda_home = ce.CUDA_HOME or "/usr/local/cuda"
    incs = [f"-I{p}" for p in ce.include_paths("cuda")] + [f"-I{os.path.join(cuda_home, 'include')}"]
    libdirs = ce.library_paths("cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}", *incs, src,
           "-o", TORCH_LIB, *[f"-L{d}" for d in libdirs], f"-L{HERE}", "-lpma", "-lc10", "-lc10_cuda", "-ltorch",
           "-ltorch_cpu", "-ltorch_cuda", "-lcudart", "-Wl,-rpath,$ORIGIN",
           *[f"-Wl,-rpath,{d}" for d in libdirs]]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"torch ops build failed:\n{r.stderr[-4000:]}")
    return TORCH_LIB


def build(verbose: bool = True) -> str:
    os.makedirs(OUT, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [_nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
    build_torch_ops(verbose)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-q" not in sys.argv))
