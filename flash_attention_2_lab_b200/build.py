"""In-tree build of the two native artefacts of this package.

* ``libfa_sm100.so``  -- the sm_100a kernel and its C ABI (include/fa_sm100.h),
  compiled by nvcc for ``compute_100a``/``sm_100a`` only.
* ``flash_attention_cuda.so`` -- the PyTorch extension module (host C++ only)
  that mirrors the reference's ``flash_attention_cuda`` binding and calls the
  C ABI; linked against ``libfa_sm100.so`` with an ``$ORIGIN`` rpath.

Both land next to this file so they travel with the source tree.  Rebuilds
happen only when a source is newer than its output (or ``force=True``).

Usage: ``python -m flash_attention_2_lab_b200.build [--force]``
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libfa_sm100.so"
EXT = PKG / "flash_attention_cuda.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _cuda_home() -> Path:
    env = os.environ.get("CUDA_HOME") or os.environ.get("CUDA_PATH")
    if env:
        return Path(env)
    nvcc = shutil.which("nvcc")
    if nvcc:
        return Path(nvcc).resolve().parent.parent
    return Path("/usr/local/cuda")


def _stale(out: Path, sources: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources)


def _run(cmd: list[str]) -> None:
    print("+", " ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build_lib(force: bool = False, verbose_ptxas: bool = False) -> Path:
    sources = [CSRC / "fa_fwd_sm100.cu", CSRC / "fa_bwd_sm100.cuh", CSRC / "sm100_ptx.cuh",
               INCLUDE / "fa_sm100.h"]
    if force or _stale(LIB, sources):
        nvcc = str(_cuda_home() / "bin" / "nvcc")
        cmd = [nvcc, *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
               "-shared", f"-I{INCLUDE}", "-o", str(LIB), str(CSRC / "fa_fwd_sm100.cu")]
        if verbose_ptxas:
            cmd.insert(1, "-Xptxas=-v")
        _run(cmd)
    return LIB


def build_ext(force: bool = False) -> Path:
    import torch
    from torch.utils import cpp_extension

    sources = [CSRC / "torch_binding.cpp", INCLUDE / "fa_sm100.h", LIB]
    if force or _stale(EXT, sources):
        torch_lib = Path(torch.__file__).resolve().parent / "lib"
        incs = cpp_extension.include_paths() + [sysconfig.get_paths()["include"],
                                                 str(_cuda_home() / "include"), str(INCLUDE)]
        abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
        cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared",
               f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_API_INCLUDE_EXTENSION_H",
               "-DTORCH_EXTENSION_NAME=flash_attention_cuda",
               *[f"-I{i}" for i in incs],
               str(CSRC / "torch_binding.cpp"), "-o", str(EXT),
               f"-L{PKG}", "-lfa_sm100", f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch",
               "-ltorch_cpu", "-ltorch_python", "-Wl,-rpath,$ORIGIN",
               f"-Wl,-rpath,{torch_lib}"]
        _run(cmd)
    return EXT


def build_all(force: bool = False) -> None:
    build_lib(force)
    build_ext(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
