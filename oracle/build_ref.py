"""Build the reference project's own CUDA extension for sm_100a -- TEST
INFRASTRUCTURE ONLY (a second parity witness and a same-GPU speed baseline).

Compiles the reference's sources where they lie (``<reference>/csrc/*.cu`` and
``bindings.cpp``, the files its setup.py:5-33 builds) with nvcc / g++ directly,
with the flags of its setup.py (``-O3 --use_fast_math -lineinfo``) and
``-gencode arch=compute_100a,code=sm_100a``, into
``oracle/_ref/flash_attention_cuda_ref.so`` (module ``flash_attention_cuda_ref``
so it cannot be confused with this library's ``flash_attention_cuda``).
Nothing is copied from the reference; the output directory is git-ignored.

    python oracle/build_ref.py REFERENCE_ROOT
"""

from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
MODULE = "flash_attention_cuda_ref"


def build(ref_root: Path) -> Path:
    import torch
    from torch.utils import cpp_extension

    csrc = ref_root / "csrc"
    if not csrc.is_dir():
        raise FileNotFoundError(f"{csrc} not found")
    OUT.mkdir(exist_ok=True)
    target = OUT / f"{MODULE}.so"
    torch_lib = Path(torch.__file__).resolve().parent / "lib"
    incs = cpp_extension.include_paths() + [sysconfig.get_paths()["include"]]
    cuda_home = Path(cpp_extension.CUDA_HOME or "/usr/local/cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    defs = [f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_API_INCLUDE_EXTENSION_H",
            f"-DTORCH_EXTENSION_NAME={MODULE}"]
    inc_flags = [f"-I{i}" for i in incs] + [f"-I{cuda_home / 'include'}"]

    def nvcc(src: Path) -> Path:
        obj = OUT / (src.stem + ".o")
        cmd = [str(cuda_home / "bin" / "nvcc"), "-c", str(src), "-o", str(obj),
               "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "--use_fast_math",
               "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", *defs, *inc_flags]
        subprocess.run(cmd, check=True)
        return obj

    def gxx(src: Path) -> Path:
        obj = OUT / (src.stem + ".o")
        cmd = ["g++", "-c", str(src), "-o", str(obj), "-O3", "-std=c++17", "-fPIC", *defs,
               *inc_flags]
        subprocess.run(cmd, check=True)
        return obj

    cu = sorted(csrc.glob("*.cu"))
    with ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        objs = list(ex.map(nvcc, cu)) + [gxx(csrc / "bindings.cpp")]
    cmd = ["g++", "-shared", "-o", str(target), *map(str, objs),
           f"-L{cuda_home / 'lib64'}", "-lcudart", f"-L{torch_lib}", "-lc10", "-lc10_cuda",
           "-ltorch", "-ltorch_cpu", "-ltorch_python", "-ltorch_cuda",
           f"-Wl,-rpath,{torch_lib}"]
    subprocess.run(cmd, check=True)
    for o in objs:
        o.unlink()
    return target


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    print(build(Path(sys.argv[1])))
