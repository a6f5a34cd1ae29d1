"""Build the reference project's own CUDA extension for sm_100a -- TEST
INFRASTRUCTURE ONLY (a second parity witness and a same-GPU speed baseline).

Compiles the reference's sources where they lie (``<reference>/csrc/*.cu`` and
``bindings.cpp``, the files its setup.py:5-33 builds) with nvcc / g++ directly,
with the flags of its setup.py (``-O3 --use_fast_math -lineinfo``) and
``-gencode arch=compute_100a,code=sm_100a``, into
``oracle/_ref/flash_attention_cuda_ref.so`` (module ``flash_attention_cuda_ref``
so it cannot be confused with this library's ``flash_attention_cuda``).
Nothing is copied from the reference; the output directory is git-ignored.

It also stages the reference's CPU path, the Python package
``flash_attention`` (``attention_reference``, flash_attention/reference.py:9-61),
unmodified into ``baseline/_ref/flash_attention/`` next to the reference's own
pip-installed extension: the reference's setup.py:5-33 declares no Python
packages, so ``pip install --target baseline/_ref`` places only the
extension.  That directory is git-ignored and travels with the working tree,
so the timed CPU baseline can run the reference's own code on the GPU host.

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


BASELINE_REF = HERE.parent / "baseline" / "_ref"


def stage_python(ref_root: Path) -> Path:
    """Copy the reference's ``flash_attention`` package files byte for byte
    into ``baseline/_ref/flash_attention/`` (git-ignored)."""
    import shutil

    src = ref_root / "flash_attention"
    if not (src / "reference.py").is_file():
        raise FileNotFoundError(f"{src / 'reference.py'} not found")
    dst = BASELINE_REF / "flash_attention"
    dst.mkdir(parents=True, exist_ok=True)
    for f in sorted(src.glob("*.py")):
        shutil.copyfile(f, dst / f.name)
    return dst


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    print(build(Path(sys.argv[1])))
    print(stage_python(Path(sys.argv[1])))
