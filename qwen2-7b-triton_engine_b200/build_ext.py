"""Build the C++ host glue of the drop-in (csrc/awq_torch_ext.cpp) in-tree:
lib/_awq_ext<ext suffix>, linked against lib/libawq_b200.so and the installed PyTorch.

Runs g++ directly with PyTorch's include and library paths (no JIT cache: the module
travels with the tree).  Skips the build when the module is newer than its sources.
Usage: python build_ext.py [--force]
"""
from __future__ import annotations

import pathlib
import subprocess
import sys
import sysconfig

HERE = pathlib.Path(__file__).resolve().parent
SRC = HERE / "csrc" / "awq_torch_ext.cpp"
HDR = HERE.parent / "include" / "awq_b200.h"
LIB = HERE / "lib"
NAME = "_awq_ext"


def target() -> pathlib.Path:
    return LIB / (NAME + sysconfig.get_config_var("EXT_SUFFIX"))


def build(force: bool = False) -> pathlib.Path:
    import torch
    import torch.utils.cpp_extension as ce

    out = target()
    deps = [SRC, HDR, LIB / "libawq_b200.so", pathlib.Path(__file__)]
    if not force and out.exists() and all(out.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return out
    torch_lib = pathlib.Path(torch.__file__).resolve().parent / "lib"
    cuda_home = ce.CUDA_HOME or "/usr/local/cuda"
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-fvisibility=hidden",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
           f"-DTORCH_EXTENSION_NAME={NAME}", "-DTORCH_API_INCLUDE_EXTENSION_H"]
    for inc in ce.include_paths() + [sysconfig.get_paths()["include"], f"{cuda_home}/include"]:
        cmd += ["-isystem", str(inc)]
    cmd += [str(SRC), "-o", str(out),
            f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
            "-ltorch_python", f"-L{LIB}", "-lawq_b200", f"-L{cuda_home}/lib64", "-lcudart",
            "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
    LIB.mkdir(exist_ok=True)
    subprocess.run(cmd, check=True)
    return out


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
