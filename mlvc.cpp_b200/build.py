"""Build libmlvc_b200.so in-tree.

1. nvcc compiles csrc/kernels/module.cu (every kernel, one translation unit)
   to an sm_100a cubin with -lineinfo.
2. The cubin is embedded into the shared library with an assembler .incbin
   (the reference embeds its fatbin the same way, cmake/EmbedBinary.cmake) and
   loaded at run time with cuModuleLoadData.
3. g++ compiles the C++ host runtime (Driver API) and the C ABI and links
   against libcuda.
4. nvcc compiles csrc/noalloc/*.cu (host and device code, CUDA runtime API)
   into an object linked with the static CUDA runtime, so the library still
   has no link-time dependency on libcudart or libcuda.

Outputs: mlvc.cpp_b200/lib/libmlvc_b200.so (git-ignored, travels with the
repository snapshot to the GPU machine).  Usage: python mlvc.cpp_b200/build.py
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CUDA = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
BUILD = HERE / "_build"
LIB = HERE / "lib" / "libmlvc_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _run(cmd):
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError(f"build step failed: {' '.join(map(str, cmd))}")
    return proc.stdout + proc.stderr


def sources():
    return sorted((HERE / "csrc").rglob("*.cu")) + sorted((HERE / "csrc").rglob("*.cuh")) + \
        sorted((HERE / "csrc").rglob("*.h")) + sorted((HERE / "csrc").rglob("*.hpp")) + \
        sorted((HERE / "csrc").rglob("*.cpp")) + [ROOT / "include" / "mlvc_b200.h", Path(__file__)]


def up_to_date():
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in sources())


def build(force=False, verbose=False):
    if not force and up_to_date():
        return LIB
    nvcc = shutil.which("nvcc") or str(CUDA / "bin" / "nvcc")
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    cubin = BUILD / "mlvc_b200_sm100a.cubin"
    out = _run([nvcc, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-cubin", "-Xptxas", "-v",
                "-o", str(cubin), str(HERE / "csrc" / "kernels" / "module.cu")])
    (BUILD / "ptxas.txt").write_text(out)
    blob = BUILD / "cubin_blob.S"
    blob.write_text(
        ".section .rodata\n.balign 128\n.global mlvc_b200_cubin_start\n.global mlvc_b200_cubin_end\n"
        f"mlvc_b200_cubin_start:\n.incbin \"{cubin}\"\nmlvc_b200_cubin_end:\n.byte 0\n"
        ".section .note.GNU-stack,\"\",@progbits\n")
    # The system g++ links libstdc++ dynamically; a statically linked copy
    # inside a library that is dlopen'ed next to the process's own libstdc++
    # crashed the Python host, so prefer it over wrapper toolchains.
    cxx = "/usr/bin/g++" if Path("/usr/bin/g++").exists() else os.environ.get("CXX", "g++")
    host = sorted((HERE / "csrc" / "host").glob("*.cpp"))
    rt_objs = []
    for cu in sorted((HERE / "csrc" / "noalloc").glob("*.cu")):
        obj = BUILD / (cu.stem + ".o")
        _run([nvcc, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-ccbin", cxx, "-Xcompiler", "-fPIC", "-c",
              "-o", str(obj), str(cu)])
        rt_objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    _run([cxx, "-std=c++20", "-O2", "-fPIC", "-shared", "-Wall", "-Wno-unused-function",
          f"-I{CUDA / 'include'}", *map(str, host), str(blob), *rt_objs,
          f"-L{CUDA / 'lib64'}", "-lcudart_static", "-lrt", "-lpthread",
          "-ldl", "-o", str(tmp)])
    os.replace(tmp, LIB)
    if verbose:
        print(out)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
