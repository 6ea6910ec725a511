"""Builds the native library: sm_100a cubin + C++ boundary -> one .so.

Steps (all in-tree so the artefacts travel with the source tree):
  1. nvcc -cubin -gencode arch=compute_100a,code=sm_100a  csrc/kernels/kernels.cu
  2. nvcc -c  csrc/native/*.cu (host code with registered device data)
  3. g++ -shared  csrc/native/*.cpp + those objects + kernel_image.S (embeds
     the cubin) + static CUDA runtime -> flight4s_b200/libflight4s_b200.so

The library needs no CUDA shared library at load time: libcuda.so.1 is
opened at first use, and the CUDA runtime used by the static-workspace
entry point is linked in statically (hidden).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libflight4s_b200.so"
CUBIN = BUILD / "flight4s_b200_kernels.cubin"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC_ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _run(cmd: list[str], quiet: bool = False) -> str:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError(f"build step failed ({proc.returncode}): {' '.join(cmd)}")
    return proc.stdout + proc.stderr


def _newer(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return False
    t = target.stat().st_mtime
    return all(s.stat().st_mtime <= t for s in sources)


def build_cubin(force: bool = False, verbose: bool = False) -> Path:
    sources = sorted((CSRC / "kernels").glob("*.cu*"))
    if not force and _newer(CUBIN, sources):
        return CUBIN
    BUILD.mkdir(exist_ok=True)
    nvcc = str(CUDA_HOME / "bin" / "nvcc")
    out = _run([nvcc, *NVCC_ARCH, "-O3", "-lineinfo", "-std=c++17", "-cubin", "-Xptxas", "-v",
                str(CSRC / "kernels" / "kernels.cu"), "-o", str(CUBIN)])
    (BUILD / "ptxas_info.txt").write_text(out)
    if verbose:
        print(out)
    return CUBIN


def build_runtime_objects(force: bool = False) -> list[Path]:
    """nvcc-compiled host+device objects linked into the library (the
    static-workspace .cu files, registered with the CUDA runtime)."""
    native = CSRC / "native"
    objs = []
    nvcc = str(CUDA_HOME / "bin" / "nvcc")
    for cu in sorted(native.glob("*.cu")):
        obj = BUILD / (cu.stem + ".o")
        deps = [cu] + sorted(native.glob("*.hpp"))
        if force or not _newer(obj, deps):
            BUILD.mkdir(exist_ok=True)
            _run([nvcc, *NVCC_ARCH, "-O3", "-std=c++17", "-c", "-Xcompiler", "-fPIC", f"-I{native}",
                  str(cu), "-o", str(obj)])
        objs.append(obj)
    return objs


def build_library(force: bool = False, verbose: bool = False) -> Path:
    cubin = build_cubin(force=force, verbose=verbose)
    objs = build_runtime_objects(force=force)
    native = CSRC / "native"
    sources = sorted(native.glob("*.cpp"))
    deps = sources + objs + sorted(native.glob("*.hpp")) + [native / "driver_functions.inc",
                                                             native / "kernel_image.S", cubin,
                                                             PKG.parent / "include" / "flight4s_b200.h"]
    if not force and _newer(LIB, deps):
        return LIB
    cxx = shutil.which("g++") or "g++"
    tmp = LIB.with_suffix(".so.tmp")
    _run([cxx, "-std=c++20", "-O2", "-fPIC", "-shared", "-Wall", "-Wextra", "-Wno-unused-parameter",
          f"-I{CUDA_HOME / 'include'}", f"-I{native}",
          f'-DF4S_KERNEL_IMAGE="{cubin}"', *map(str, sources), *map(str, objs), str(native / "kernel_image.S"),
          f"-L{CUDA_HOME / 'lib64'}", "-lcudart_static", "-lrt", "-lpthread",
          # The C++ runtime is linked in and hidden, so the library can be
          # loaded into any host process (a JVM, Python) without its
          # libstdc++ symbols interposing with the host's.
          "-static-libstdc++", "-static-libgcc", "-Wl,--exclude-libs,ALL",
          "-ldl", "-o", str(tmp)])
    tmp.replace(LIB)
    return LIB


def main() -> None:
    force = "--force" in sys.argv
    lib = build_library(force=force, verbose="-v" in sys.argv)
    print(lib)


if __name__ == "__main__":
    main()
