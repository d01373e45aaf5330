"""Builds libtitan_b200.so in-tree.

1. Every kernels/*.cu is compiled by nvcc to an sm_100a cubin
   (-gencode arch=compute_100a,code=sm_100a -O3 -lineinfo).
2. The cubins are embedded into the host library with `.incbin`, so the
   shared object is self-contained and loads them with cuModuleLoadData.
3. The host sources (C++17, no CUDA runtime, libcuda/libnccl opened with
   dlopen at run time) are compiled and linked into
   titan_rs_b200/libtitan_b200.so.

Run:  python -m titan_rs_b200.build   (or call build()).
"""
from __future__ import annotations

import hashlib
import os
import pathlib
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
KERNELS = CSRC / "kernels"
HOST = CSRC / "host"
OUT_DIR = PKG / "_build"
LIB = PKG / "libtitan_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and pathlib.Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the sm_100a kernels cannot be built")


def _cxx() -> str:
    for cand in ("/usr/bin/g++", os.environ.get("CXX"), shutil.which("g++")):
        if cand and pathlib.Path(cand).exists():
            return cand
    raise RuntimeError("no C++ compiler found")


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"command failed ({proc.returncode}): {' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")


def _digest(paths) -> str:
    h = hashlib.sha256()
    for p in sorted(paths):
        h.update(str(p.relative_to(ROOT)).encode())
        h.update(p.read_bytes())
    return h.hexdigest()


def _compile_cubin(src: pathlib.Path, verbose: bool) -> pathlib.Path:
    out = OUT_DIR / (src.stem + ".cubin")
    cmd = [_nvcc(), "-cubin", *ARCH, "-O3", "-lineinfo", "-std=c++17", "-I", str(KERNELS), "-I",
           str(ROOT / "include"), str(src), "-o", str(out)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    _run(cmd)
    return out


def build(verbose: bool = False, force: bool = False) -> pathlib.Path:
    """Compiles all kernels and the host library; returns the .so path."""
    OUT_DIR.mkdir(exist_ok=True)
    kernel_srcs = sorted(KERNELS.glob("*.cu"))
    headers = sorted(KERNELS.glob("*.cuh")) + sorted(HOST.glob("*.hpp")) + [ROOT / "include" / "titan_b200.h"]
    host_srcs = sorted(HOST.glob("*.cpp"))
    runtime_srcs = sorted((CSRC / "noalloc").glob("*.cu"))
    stamp = OUT_DIR / "stamp"
    digest = _digest(kernel_srcs + headers + host_srcs + runtime_srcs + [pathlib.Path(__file__)])
    if not force and LIB.exists() and stamp.exists() and stamp.read_text() == digest:
        return LIB

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        cubins = list(ex.map(lambda s: _compile_cubin(s, verbose), kernel_srcs))

    # .incbin embedding: one symbol pair per cubin, 64-byte aligned.
    lines = ['#include "../csrc/host/internal.hpp"', ""]
    table = []
    for cubin in cubins:
        name = cubin.stem
        sym = f"tbk_cubin_{name}"
        lines.append(
            f'asm(".section .rodata\\n.balign 64\\n.global {sym}\\n{sym}:\\n.incbin \\"{cubin}\\"\\n'
            f'.global {sym}_end\\n{sym}_end:\\n.byte 0\\n.previous\\n");')
        lines.append(f'extern "C" const unsigned char {sym}[]; extern "C" const unsigned char {sym}_end[];')
        table.append((name, sym))
    lines.append("namespace tb {")
    lines.append("const EmbeddedCubin* embedded_cubins(size_t* count) {")
    lines.append("  static const EmbeddedCubin table[] = {")
    for name, sym in table:
        lines.append(f'    {{"{name}", {sym}, (size_t)({sym}_end - {sym})}},')
    lines.append("  };")
    lines.append(f"  *count = {len(table)};")
    lines.append("  return table;")
    lines.append("}")
    lines.append("}  // namespace tb")
    embed = OUT_DIR / "embedded_cubins.cpp"
    embed.write_text("\n".join(lines) + "\n")

    cuda_inc = "/usr/local/cuda/include"
    objs = []

    def compile_host(src: pathlib.Path) -> pathlib.Path:
        obj = OUT_DIR / (src.stem + ".o")
        _run([_cxx(), "-std=c++17", "-O2", "-fPIC", "-Wall", "-Wextra", "-Wno-unused-parameter",
              "-I", cuda_inc, "-I", str(ROOT / "include"), "-DTB_BUILDING_LIBRARY", "-c", str(src), "-o", str(obj)])
        return obj

    def compile_runtime_unit(src: pathlib.Path) -> pathlib.Path:
        # Host+device translation units that use the CUDA runtime API (static cudart).
        obj = OUT_DIR / (src.stem + ".o")
        _run([_nvcc(), "-c", *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", str(KERNELS),
              "-I", str(ROOT / "include"), str(src), "-o", str(obj)])
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_host, host_srcs + [embed]))
        objs += list(ex.map(compile_runtime_unit, runtime_srcs))
    tmp = LIB.with_suffix(".so.tmp")
    _run([_cxx(), "-shared", "-o", str(tmp), *map(str, objs), "-L/usr/local/cuda/lib64", "-lcudart_static", "-lrt",
          "-ldl", "-lpthread", "-Wl,--version-script=" + str(HOST / "exports.map")])
    os.replace(tmp, LIB)
    stamp.write_text(digest)
    return LIB


if __name__ == "__main__":
    path = build(verbose="-v" in sys.argv, force="--force" in sys.argv)
    print(path)
