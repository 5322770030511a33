"""Builds the native library in-tree: rustyneedle_b200/_native/libneedle_b200.so.

Every translation unit is compiled by nvcc for sm_100a only, with
-fmad=false (no multiply-add contraction: the reference's float arithmetic is
reproduced operation by operation) and host code with -ffp-contract=off.
The build also writes the host-libm exponential table the library reads at
model open (glibc_expf_exceptions.bin, beside the library).
"""

from __future__ import annotations

import concurrent.futures
import ctypes
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "_native")
LIBRARY = os.path.join(OUT, "libneedle_b200.so")
EXPF_TABLE = os.path.join(OUT, "glibc_expf_exceptions.bin")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

SOURCES = ["kernels.cu", "grammar.cu", "runtime.cu", "archive.cpp", "expf_table.cpp", "call_grammar.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-fmad=false", "--expt-relaxed-constexpr",
                     "-Xcompiler", "-fPIC,-ffp-contract=off,-O3", f"-I{INCLUDE}"]


def _nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if candidate and (os.path.isabs(candidate) and os.path.exists(candidate) or not os.path.isabs(candidate)):
            return candidate
    return "nvcc"


def _headers() -> list[str]:
    names = [os.path.join(SRC, f) for f in os.listdir(SRC) if f.endswith((".h", ".cuh"))]
    return names + [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]


def _stale(target: str, inputs: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(i) > t for i in inputs)


def _compile(source: str, verbose: bool) -> str:
    obj = os.path.join(OUT, "obj", os.path.basename(source) + ".o")
    src = os.path.join(SRC, source)
    if _stale(obj, [src] + _headers() + [__file__]):
        cmd = [_nvcc()] + NVCC_FLAGS + ["-c", src, "-o", obj]
        if source.endswith(".cu") and verbose:
            cmd += ["-Xptxas", "-v"]
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"nvcc failed on {source}:\n{result.stderr}")
        if verbose and result.stderr:
            sys.stderr.write(result.stderr)
    return obj


def build(verbose: bool = False, expf_table: bool = True) -> str:
    """Compiles the library (incrementally) and its expf table; returns the .so path."""
    os.makedirs(os.path.join(OUT, "obj"), exist_ok=True)
    with concurrent.futures.ThreadPoolExecutor(max_workers=len(SOURCES)) as pool:
        objects = list(pool.map(lambda s: _compile(s, verbose), SOURCES))
    if _stale(LIBRARY, objects):
        cmd = [_nvcc()] + ARCH + ["-shared", "-o", LIBRARY] + objects + ["-lpthread", "-ldl"]
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"link failed:\n{result.stderr}")
    if expf_table and not os.path.exists(EXPF_TABLE):
        lib = ctypes.CDLL(LIBRARY)
        lib.nb_build_expf_table.argtypes = [ctypes.c_char_p]
        lib.nb_build_expf_table.restype = ctypes.c_int
        status = lib.nb_build_expf_table(EXPF_TABLE.encode())
        if status != 0:
            raise RuntimeError(f"expf table build failed with status {status}")
    return LIBRARY


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
