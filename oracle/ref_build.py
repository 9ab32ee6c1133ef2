"""Build recipe for oracle/_ref/libref_cpu.so: the reference's own AVX2 CPU kernels
(src/cpu_backend/gemm_avx2.cpp, src/cpu_backend/dequantize_cpu.cpp), compiled from the
reference tree where they lie with the reference's flags (CMakeLists.txt:16), plus
oracle/ref_shim.cpp's C entry points.  Benchmark infrastructure only: bench.py times these
kernels as the reference CPU path; nothing in the product loads the library.

The reference tree is only present where the repository is developed; elsewhere (a GPU box)
the library built here travels with the snapshot and build() leaves it alone.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
LIB = os.path.join(OUT_DIR, "libref_cpu.so")
REF_ROOT = os.environ.get("ULB_REFERENCE_ROOT", "/root/reference")
SOURCES = ["src/cpu_backend/gemm_avx2.cpp", "src/cpu_backend/dequantize_cpu.cpp"]
REF_FLAGS = ["-mavx2", "-mfma", "-mf16c", "-O3", "-ffast-math"]


def build(force: bool = False):
    srcs = [os.path.join(REF_ROOT, s) for s in SOURCES]
    if not all(os.path.exists(s) for s in srcs):
        return LIB if os.path.exists(LIB) else None
    shim = os.path.join(HERE, "ref_shim.cpp")
    deps = srcs + [shim, os.path.abspath(__file__)]
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(d) for d in deps):
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    cmd = (["g++", "-std=c++17", "-fPIC", "-shared", "-fvisibility=hidden"] + REF_FLAGS +
           ["-I" + os.path.join(REF_ROOT, "src/cpu_backend"), "-o", LIB + ".tmp"] + srcs + [shim])
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
