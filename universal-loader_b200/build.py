"""Build recipe for the native parts of the package.

  libulb_cuda.so   the C ABI (include/ulb.h) over the sm_100a kernels   (nvcc)
  vulkangguf*.so   the reference-compatible Python module (pybind11)  (g++)

Everything is built in-tree so the built files travel with the repository snapshot.
"""
import concurrent.futures as cf
import os
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
ENGINE = os.path.join(CSRC, "engine")
BUILD = os.path.join(PKG, "_build")
INCLUDE = os.path.join(ROOT, "include")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CUDA_HOME = os.path.dirname(os.path.dirname(NVCC))

CU_SOURCES = ["runtime.cu", "qgemv.cu", "qgemm_tc.cu", "attention.cu", "sampling.cu", "model.cu", "spec.cu"]
CUDA_LIB = os.path.join(PKG, "libulb_cuda.so")
BUILD_TRACE = os.path.join(PKG, "_build_trace")
CUDA_LIB_TRACE = os.path.join(PKG, "libulb_cuda_trace.so")
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
              "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
              "-I" + INCLUDE, "-I" + CSRC]


def _newer(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".h")]
    return hs + [os.path.join(INCLUDE, "ulb.h")]


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed: %s\n%s%s" % (" ".join(cmd), r.stdout, r.stderr))
    return r.stdout + r.stderr


def build_cuda(verbose=False, trace=False):
    """libulb_cuda.so; trace=True: libulb_cuda_trace.so, the same sources with the CTA timeline
    trace compiled in (-DULB_TRACE), under the same soname so the Python module binds to it
    when it is loaded first (bench.py --mode trace)."""
    bdir = BUILD_TRACE if trace else BUILD
    lib_path = CUDA_LIB_TRACE if trace else CUDA_LIB
    os.makedirs(bdir, exist_ok=True)
    hdrs = _headers()
    jobs = []
    objs = []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(bdir, src + ".o")
        objs.append(o)
        if _newer(o, [s] + hdrs):
            extra = (["-Xptxas", "-v"] if verbose else []) + (["-DULB_TRACE"] if trace else [])
            jobs.append(([NVCC] + NVCC_FLAGS + extra + ["-c", s, "-o", o], src))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for out, (cmd, src) in zip(ex.map(lambda j: _run(j[0]), jobs), jobs):
            if verbose and out.strip():
                print("== %s\n%s" % (src, out))
    if _newer(lib_path, objs):
        tmp = lib_path + ".tmp"
        _run([NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-Xlinker", "-soname=libulb_cuda.so",
              "-o", tmp] + objs + ["-lnccl"])
        os.replace(tmp, lib_path)
    return lib_path


def pybind_module_path():
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return os.path.join(PKG, "vulkangguf" + suffix)


def build_engine():
    import pybind11

    out = pybind_module_path()
    srcs = sorted(os.path.join(ENGINE, f) for f in os.listdir(ENGINE) if f.endswith(".cpp"))
    hdrs = sorted(os.path.join(ENGINE, f) for f in os.listdir(ENGINE) if f.endswith(".h")) + _headers()
    if not _newer(out, srcs + hdrs + [CUDA_LIB]):
        return out
    os.makedirs(BUILD, exist_ok=True)
    py_inc = sysconfig.get_paths()["include"]
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden", "-Wall", "-Wno-unused-function",
           "-I" + INCLUDE, "-I" + CSRC, "-I" + ENGINE, "-I" + pybind11.get_include(), "-I" + py_inc] + srcs + [
        "-L" + PKG, "-l:libulb_cuda.so", "-Wl,-rpath,$ORIGIN", "-pthread", "-o", out + ".tmp"]
    _run(cmd)
    os.replace(out + ".tmp", out)
    return out


def build(verbose=False, trace=True):
    lib = build_cuda(verbose=verbose)
    if trace:
        build_cuda(trace=True)
    mod = None
    if os.path.isdir(ENGINE) and any(f.endswith(".cpp") for f in os.listdir(ENGINE)):
        mod = build_engine()
    return lib, mod


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
