"""Build recipe for the sm_100a kernel library and the PureAttention host module.

    python pure-attention_b200/build.py            # kernels + host module
    python pure-attention_b200/build.py kernels    # libpa_kernels.so only

Everything is built in-tree (objects under pure-attention_b200/_build/):
  libpa_kernels.so   the C-ABI library (include/pa_kernels.h), nvcc -> sm_100a
  PureAttention*.so  the pybind11 host module (reference operator surface)
"""
import concurrent.futures
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
           "-I" + os.path.join(REPO, "include"), "-I" + CSRC]

KERNEL_SOURCES = [
    "attn_fwd.cu",
    "attn_bwd.cu",
    "fp32_split.cu",
    "layernorm.cu",
    "elementwise.cu",
    "gemm.cu",
    "training.cu",
    "capi.cu",
    "attn_bwd_noalloc.cu",
]

LIB = os.path.join(HERE, "libpa_kernels.so")


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError("build step failed: " + os.path.basename(cmd[-1]))
    return r


def _newer(target, deps):
    if not os.path.exists(target):
        return False
    t = os.path.getmtime(target)
    return all(os.path.getmtime(d) <= t for d in deps)


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs.append(os.path.join(REPO, "include", "pa_kernels.h"))
    return hs


def build_kernels(force=False):
    """Compile every .cu for sm_100a and link libpa_kernels.so."""
    os.makedirs(OBJ, exist_ok=True)
    hdrs = _headers()
    jobs = []
    objs = []
    for src in KERNEL_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJ, src.replace(".cu", ".o"))
        objs.append(o)
        if force or not _newer(o, [s] + hdrs):
            jobs.append(ARCH + NVFLAGS + ["-c", s, "-o", o])
    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        list(ex.map(lambda c: _run([NVCC] + c), jobs))
    if force or jobs or not _newer(LIB, objs):
        _run([NVCC] + ARCH + ["-shared", "-o", LIB] + objs)
    return LIB


HOST = os.path.join(HERE, "host")
HOST_SOURCES = ["src/Tensor.cpp", "src/Autograd.cpp", "src/Functional.cpp", "src/Adam.cpp",
                "src/layers.cpp", "bindings.cpp"]


def build_host(force=False):
    """Compile the C++ host layer + pybind11 bindings into PureAttention<ext>.so,
    linked against libpa_kernels.so (found next to it at run time)."""
    import pybind11
    ext = sysconfig.get_config_var("EXT_SUFFIX")
    out = os.path.join(HERE, "PureAttention" + ext)
    srcs = [os.path.join(HOST, f) for f in HOST_SOURCES]
    hdrs = []
    for root, _, files in os.walk(HOST):
        hdrs += [os.path.join(root, f) for f in files if f.endswith(".h")]
    hdrs.append(os.path.join(REPO, "include", "pa_kernels.h"))
    if not force and _newer(out, srcs + hdrs + [LIB]):
        return out
    os.makedirs(OBJ, exist_ok=True)
    inc = ["-I" + os.path.join(HOST, "include"), "-I" + os.path.join(HOST, "src"),
           "-I" + os.path.join(REPO, "include"), "-I/usr/local/cuda/include",
           "-I" + pybind11.get_include(), "-I" + sysconfig.get_paths()["include"]]
    flags = ["-O2", "-std=c++20", "-fPIC", "-Wall", "-fvisibility=hidden"]
    objs = []
    jobs = []
    for src in srcs:
        o = os.path.join(OBJ, "host_" + os.path.basename(src).replace(".cpp", ".o"))
        objs.append(o)
        jobs.append(["g++"] + flags + inc + ["-c", src, "-o", o])
    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        list(ex.map(_run, jobs))
    _run(["g++", "-shared", "-o", out] + objs +
         ["-L" + HERE, "-lpa_kernels", "-Wl,-rpath,$ORIGIN",
          "-L/usr/local/cuda/lib64", "-lcudart_static", "-ldl", "-lrt", "-lpthread"])
    return out


def build_all(force=False):
    build_kernels(force)
    build_host(force)


if __name__ == "__main__":
    what = sys.argv[1] if len(sys.argv) > 1 else "all"
    force = "--force" in sys.argv
    if what == "kernels":
        print(build_kernels(force))
    else:
        build_all(force)
        print("built", LIB)
