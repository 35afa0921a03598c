"""Build the native parts of kinetic-rt-b200 in-tree.

Outputs (all under python/kinetic_rt/):
  libkrt.so                  CUDA kernels + the C ABI of include/krt.h (sm_100a)
  kernels/fused_rmsnorm_qkv_rope.sm_100a.cubin
                             kernel image that AOTEngine packs into .kin files
  _core.<ext>                pybind11 module over the C++ runtime (real CUDA)
  _core_mock.<ext>           the same runtime over a host-only fake of the CUDA
                             runtime, for headless host-logic tests

    python kinetic-rt_b200/build.py [--only lib|cubin|core|mock] [-j N]

Rebuilds a target only when one of its inputs is newer than the output.
"""
import argparse
import glob
import os
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
RUNTIME = os.path.join(CSRC, "runtime")
PKG = os.path.join(HERE, "python", "kinetic_rt")
INCLUDE = os.path.join(REPO, "include")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CUDA_INC = "/usr/local/cuda/include"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
EXT = sysconfig.get_config_var("EXT_SUFFIX")

LIB_SOURCES = ["capi.cu", "qkv_generic.cu", "qkv_prep.cu", "qkv_decode.cu", "qkv_decode_noalloc.cu", "qkv_prefill.cu", "gemm_ar.cu", "comm.cu", "attn_decode.cu", "attn_prefill.cu", "proj_persistent.cu"]


def _pybind_includes():
    import pybind11
    return [pybind11.get_include(), sysconfig.get_paths()["include"]]


def _newer(out, inputs):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(i) > t for i in inputs if os.path.exists(i))


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {os.path.basename(cmd[-1])}")
    return r


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h")) + glob.glob(os.path.join(RUNTIME, "*.h"))


def build_lib(jobs=8):
    out = os.path.join(PKG, "libkrt.so")
    srcs = [os.path.join(CSRC, s) for s in LIB_SOURCES if os.path.exists(os.path.join(CSRC, s))]
    objdir = os.path.join(HERE, "_build", "lib")
    os.makedirs(objdir, exist_ok=True)
    objs = []

    def compile_one(src):
        obj = os.path.join(objdir, os.path.basename(src) + ".o")
        if _newer(obj, [src] + _headers()):
            _run([NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
                  "-Xptxas", "-v", "--expt-relaxed-constexpr", "-I", INCLUDE, "-c", src, "-o", obj])
        return obj

    with ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(compile_one, srcs))
    if _newer(out, objs):
        vs = os.path.join(objdir, "exports.map")
        with open(vs, "w") as f:
            f.write("{ global: krt_*; local: *; };\n")
        tmp = out + ".tmp"  # linked aside and renamed: a reader never sees a half-written library
        _run([NVCC, *ARCH, "-shared", "-cudart", "static", "-Xlinker", f"--version-script={vs}",
              "-Xlinker", "--exclude-libs,ALL", *objs, "-o", tmp])
        os.replace(tmp, out)
    return out


def build_cubin():
    out_dir = os.path.join(PKG, "kernels")
    os.makedirs(out_dir, exist_ok=True)
    out = os.path.join(out_dir, "fused_rmsnorm_qkv_rope.sm_100a.cubin")
    src = os.path.join(CSRC, "aot_kernel.cu")
    if _newer(out, [src] + _headers()):
        _run([NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-cubin", src, "-o", out])
    return out


def _runtime_sources():
    return sorted(glob.glob(os.path.join(RUNTIME, "*.cpp"))) + [os.path.join(CSRC, "bindings", "python_bindings.cpp")]


def build_core(mock=False, jobs=8):
    name = "_core_mock" if mock else "_core"
    out = os.path.join(PKG, name + EXT)
    srcs = _runtime_sources()
    objdir = os.path.join(HERE, "_build", name)
    os.makedirs(objdir, exist_ok=True)
    defs = ["-DKRT_MOCK_CUDA=1", f"-DKRT_MODULE_NAME={name}"] if mock else [f"-DKRT_MODULE_NAME={name}"]
    incs = ["-I", INCLUDE, "-I", RUNTIME] + sum((["-I", p] for p in _pybind_includes()), [])
    if not mock:
        incs += ["-I", CUDA_INC]

    def compile_one(src):
        obj = os.path.join(objdir, os.path.basename(src) + ".o")
        if _newer(obj, [src] + _headers()):
            _run(["g++", "-O2", "-std=c++17", "-fPIC", "-fvisibility=hidden", *defs, *incs, "-c", src, "-o", obj])
        return obj

    with ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(compile_one, srcs))
    lib = os.path.join(PKG, "libkrt.so")
    deps = objs + ([] if mock else [lib])
    if _newer(out, deps):
        if mock:
            _run(["g++", "-shared", "-fPIC", *objs, "-o", out, "-lpthread"])
        else:
            _run([NVCC, *ARCH, "-shared", "-cudart", "static", "-Xlinker", "--exclude-libs,ALL", *objs,
                  "-L", PKG, "-lkrt", "-Xlinker", "-rpath,$ORIGIN", "-o", out])
    return out


def build_all(jobs=8, only=None):
    outs = []
    if only in (None, "lib"):
        outs.append(build_lib(jobs))
    if only in (None, "cubin"):
        outs.append(build_cubin())
    have_runtime = os.path.exists(os.path.join(CSRC, "bindings", "python_bindings.cpp"))
    if only in (None, "core") and have_runtime:
        outs.append(build_core(False, jobs))
    if only in (None, "mock") and have_runtime:
        outs.append(build_core(True, jobs))
    return outs


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", choices=["lib", "cubin", "core", "mock"])
    ap.add_argument("-j", type=int, default=8)
    args = ap.parse_args()
    for o in build_all(args.j, args.only):
        print(o)
