"""Run the reference's own Python tests, unmodified, against this build.

    KINETIC_REFERENCE=<reference root or its tests directory> python tests/run_reference_suite.py [--gpu | --host]

The reference's tests import `python.kinetic_rt` (and its fusion_forge /
hardware_probe modules); here that name resolves to this repository's
package (kinetic-rt_b200/python/kinetic_rt), because the package root is put
first on PYTHONPATH and pytest runs from a scratch directory in which the
reference's own `python/` tree is not importable.  Nothing is copied or
edited; the path comes only from KINETIC_REFERENCE.

--gpu   tests/test_fusion.py against the CUDA runtime (python.kinetic_rt._core):
        the .kin bridge and the known-answer math through the
        fused_rmsnorm_qkv_rope[grid](...) call with CPU tensors (needs a B200).
--cpp   tests/test_request_context.cpp, the reference's C++ test of its
        RequestContext, compiled with g++ against this build's
        kinetic-rt_b200/csrc/runtime/RequestContext.cpp (its header found first on
        the include path) and run.
--host  the tests that drive the runtime with fake stream pointers and host
        buffers (test_graph, test_aot, test_validation, test_distributed,
        test_hardware_probe) against the host-only build
        (KINETIC_MOCK_CUDA=1 selects python.kinetic_rt._core_mock), as the
        reference runs them against its HIP/RCCL mocks, with
        KINETIC_ALLOW_MOCKS=1 as those runs need (src/AOTEngine.cpp:385-391).

Exit status: pytest's.
"""
import os
import subprocess
import sys
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(ROOT, "kinetic-rt_b200")

GPU_TESTS = ["test_fusion.py"]
HOST_TESTS = ["test_graph.py", "test_aot.py", "test_validation.py", "test_distributed.py", "test_hardware_probe.py"]


CPP_TESTS = ["test_request_context.cpp"]


def run_cpp(tests_dir):
    """Compile and run the reference's C++ RequestContext test against this
    build's implementation; returns the test binary's exit status."""
    runtime = os.path.join(PKG_ROOT, "csrc", "runtime")
    src = os.path.join(tests_dir, CPP_TESTS[0])
    if not os.path.exists(src):
        print(f"no {CPP_TESTS[0]} under {tests_dir}", file=sys.stderr)
        return 4
    with tempfile.TemporaryDirectory() as scratch:
        exe = os.path.join(scratch, "test_request_context")
        rc = subprocess.call(["g++", "-O1", "-std=c++17", "-I", runtime, src,
                              os.path.join(runtime, "RequestContext.cpp"), "-o", exe, "-lpthread"])
        if rc != 0:
            return rc
        return subprocess.call([exe], cwd=scratch)


def run(tests_dir, which, extra=()):
    tests_dir = os.path.abspath(tests_dir)  # pytest runs from a scratch directory
    if os.path.isdir(os.path.join(tests_dir, "tests")):
        tests_dir = os.path.join(tests_dir, "tests")
    if which == "cpp":
        return run_cpp(tests_dir)
    files = [os.path.join(tests_dir, f) for f in (GPU_TESTS if which == "gpu" else HOST_TESTS)]
    files = [f for f in files if os.path.exists(f)]
    if not files:
        print(f"no reference tests found under {tests_dir}", file=sys.stderr)
        return 4
    env = dict(os.environ)
    env["PYTHONPATH"] = PKG_ROOT + os.pathsep + env.get("PYTHONPATH", "")
    if which == "host":
        # the host-only build, and the mock-artifact gate opened as the
        # reference's own mock test runs need it (src/AOTEngine.cpp:385-391)
        env["KINETIC_MOCK_CUDA"] = "1"
        env["KINETIC_ALLOW_MOCKS"] = "1"
    else:
        env.pop("KINETIC_MOCK_CUDA", None)
    with tempfile.TemporaryDirectory() as scratch:
        cmd = [sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", "--rootdir", scratch,
               "--import-mode=importlib", *extra, *files]
        return subprocess.call(cmd, cwd=scratch, env=env)


def main():
    tests_dir = os.environ.get("KINETIC_REFERENCE")
    if not tests_dir:
        print("set KINETIC_REFERENCE to the reference's tests directory", file=sys.stderr)
        return 2
    which = "gpu" if "--gpu" in sys.argv else "cpp" if "--cpp" in sys.argv else "host"
    return run(tests_dir, which, [a for a in sys.argv[1:] if a not in ("--gpu", "--host", "--cpp")])


if __name__ == "__main__":
    sys.exit(main())
