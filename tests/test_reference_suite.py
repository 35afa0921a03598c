"""The reference's own Python tests, unmodified, against this build
(tests/run_reference_suite.py).  Runs only when KINETIC_REFERENCE names the
reference's root (or its tests directory); the host-side tests need no GPU, test_fusion.py
needs a B200."""
import os
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def _run(which):
    tests_dir = os.environ.get("KINETIC_REFERENCE")
    if not tests_dir or not os.path.isdir(tests_dir):
        pytest.skip("KINETIC_REFERENCE does not name the reference's directory")
    sys.path.insert(0, HERE)
    import run_reference_suite
    return run_reference_suite.run(tests_dir, which)


def test_reference_host_tests_pass_unmodified():
    assert _run("host") == 0


def test_reference_request_context_cpp_test_passes_unmodified():
    """The reference's tests/test_request_context.cpp against this build's
    RequestContext (g++, no GPU)."""
    assert _run("cpp") == 0


@pytest.mark.gpu
def test_reference_fusion_test_passes_unmodified():
    pytest.importorskip("torch")
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    assert _run("gpu") == 0
