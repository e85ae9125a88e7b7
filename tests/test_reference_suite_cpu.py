"""The reference's own CPU tests of the linear path, unchanged, with this engine registered as ``easyfhe``.

These are the plan / key-set / packing / fake-backend tests of the files whose GPU tests
``tests/test_gpu_reference_suite.py`` runs; they exercise the compatibility layer's module wiring (``easyfhe.fhe``,
``easyfhe.cuda``, the packer replacement, monkeypatching of ``fhe`` names by the reference's tests) without a GPU.
"""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_TESTS = os.path.join(ROOT, "baseline", "_ref", "tests")
FILES = ["test_linear.py", "test_shifted_lane.py", "test_structured_weight.py", "test_qkv.py", "test_mlp.py",
         "test_linear_encode_pipeline.py", "test_parallel_wire.py", "test_parallel_ownership.py"]


def test_reference_cpu_tests_pass_through_the_compatibility_layer():
    paths = [os.path.join(REF_TESTS, f) for f in FILES]
    if not all(os.path.exists(p) for p in paths):
        pytest.skip("the reference is not installed (python tests/install_reference.py <checkout>)")
    cmd = [sys.executable, "-m", "pytest", "-p", "tests.easyfhe_shim_plugin", *paths, "-m", "not gpu", "-q",
           "-p", "no:cacheprovider", "--tb=short"]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    res = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600, env=env)
    tail = "\n".join((res.stdout + res.stderr).strip().splitlines()[-30:])
    assert res.returncode == 0, tail
    assert " passed" in tail and " failed" not in tail, tail
