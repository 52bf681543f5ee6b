"""The reference's own kernel test suites, run against this library.

oracle/Makefile (target ref_suites) compiles the reference's
tests/test_cuda_ops.cpp, test_attention.cpp and test_sampler.cpp unmodified,
where they lie, against the compatibility headers in
serving-engine_b200/compat (the reference's engine::cuda / SamplerGPU API as
inline wrappers over the C-ABI) and links libb2engine.so: the reference's
seeded shapes, CPU references and tolerances then check this library's
kernels, and the suites building unchanged shows the drop-in boundary.
The binaries are built where the reference sources exist and travel to the
GPU box prebuilt; each runs as its own process.
"""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SUITES = ["test_cuda_ops", "test_attention", "test_sampler"]


@pytest.mark.parametrize("suite", SUITES)
def test_reference_suite_passes(cuda, suite):
    exe = os.path.join(ROOT, "oracle", "_ref", suite)
    if not os.path.exists(exe):
        pytest.skip("reference suites not built (make -C oracle ref_suites where the reference sources exist)")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=900, cwd=ROOT)
    tail = (r.stdout + r.stderr)[-4000:]
    assert r.returncode == 0, tail
    assert "Status: SUCCESS!" in r.stdout, tail
