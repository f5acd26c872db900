"""The PyFlameRT Backend plugin (CudaBackend, pyflamert_b200/backend) run
inside the reference runtime: tests/native/test_cuda_backend.cpp builds graphs
with the reference's Graph/Node/Tensor, runs them on CudaBackend and on the
reference's CPUExecutor, and compares (bit-exact for the int8 paths, normwise
<= 1e-5 for fp32)."""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "tests", "native", "_build", "test_cuda_backend")


def test_cuda_backend_against_cpu_executor():
    assert os.path.exists(EXE), "build it with python -m pyflamert_b200.build (needs the reference headers)"
    r = subprocess.run([EXE], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    failed = [l for l in r.stdout.splitlines() if l.startswith("FAIL")]
    assert r.returncode == 0 and not failed, (failed, r.stderr[-2000:])
    assert r.stdout.count("PASS ") >= 12


SEAM = os.path.join(ROOT, "tests", "native", "_build", "test_session_seam")


def test_inference_session_device_cuda():
    """The reference's InferenceSession with device="cuda" (seam edits applied
    at build time) against device="cpu" on the same .pfm model."""
    assert os.path.exists(SEAM), "build it with python -m pyflamert_b200.build (needs the reference sources)"
    r = subprocess.run([SEAM], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0 and "FAIL" not in r.stdout, (r.stdout[-3000:], r.stderr[-2000:])
    assert r.stdout.count("PASS ") == 4
