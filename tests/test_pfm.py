"""The .pfm fast path (pyflamert_b200/backend/pfm_image.{hpp,cpp} and
CudaBackend::prepare) against the reference's own loader,
PyFlameFormat::load (src/io/pyflame_format.cpp:392-460), compiled from the
reference's sources into tests/native/test_pfm_fast.cpp.

CPU: the same Graph from both loaders, and the same InvalidModelError text for
every truncation of a model file and for targeted corruptions (bad magic,
version, string/data size limits, dtype, dims, attribute type).
GPU: a model opened through PfmImage and prepared by CudaBackend::prepare gives
bit-identical outputs to the reference-loaded model prepared lazily."""
import json
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "tests", "native", "_build", "test_pfm_fast")


def _exe():
    if not os.path.exists(EXE):
        from pyflamert_b200 import build
        if build.reference_include() is None:
            pytest.skip("needs the PyFlameRT sources to build tests/native/test_pfm_fast")
        build.build_cuda()
        build.build_backend()
        build.build_oracle()
        build.build_pfm_test()
    assert os.path.exists(EXE)
    return EXE


def test_pfm_parse_and_error_parity():
    r = subprocess.run([_exe(), "--cpu"], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0 and "FAIL" not in r.stdout, (r.stdout[-3000:], r.stderr[-2000:])
    assert r.stdout.count("PASS ") == 3


@pytest.mark.gpu
def test_pfm_fast_path_outputs_match_reference_loader():
    assert os.path.exists(EXE), "build it with python -m pyflamert_b200.build (needs the reference sources)"
    r = subprocess.run([EXE], capture_output=True, text=True, timeout=900)
    print(r.stdout)
    assert r.returncode == 0 and "FAIL" not in r.stdout, (r.stdout[-3000:], r.stderr[-2000:])
    assert r.stdout.count("PASS PfmFastPathMatchesReferenceLoader") == 3
    t = json.loads(next(l for l in r.stdout.splitlines() if l.startswith("PFM_TIMING")).split(" ", 1)[1])
    assert t["bytes"] > 0 and t["fast_ms"] > 0 and t["reference_ms"] > 0
