"""The batching caller (cuda::DynamicBatcher, pyflamert_b200/backend/batcher.{hpp,cpp}),
mirroring the reference's DynamicBatcher (include/pyflame_rt/batching/
dynamic_batcher.hpp; src/batching/dynamic_batcher.cpp does not compile).  Every
batched response is compared with the same request run alone
(tests/native/test_batcher.cpp).

CPU: the host logic on the reference's CPUExecutor as the backends.
GPU: the same on CudaBackend, and config 2's layer for single-row requests,
one at a time vs batched."""
import json
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "tests", "native", "_build", "test_batcher")


def _exe():
    if not os.path.exists(EXE):
        from pyflamert_b200 import build
        if build.reference_include() is None:
            pytest.skip("needs the PyFlameRT sources to build tests/native/test_batcher")
        build.build_cuda()
        build.build_backend()
        build.build_oracle()
        build.build_batcher_test()
    assert os.path.exists(EXE)
    return EXE


def test_batcher_host_logic_on_cpu_executor():
    r = subprocess.run([_exe(), "--cpu"], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0 and "FAIL" not in r.stdout, (r.stdout[-3000:], r.stderr[-2000:])
    assert r.stdout.count("PASS ") == 6


@pytest.mark.gpu
def test_batcher_on_cuda_backend():
    assert os.path.exists(EXE), "build it with python -m pyflamert_b200.build (needs the reference sources)"
    r = subprocess.run([EXE], capture_output=True, text=True, timeout=900)
    print(r.stdout)
    assert r.returncode == 0 and "FAIL" not in r.stdout, (r.stdout[-3000:], r.stderr[-2000:])
    t = json.loads(next(l for l in r.stdout.splitlines() if l.startswith("BATCH_TIMING")).split(" ", 1)[1])
    assert t["batched_rps"] > t["alone_rps"]
