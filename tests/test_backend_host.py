"""Host-side logic of the PyFlameRT Backend plugin that needs no GPU:
tests/native/test_cuda_backend.cpp --cpu checks the batch-split plan of a
multi-GPU CudaBackend (which graphs split by rows, and the row ranges) and the
parsing of SessionOptions.device strings ("cuda", "cuda:<n>", "cuda:<n>,<m>",
PFRT_CUDA_DEVICES).  The split itself runs on the GPU in
tests/test_gpu_backend.py."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "tests", "native", "_build", "test_cuda_backend")


def test_batch_split_plan_and_device_strings():
    if not os.path.exists(EXE):
        from pyflamert_b200 import build
        if build.reference_include() is None:
            pytest.skip("needs the PyFlameRT sources to build tests/native/test_cuda_backend")
        build.build_cuda()
        build.build_backend()
        build.build_oracle()
        build.build_native_tests()
    r = subprocess.run([EXE, "--cpu"], capture_output=True, text=True, timeout=120)
    print(r.stdout)
    assert r.returncode == 0 and "FAIL" not in r.stdout, (r.stdout[-2000:], r.stderr[-2000:])
    assert r.stdout.count("PASS ") == 3
