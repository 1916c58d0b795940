"""The reference's own CUDA test file (tests/test_cuda.cpp), compiled
unchanged (gtest-compatible shim, oracle/gtest_shim) against
(a) the reference kernels and (b) the b200 kernels behind the C++ adapter
(qwen2.5-jetson-inference_b200/adapter/infer_cuda_linear.cpp).  Built by
``make -C oracle reftests`` where the reference sources exist; the binaries
travel with the repository snapshot."""
import os
import re
import subprocess

import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("binary", ["test_cuda_b200", "test_cuda_reference"])
def test_reference_cuda_suite(cuda, b200, binary):
    path = os.path.join(REPO, "oracle", "_ref", binary)
    if not os.path.exists(path):
        pytest.skip(f"{binary} not built (needs the reference sources)")
    proc = subprocess.run([path], capture_output=True, text=True, timeout=600)
    m = re.search(r"SUMMARY passed=(\d+) failed=(\d+) skipped=(\d+)", proc.stdout)
    assert m, proc.stdout[-2000:] + proc.stderr[-2000:]
    passed, failed, skipped = map(int, m.groups())
    assert failed == 0 and proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    assert passed == 9 and skipped == 0
