"""The reference's own C++ code paths (dispatchers, autograd, Linear, conv backward,
OpRegistry) on CUDA tensors, with the GEMM/conv entry points of include/TensorOps.hpp:703-712
served by this library through minitensor_b200/overlay/gpu_ops_b200.cpp.

The test binary is built by minitensor_b200.build.build_dropin() where the reference
checkout exists (its headers and src/gpu_ops.cpp are compiled from where they lie) and
travels with the other built files."""
import os
import subprocess

import pytest
import torch

from minitensor_b200 import build

pytestmark = pytest.mark.gpu


def test_reference_paths_run_on_the_engine():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    # Built by build_dropin() where the reference checkout exists; the binary travels with
    # the other built files, so its absence on a GPU machine is a failure, not a skip.
    assert os.path.exists(build.DROPIN_BIN), "drop-in test binary not built: run build.build_dropin()"
    r = subprocess.run([build.DROPIN_BIN], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "ALL PASSED" in r.stdout
