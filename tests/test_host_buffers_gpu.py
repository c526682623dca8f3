"""GPU parity tests of the GEMM on host buffers (mt_matmul_host): row panels of A copied in,
GEMMs and copies out overlapped on three streams, checked against the CPU oracle."""
import numpy as np
import pytest
import torch

from minitensor_b200 import inputs
from parity import absmm, check, host

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode", ["strict", "tf32", "tf32x3"])
def test_matmul_host_pinned_in_panels(eng, port, mode):
    M, K, N = 1000, 520, 1200
    A = inputs.uniform((M, K), -1, 1, 130)
    B = inputs.uniform((K, N), -1, 1, 131)
    Ah, Bh = torch.from_numpy(A).pin_memory(), torch.from_numpy(B).pin_memory()
    C = torch.full((M, N), float("nan")).pin_memory()
    eng.matmul_host(Ah, Bh, C, mode=mode, panels=3)
    assert eng.last_path().startswith("matmul_host 3 panels"), eng.last_path()
    check(mode, C.numpy(), port.matmul(A, B), absmm(A, B), K, "host buffers, 3 panels")


def test_matmul_host_matches_device_gemm_and_reuses_workspace(eng):
    M, K, N = 777, 256, 640
    A = inputs.uniform((M, K), -1, 1, 132)
    B = inputs.uniform((K, N), -1, 1, 133)
    ws = torch.empty(eng.matmul_host_workspace_bytes(M, K, N), dtype=torch.uint8, device="cuda")
    C1 = eng.matmul_host(torch.from_numpy(A), torch.from_numpy(B), mode="tf32x3", panels=1, workspace=ws)
    Cd = torch.empty(M, N, device="cuda")
    eng.gemm(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), Cd, mode="tf32x3")
    # One panel is the same single GEMM as the device call: bitwise equal.
    assert np.array_equal(C1.numpy(), host(Cd))
    # Pageable buffers, several panels, the same workspace again: within tolerance.
    C2 = eng.matmul_host(torch.from_numpy(A), torch.from_numpy(B), mode="tf32x3", panels=4, workspace=ws)
    check("tf32x3", C2.numpy(), host(Cd), absmm(A, B), K, "pageable, 4 panels")


def test_matmul_host_k0_and_empty(eng):
    A = torch.empty(300, 0)
    B = torch.empty(0, 50)
    C = torch.full((300, 50), 7.0)
    eng.matmul_host(A, B, C, mode="tf32")
    assert torch.count_nonzero(C) == 0
    C0 = eng.matmul_host(torch.empty(0, 8), torch.ones(8, 5))
    assert tuple(C0.shape) == (0, 5)


def test_matmul_host_config5_rows(eng, port):
    """The benchmark's 8192^3 configuration from pinned host buffers (default panels),
    checked on sampled rows against the oracle."""
    A, B = inputs.config5()
    Ah, Bh = torch.from_numpy(A).pin_memory(), torch.from_numpy(B).pin_memory()
    C = eng.matmul_host(Ah, Bh, mode="tf32x3")
    assert eng.last_path().startswith("matmul_host 8 panels"), eng.last_path()
    Ch = C.numpy()
    for r in (0, 1023, 1024, 4095, 8191):
        check("tf32x3", Ch[r:r + 1], port.matmul_rows(A, B, r, r + 1, 1), absmm(A[r:r + 1], B), 8192,
              f"config5 row {r}")
