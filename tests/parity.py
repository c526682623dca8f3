"""Parity metric shared by the GPU tests.

rel_err = max_ij |C_gpu - C_ref|_ij / D_ij, D = |A|.|B| (the magnitude of the exact
product; computed in float64 -- it only scales the error, so it needs no bit-exactness).
Thresholds (stated in the project's north star):
    strict fp32 and 3xTF32: rel_err <= 1e-5 * sqrt(K)
    TF32:                   rel_err <= 2e-3 * sqrt(K)
"""
import math

import numpy as np
import torch

TOL = {"strict": 1e-5, "tf32x3": 1e-5, "tf32": 2e-3}


def tol(mode: str, K: int) -> float:
    return TOL[mode] * math.sqrt(max(K, 1))


def rel_err(C, C_ref, D) -> float:
    C = np.asarray(C, np.float64)
    C_ref = np.asarray(C_ref, np.float64)
    D = np.asarray(D, np.float64)
    if C.size == 0:
        return 0.0
    err = np.abs(C - C_ref)
    return float(np.max(err / np.maximum(D, 1e-30)))


def absmm(A, B):
    """|A|.|B| in float64 for 2-D or batched operands (numpy broadcasting)."""
    return np.matmul(np.abs(np.asarray(A, np.float64)), np.abs(np.asarray(B, np.float64)))


def dev(x, device="cuda"):
    return torch.from_numpy(np.ascontiguousarray(x)).to(device)


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def check(mode, C_gpu, C_ref, D, K, what=""):
    r = rel_err(C_gpu, C_ref, D)
    assert np.all(np.isfinite(C_gpu)), f"{what}: non-finite output"
    assert r <= tol(mode, K), f"{what} [{mode}] rel_err {r:.3e} > {tol(mode, K):.3e}"
    return r
