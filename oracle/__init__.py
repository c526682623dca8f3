"""CPU oracle for the fp32 GEMM path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / reference legs of
``bench.py`` may import this package. It is the checker, never the thing measured or
shipped: the engine in ``minitensor_b200`` does not import it and fails loudly when its
CUDA library is missing.

Two backends, same signatures (numpy float32 arrays in, numpy float32 arrays out):

* ``Port``  -- ``liboracle.so``: the plain-C restatement in ``mt_oracle.c`` (each
  function cites the reference line it follows).
* ``Ref``   -- ``_ref/libref_cpu.so``: the reference's own CPU code (its headers compiled
  from source by ``oracle/Makefile``). Present when the build ran in a container that
  had the reference checkout; it travels with the other built files.

``Port`` is pinned bit-exactly against ``Ref`` and against the reference's known-answer
tests in ``tests/test_oracle.py``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libref_cpu.so")

_f = ctypes.POINTER(ctypes.c_float)
_i64 = ctypes.c_int64


def _p(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"] or a.ndim == 0
    return a.ctypes.data_as(_f)


def build(ref_include: str | None = None) -> None:
    """Compile liboracle.so (and _ref/libref_cpu.so when the reference headers exist)."""
    subprocess.check_call(["make", "-s", "-C", HERE, "all"])
    # The reference checkout: $MT_REFERENCE_ROOT, else a "reference" directory beside the repo.
    root = os.environ.get("MT_REFERENCE_ROOT",
                          os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))
    inc = ref_include or os.path.join(root, "include")
    if os.path.isdir(inc):
        subprocess.check_call(["make", "-s", "-C", HERE, "ref", f"REF_INCLUDE={inc}"])


def out_size(n: int, pad: int, k: int, stride: int) -> int:
    """include/TensorOps.hpp:17-20 safe_out_size."""
    if n + 2 * pad < k:
        return 0
    return (n + 2 * pad - k) // stride + 1


class Port:
    """ctypes front of the C restatement (mt_oracle.c)."""

    def __init__(self, path: str = PORT_SO):
        if not os.path.exists(path):
            build()
        self.lib = ctypes.CDLL(path)
        L = self.lib
        L.orc_matmul.argtypes = [_f, _f, _f, _i64, _i64, _i64]
        L.orc_matmul_strided.argtypes = [_f, _i64, _i64, _f, _i64, _i64, _f, _i64, _i64, _i64, _i64, _i64]
        L.orc_matmul_rows_mt.argtypes = [_f, _f, _f, _i64, _i64, _i64, _i64, _i64, ctypes.c_int]
        L.orc_bmm.argtypes = [_f, _i64, _i64, _i64, _f, _i64, _i64, _i64, _f, _i64, _i64, _i64, _i64]
        L.orc_linear_fwd.argtypes = [_f, _f, _f, _f, _i64, _i64, _i64]
        L.orc_conv2d_fwd.argtypes = [_f, _f, _f, _f] + [_i64] * 9 + [ctypes.c_int]
        L.orc_conv2d_bwd_input.argtypes = [_f, _f, _f] + [_i64] * 9 + [ctypes.c_int]
        L.orc_conv2d_bwd_weight.argtypes = [_f, _f, _f] + [_i64] * 9 + [ctypes.c_int]
        L.orc_conv2d_bwd_bias.argtypes = [_f, _f, _i64, _i64, _i64, _i64]

    def matmul(self, A, B):
        M, K = A.shape
        N = B.shape[1]
        C = np.empty((M, N), np.float32)
        self.lib.orc_matmul(_p(np.ascontiguousarray(A)), _p(np.ascontiguousarray(B)), _p(C), M, K, N)
        return C

    def matmul_strided(self, A, B):
        """A, B may be any numpy views (transposes, slices); strides are passed through."""
        M, K = A.shape
        N = B.shape[1]
        C = np.empty((M, N), np.float32)
        sa = [s // 4 for s in A.strides]
        sb = [s // 4 for s in B.strides]
        pa = ctypes.cast(A.__array_interface__["data"][0], _f)
        pb = ctypes.cast(B.__array_interface__["data"][0], _f)
        self.lib.orc_matmul_strided(pa, sa[0], sa[1], pb, sb[0], sb[1], _p(C), N, 1, M, K, N)
        return C

    def matmul_rows(self, A, B, r0, r1, threads=1, timing=False):
        M, K = A.shape
        N = B.shape[1]
        C = np.zeros((M, N), np.float32)
        t0 = time.perf_counter()
        self.lib.orc_matmul_rows_mt(_p(A), _p(B), _p(C), M, K, N, r0, r1, threads)
        dt = time.perf_counter() - t0
        return (C[r0:r1], dt) if timing else C[r0:r1]

    def bmm(self, A, B):
        """A [b,M,K], B [b,K,N]; a numpy broadcast view (stride 0) is honoured."""
        bt, M, K = A.shape
        N = B.shape[2]
        C = np.empty((bt, M, N), np.float32)
        sa = [s // 4 for s in A.strides]
        sb = [s // 4 for s in B.strides]
        pa = ctypes.cast(A.__array_interface__["data"][0], _f)
        pb = ctypes.cast(B.__array_interface__["data"][0], _f)
        self.lib.orc_bmm(pa, sa[0], sa[1], sa[2], pb, sb[0], sb[1], sb[2], _p(C), bt, M, K, N)
        return C

    def linear_fwd(self, X, W, bias):
        M, K = X.shape
        N = W.shape[1]
        Y = np.empty((M, N), np.float32)
        self.lib.orc_linear_fwd(_p(X), _p(W), _p(bias.reshape(-1)) if bias is not None else None, _p(Y), M, K, N)
        return Y

    def conv2d(self, x, w, bias, stride, pad, threads=1):
        N, C, H, W = x.shape
        Co, _, kh, kw = w.shape
        y = np.empty((N, Co, out_size(H, pad, kh, stride), out_size(W, pad, kw, stride)), np.float32)
        self.lib.orc_conv2d_fwd(_p(x), _p(w), _p(bias) if bias is not None else None, _p(y),
                                N, C, H, W, Co, kh, kw, stride, pad, threads)
        return y

    def conv2d_bwd_input(self, dy, w, x_shape, stride, pad, threads=1):
        N, C, H, W = x_shape
        Co, _, kh, kw = w.shape
        dx = np.empty((N, C, H, W), np.float32)
        self.lib.orc_conv2d_bwd_input(_p(dy), _p(w), _p(dx), N, C, H, W, Co, kh, kw, stride, pad, threads)
        return dx

    def conv2d_bwd_weight(self, dy, x, w_shape, stride, pad, threads=1):
        N, C, H, W = x.shape
        Co, _, kh, kw = w_shape
        dw = np.empty((Co, C, kh, kw), np.float32)
        self.lib.orc_conv2d_bwd_weight(_p(dy), _p(x), _p(dw), N, C, H, W, Co, kh, kw, stride, pad, threads)
        return dw

    def conv2d_bwd_bias(self, dy):
        N, Co, Ho, Wo = dy.shape
        db = np.empty((Co,), np.float32)
        self.lib.orc_conv2d_bwd_bias(_p(dy), _p(db), N, Co, Ho, Wo)
        return db


class Ref:
    """ctypes front of the reference's own CPU code (_ref/libref_cpu.so)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.lib = ctypes.CDLL(path)
        L = self.lib
        L.ref_matmul.argtypes = [_f, _f, _f, _i64, _i64, _i64]
        L.ref_matmul_t.argtypes = [_f, _f, _f, _i64, _i64, _i64, ctypes.c_int, ctypes.c_int]
        L.ref_matmul_rowslice.argtypes = [_f, _f, _f, _i64, _i64, _i64, _i64, _i64]
        L.ref_bmm.argtypes = [_f, _f, _f, _i64, _i64, _i64, _i64, ctypes.c_int]
        L.ref_linear.argtypes = [_f, _f, _f, _f, _f, _f, _f, _i64, _i64, _i64]
        L.ref_conv2d.argtypes = [_f, _f, _f, _f] + [_i64] * 9
        L.ref_conv2d_backward.argtypes = [_f, _f, _f, _f, _f, _f] + [_i64] * 9
        L.ref_matmul_rows_mt.argtypes = [_f, _f, _f, _i64, _i64, _i64, _i64, _i64, ctypes.c_int,
                                         ctypes.POINTER(ctypes.c_double)]
        L.ref_normal.argtypes = [ctypes.c_uint32, ctypes.c_float, ctypes.c_float, _f, _i64]
        L.ref_conv2d_first_weight.argtypes = [_i64, _i64, _i64, _f]

    @staticmethod
    def _ok(rc):
        if rc != 0:
            raise RuntimeError("reference CPU call threw")

    def matmul(self, A, B):
        M, K = A.shape
        N = B.shape[1]
        C = np.empty((M, N), np.float32)
        self._ok(self.lib.ref_matmul(_p(A), _p(B), _p(C), M, K, N))
        return C

    def matmul_t(self, A_store, B_store, M, K, N, ta, tb):
        C = np.empty((M, N), np.float32)
        self._ok(self.lib.ref_matmul_t(_p(A_store), _p(B_store), _p(C), M, K, N, int(ta), int(tb)))
        return C

    def matmul_rowslice(self, A, B, r0, r1):
        M, K = A.shape
        N = B.shape[1]
        C = np.empty((r1 - r0, N), np.float32)
        self._ok(self.lib.ref_matmul_rowslice(_p(A), _p(B), _p(C), M, K, N, r0, r1))
        return C

    def matmul_rows(self, A, B, r0, r1, threads=1, timing=False):
        """C rows [r0, r1) by the reference's matmul_cpu on row slices; with timing=True
        also returns the seconds spent in matmul_cpu (excluding input copies)."""
        M, K = A.shape
        N = B.shape[1]
        C = np.empty((r1 - r0, N), np.float32)
        sec = ctypes.c_double(0.0)
        self._ok(self.lib.ref_matmul_rows_mt(_p(A), _p(B), _p(C), M, K, N, r0, r1, threads, ctypes.byref(sec)))
        return (C, sec.value) if timing else C

    def bmm(self, A, B, b_bcast):
        bt, M, K = A.shape
        N = B.shape[-1]
        C = np.empty((bt, M, N), np.float32)
        self._ok(self.lib.ref_bmm(_p(A), _p(B), _p(C), bt, M, K, N, int(b_bcast)))
        return C

    def linear(self, X, W, bias, dY):
        M, K = X.shape
        N = W.shape[1]
        Y = np.empty((M, N), np.float32)
        dX = np.empty((M, K), np.float32)
        dW = np.empty((K, N), np.float32)
        self._ok(self.lib.ref_linear(_p(X), _p(W), _p(bias.reshape(-1)) if bias is not None else None,
                                     _p(dY), _p(Y), _p(dX), _p(dW), M, K, N))
        return Y, dX, dW

    def conv2d(self, x, w, bias, stride, pad):
        N, C, H, W = x.shape
        Co, _, kh, kw = w.shape
        y = np.empty((N, Co, out_size(H, pad, kh, stride), out_size(W, pad, kw, stride)), np.float32)
        self._ok(self.lib.ref_conv2d(_p(x), _p(w), _p(bias) if bias is not None else None, _p(y),
                                     N, C, H, W, Co, kh, kw, stride, pad))
        return y

    def normal(self, n, mean, stddev, seed):
        """The first n draws of std::normal_distribution<float>(mean, stddev) on std::mt19937(seed)."""
        out = np.empty(n, np.float32)
        self._ok(self.lib.ref_normal(seed, mean, stddev, _p(out), n))
        return out

    def conv2d_first_weight(self, out_ch, in_ch, k):
        """Weights of the first Conv2D<float> constructed in this process (seed 42)."""
        out = np.empty((out_ch, in_ch, k, k), np.float32)
        self._ok(self.lib.ref_conv2d_first_weight(out_ch, in_ch, k, _p(out)))
        return out

    def conv2d_backward(self, dy, x, w, stride, pad):
        N, C, H, W = x.shape
        Co, _, kh, kw = w.shape
        dx = np.empty((N, C, H, W), np.float32)
        dw = np.empty((Co, C, kh, kw), np.float32)
        db = np.empty((Co,), np.float32)
        self._ok(self.lib.ref_conv2d_backward(_p(dy), _p(x), _p(w), _p(dx), _p(dw), _p(db),
                                              N, C, H, W, Co, kh, kw, stride, pad))
        return dx, dw, db


def have_ref() -> bool:
    return os.path.exists(REF_SO)


def parity_ratio(C, C_ref, D):
    """max_ij |C - C_ref| / D_ij with D = |A|.|B| from the same oracle (0/0 -> 0)."""
    C = np.asarray(C, np.float64)
    C_ref = np.asarray(C_ref, np.float64)
    D = np.asarray(D, np.float64)
    err = np.abs(C - C_ref)
    tiny = np.finfo(np.float32).tiny
    return float(np.max(err / np.maximum(D, tiny))) if err.size else 0.0
