"""CPU tests of the C ABI boundary: the library loads, exports every function that
include/*.h declares, and rejects bad arguments with the reference's error semantics
before touching the device."""
import ctypes
import glob
import os
import re

import pytest
import torch

from minitensor_b200 import engine

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = []
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        names += re.findall(r"MT_API\s+[\w\s\*]+?\b(mt_\w+)\s*\(", src)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared_functions()
    for n in ("mt_matmul_gpu", "mt_matmul_gpu_strided", "mt_bmm_gpu", "mt_linear_fwd_gpu", "mt_gemm"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = engine.lib()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_version_and_default_mode():
    assert "sm_100a" in engine.version()
    assert engine.lib().mt_get_default_mode() in (0, 1, 2)


def _t(*shape):
    return torch.zeros(shape, dtype=torch.float32)


@pytest.mark.parametrize("fn", ["matmul_gpu", "matmul_gpu_strided", "matmul_gpu_v2", "matmul_gpu_bk16"])
def test_matmul_shape_errors_raise_value_error(fn):
    # include/TensorOps.hpp:995-1005: std::invalid_argument on mismatched inner dims.
    with pytest.raises(ValueError, match="Dimension mismatch"):
        getattr(engine, fn)(_t(2, 3), _t(4, 2), _t(2, 2))
    with pytest.raises(ValueError, match="2-D"):
        getattr(engine, fn)(_t(2, 3, 1), _t(3, 2), _t(2, 2))
    with pytest.raises(ValueError, match="C must be"):
        getattr(engine, fn)(_t(2, 3), _t(3, 2), _t(3, 3))


def test_bmm_shape_errors():
    # include/TensorOps.hpp:937-943.
    with pytest.raises(ValueError, match="batch dimension mismatch"):
        engine.bmm_gpu(_t(2, 3, 4), _t(3, 4, 5), _t(2, 3, 5))
    with pytest.raises(ValueError, match="inner dimension mismatch"):
        engine.bmm_gpu(_t(2, 3, 4), _t(2, 5, 5), _t(2, 3, 5))
    with pytest.raises(ValueError, match="3-D"):
        engine.bmm_gpu(_t(3, 4), _t(4, 5), _t(3, 5))


def test_dispatcher_errors():
    with pytest.raises(ValueError, match="Dimension mismatch"):
        engine.matmul(_t(2, 3), _t(2, 3))
    with pytest.raises(ValueError, match="bmm requires 3D"):
        engine.bmm(_t(2, 3), _t(3, 2))
    with pytest.raises(ValueError, match="float32"):
        engine.view(torch.zeros(2, 2, dtype=torch.float64))


def test_gemm_argument_errors():
    lib = engine.lib()
    a, b, c = engine.view(_t(2, 3)), engine.view(_t(3, 2)), engine.view(_t(2, 2))
    rc = lib.mt_gemm(ctypes.byref(a), ctypes.byref(b), ctypes.byref(c), None, 0, 7, None)
    assert rc == engine.MT_EINVAL and b"bad mode" in lib.mt_last_error()
    rc = lib.mt_gemm(ctypes.byref(a), ctypes.byref(b), ctypes.byref(c), None, 64, 0, None)
    assert rc == engine.MT_EINVAL
    rc = lib.mt_gemm(None, ctypes.byref(b), ctypes.byref(c), None, 0, 0, None)
    assert rc == engine.MT_EINVAL


def test_view_carries_offset_and_strides():
    base = torch.arange(48, dtype=torch.float32).reshape(6, 8)
    v = engine.view(base[2:5, 1:7].t())
    assert v.offset == 2 * 8 + 1 and v.ndim == 2
    assert list(v.shape)[:2] == [6, 3] and list(v.strides)[:2] == [1, 8]
    e = engine.view(torch.zeros(1, 4, 5).expand(3, 4, 5))
    assert list(e.strides)[:3] == [0, 5, 1]


def test_sum_rows_argument_errors():
    lib = engine.lib()
    x3, out = engine.view(_t(2, 3, 4)), engine.view(_t(4))
    assert lib.mt_sum_rows_gpu(ctypes.byref(x3), ctypes.byref(out), None) == engine.MT_EINVAL
    assert b"2-D" in lib.mt_last_error()
    x, wrong = engine.view(_t(5, 4)), engine.view(_t(3))
    assert lib.mt_sum_rows_gpu(ctypes.byref(x), ctypes.byref(wrong), None) == engine.MT_EINVAL
    assert b"columns" in lib.mt_last_error()
    two_rows = engine.view(_t(2, 4))
    assert lib.mt_sum_rows_gpu(ctypes.byref(x), ctypes.byref(two_rows), None) == engine.MT_EINVAL
    assert lib.mt_sum_rows_gpu(None, ctypes.byref(out), None) == engine.MT_EINVAL


def test_copy_rows_and_multi_gpu_argument_errors():
    lib = engine.lib()
    assert lib.mt_copy_rows_async(None, 64, None, 64, 16, 4, None) == engine.MT_EINVAL
    buf = ctypes.create_string_buffer(64)
    p = ctypes.cast(buf, ctypes.c_void_p)
    assert lib.mt_copy_rows_async(p, 8, p, 64, 16, 4, None) == engine.MT_EINVAL   # pitch < width
    assert lib.mt_copy_rows_async(p, 64, p, 64, 16, 0, None) == engine.MT_OK      # nothing to copy
    a, b, c = engine.view(_t(2, 3)), engine.view(_t(3, 2)), engine.view(_t(2, 2))
    rc = lib.mt_gemm_multi(ctypes.byref(a), ctypes.byref(b), ctypes.byref(c), None, 2, None, 0, 0, None)
    assert rc == engine.MT_EINVAL and b"extra_dst" in lib.mt_last_error()
    rc = lib.mt_gemm_multi(ctypes.byref(a), ctypes.byref(b), ctypes.byref(c), None, 9, None, 0, 0, None)
    assert rc == engine.MT_EINVAL
    flags = (ctypes.c_void_p * 2)(None, None)
    rc = lib.mt_peer_barrier(flags, 0, 9, 1, 1000, None)
    assert rc == engine.MT_EINVAL


def test_gemm_bias_is_checked_before_the_call():
    # The C ABI takes a raw bias pointer: its length, type and layout are checked above it.
    A, B, C = _t(4, 3), _t(3, 5), _t(4, 5)
    with pytest.raises(ValueError, match="5 elements"):
        engine.gemm(A, B, C, bias=_t(4), epi=engine.EPI_BIAS_COL)
    with pytest.raises(ValueError, match="4 elements"):
        engine.gemm(A, B, C, bias=_t(5), epi=engine.EPI_BIAS_ROW)
    with pytest.raises(ValueError, match="without a bias epilogue"):
        engine.gemm(A, B, C, bias=_t(5), epi=engine.EPI_RELU)
    with pytest.raises(ValueError, match="float32"):
        engine.gemm(A, B, C, bias=torch.zeros(5, dtype=torch.float64), epi=engine.EPI_BIAS_COL)
    with pytest.raises(ValueError, match="contiguous"):
        engine.gemm(A, B, C, bias=_t(5, 2)[:, 0], epi=engine.EPI_BIAS_COL)


def _sms():
    return torch.cuda.get_device_properties(0).multi_processor_count if torch.cuda.is_available() else 0


@pytest.mark.parametrize("mode,x3", [("tf32", False), ("tf32x3", True)])
def test_workspace_query_describes_dw_by_shape(mode, x3):
    # Host-only: dW is described by its shape alone; the conv stride and padding pass through.
    from wgrad_plan import tma_bytes
    N, C, H, W, Co, k = 2, 32, 8, 8, 32, 3
    n = engine.conv2d_wgrad_workspace_bytes(_t(N, Co, H, W), _t(N, C, H, W), (Co, C, k, k), 1, 1, mode)
    want, _ = tma_bytes(N, C, H, W, Co, k, k, H, W, _sms(), x3)
    assert n == want > 0
    # x given as a channels-last copy (mt_nchw_to_nhwc's layout): read in place, no NHWC copy.
    x_cl = _t(N, C, H, W).contiguous(memory_format=torch.channels_last)
    n_cl = engine.conv2d_wgrad_workspace_bytes(_t(N, Co, H, W), x_cl, (Co, C, k, k), 1, 1, mode)
    assert n_cl == tma_bytes(N, C, H, W, Co, k, k, H, W, _sms(), x3, x_in_place=True)[0] < n
    # Stride 2: the gather plan, whose only scratch is the split-K partials.
    n2 = engine.conv2d_wgrad_workspace_bytes(_t(N, Co, 4, 4), _t(N, C, H, W), (Co, C, k, k), 2, 1, mode)
    from wgrad_plan import gather_bytes
    assert n2 == gather_bytes(N, C, Co, k, k, 4, 4, _sms())[0]
    # A stride or padding that does not produce dy's shape: 0 bytes, not a crash.
    assert engine.conv2d_wgrad_workspace_bytes(_t(N, Co, H, W), _t(N, C, H, W), (Co, C, k, k), 2, 1, mode) == 0
    assert engine.conv2d_wgrad_workspace_bytes(_t(N, Co, H, W), _t(N, C, H, W), (Co, C, k, k), 1, 0, mode) == 0
    # Strict fp32: one partial sum per image (N x C_in*kh*kw x C_out floats).
    assert engine.conv2d_wgrad_workspace_bytes(_t(N, Co, H, W), _t(N, C, H, W), (Co, C, k, k), 1, 1,
                                               "strict") == N * C * k * k * Co * 4


def test_bmm_backward_shape_errors():
    with pytest.raises(ValueError, match="3D"):
        engine.bmm_backward(_t(3, 4), _t(4, 5), _t(3, 5))
    with pytest.raises(ValueError, match="batch dimension mismatch"):
        engine.bmm_backward(_t(2, 3, 4), _t(3, 4, 5), _t(2, 3, 5))
    with pytest.raises(ValueError, match="dC must be"):
        engine.bmm_backward(_t(2, 3, 4), _t(2, 4, 5), _t(2, 3, 4))
    with pytest.raises(ValueError, match="dC must be"):
        engine.bmm_backward(_t(2, 3, 4), _t(2, 5, 5), _t(2, 3, 5))


def test_matmul_host_argument_errors():
    # Checked before any device call, so these run without a GPU.
    lib = engine.lib()
    buf = ctypes.create_string_buffer(4096)
    p = ctypes.cast(buf, ctypes.c_void_p)
    assert lib.mt_matmul_host(p, p, p, 4, 4, 4, 7, 0, None, 0, None) == engine.MT_EINVAL   # mode
    assert b"bad mode" in lib.mt_last_error()
    assert lib.mt_matmul_host(None, p, p, 4, 4, 4, 0, 0, None, 0, None) == engine.MT_EINVAL
    assert lib.mt_matmul_host(p, p, None, 4, 4, 4, 0, 0, None, 0, None) == engine.MT_EINVAL
    assert lib.mt_matmul_host(p, p, p, 1 << 31, 4, 4, 0, 0, None, 0, None) == engine.MT_EINVAL
    need = lib.mt_matmul_host_workspace_bytes(4, 4, 4)
    assert need >= 3 * 4 * 4 * 4
    assert lib.mt_matmul_host(p, p, p, 4, 4, 4, 0, 0, p, need - 1, None) == engine.MT_EINVAL
    assert b"workspace" in lib.mt_last_error()
    assert lib.mt_matmul_host(p, p, p, 0, 4, 4, 0, 0, None, 0, None) == engine.MT_OK   # empty C
    assert lib.mt_matmul_host(None, None, p, 4, 0, 0, 0, 0, None, 0, None) == engine.MT_OK


def test_matmul_host_workspace_layout():
    # A, B and C each start on a 256-byte boundary; the total covers all three.
    for M, K, N in [(1, 1, 1), (1000, 520, 1200), (8192, 8192, 8192), (3, 0, 5)]:
        n = engine.matmul_host_workspace_bytes(M, K, N)
        up = lambda x: (x + 255) // 256 * 256
        assert n == up(M * K * 4) + up(K * N * 4) + M * N * 4


def test_matmul_host_python_checks():
    with pytest.raises(ValueError, match="Dimension mismatch"):
        engine.matmul_host(_t(3, 4), _t(5, 2))
    with pytest.raises(ValueError, match="2-D"):
        engine.matmul_host(_t(3, 4, 1), _t(4, 2))
    with pytest.raises(ValueError, match="C must be"):
        engine.matmul_host(_t(3, 4), _t(4, 2), C=_t(2, 3))
    with pytest.raises(ValueError, match="host tensor"):
        engine.matmul_host(_t(3, 4).t(), _t(3, 2))


def test_linear_bias_layout_checked_before_the_call():
    # The fused epilogue reads the bias densely; a strided bias view is refused up front.
    lib = engine.lib()
    X, W, Y = engine.view(_t(2, 3)), engine.view(_t(3, 4)), engine.view(_t(2, 4))
    base = torch.zeros(4, 2)
    col_strided = engine.view(base[:, :1])          # [4, 1] with row stride 2
    assert lib.mt_linear_fwd_gpu(ctypes.byref(X), ctypes.byref(W), ctypes.byref(col_strided),
                                 ctypes.byref(Y), 0, None) == engine.MT_EINVAL
    assert b"contiguous" in lib.mt_last_error()
    row_strided = engine.view(torch.zeros(1, 8)[:, ::2])   # [1, 4] with stride 2
    assert lib.mt_linear_fwd_gpu(ctypes.byref(X), ctypes.byref(W), ctypes.byref(row_strided),
                                 ctypes.byref(Y), 0, None) == engine.MT_EINVAL
    short = engine.view(_t(1, 3))
    assert lib.mt_linear_fwd_gpu(ctypes.byref(X), ctypes.byref(W), ctypes.byref(short),
                                 ctypes.byref(Y), 0, None) == engine.MT_EINVAL
    assert b"out_features" in lib.mt_last_error()


def test_peer_barrier_refuses_unbounded_timeout():
    # Checked before any device call: a limit above 60 s is refused, so no wait is unbounded.
    lib = engine.lib()
    flags = (ctypes.c_void_p * 1)(None)
    rc = lib.mt_peer_barrier(flags, 0, 1, 1, 2**64 - 1, None)
    assert rc == engine.MT_EINVAL
    assert b"timeout" in lib.mt_last_error()


def test_scratch_allocator_needs_both_functions():
    lib = engine.lib()
    fn = ctypes.CFUNCTYPE(ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p)(lambda b, d, c: None)
    assert lib.mt_set_scratch_allocator(ctypes.cast(fn, ctypes.c_void_p), None, None) == engine.MT_EINVAL
    assert b"both" in lib.mt_last_error()
    assert lib.mt_set_scratch_allocator(None, None, None) == engine.MT_OK   # back to stream-ordered
    a, b = engine.scratch_counts()
    assert a >= 0 and b >= 0


def test_nchw_to_nhwc_argument_errors():
    # Checked before any device call: shapes, the output's channels-last layout, C % 4.
    lib = engine.lib()
    x = _t(2, 8, 5, 6)
    v = engine.view
    bad = [(x, _t(2, 8, 5, 7).contiguous(memory_format=torch.channels_last), b"shape"),
           (x, _t(2, 8, 5, 6), b"channels-last"),
           (_t(2, 6, 5, 6), _t(2, 6, 5, 6).contiguous(memory_format=torch.channels_last), b"channels-last")]
    for a, o, msg in bad:
        assert lib.mt_nchw_to_nhwc(ctypes.byref(v(a)), ctypes.byref(v(o)), None) == engine.MT_EINVAL
        assert msg in lib.mt_last_error()
    assert lib.mt_nchw_to_nhwc(None, ctypes.byref(v(x)), None) == engine.MT_EINVAL
