"""The weight gradient that allocates nothing (mt_conv2d_wgrad_noalloc).

Some callers cannot let a library allocate device memory during a call: a CUDA-graph
capture that must not contain allocation nodes, a host application that owns every byte
of device memory, or a latency-critical loop where an allocation could block. This entry
point keeps its split-K partials in a fixed array inside the library instead, and always
takes the gather weight-gradient kernel (whose only scratch is those partials). The test
calls it through the C ABI twice in a row and checks each result against the allocating
entry point (mt_conv2d_wgrad) within the parity tolerance used by the other tests; it
also checks that the calls leave the device's free memory unchanged and that a problem
too large for the fixed array is refused with a clear error.

The file is named so that pytest collects it last.
"""
import ctypes

import pytest
import torch

from minitensor_b200 import engine, inputs
from parity import check, host
from wgrad_plan import gather_bytes

pytestmark = pytest.mark.gpu

LIMIT = 8 << 20   # bytes of the library's fixed scratch array


def _bind():
    L = engine.lib()
    P = ctypes.POINTER(engine.MtTensor)
    L.mt_conv2d_wgrad_noalloc.argtypes = [P, P, P, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int, ctypes.c_void_p]
    L.mt_conv2d_wgrad_noalloc.restype = ctypes.c_int
    return L


def _noalloc(L, dy, x, dw, stride, pad, mode):
    return L.mt_conv2d_wgrad_noalloc(ctypes.byref(engine.view(dy)), ctypes.byref(engine.view(x)),
                                     ctypes.byref(engine.view(dw)), stride, pad, engine._mode(mode),
                                     engine._stream(None))


def _sms():
    return torch.cuda.get_device_properties(0).multi_processor_count


@pytest.mark.parametrize("mode", ["tf32x3", "tf32"])
def test_noalloc_wgrad_matches_allocating_entry_point(mode):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    L = _bind()
    N, C, H, W, Co, k = 8, 64, 28, 28, 64, 3
    x = torch.from_numpy(inputs.normal((N, C, H, W), 1.0, 501)).cuda()
    dy = torch.from_numpy(inputs.normal((N, Co, H, W), 1.0, 502)).cuda()
    w_shape = (Co, C, k, k)
    need, splits = gather_bytes(N, C, Co, k, k, H, W, _sms())
    assert splits > 1 and 0 < need <= LIMIT     # split-K partials that fit the fixed array

    dw_na = torch.empty(w_shape, device="cuda")
    # First call on the device: looks up the array's address (done before any capture).
    engine._check(_noalloc(L, dy, x, dw_na, 1, 1, mode))
    torch.cuda.synchronize()
    path = engine.last_path()
    assert "gather" in path and f"splits={splits}" in path, path
    denom = torch.nn.grad.conv2d_weight(x.abs().double(), w_shape, dy.abs().double(), stride=1, padding=1)
    for call in range(2):
        dw_na.fill_(float("nan"))
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        engine._check(_noalloc(L, dy, x, dw_na, 1, 1, mode))
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] == free_before, "the no-allocation call changed free device memory"
        _, dw_ref, _ = engine.conv2d_backward(dy, x, torch.empty(w_shape, device="cuda"), 1, 1,
                                              need=("weight",), mode=mode)
        check(mode, host(dw_na), host(dw_ref), denom.cpu().numpy(), N * H * W, f"no-alloc call {call}")
    assert engine.device_status(reset=True) == 0


def test_noalloc_wgrad_rejects_oversized_problem():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    L = _bind()
    # 512 x 512 x 3 x 3 weights: 72 tiles on 148 SMs -> 2 splits of 9.4 MB each.
    N, C, H, W, Co, k = 4, 512, 14, 14, 512, 3
    need, splits = gather_bytes(N, C, Co, k, k, H, W, _sms())
    assert splits > 1 and need > LIMIT
    x = torch.zeros(N, C, H, W, device="cuda")
    dy = torch.zeros(N, Co, H, W, device="cuda")
    dw = torch.empty(Co, C, k, k, device="cuda")
    rc = _noalloc(L, dy, x, dw, 1, 1, "tf32x3")
    assert rc == engine.MT_EINVAL
    assert b"static scratch" in L.mt_last_error()
