"""Python front of libmtgemm.so -- the reference's GPU GEMM interface, mirrored.

The names, argument meaning and error behaviour follow the reference's C++ entry points
(include/TensorOps.hpp:703-712 and the dispatchers at :933-1149):

* ``matmul_gpu(A, B, C)`` & co. write into a caller-allocated ``C``; shape errors raise
  ``ValueError`` (the reference throws ``std::invalid_argument``), CUDA failures raise
  ``RuntimeError`` (``GPU_CHECK`` throws ``std::runtime_error``).
* ``matmul(A, B)``, ``bmm(A, B)``, ``linear_forward`` ... allocate the output like the
  reference dispatchers do.

Tensors are torch CUDA tensors used purely as device memory: each is passed to the C ABI
as (storage base, view offset, shape, strides) -- the fields of the reference's
TensorImpl -- so transposed, sliced and expanded (stride-0) views are consumed in place.
There is no CPU or library fallback: if libmtgemm.so is missing this module raises.
"""
from __future__ import annotations

import ctypes
import os

import torch

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libmtgemm.so")

MAX_DIMS = 8
MT_OK, MT_EINVAL, MT_EUNSUPPORTED, MT_ECUDA, MT_ETIMEOUT, MT_ENOMEM = range(6)
MODE_DEFAULT, STRICT_FP32, TF32, TF32X3 = -1, 0, 1, 2
MODES = {"default": MODE_DEFAULT, "strict": STRICT_FP32, "tf32": TF32, "tf32x3": TF32X3}
EPI_NONE, EPI_BIAS_ROW, EPI_BIAS_COL, EPI_RELU = 0, 1, 2, 4


class MtTensor(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("offset", ctypes.c_uint64),
        ("ndim", ctypes.c_uint32),
        ("shape", ctypes.c_uint64 * MAX_DIMS),
        ("strides", ctypes.c_uint64 * MAX_DIMS),
    ]


_lib = None


def lib() -> ctypes.CDLL:
    """Loads libmtgemm.so (built in-tree by ``python -m minitensor_b200.build``)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m minitensor_b200.build`")
    L = ctypes.CDLL(LIB_PATH)
    P = ctypes.POINTER(MtTensor)
    vp = ctypes.c_void_p
    for name in ("mt_matmul_gpu", "mt_matmul_gpu_strided", "mt_matmul_gpu_v2", "mt_matmul_gpu_bk16",
                 "mt_bmm_gpu"):
        fn = getattr(L, name)
        fn.argtypes = [P, P, P, vp]
        fn.restype = ctypes.c_int
    L.mt_linear_fwd_gpu.argtypes = [P, P, P, P, ctypes.c_int, vp]
    L.mt_linear_fwd_gpu.restype = ctypes.c_int
    L.mt_gemm.argtypes = [P, P, P, vp, ctypes.c_int, ctypes.c_int, vp]
    L.mt_gemm.restype = ctypes.c_int
    u64 = ctypes.c_uint64
    for name in ("mt_conv2d_gpu", "mt_conv2d_gpu_strided"):
        fn = getattr(L, name)
        fn.argtypes = [P, P, P, P, u64, u64, vp]
        fn.restype = ctypes.c_int
    for name in ("mt_conv2d_backward_input_gpu", "mt_conv2d_backward_weight_gpu"):
        fn = getattr(L, name)
        fn.argtypes = [P, P, P, u64, u64, vp]
        fn.restype = ctypes.c_int
    L.mt_conv2d_backward_bias_gpu.argtypes = [P, P, vp]
    L.mt_conv2d_backward_bias_gpu.restype = ctypes.c_int
    L.mt_conv2d_fwd.argtypes = [P, P, P, P, u64, u64, ctypes.c_int, vp]
    L.mt_conv2d_fwd.restype = ctypes.c_int
    L.mt_conv2d_dgrad.argtypes = [P, P, P, u64, u64, ctypes.c_int, vp]
    L.mt_conv2d_dgrad.restype = ctypes.c_int
    L.mt_conv2d_wgrad.argtypes = [P, P, P, u64, u64, ctypes.c_int, vp, ctypes.c_size_t, vp]
    L.mt_conv2d_wgrad.restype = ctypes.c_int
    L.mt_conv2d_wgrad_workspace_bytes.argtypes = [P, P, P, u64, u64, ctypes.c_int]
    L.mt_conv2d_wgrad_workspace_bytes.restype = ctypes.c_size_t
    L.mt_nchw_to_nhwc.argtypes = [P, P, vp]
    L.mt_nchw_to_nhwc.restype = ctypes.c_int
    L.mt_sum_rows_gpu.argtypes = [P, P, vp]
    L.mt_sum_rows_gpu.restype = ctypes.c_int
    L.mt_conv2d_wgrad_noalloc.argtypes = [P, P, P, u64, u64, ctypes.c_int, vp]
    L.mt_conv2d_wgrad_noalloc.restype = ctypes.c_int
    # multi-GPU entry points (used by sharded.py)
    L.mt_ipc_get_handle.argtypes = [vp, vp, ctypes.POINTER(u64)]
    L.mt_ipc_get_handle.restype = ctypes.c_int
    L.mt_ipc_open.argtypes = [vp, u64, ctypes.POINTER(vp)]
    L.mt_ipc_open.restype = ctypes.c_int
    L.mt_ipc_close.argtypes = [vp, u64]
    L.mt_ipc_close.restype = ctypes.c_int
    L.mt_gemm_multi.argtypes = [P, P, P, vp, ctypes.c_int, vp, ctypes.c_int, ctypes.c_int, vp]
    L.mt_gemm_multi.restype = ctypes.c_int
    L.mt_peer_barrier.argtypes = [vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, u64, vp]
    L.mt_peer_barrier.restype = ctypes.c_int
    L.mt_copy_rows_async.argtypes = [vp, u64, vp, u64, u64, u64, vp]
    L.mt_copy_rows_async.restype = ctypes.c_int
    L.mt_matmul_host.argtypes = [vp, vp, vp, u64, u64, u64, ctypes.c_int, ctypes.c_int, vp, ctypes.c_size_t, vp]
    L.mt_matmul_host.restype = ctypes.c_int
    L.mt_matmul_host_workspace_bytes.argtypes = [u64, u64, u64]
    L.mt_matmul_host_workspace_bytes.restype = ctypes.c_size_t
    L.mt_set_scratch_allocator.argtypes = [vp, vp, vp]
    L.mt_set_scratch_allocator.restype = ctypes.c_int
    L.mt_scratch_counts.argtypes = [ctypes.POINTER(u64), ctypes.POINTER(u64)]
    L.mt_scratch_counts.restype = None
    L.mt_set_default_mode.argtypes = [ctypes.c_int]
    L.mt_set_default_mode.restype = ctypes.c_int
    L.mt_get_default_mode.restype = ctypes.c_int
    L.mt_last_error.restype = ctypes.c_char_p
    L.mt_last_path.restype = ctypes.c_char_p
    L.mt_launch_count.restype = ctypes.c_uint64
    L.mt_device_status.argtypes = [ctypes.c_int]
    L.mt_device_status.restype = ctypes.c_int
    L.mt_version.restype = ctypes.c_char_p
    _lib = L
    return L


_cuda_present = None


def _gpu_present() -> bool:
    global _cuda_present
    if _cuda_present is None:
        _cuda_present = torch.cuda.is_available()
    return _cuda_present


def view(t: torch.Tensor | None) -> MtTensor | None:
    """A torch tensor as an mt_tensor: storage base + element offset + shape + strides.

    The C ABI takes device pointers only. Where a GPU is present a host tensor is refused
    here, before any kernel could read a host address (the reference's dispatchers refuse
    mixed devices the same way, include/TensorOps.hpp:995-997). Without a GPU no kernel
    can launch, so host tensors still reach the library's argument checks."""
    if t is None:
        return None
    if t.dtype != torch.float32:
        raise ValueError(f"expected float32, got {t.dtype}")
    if t.dim() > MAX_DIMS:
        raise ValueError("Exceeded MAX_DIMS")
    if not t.is_cuda and _gpu_present():
        raise ValueError(f"expected a CUDA tensor, got one on {t.device}")
    v = MtTensor()
    v.data = t.untyped_storage().data_ptr() if t.numel() else 0
    v.offset = t.storage_offset()
    v.ndim = t.dim()
    for i, (s, st) in enumerate(zip(t.shape, t.stride())):
        v.shape[i] = s
        v.strides[i] = st
    return v


def _stream(stream) -> int | None:
    if stream is None:
        # torch's current stream (the role of the reference's active_stream()).
        return torch.cuda.current_stream().cuda_stream if torch.cuda.is_available() else None
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    return int(stream)


def _check(rc: int) -> None:
    if rc == MT_OK:
        return
    msg = lib().mt_last_error().decode()
    if rc == MT_EINVAL:
        raise ValueError(msg)
    raise RuntimeError(f"mtgemm status {rc}: {msg}")


def _ref(v):
    return ctypes.byref(v) if v is not None else None


def _call3(name, A, B, C, stream):
    a, b, c = view(A), view(B), view(C)
    _check(getattr(lib(), name)(_ref(a), _ref(b), _ref(c), _stream(stream)))


# ---- the reference's *_gpu entry points (caller-allocated output) --------------------

def matmul_gpu(A, B, C, stream=None):
    """include/TensorOps.hpp:703."""
    _call3("mt_matmul_gpu", A, B, C, stream)


def matmul_gpu_strided(A, B, C, stream=None):
    """include/TensorOps.hpp:704."""
    _call3("mt_matmul_gpu_strided", A, B, C, stream)


def matmul_gpu_v2(A, B, C, stream=None):
    """include/TensorOps.hpp:705."""
    _call3("mt_matmul_gpu_v2", A, B, C, stream)


def matmul_gpu_bk16(A, B, C, stream=None):
    """include/TensorOps.hpp:706."""
    _call3("mt_matmul_gpu_bk16", A, B, C, stream)


def bmm_gpu(A, B, C, stream=None):
    """One launch for bmm (include/TensorOps.hpp:933-991); stride-0 batch = broadcast."""
    _call3("mt_bmm_gpu", A, B, C, stream)


def linear_fwd_gpu(X, W, bias, Y, relu=False, stream=None):
    """Linear<float>::forward (include/Module.hpp:112-114) with the bias add fused."""
    x, w, b, y = view(X), view(W), view(bias), view(Y)
    _check(lib().mt_linear_fwd_gpu(_ref(x), _ref(w), _ref(b), _ref(y), int(bool(relu)), _stream(stream)))


def gemm(A, B, C, bias=None, epi=EPI_NONE, mode=MODE_DEFAULT, stream=None):
    """C = epi(A @ B) for 2-D or 3-D views with an explicit precision mode."""
    if isinstance(mode, str):
        mode = MODES[mode]
    a, b, c = view(A), view(B), view(C)
    _check(lib().mt_gemm(_ref(a), _ref(b), _ref(c), _bias_ptr(bias, epi, C), int(epi), int(mode),
                         _stream(stream)))


def _bias_ptr(bias, epi, C):
    """The raw bias pointer of mt_gemm, after checking what the C ABI cannot: a dense
    float32 vector of M (EPI_BIAS_ROW) or N (EPI_BIAS_COL) elements on C's device."""
    if bias is None:
        return None
    if not epi & (EPI_BIAS_ROW | EPI_BIAS_COL):
        raise ValueError("bias given without a bias epilogue (EPI_BIAS_ROW or EPI_BIAS_COL)")
    view(bias)   # dtype and device
    want = C.shape[-2] if epi & EPI_BIAS_ROW else C.shape[-1]
    if bias.numel() != want:
        raise ValueError(f"bias must have {want} elements, got {bias.numel()}")
    if not bias.is_contiguous():
        raise ValueError("bias must be contiguous")
    if bias.device != C.device:
        raise ValueError("bias and C must be on the same device")
    return bias.data_ptr()


# ---- allocating dispatchers (include/TensorOps.hpp:933-1045, include/Module.hpp) ------

def matmul(A, B, mode=MODE_DEFAULT, stream=None):
    """matmul(A, B) -> C (include/TensorOps.hpp:993-1045)."""
    if A.device != B.device:
        raise ValueError("Tensors must be on the same device for matmul.")
    if A.dim() != 2 or B.dim() != 2:
        raise ValueError("matmul currently only supports 2D tensors.")
    if A.shape[1] != B.shape[0]:
        raise ValueError("Dimension mismatch: A columns must match B rows.")
    C = torch.empty((A.shape[0], B.shape[1]), dtype=torch.float32, device=A.device)
    gemm(A, B, C, mode=mode, stream=stream)
    return C


def bmm(A, B, mode=MODE_DEFAULT, stream=None):
    """bmm(A, B) -> C (include/TensorOps.hpp:933-991), broadcast operands read in place."""
    if A.device != B.device:
        raise ValueError("Tensors must be on the same device for bmm.")
    if A.dim() != 3 or B.dim() != 3:
        raise ValueError("bmm requires 3D tensors.")
    if A.shape[0] != B.shape[0]:
        raise ValueError("bmm: batch dimension mismatch.")
    if A.shape[2] != B.shape[1]:
        raise ValueError("bmm: inner dimension mismatch (A.K != B.K).")
    C = torch.empty((A.shape[0], A.shape[1], B.shape[2]), dtype=torch.float32, device=A.device)
    gemm(A, B, C, mode=mode, stream=stream)
    return C


def linear_forward(x, W, bias=None, relu=False, mode=MODE_DEFAULT, stream=None):
    """Linear<float>::forward: x [M,in] @ W [in,out] + bias [1,out] (optional ReLU fused)."""
    Y = torch.empty((x.shape[0], W.shape[1]), dtype=torch.float32, device=x.device)
    epi = (EPI_BIAS_COL if bias is not None else 0) | (EPI_RELU if relu else 0)
    gemm(x, W, Y, bias=bias.reshape(-1) if bias is not None else None, epi=epi, mode=mode, stream=stream)
    return Y


_side_streams = {}


def _side_stream(device):
    """One extra stream per device for work that overlaps the caller's stream."""
    key = torch.device(device).index if torch.device(device).index is not None else torch.cuda.current_device()
    if key not in _side_streams:
        _side_streams[key] = torch.cuda.Stream(device=key)
    return _side_streams[key]


def linear_backward_into(x, W, dY, dX, dW, db, mode=MODE_DEFAULT, stream=None):
    """MatmulBackward for Linear into caller buffers. dX = dY @ W^T runs on `stream`; dW =
    x^T @ dY and db run at the same time on a side stream, since neither waits for the
    other and each fills only part of the GPU at Linear sizes. Events fork the side stream
    from `stream` and join it back, so `stream` orders everything that follows, CUDA-graph
    capture included."""
    if stream is None:
        s0 = torch.cuda.current_stream(x.device)
    elif isinstance(stream, torch.cuda.Stream):
        s0 = stream
    else:
        s0 = torch.cuda.ExternalStream(int(stream), device=x.device)
    side = _side_stream(x.device)
    fork = torch.cuda.Event()
    fork.record(s0)
    side.wait_event(fork)
    gemm(dY, W.t(), dX, mode=mode, stream=s0)
    with torch.cuda.stream(side):
        gemm(x.t(), dY, dW, mode=mode, stream=side)
        sum_rows(dY, db, stream=side)
    join = torch.cuda.Event()
    join.record(side)
    s0.wait_event(join)
    return dX, dW, db


def linear_backward(x, W, dY, mode=MODE_DEFAULT, stream=None):
    """MatmulBackward for Linear (include/Autograd.hpp:124-141): dX = dY @ W^T and
    dW = x^T @ dY, both read through transposed views (no copies), plus the bias gradient
    db = the sum of dY over rows (the reference's unbroadcast of the bias add,
    include/TensorOps.hpp:1305-1345). dX and (dW, db) run concurrently on two streams."""
    dX = torch.empty_like(x)
    dW = torch.empty_like(W)
    db = torch.empty((1, dY.shape[1]), dtype=torch.float32, device=dY.device)
    return linear_backward_into(x, W, dY, dX, dW, db, mode=mode, stream=stream)


def matmul_host(A, B, C=None, mode=MODE_DEFAULT, panels=0, workspace=None, stream=None, sync=True):
    """C = A @ B for host (CPU) float32 tensors through mt_matmul_host: the copies in, the
    GEMM and the copies out overlap by row panels (pin A, B and C for the overlap). With
    sync=True (the reference's to() is blocking) the call waits for `stream`; with
    sync=False C is valid once the stream has completed."""
    for name, t in (("A", A), ("B", B)):
        if t.dim() != 2:
            raise ValueError(f"matmul_host: {name} must be 2-D")
    M, K = A.shape
    if B.shape[0] != K:
        raise ValueError("Dimension mismatch: A columns must match B rows.")
    N = B.shape[1]
    if C is None:
        pin = A.is_pinned() and B.is_pinned()
        C = torch.empty((M, N), dtype=torch.float32, pin_memory=pin)
    for name, t in (("A", A), ("B", B), ("C", C)):
        if t.dtype != torch.float32 or t.is_cuda or not t.is_contiguous():
            raise ValueError(f"matmul_host: {name} must be a contiguous float32 host tensor")
    if tuple(C.shape) != (M, N):
        raise ValueError(f"matmul_host: C must be [{M}, {N}]")
    ws, ws_bytes = None, 0
    if workspace is not None:
        if not workspace.is_cuda or not workspace.is_contiguous():
            raise ValueError("matmul_host: workspace must be a contiguous CUDA tensor")
        ws, ws_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    s = _stream(stream)
    _check(lib().mt_matmul_host(A.data_ptr() if A.numel() else None, B.data_ptr() if B.numel() else None,
                                C.data_ptr() if C.numel() else None, M, K, N, _mode(mode), int(panels), ws,
                                ws_bytes, s))
    if sync and torch.cuda.is_available():
        if stream is None:
            torch.cuda.current_stream().synchronize()
        else:
            torch.cuda.ExternalStream(s).synchronize()
    return C


def matmul_host_workspace_bytes(M, K, N) -> int:
    return int(lib().mt_matmul_host_workspace_bytes(M, K, N))


def bmm_backward(A, B, dC, mode=MODE_DEFAULT, stream=None):
    """Gradients of C = bmm(A, B): dA[i] = dC[i] . B[i]^T and dB[i] = A[i]^T . dC[i], read
    through transposed views (no copies).

    The reference's MatmulBackward transposes dims 0 and 1 (include/Autograd.hpp:133,139),
    which is only right for 2-D operands; this is the batched form. An operand that is a
    broadcast view (batch stride 0, the expand of a [1, ., .] tensor) gets the batch sum
    of its gradient as [1, ., .], which is what accumulating into the expanded source means.
    For a broadcast B with batch-contiguous A and dC that sum is ONE GEMM whose k runs over
    (batch, row). Otherwise the per-batch gradients go to a scratch tensor and
    mt_sum_rows_gpu adds them in batch order."""
    if A.dim() != 3 or B.dim() != 3 or dC.dim() != 3:
        raise ValueError("bmm_backward requires 3D tensors.")
    bt, M, K = A.shape
    N = B.shape[2]
    if B.shape[0] != bt or dC.shape[0] != bt:
        raise ValueError("bmm_backward: batch dimension mismatch.")
    if B.shape[1] != K or tuple(dC.shape[1:]) != (M, N):
        raise ValueError("bmm_backward: dC must be [batch, M, N] for A [batch, M, K] and B [batch, K, N].")
    dev = A.device

    def grad(X, Y, rows, cols, reduce, fold):
        """X [bt, rows, k] . Y [bt, k, cols], batch-summed to [1, rows, cols] if `reduce`."""
        if not reduce or bt == 1:
            out = torch.empty((bt, rows, cols), dtype=torch.float32, device=dev)
            gemm(X, Y, out, mode=mode, stream=stream)
            return out
        out = torch.empty((1, rows, cols), dtype=torch.float32, device=dev)
        if fold is not None:
            gemm(fold[0], fold[1], out[0], mode=mode, stream=stream)
            return out
        part = torch.empty((bt, rows, cols), dtype=torch.float32, device=dev)
        gemm(X, Y, part, mode=mode, stream=stream)
        sum_rows(part.view(bt, rows * cols), out.view(rows * cols), stream=stream)
        return out

    a_bcast = bt > 1 and A.stride(0) == 0
    b_bcast = bt > 1 and B.stride(0) == 0
    fold_b = None
    if b_bcast and A.is_contiguous() and dC.is_contiguous():
        # sum_i A[i]^T dC[i] = (A as [bt*M, K])^T . (dC as [bt*M, N])
        fold_b = (A.reshape(bt * M, K).t(), dC.reshape(bt * M, N))
    dA = grad(dC, B.transpose(1, 2), M, K, a_bcast, None)
    dB = grad(A.transpose(1, 2), dC, K, N, b_bcast, fold_b)
    return dA, dB


def sum_rows(X, out, stream=None):
    """out[n] = sum over m of X[m, n] (X 2-D, out [N] or [1, N])."""
    _check(lib().mt_sum_rows_gpu(_ref(view(X)), _ref(view(out)), _stream(stream)))


# ---- Conv2D (include/TensorOps.hpp:708-712, :1076-1149) --------------------------------

def out_size(n, pad, k, stride):
    """include/TensorOps.hpp:17-20 safe_out_size."""
    return 0 if n + 2 * pad < k else (n + 2 * pad - k) // stride + 1


def _mode(mode):
    return MODES[mode] if isinstance(mode, str) else int(mode)


def conv2d_gpu(x, w, bias, y, stride, padding, stream=None):
    """include/TensorOps.hpp:708; y is caller-allocated [N, C_out, H_out, W_out]."""
    _check(lib().mt_conv2d_gpu(_ref(view(x)), _ref(view(w)), _ref(view(bias)), _ref(view(y)),
                               stride, padding, _stream(stream)))


def conv2d_gpu_strided(x, w, bias, y, stride, padding, stream=None):
    """include/TensorOps.hpp:709 (non-contiguous input views)."""
    _check(lib().mt_conv2d_gpu_strided(_ref(view(x)), _ref(view(w)), _ref(view(bias)), _ref(view(y)),
                                       stride, padding, _stream(stream)))


def conv2d_backward_input_gpu(dy, w, dx, stride, padding, stream=None):
    """include/TensorOps.hpp:710."""
    _check(lib().mt_conv2d_backward_input_gpu(_ref(view(dy)), _ref(view(w)), _ref(view(dx)), stride, padding,
                                              _stream(stream)))


def conv2d_backward_weight_gpu(dy, x, dw, stride, padding, stream=None):
    """include/TensorOps.hpp:711."""
    _check(lib().mt_conv2d_backward_weight_gpu(_ref(view(dy)), _ref(view(x)), _ref(view(dw)), stride, padding,
                                               _stream(stream)))


def conv2d_backward_bias_gpu(dy, db, stream=None):
    """include/TensorOps.hpp:712."""
    _check(lib().mt_conv2d_backward_bias_gpu(_ref(view(dy)), _ref(view(db)), _stream(stream)))


def nchw_to_nhwc(x, out=None, stream=None):
    """Channels-last copy of a 4-D (N, C, H, W) tensor through mt_nchw_to_nhwc; C must be a
    multiple of 4. The stride-1 tensor-core convolutions read such a copy in place, so a step
    that runs the forward and the weight gradient on the same input transforms it once."""
    if x.dim() != 4:
        raise ValueError("nchw_to_nhwc expects a 4-D tensor")
    if out is None:
        out = torch.empty_like(x, memory_format=torch.channels_last)
    _check(lib().mt_nchw_to_nhwc(_ref(view(x)), _ref(view(out)), _stream(stream)))
    return out


def conv2d(x, w, bias=None, stride=1, padding=0, mode=MODE_DEFAULT, stream=None):
    """conv2d(input, weight, bias, stride, padding) -> output (include/TensorOps.hpp:1076-1110)."""
    if x.dim() != 4 or w.dim() != 4:
        raise ValueError("conv2d expects 4-D input and weight")
    N, _, H, W = x.shape
    Co, _, kh, kw = w.shape
    y = torch.empty((N, Co, out_size(H, padding, kh, stride), out_size(W, padding, kw, stride)),
                    dtype=torch.float32, device=x.device)
    _check(lib().mt_conv2d_fwd(_ref(view(x)), _ref(view(w)), _ref(view(bias)), _ref(view(y)), stride, padding,
                               _mode(mode), _stream(stream)))
    return y


def conv2d_backward(dy, x, w, stride=1, padding=0, need=("input", "weight", "bias"), mode=MODE_DEFAULT,
                    workspace=None, stream=None):
    """Conv2DBackward (include/Autograd.hpp:481-509): (dx, dw, db), each None unless asked for."""
    dx = dw = db = None
    s = _stream(stream)
    if "input" in need:
        dx = torch.empty_like(x, memory_format=torch.contiguous_format)
        _check(lib().mt_conv2d_dgrad(_ref(view(dy)), _ref(view(w)), _ref(view(dx)), stride, padding, _mode(mode), s))
    if "weight" in need:
        dw = torch.empty(w.shape, dtype=torch.float32, device=w.device)
        ws_ptr = workspace.data_ptr() if workspace is not None else None
        ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
        _check(lib().mt_conv2d_wgrad(_ref(view(dy)), _ref(view(x)), _ref(view(dw)), stride, padding, _mode(mode),
                                     ws_ptr, ws_bytes, s))
    if "bias" in need:
        db = torch.empty((dy.shape[1],), dtype=torch.float32, device=dy.device)
        _check(lib().mt_conv2d_backward_bias_gpu(_ref(view(dy)), _ref(view(db)), s))
    return dx, dw, db


def conv2d_wgrad_workspace_bytes(dy, x, w_shape, stride, padding, mode=MODE_DEFAULT):
    # dW is described by shape alone (contiguous, no storage): only its sizes are read.
    v = MtTensor()
    v.ndim = 4
    elem_stride = 1
    for i in reversed(range(4)):
        v.shape[i] = w_shape[i]
        v.strides[i] = elem_stride
        elem_stride *= w_shape[i]
    return int(lib().mt_conv2d_wgrad_workspace_bytes(_ref(view(dy)), _ref(view(x)), _ref(v), stride, padding,
                                                     _mode(mode)))


# ---- settings and diagnostics ---------------------------------------------------------

def set_default_mode(mode) -> int:
    if isinstance(mode, str):
        mode = MODES[mode]
    return lib().mt_set_default_mode(int(mode))


def last_path() -> str:
    return lib().mt_last_path().decode()


def launch_count() -> int:
    return int(lib().mt_launch_count())


def device_status(reset: bool = True) -> int:
    return int(lib().mt_device_status(1 if reset else 0))


def scratch_counts() -> tuple[int, int]:
    """(stream-ordered, from the installed allocator) scratch buffers obtained so far."""
    a, b = ctypes.c_uint64(0), ctypes.c_uint64(0)
    lib().mt_scratch_counts(ctypes.byref(a), ctypes.byref(b))
    return int(a.value), int(b.value)


def version() -> str:
    return lib().mt_version().decode()
