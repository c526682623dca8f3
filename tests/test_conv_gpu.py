"""GPU parity tests for Conv2D as implicit GEMM (forward, input-grad, weight-grad,
bias-grad) through the C ABI, against the CPU oracle and the reference's golden vectors."""
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from minitensor_b200 import inputs
from parity import check, dev, host

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden_v1.npz")
MODES = ["strict", "tf32", "tf32x3"]
THREADS = max(1, min(32, os.cpu_count() or 1))


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLDEN)


# Error denominators |x|*|w| for each product (float64; they only scale the error).
def d_fwd(x, w, s, p):
    return F.conv2d(torch.from_numpy(np.abs(x)).double(), torch.from_numpy(np.abs(w)).double(),
                    stride=s, padding=p).numpy()


def d_dgrad(dy, w, x_shape, s, p):
    return torch.nn.grad.conv2d_input(x_shape, torch.from_numpy(np.abs(w)).double(),
                                      torch.from_numpy(np.abs(dy)).double(), stride=s, padding=p).numpy()


def d_wgrad(dy, x, w_shape, s, p):
    return torch.nn.grad.conv2d_weight(torch.from_numpy(np.abs(x)).double(), w_shape,
                                       torch.from_numpy(np.abs(dy)).double(), stride=s, padding=p).numpy()


def run_all(eng, x, w, b, dy, s, p, mode):
    xd, wd = dev(x), dev(w)
    bd = dev(b) if b is not None else None
    y = eng.conv2d(xd, wd, bd, s, p, mode=mode)
    dx, dw, db = eng.conv2d_backward(dev(dy), xd, wd, s, p, mode=mode)
    return host(y), host(dx), host(dw), host(db)


@pytest.mark.parametrize("mode", MODES)
def test_golden_conv(eng, gold, mode):
    # spatial_test.cpp:155-185 known answer [12, 16, 24, 28].
    y = eng.conv2d(dev(gold["convk_x"]), dev(gold["convk_w"]), dev(gold["convk_b"]), 1, 0, mode=mode)
    assert np.allclose(host(y).ravel(), [12, 16, 24, 28], rtol=1e-6)
    # spatial_test.cpp:209-230 device equivalence (stride 2, pad 1): rtol 1e-3, atol 1e-4.
    x, w, b = gold["conveq_x"], gold["conveq_w"], gold["conveq_b"]
    y = host(eng.conv2d(dev(x), dev(w), dev(b), 2, 1, mode=mode))
    ref = gold["conveq_y"]
    assert np.all(np.abs(y - ref) <= 1e-4 + 1e-3 * np.abs(ref))
    for i in range(4):
        s, p = gold[f"conv{i}_meta"].tolist()
        x, w, b, dy = (gold[f"conv{i}_{k}"] for k in ("x", "w", "b", "dy"))
        y, dx, dw, db = run_all(eng, x, w, b, dy, s, p, mode)
        K = x.shape[1] * w.shape[2] * w.shape[3]
        check(mode, y, gold[f"conv{i}_y"], d_fwd(x, w, s, p) + np.abs(b)[None, :, None, None], K, f"conv{i} fwd")
        check(mode, dx, gold[f"conv{i}_dx"], d_dgrad(dy, w, x.shape, s, p), w.shape[0] * w.shape[2] * w.shape[3],
              f"conv{i} dgrad")
        check(mode, dw, gold[f"conv{i}_dw"], d_wgrad(dy, x, w.shape, s, p), dy.shape[0] * dy.shape[2] * dy.shape[3],
              f"conv{i} wgrad")
        assert np.allclose(db, gold[f"conv{i}_db"], rtol=1e-5, atol=1e-5), f"conv{i} bias grad"


@pytest.mark.parametrize("mode", MODES)
def test_config4_resnet_3x3(eng, port, mode):
    x, w, b, dy = inputs.config4()
    xd, wd, dyd = dev(x), dev(w), dev(dy)
    y = host(eng.conv2d(xd, wd, dev(b), 1, 1, mode=mode))
    want = "conv_simt_fwd_fp32" if mode == "strict" else "conv_umma_fwd_" + mode
    assert eng.last_path().startswith(want), eng.last_path()
    yr = port.conv2d(x, w, b, 1, 1, threads=THREADS)
    check(mode, y, yr, d_fwd(x, w, 1, 1), 576, "config4 fwd")
    _, dw, _ = eng.conv2d_backward(dyd, xd, wd, 1, 1, need=("weight",), mode=mode)
    path = eng.last_path()
    dwr = port.conv2d_bwd_weight(dy, x, w.shape, 1, 1, threads=THREADS)
    check(mode, host(dw), dwr, d_wgrad(dy, x, w.shape, 1, 1), 32 * 56 * 56, f"config4 wgrad ({path})")
    dx, _, _ = eng.conv2d_backward(dyd, xd, wd, 1, 1, need=("input",), mode=mode)
    dxr = port.conv2d_bwd_input(dy, w, x.shape, 1, 1, threads=THREADS)
    check(mode, host(dx), dxr, d_dgrad(dy, w, x.shape, 1, 1), 576, "config4 dgrad")


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("shape", [
    # N, C, H, W, Co, k, stride, pad
    (1, 3, 7, 9, 5, 3, 1, 1),
    (2, 17, 13, 11, 33, 3, 2, 1),
    (3, 8, 10, 10, 130, 1, 1, 0),
    (2, 5, 9, 12, 7, 5, 2, 2),
    (1, 64, 14, 14, 256, 3, 1, 1),
    (4, 2, 6, 6, 3, 7, 1, 3),
    (1, 4, 5, 140, 8, 3, 1, 1),       # stride-1 rows wider than one pitched tile
    (2, 40, 9, 20, 48, 3, 1, 0),      # no padding, channels not a multiple of 32
])
def test_conv_shapes(eng, port, mode, shape):
    N, C, H, W, Co, k, s, p = shape
    x = inputs.normal((N, C, H, W), 1.0, 1000 + C)
    w = inputs.normal((Co, C, k, k), float(np.sqrt(2.0 / (C * k * k))), 1100 + Co)
    b = inputs.normal((Co,), 0.1, 1200)
    Ho, Wo = (H + 2 * p - k) // s + 1, (W + 2 * p - k) // s + 1
    dy = inputs.normal((N, Co, Ho, Wo), 1.0, 1300)
    y, dx, dw, db = run_all(eng, x, w, b, dy, s, p, mode)
    K = C * k * k
    check(mode, y, port.conv2d(x, w, b, s, p), d_fwd(x, w, s, p) + np.abs(b)[None, :, None, None], K, f"{shape} fwd")
    check(mode, dx, port.conv2d_bwd_input(dy, w, x.shape, s, p), d_dgrad(dy, w, x.shape, s, p), Co * k * k,
          f"{shape} dgrad")
    check(mode, dw, port.conv2d_bwd_weight(dy, x, w.shape, s, p), d_wgrad(dy, x, w.shape, s, p), N * Ho * Wo,
          f"{shape} wgrad")
    assert np.allclose(db, port.conv2d_bwd_bias(dy), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("mode", ["tf32x3", "strict"])
def test_strided_input_view(eng, port, mode):
    # spatial_test.cpp:259-281: an NHWC buffer viewed as NCHW via transposes (non-contiguous).
    nhwc = (np.arange(2 * 16 * 16 * 3, dtype=np.float32) * np.float32(0.1)).reshape(2, 16, 16, 3)
    xv = dev(nhwc).transpose(1, 3).transpose(2, 3)
    assert not xv.is_contiguous()
    w = np.full((8, 3, 3, 3), 0.5, np.float32)
    b = np.zeros(8, np.float32)
    y = torch.empty(2, 8, 16, 16, device="cuda")
    eng.set_default_mode(mode)
    try:
        eng.conv2d_gpu_strided(xv, dev(w), dev(b), y, 1, 1)
    finally:
        eng.set_default_mode("tf32x3")
    x = np.ascontiguousarray(nhwc.transpose(0, 3, 1, 2))
    check(mode, host(y), port.conv2d(x, w, b, 1, 1), d_fwd(x, w, 1, 1), 27, "strided view")


def test_explicit_workspace_matches_pool(eng):
    x, w, _, dy = (a[:4] if a.ndim == 4 and a.shape[0] == 32 else a for a in inputs.config4())
    xd, wd, dyd = dev(x), dev(w), dev(dy)
    nbytes = eng.conv2d_wgrad_workspace_bytes(dyd, xd, w.shape, 1, 1, mode="tf32x3")
    assert nbytes > 0
    ws = torch.empty(nbytes // 4 + 1, device="cuda")
    _, dw1, _ = eng.conv2d_backward(dyd, xd, wd, 1, 1, need=("weight",), mode="tf32x3", workspace=ws)
    _, dw2, _ = eng.conv2d_backward(dyd, xd, wd, 1, 1, need=("weight",), mode="tf32x3")
    assert torch.equal(dw1, dw2)   # same split plan and reduction order: bit-identical
    with pytest.raises(ValueError, match="workspace"):
        eng.conv2d_backward(dyd, xd, wd, 1, 1, need=("weight",), mode="tf32x3", workspace=ws[:8])


def test_conv_errors_and_empty(eng):
    x = torch.zeros(2, 3, 8, 8, device="cuda")
    w = torch.zeros(4, 5, 3, 3, device="cuda")
    with pytest.raises(ValueError, match="C_in"):
        eng.conv2d(x, w, None, 1, 1)
    w = torch.zeros(4, 3, 3, 3, device="cuda")
    y = torch.zeros(2, 4, 7, 7, device="cuda")
    with pytest.raises(ValueError, match="output must be"):
        eng.conv2d_gpu(x, w, None, y, 1, 1)
    # Kernel larger than the padded input: safe_out_size gives 0 -> empty output.
    y = eng.conv2d(torch.zeros(1, 3, 2, 2, device="cuda"), torch.zeros(4, 3, 5, 5, device="cuda"), None, 1, 1)
    assert tuple(y.shape) == (1, 4, 0, 0)


def test_device_status_clean_after_conv(eng):
    assert eng.device_status(reset=True) == 0


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("shape", [
    # N, C, H, W, Co, kh, kw, stride, pad
    (2, 6, 9, 11, 10, 3, 5, 1, 1),
    (1, 33, 8, 12, 20, 1, 3, 1, 0),
    (1, 64, 10, 10, 64, 3, 1, 1, 0),
    (2, 4, 10, 7, 6, 5, 2, 2, 1),
])
def test_conv_non_square_filters(eng, port, mode, shape):
    """kh != kw with the reference's single padding: the stride-1 input gradient cannot be
    the forward kernel on flipped weights (that needs kh-1-pad down and kw-1-pad across)."""
    N, C, H, W, Co, kh, kw, s, p = shape
    x = inputs.normal((N, C, H, W), 1.0, 1400 + C)
    w = inputs.normal((Co, C, kh, kw), float(np.sqrt(2.0 / (C * kh * kw))), 1500 + Co)
    b = inputs.normal((Co,), 0.1, 1600)
    Ho, Wo = (H + 2 * p - kh) // s + 1, (W + 2 * p - kw) // s + 1
    dy = inputs.normal((N, Co, Ho, Wo), 1.0, 1700)
    y, dx, dw, db = run_all(eng, x, w, b, dy, s, p, mode)
    check(mode, y, port.conv2d(x, w, b, s, p), d_fwd(x, w, s, p) + np.abs(b)[None, :, None, None], C * kh * kw,
          f"{shape} fwd")
    check(mode, dx, port.conv2d_bwd_input(dy, w, x.shape, s, p), d_dgrad(dy, w, x.shape, s, p), Co * kh * kw,
          f"{shape} dgrad")
    check(mode, dw, port.conv2d_bwd_weight(dy, x, w.shape, s, p), d_wgrad(dy, x, w.shape, s, p), N * Ho * Wo,
          f"{shape} wgrad")
    assert np.allclose(db, port.conv2d_bwd_bias(dy), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("mode", ["tf32", "tf32x3"])
def test_conv_per_tap_fallback(eng, port, mode):
    """A 25x25 filter: the smallest halo tile (1 pixel wide, pitch 25, 30 rows) takes 94 KB,
    so the 3xTF32 forward's two hi/lo halo slot pairs exceed the 227 KB of shared memory and
    it takes the per-tap TMA kernel (one activation box per tap); TF32 still fits the halo
    kernel. Both are checked against the oracle, with the input-grad and weight-grad."""
    N, C, H, W, Co, k, s, p = 1, 32, 30, 30, 16, 25, 1, 12
    x = inputs.normal((N, C, H, W), 1.0, 1800)
    w = inputs.normal((Co, C, k, k), float(np.sqrt(2.0 / (C * k * k))), 1801)
    b = inputs.normal((Co,), 0.1, 1802)
    dy = inputs.normal((N, Co, H, W), 1.0, 1803)
    xd, wd = dev(x), dev(w)
    y = eng.conv2d(xd, wd, dev(b), s, p, mode=mode)
    want = "tma bn=" if mode == "tf32x3" else "tma_halo"
    assert want in eng.last_path(), eng.last_path()
    dx, dw, _ = eng.conv2d_backward(dev(dy), xd, wd, s, p, need=("input", "weight"), mode=mode)
    check(mode, host(y), port.conv2d(x, w, b, s, p), d_fwd(x, w, s, p) + np.abs(b)[None, :, None, None],
          C * k * k, "per-tap fwd")
    check(mode, host(dx), port.conv2d_bwd_input(dy, w, x.shape, s, p), d_dgrad(dy, w, x.shape, s, p), Co * k * k,
          "per-tap dgrad")
    check(mode, host(dw), port.conv2d_bwd_weight(dy, x, w.shape, s, p), d_wgrad(dy, x, w.shape, s, p), N * H * W,
          "per-tap shape wgrad")


def test_strict_wgrad_paths(eng, port):
    """Strict weight-grad: per-image partials in scratch, in a caller workspace, and, with a
    workspace too small for them, the direct kernel -- all within the strict bound."""
    N, C, H, W, Co, k = 3, 6, 11, 9, 10, 3
    x = inputs.normal((N, C, H, W), 1.0, 1401)
    dy = inputs.normal((N, Co, H, W), 1.0, 1402)
    w = np.zeros((Co, C, k, k), np.float32)
    ref = port.conv2d_bwd_weight(dy, x, w.shape, 1, 1)
    D = d_wgrad(dy, x, w.shape, 1, 1)
    need = eng.conv2d_wgrad_workspace_bytes(dev(dy), dev(x), w.shape, 1, 1, mode="strict")
    assert need == N * C * k * k * Co * 4
    for ws, path in ((None, "conv_simt_wgrad_fp32"), (torch.empty(need // 4, device="cuda"), "conv_simt_wgrad_fp32"),
                     (torch.empty(need // 8, device="cuda"), "conv_direct_wgrad_fp32")):
        _, dw, _ = eng.conv2d_backward(dev(dy), dev(x), dev(w), 1, 1, need=("weight",), mode="strict", workspace=ws)
        assert eng.last_path() == path, eng.last_path()
        check("strict", host(dw), ref, D, N * H * W, path)


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("stride", [1, 2])
def test_channels_last_inputs(eng, port, mode, stride):
    """mt_nchw_to_nhwc's copy is the same tensor in the layout the stride-1 tensor-core
    kernels work on: the forward and the weight gradient read x from it in place, the
    input gradient dy (path " nhwc_in"), with results bitwise those of the NCHW inputs. Other
    paths (stride 2, strict fp32) read the copy as any strided view, also bitwise equal."""
    N, C, H, W, Co, k, p = 3, 64, 18, 20, 48, 3, 1   # W % 4 == 0: dy's rows suit the TMA weight-grad
    x = inputs.normal((N, C, H, W), 1.0, 1501)
    w = inputs.normal((Co, C, k, k), 0.05, 1502)
    b = inputs.normal((Co,), 0.1, 1503)
    Ho, Wo = (H + 2 * p - k) // stride + 1, (W + 2 * p - k) // stride + 1
    dy = inputs.normal((N, Co, Ho, Wo), 1.0, 1504)
    xd, wd, bd, dyd = dev(x), dev(w), dev(b), dev(dy)
    x_cl = eng.nchw_to_nhwc(xd)
    assert x_cl.stride() == (H * W * C, 1, W * C, C) and torch.equal(x_cl, xd)
    dy_cl = eng.nchw_to_nhwc(dyd)
    assert torch.equal(dy_cl, dyd)
    in_place = stride == 1 and mode != "strict"

    y0 = eng.conv2d(xd, wd, bd, stride, p, mode=mode)
    y1 = eng.conv2d(x_cl, wd, bd, stride, p, mode=mode)
    assert ("nhwc_in" in eng.last_path()) == in_place, eng.last_path()
    assert torch.equal(y0, y1)
    dx0, dw0, _ = eng.conv2d_backward(dyd, xd, wd, stride, p, need=("input", "weight"), mode=mode)
    _, dw1, _ = eng.conv2d_backward(dyd, x_cl, wd, stride, p, need=("weight",), mode=mode)
    assert ("nhwc_in" in eng.last_path()) == in_place, eng.last_path()
    assert torch.equal(dw0, dw1)
    dx1, _, _ = eng.conv2d_backward(dy_cl, xd, wd, stride, p, need=("input",), mode=mode)
    assert ("nhwc_in" in eng.last_path()) == in_place, eng.last_path()
    assert torch.equal(dx0, dx1)
    check(mode, host(y1), port.conv2d(x, w, b, stride, p, THREADS), d_fwd(x, w, stride, p) + np.abs(b)[None, :, None, None],
          C * k * k, "fwd from channels-last x")
    check(mode, host(dw1), port.conv2d_bwd_weight(dy, x, w.shape, stride, p, THREADS),
          d_wgrad(dy, x, w.shape, stride, p), N * Ho * Wo, "wgrad from channels-last x")


def test_nchw_to_nhwc_views_and_errors(eng):
    """The copy from a strided NCHW view (a crop), and the layouts the output must have."""
    base = torch.randn(2, 40, 17, 23, device="cuda")
    xv = base[:, 4:36, 1:16, 2:21]                     # 32 channels, not contiguous
    out = eng.nchw_to_nhwc(xv)
    assert torch.equal(out, xv) and out.stride() == (15 * 19 * 32, 1, 19 * 32, 32)
    with pytest.raises(ValueError, match="channels-last"):
        eng.nchw_to_nhwc(xv, out=torch.empty(2, 32, 15, 19, device="cuda"))       # NCHW output
    with pytest.raises(ValueError, match="channels-last"):
        x6 = torch.randn(1, 6, 4, 4, device="cuda")                              # C % 4 != 0
        eng.nchw_to_nhwc(x6, out=torch.empty_like(x6, memory_format=torch.channels_last))
    with pytest.raises(ValueError, match="shape"):
        eng.nchw_to_nhwc(xv, out=torch.empty(2, 32, 15, 18, device="cuda").to(memory_format=torch.channels_last))


def test_cta_pair_forward_matches_one_cta(eng, port, tmp_path):
    """The CTA-pair halo forward (M = 256 over two SMs; opt-in with MT_CONV_PAIR=1, since it
    measured slower than one CTA per tile) runs every output through the same MMA k-steps,
    so its results must equal the one-CTA kernel's bit for bit: config 4's forward and
    input gradient in both tensor-core precisions, and a shape whose last pair has its
    second tile past the right edge."""
    import subprocess
    import sys
    script = os.path.join(os.path.dirname(__file__), "conv_pair_cases.py")
    res = {}
    for flag in ("1", "0"):
        out = str(tmp_path / f"pair{flag}.npz")
        env = dict(os.environ, MT_CONV_PAIR=flag)
        r = subprocess.run([sys.executable, script, out], env=env, capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
        res[flag] = np.load(out)
    pair, one = res["1"], res["0"]
    names = [k for k in pair.files if not k.startswith("path_")]
    assert len(names) == 6
    for k in names:
        assert str(pair["path_" + k]).endswith(" pair"), (k, str(pair["path_" + k]))
        assert " pair" not in str(one["path_" + k]), (k, str(one["path_" + k]))
        assert np.array_equal(pair[k], one[k]), k
    x, w, b, _ = inputs.config4()
    xs = np.ascontiguousarray(x[:2])
    check("tf32x3", pair["fwd_tf32x3"][:2], port.conv2d(xs, w, b, 1, 1, THREADS),
          d_fwd(xs, w, 1, 1) + np.abs(b)[None, :, None, None], 576, "pair forward, images 0-1")
