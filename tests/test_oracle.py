"""CPU tests: pin the oracle (oracle/mt_oracle.c) before trusting it.

1. The reference's own known-answer tests, restated on the oracle.
2. Bit-exact agreement with golden vectors computed by the reference's own code
   (tests/golden/golden_v1.npz, made by tests/golden/make_golden.py).
3. Bit-exact agreement with the reference build (oracle/_ref) on fresh seeded inputs.
"""
import os

import numpy as np
import pytest

from minitensor_b200 import inputs

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden_v1.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLDEN)


# ---------------------------------------------------------------- known answers -----

def test_known_matmul(port):
    # test/tensor_test.cpp:258-283 (CPU) and :285-317 (GPU): [58, 64, 139, 154].
    A = np.arange(1, 7, dtype=np.float32).reshape(2, 3)
    B = np.arange(7, 13, dtype=np.float32).reshape(3, 2)
    assert port.matmul(A, B).ravel().tolist() == [58.0, 64.0, 139.0, 154.0]


def test_known_matmul_backward(port):
    # test/tensor_test.cpp:368-419: C = A.B, dC = ones -> dA = dC.B^T, dB = A^T.dC.
    A = np.arange(1, 7, dtype=np.float32).reshape(2, 3)
    B = np.arange(7, 13, dtype=np.float32).reshape(3, 2)
    g = np.ones((2, 2), np.float32)
    dA = port.matmul_strided(g, B.T)
    dB = port.matmul_strided(A.T, g)
    assert dA.ravel().tolist() == [15, 19, 23, 15, 19, 23]
    assert dB.ravel().tolist() == [5, 5, 7, 7, 9, 9]


def test_known_fill_gradients(port):
    # test/tensor_test.cpp:490-510 and test/engien_test.cpp:80-99: fill 2 / 3.
    A = np.full((2, 3), 2.0, np.float32)
    B = np.full((3, 2), 3.0, np.float32)
    assert port.matmul(A, B)[0, 0] == 18.0
    g = np.ones((2, 2), np.float32)
    assert port.matmul_strided(g, B.T)[0, 0] == 6.0
    assert port.matmul_strided(A.T, g)[0, 0] == 4.0


def test_known_conv(port):
    # test/spatial_test.cpp:155-185: 3x3 input 1..9, 2x2 ones filter -> [12, 16, 24, 28].
    x = np.arange(1, 10, dtype=np.float32).reshape(1, 1, 3, 3)
    w = np.ones((1, 1, 2, 2), np.float32)
    y = port.conv2d(x, w, np.zeros(1, np.float32), 1, 0)
    assert y.ravel().tolist() == [12.0, 16.0, 24.0, 28.0]


def test_benchmark_selfcheck(port):
    # test/benchmark.cpp:696-725: contiguous vs strided path agree (max_err < 1e-4).
    for M, K, N in [(32, 32, 32), (1, 256, 1)]:
        i = np.arange(M * K)
        A = (((i * 131) % 997).astype(np.float32) / np.float32(997)).reshape(M, K)
        j = np.arange(K * N)
        B = (((j * 131) % 997).astype(np.float32) / np.float32(997)).reshape(K, N)
        assert np.max(np.abs(port.matmul(A, B) - port.matmul_strided(A, B))) < 1e-4


def test_conv_gradcheck(port):
    # test/spatial_test.cpp:286-320 run_conv2d_gradcheck on the oracle: loss = sum(conv),
    # central differences eps 1e-3, tolerance atol 1e-3 + rtol 1e-2, first 100 elements.
    rs = np.random.RandomState(42)
    x = rs.uniform(-0.1, 0.1, (2, 3, 5, 5)).astype(np.float32)
    w = rs.uniform(-0.1, 0.1, (4, 3, 3, 3)).astype(np.float32)
    b = rs.uniform(-0.1, 0.1, (4,)).astype(np.float32)
    y = port.conv2d(x, w, b, 1, 0)
    dy = np.ones_like(y)
    grads = {"x": port.conv2d_bwd_input(dy, w, x.shape, 1, 0),
             "w": port.conv2d_bwd_weight(dy, x, w.shape, 1, 0),
             "b": port.conv2d_bwd_bias(dy)}
    params = {"x": x, "w": w, "b": b}
    eps = 1e-3
    for name, p in params.items():
        flat = p.reshape(-1)
        for i in range(min(flat.size, 100)):
            orig = flat[i]
            flat[i] = orig + eps
            lp = float(port.conv2d(x, w, b, 1, 0).sum(dtype=np.float32))
            flat[i] = orig - eps
            ln = float(port.conv2d(x, w, b, 1, 0).sum(dtype=np.float32))
            flat[i] = orig
            num = (lp - ln) / (2 * eps)
            ana = float(grads[name].reshape(-1)[i])
            assert abs(num - ana) <= 1e-3 + 1e-2 * abs(num), (name, i, num, ana)


# ---------------------------------------------------------------- golden vectors ----

def test_golden_matmul(port, gold):
    for key in [k[:-2] for k in gold.files if k.endswith("_C") and (k.startswith("mm") or k.startswith("bench"))
                and not k.startswith("mmt")]:
        C = port.matmul(gold[key + "_A"], gold[key + "_B"])
        assert np.array_equal(C, gold[key + "_C"]), key


def test_golden_transposed_views(port, gold):
    for i in range(3):
        M, K, N, ta, tb = gold[f"mmt{i}_meta"].tolist()
        As, Bs = gold[f"mmt{i}_As"], gold[f"mmt{i}_Bs"]
        A = As.T if ta else As
        B = Bs.T if tb else Bs
        assert np.array_equal(port.matmul_strided(A, B), gold[f"mmt{i}_C"]), i


def test_golden_row_slice(port, gold):
    r0, r1 = gold["rows_meta"].tolist()
    C = port.matmul_strided(gold["rows_A"][r0:r1], gold["rows_B"])
    assert np.array_equal(C, gold["rows_C"])


def test_golden_bmm(port, gold):
    A, B0 = gold["bmmb_A"], gold["bmmb_B0"]
    Bx = np.broadcast_to(B0, (A.shape[0],) + B0.shape[1:])
    assert Bx.strides[0] == 0
    assert np.array_equal(port.bmm(A, Bx), gold["bmmb_C"])
    assert np.array_equal(port.bmm(gold["bmm_A"], gold["bmm_B"]), gold["bmm_C"])


def test_golden_linear(port, gold):
    X, W, b, dY = gold["lin_X"], gold["lin_W"], gold["lin_b"], gold["lin_dY"]
    assert np.array_equal(port.linear_fwd(X, W, b), gold["lin_Y"])
    assert np.array_equal(port.matmul_strided(dY, W.T), gold["lin_dX"])
    assert np.array_equal(port.matmul_strided(X.T, dY), gold["lin_dW"])


def test_golden_conv(port, gold):
    assert np.array_equal(port.conv2d(gold["convk_x"], gold["convk_w"], gold["convk_b"], 1, 0), gold["convk_y"])
    assert np.array_equal(port.conv2d(gold["conveq_x"], gold["conveq_w"], gold["conveq_b"], 2, 1), gold["conveq_y"])
    for i in range(4):
        s, p = gold[f"conv{i}_meta"].tolist()
        x, w, b, dy = (gold[f"conv{i}_{k}"] for k in ("x", "w", "b", "dy"))
        assert np.array_equal(port.conv2d(x, w, b, s, p), gold[f"conv{i}_y"]), i
        assert np.array_equal(port.conv2d_bwd_input(dy, w, x.shape, s, p), gold[f"conv{i}_dx"]), i
        assert np.array_equal(port.conv2d_bwd_weight(dy, x, w.shape, s, p), gold[f"conv{i}_dw"]), i
        assert np.array_equal(port.conv2d_bwd_bias(dy), gold[f"conv{i}_db"]), i


def test_threaded_oracle_matches_single_thread(port):
    A = inputs.uniform((96, 70), -1, 1, 11)
    B = inputs.uniform((70, 50), -1, 1, 12)
    assert np.array_equal(port.matmul_rows(A, B, 10, 90, threads=4), port.matmul(A, B)[10:90])
    x = inputs.normal((3, 4, 9, 9), 1.0, 13)
    w = inputs.normal((5, 4, 3, 3), 0.3, 14)
    dy = inputs.normal((3, 5, 9, 9), 1.0, 15)
    assert np.array_equal(port.conv2d(x, w, None, 1, 1, threads=3), port.conv2d(x, w, None, 1, 1))
    assert np.array_equal(port.conv2d_bwd_weight(dy, x, w.shape, 1, 1, threads=3),
                          port.conv2d_bwd_weight(dy, x, w.shape, 1, 1))


# ---------------------------------------------------------------- vs reference build -

def test_port_matches_reference_build(port, ref):
    for i, (M, K, N) in enumerate([(19, 31, 23), (64, 128, 32)]):
        A = inputs.uniform((M, K), -1, 1, 900 + i)
        B = inputs.uniform((K, N), -1, 1, 950 + i)
        assert np.array_equal(port.matmul(A, B), ref.matmul(A, B))
        assert np.array_equal(port.matmul_rows(A, B, 3, M, threads=2), ref.matmul_rows(A, B, 3, M, threads=3))
    x = inputs.normal((2, 3, 7, 6), 1.0, 960)
    w = inputs.normal((4, 3, 3, 3), 0.5, 961)
    b = inputs.normal((4,), 0.1, 962)
    y = port.conv2d(x, w, b, 2, 1)
    assert np.array_equal(y, ref.conv2d(x, w, b, 2, 1))
    dy = inputs.normal(y.shape, 1.0, 963)
    dx, dw, db = ref.conv2d_backward(dy, x, w, 2, 1)
    assert np.array_equal(port.conv2d_bwd_input(dy, w, x.shape, 2, 1), dx)
    assert np.array_equal(port.conv2d_bwd_weight(dy, x, w.shape, 2, 1), dw)
    assert np.array_equal(port.conv2d_bwd_bias(dy), db)


def test_port_matches_reference_build_sweep(port, ref):
    """Seeded sweep of small shapes, layouts, strides and paddings: the C restatement and
    the reference's own CPU code agree bit for bit (same loop order, same fp32 sums)."""
    rs = np.random.RandomState(2024)
    for i in range(24):
        M, K, N = (int(v) for v in rs.randint(1, 40, size=3))
        ta, tb = int(rs.randint(2)), int(rs.randint(2))
        A_store = inputs.uniform((K, M) if ta else (M, K), -1, 1, 3000 + i)
        B_store = inputs.uniform((N, K) if tb else (K, N), -1, 1, 3100 + i)
        A = A_store.T if ta else A_store
        B = B_store.T if tb else B_store
        got = port.matmul_strided(A, B)
        assert np.array_equal(got, ref.matmul_t(A_store, B_store, M, K, N, ta, tb)), (M, K, N, ta, tb)
        if not ta and not tb:
            assert np.array_equal(port.matmul(A, B), ref.matmul(A, B))
    for i in range(8):
        bt, M, K, N = (int(v) for v in rs.randint(1, 12, size=4))
        A = inputs.normal((bt, M, K), 1.0, 3200 + i)
        bc = bool(i % 2)
        B = inputs.normal((1 if bc else bt, K, N), 1.0, 3300 + i)
        Bv = np.broadcast_to(B, (bt, K, N)) if bc else B
        assert np.array_equal(port.bmm(A, Bv), ref.bmm(A, B, bc)), (bt, M, K, N, bc)
    for i in range(6):
        M, K, N = (int(v) for v in rs.randint(1, 30, size=3))
        X = inputs.normal((M, K), 1.0, 3400 + i)
        W = inputs.normal((K, N), 0.3, 3500 + i)
        b = inputs.normal((1, N), 0.1, 3600 + i)
        dY = inputs.normal((M, N), 1.0, 3700 + i)
        Y, dX, dW = ref.linear(X, W, b, dY)
        assert np.array_equal(port.linear_fwd(X, W, b), Y)
        assert np.array_equal(port.matmul_strided(dY, W.T), dX)
        assert np.array_equal(port.matmul_strided(X.T, dY), dW)
    for i in range(24):
        N, C, Co = (int(v) for v in rs.randint(1, 5, size=3))
        H, W = (int(v) for v in rs.randint(1, 10, size=2))
        kh, kw = (int(v) for v in rs.choice([1, 2, 3, 5], size=2))
        stride, pad = int(rs.randint(1, 4)), int(rs.randint(0, 3))
        x = inputs.normal((N, C, H, W), 1.0, 3800 + i)
        w = inputs.normal((Co, C, kh, kw), 0.5, 3900 + i)
        b = inputs.normal((Co,), 0.1, 4000 + i) if i % 3 else None
        case = (N, C, H, W, Co, kh, kw, stride, pad)
        y = port.conv2d(x, w, b, stride, pad)
        assert np.array_equal(y, ref.conv2d(x, w, b, stride, pad)), case
        if y.size == 0:
            continue
        dy = inputs.normal(y.shape, 1.0, 4100 + i)
        dx, dw, db = ref.conv2d_backward(dy, x, w, stride, pad)
        assert np.array_equal(port.conv2d_bwd_input(dy, w, x.shape, stride, pad), dx), case
        assert np.array_equal(port.conv2d_bwd_weight(dy, x, w.shape, stride, pad), dw), case
        assert np.array_equal(port.conv2d_bwd_bias(dy), db), case


def test_normal_inputs_match_libstdcxx(ref):
    # The synthetic normals are libstdc++'s normal_distribution<float> on mt19937(seed), bit
    # for bit: odd and even lengths (the polar method makes values in pairs), the stds the
    # configurations use, and seeds 0..7 and 42.
    for seed, std, n in [(0, 1.0, 1), (1, 1.0, 2), (2, 1.0, 7), (3, 1.0, 4097), (4, 0.125, 131072),
                         (5, 0.125, 32768), (6, 1.0, 100001), (7, 1.0, 65536),
                         (42, inputs.he_std_conv(576), 36864), (42, inputs.he_std_linear(1024), 50000)]:
        got = inputs.normal((n,), std, seed)
        want = ref.normal(n, 0.0, float(np.float32(std)), seed)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (seed, std, n)


def test_config4_weight_is_the_reference_first_conv2d(ref):
    # include/Module.hpp:226-232: the first Conv2D<float> draws He-normal weights from mt19937(42).
    W = inputs.config4()[1]
    assert np.array_equal(W.view(np.uint32), ref.conv2d_first_weight(64, 64, 3).view(np.uint32))


def test_uniform_inputs_match_libstdcxx_canonical(port):
    # uniform() restates generate_canonical<float> + uniform_real_distribution<float>;
    # the C generator (inputs_gen.c) does the same from its own MT19937, so both agree.
    import ctypes
    L = inputs._gen()
    L.mtin_uniform_f32.argtypes = [ctypes.c_uint32, ctypes.c_float, ctypes.c_float,
                                   ctypes.POINTER(ctypes.c_float), ctypes.c_size_t]
    for seed, n in [(0, 5), (1, 100003)]:
        out = np.empty(n, np.float32)
        L.mtin_uniform_f32(seed, -1.0, 1.0, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), n)
        assert np.array_equal(out, inputs.uniform((n,), -1.0, 1.0, seed))
