"""GPU parity tests for the GEMM family (matmul / strided views / bmm / Linear) through
the C ABI, against the CPU oracle (oracle/, pinned to the reference) and the golden
vectors made by the reference's own code."""
import os

import numpy as np
import pytest
import torch

from minitensor_b200 import inputs
from parity import absmm, check, dev, host

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden_v1.npz")
MODES = ["strict", "tf32", "tf32x3"]
THREADS = max(1, min(16, os.cpu_count() or 1))


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLDEN)


def run(eng, A, B, mode, C=None):
    if C is None:
        C = torch.empty((A.shape[0], B.shape[1]), dtype=torch.float32, device="cuda")
    eng.gemm(A, B, C, mode=mode)
    return C


# ------------------------------------------------------------------ golden vectors ---

@pytest.mark.parametrize("mode", MODES)
def test_golden_matmul(eng, gold, mode):
    keys = [k[:-2] for k in gold.files if k.endswith("_C") and (k.startswith("mm") or k.startswith("bench"))
            and not k.startswith("mmt")]
    for key in keys:
        A, B, Cr = gold[key + "_A"], gold[key + "_B"], gold[key + "_C"]
        C = host(run(eng, dev(A), dev(B), mode))
        check(mode, C, Cr, absmm(A, B), A.shape[1], key)
    # The reference's own GPU known answer (test/tensor_test.cpp:285-317) via matmul_gpu.
    A, B = dev(gold["mm_known_A"]), dev(gold["mm_known_B"])
    C = torch.empty(2, 2, device="cuda")
    eng.matmul_gpu(A, B, C)
    assert host(C).ravel().tolist() == [58.0, 64.0, 139.0, 154.0]


@pytest.mark.parametrize("mode", MODES)
def test_golden_views(eng, gold, mode):
    for i in range(3):
        M, K, N, ta, tb = gold[f"mmt{i}_meta"].tolist()
        As, Bs = dev(gold[f"mmt{i}_As"]), dev(gold[f"mmt{i}_Bs"])
        A = As.t() if ta else As
        B = Bs.t() if tb else Bs
        An, Bn = (gold[f"mmt{i}_As"].T if ta else gold[f"mmt{i}_As"]), (gold[f"mmt{i}_Bs"].T if tb else gold[f"mmt{i}_Bs"])
        C = host(run(eng, A, B, mode))
        check(mode, C, gold[f"mmt{i}_C"], absmm(An, Bn), K, f"mmt{i}")
    r0, r1 = gold["rows_meta"].tolist()
    A = dev(gold["rows_A"])[r0:r1]
    C = torch.empty((r1 - r0, gold["rows_B"].shape[1]), device="cuda")
    eng.matmul_gpu(A, dev(gold["rows_B"]), C)  # contiguous view with an offset
    check("tf32x3" if mode != "strict" else mode, host(C), gold["rows_C"],
          absmm(gold["rows_A"][r0:r1], gold["rows_B"]), A.shape[1], "row slice")


@pytest.mark.parametrize("mode", MODES)
def test_golden_bmm_and_linear(eng, gold, mode):
    A, B0 = gold["bmmb_A"], gold["bmmb_B0"]
    Bx = dev(B0).expand(A.shape[0], -1, -1)
    assert Bx.stride(0) == 0
    C = torch.empty((A.shape[0], A.shape[1], B0.shape[2]), device="cuda")
    eng.gemm(dev(A), Bx, C, mode=mode)
    check(mode, host(C), gold["bmmb_C"], absmm(A, B0), A.shape[2], "bmm broadcast")
    eng.gemm(dev(gold["bmm_A"]), dev(gold["bmm_B"]), C, mode=mode)
    check(mode, host(C), gold["bmm_C"], absmm(gold["bmm_A"], gold["bmm_B"]), A.shape[2], "bmm")

    X, W, b, dY = (gold[k] for k in ("lin_X", "lin_W", "lin_b", "lin_dY"))
    Y = eng.linear_forward(dev(X), dev(W), dev(b), mode=mode)
    check(mode, host(Y), gold["lin_Y"], absmm(X, W) + np.abs(b), X.shape[1], "linear fwd")
    dX, dW, db = eng.linear_backward(dev(X), dev(W), dev(dY), mode=mode)
    check(mode, host(dX), gold["lin_dX"], absmm(dY, W.T), W.shape[1], "linear dX")
    check(mode, host(dW), gold["lin_dW"], absmm(X.T, dY), X.shape[0], "linear dW")
    assert np.allclose(host(db).ravel(), dY.sum(0, dtype=np.float64), rtol=1e-5, atol=1e-4)


# ------------------------------------------------------------------ configurations ---

@pytest.mark.parametrize("mode", MODES)
def test_config1_512(eng, port, mode):
    A, B = inputs.config1()
    C = host(run(eng, dev(A), dev(B), mode))
    if mode != "strict":
        assert eng.last_path().startswith("umma_" + mode), eng.last_path()
    check(mode, C, port.matmul(A, B), absmm(A, B), 512, "config1")


@pytest.mark.parametrize("mode", MODES)
def test_config2_linear(eng, port, mode):
    X, W, b, dY = inputs.config2()
    Xd, Wd, bd, dYd = dev(X), dev(W), dev(b), dev(dY)
    Y = host(eng.linear_forward(Xd, Wd, bd, mode=mode))
    Yr = port.matmul_rows(X, W, 0, X.shape[0], THREADS) + b
    check(mode, Y, Yr, absmm(X, W), 1024, "config2 fwd")
    dX, dW, _ = eng.linear_backward(Xd, Wd, dYd, mode=mode)
    # dX = dY.W^T and dW = X^T.dY: same per-element k order as matmul_cpu_strided.
    dXr = port.matmul_rows(dY, np.ascontiguousarray(W.T), 0, 256, THREADS)
    check(mode, host(dX), dXr, absmm(dY, W.T), 4096, "config2 dX (NT)")
    XT = np.ascontiguousarray(X.T)
    dWr = port.matmul_rows(XT, dY, 0, 1024, THREADS)
    check(mode, host(dW), dWr, absmm(XT, dY), 256, "config2 dW (TN)")
    # db: the sum of dY over the batch (fp32 adds in a fixed order, every mode).
    db = host(eng.linear_backward(Xd, Wd, dYd, mode=mode)[2]).ravel()
    ref = dY.astype(np.float64).sum(0)
    assert np.max(np.abs(db - ref) / np.abs(dY).astype(np.float64).sum(0)) < 1e-6


@pytest.mark.parametrize("shape", [(256, 4096), (1, 7), (77, 33), (1000, 65), (0, 5)])
def test_sum_rows(eng, shape):
    """out[n] = sum over rows; X read through a transposed view, out a strided [1, N] row."""
    M, N = shape
    base = inputs.uniform((N, M), -1, 1, 61)          # X = base^T: column stride 1 in memory rows
    X = dev(base).t()
    out_buf = torch.full((3, N), 5.0, device="cuda")
    out = out_buf[1:2]                                 # [1, N] window of a larger buffer
    eng.sum_rows(X, out)
    first = host(out).ravel()
    eng.sum_rows(X, out)
    assert np.array_equal(host(out).ravel(), first)   # deterministic
    ref = base.T.astype(np.float64).sum(0)
    bound = np.abs(base.T).astype(np.float64).sum(0) + 1e-30
    assert np.max(np.abs(first - ref) / bound) < 1e-6
    assert np.all(host(out_buf)[[0, 2]] == 5.0)        # neighbours untouched


@pytest.mark.parametrize("mode", ["tf32", "tf32x3"])
def test_split_k_ragged_with_bias(eng, port, mode):
    """Few output tiles and a long K: split-K partials, ordered sum, fused bias epilogue."""
    M, N, K = 200, 136, 5000
    A = inputs.uniform((M, K), -1, 1, 63)
    B = inputs.uniform((K, N), -1, 1, 64)
    bn = inputs.uniform((N,), -1, 1, 65)
    C = torch.empty(M, N, device="cuda")
    eng.gemm(dev(A), dev(B), C, bias=dev(bn), epi=eng.EPI_BIAS_COL, mode=mode)
    assert "splitk=" in eng.last_path(), eng.last_path()
    check(mode, host(C), port.matmul(A, B) + bn, absmm(A, B) + np.abs(bn), K, "split-K")


@pytest.mark.parametrize("mode", MODES)
def test_config3_bmm_broadcast(eng, port, mode):
    A, B0 = inputs.config3()
    Bx = dev(B0).expand(64, 64, 512)
    C = torch.empty(64, 512, 512, device="cuda")
    eng.bmm_gpu(dev(A), Bx, C) if mode == "tf32x3" else eng.gemm(dev(A), Bx, C, mode=mode)
    Cr = port.bmm(A, np.broadcast_to(B0, (64, 64, 512)))
    check(mode, host(C), Cr, absmm(A, B0), 64, "config3")


@pytest.mark.parametrize("mode", ["tf32", "tf32x3", "strict"])
def test_config5_8192_sampled_rows(eng, port, mode):
    A, B = inputs.config5()
    Ad, Bd = dev(A), dev(B)
    C = torch.empty(8192, 8192, device="cuda")
    eng.gemm(Ad, Bd, C, mode=mode)
    rows = [0, 1, 127, 128, 4095, 8191]
    rng = np.random.RandomState(5)
    rows += sorted(rng.choice(8192, 10, replace=False).tolist())
    Ch = host(C)
    for r in rows:
        Cr = port.matmul_rows(A, B, r, r + 1, 1)
        check(mode, Ch[r:r + 1], Cr, absmm(A[r:r + 1], B), 8192, f"config5 row {r}")
    # Size-independent property: the column sums of C equal (1^T A) B.
    colsum = np.abs(Ch.astype(np.float64).sum(0) - A.astype(np.float64).sum(0) @ B.astype(np.float64))
    bound = np.abs(A).astype(np.float64).sum(0) @ np.abs(B).astype(np.float64)
    assert np.max(colsum / bound) < 1e-3


# ------------------------------------------------------------------ layouts & edges ---

def padded(shape, seed, pad=4):
    """A float32 matrix stored with a leading dimension rounded up to `pad` elements:
    returns (numpy view, the same view on the GPU)."""
    r, c = shape
    ld = (c + pad - 1) // pad * pad
    base = inputs.uniform((r, ld), -1, 1, seed)
    return base[:, :c], dev(base)[:, :c]


@pytest.mark.parametrize("mode", ["tf32", "tf32x3", "strict"])
@pytest.mark.parametrize("layout", ["NN", "NT", "TN", "TT"])
def test_layouts_ragged(eng, port, mode, layout):
    shapes = [(257, 383, 511), (129, 65, 1), (1, 7, 300), (63, 127, 129), (300, 200, 33), (128, 256, 96)]
    for i, (M, N, K) in enumerate(shapes):
        a_np, a_t = padded((K, M) if layout[0] == "T" else (M, K), 10 * i + 1)
        b_np, b_t = padded((N, K) if layout[1] == "T" else (K, N), 10 * i + 2)
        A = a_t.t() if layout[0] == "T" else a_t
        B = b_t.t() if layout[1] == "T" else b_t
        An = a_np.T if layout[0] == "T" else a_np
        Bn = b_np.T if layout[1] == "T" else b_np
        C = host(run(eng, A, B, mode))
        if mode != "strict":
            assert eng.last_path().startswith("umma_" + mode), (layout, M, N, K, eng.last_path())
        check(mode, C, port.matmul_strided(An, Bn), absmm(An, Bn), K, f"{layout} {M}x{N}x{K}")


@pytest.mark.parametrize("mode", ["tf32", "tf32x3"])
def test_unaligned_views_use_simt_and_stay_correct(eng, port, mode):
    # Row stride 383 floats is not 16-byte aligned: the tensor-core kernel cannot take it.
    A = inputs.uniform((200, 383), -1, 1, 31)
    B = inputs.uniform((383, 150), -1, 1, 32)
    C = host(run(eng, dev(A), dev(B), mode))
    assert eng.last_path().startswith("simt"), eng.last_path()
    check(mode, C, port.matmul(A, B), absmm(A, B), 383, "unaligned")


@pytest.mark.parametrize("mode", MODES)
def test_epilogues_and_k0(eng, port, mode):
    M, N, K = 200, 264, 96
    A = inputs.uniform((M, K), -1, 1, 41)
    B = inputs.uniform((K, N), -1, 1, 42)
    bn = inputs.uniform((N,), -1, 1, 43)
    bm = inputs.uniform((M,), -1, 1, 44)
    base = port.matmul(A, B)
    D = absmm(A, B)
    C = torch.empty(M, N, device="cuda")
    eng.gemm(dev(A), dev(B), C, bias=dev(bn), epi=eng.EPI_BIAS_COL | eng.EPI_RELU, mode=mode)
    check(mode, host(C), np.maximum(base + bn, 0), D + np.abs(bn), K, "bias col + relu")
    eng.gemm(dev(A), dev(B), C, bias=dev(bm), epi=eng.EPI_BIAS_ROW, mode=mode)
    check(mode, host(C), base + bm[:, None], D + np.abs(bm)[:, None], K, "bias row")
    # K == 0: the empty sum; C = epi(0).
    A0 = torch.empty(M, 0, device="cuda")
    B0 = torch.empty(0, N, device="cuda")
    eng.gemm(A0, B0, C, bias=dev(bn), epi=eng.EPI_BIAS_COL, mode=mode)
    assert np.array_equal(host(C), np.broadcast_to(bn, (M, N)))


@pytest.mark.parametrize("mode", ["tf32", "tf32x3", "strict"])
def test_output_guard_bands(eng, port, mode):
    # C is a window of a larger buffer; everything outside the window must be untouched.
    M, N, K = 300, 260, 128
    A = inputs.uniform((M, K), -1, 1, 51)
    B = inputs.uniform((K, N), -1, 1, 52)
    big = torch.full((M + 16, N + 20), 12345.0, device="cuda")
    C = big[8:8 + M, 4:4 + N]
    eng.gemm(dev(A), dev(B), C, mode=mode)
    h = host(big)
    mask = np.ones_like(h, dtype=bool)
    mask[8:8 + M, 4:4 + N] = False
    assert np.all(h[mask] == 12345.0)
    check(mode, h[8:8 + M, 4:4 + N], port.matmul(A, B), absmm(A, B), K, "guarded")


def test_column_major_output(eng, port):
    M, N, K = 160, 96, 64
    A = inputs.uniform((M, K), -1, 1, 61)
    B = inputs.uniform((K, N), -1, 1, 62)
    Ct = torch.empty(N, M, device="cuda")
    eng.gemm(dev(A), dev(B), Ct.t(), mode="tf32x3")
    check("tf32x3", host(Ct).T, port.matmul(A, B), absmm(A, B), K, "column-major C")


def test_device_status_clean(eng):
    assert eng.device_status(reset=True) == 0


# ------------------------------------------------------- CTA-pair (256-row) kernel ---

@pytest.mark.parametrize("mode", ["tf32", "tf32x3"])
@pytest.mark.parametrize("layout", ["NN", "NT", "TN", "TT"])
def test_pair_kernel_ragged_layouts(eng, port, mode, layout):
    """Outputs with >= 74 tiles of 256 x 256 run on CTA pairs (M = 256 per MMA, B split
    across the two SMs). Ragged M, N and K so that the odd CTA's rows, the second B half
    and the k tail all meet the zero-filled edge; checked on sampled rows (both halves
    of a pair tile) and sampled columns (both B halves) against the oracle."""
    M, N, K = 2381, 2355, 301
    a_np, a_t = padded((K, M) if layout[0] == "T" else (M, K), 91)
    b_np, b_t = padded((N, K) if layout[1] == "T" else (K, N), 92)
    A = a_t.t() if layout[0] == "T" else a_t
    B = b_t.t() if layout[1] == "T" else b_t
    An = np.ascontiguousarray(a_np.T if layout[0] == "T" else a_np)
    Bn = np.ascontiguousarray(b_np.T if layout[1] == "T" else b_np)
    bn = inputs.uniform((N,), -1, 1, 93)
    C = torch.empty(M, N, device="cuda")
    eng.gemm(A, B, C, bias=dev(bn), epi=eng.EPI_BIAS_COL | eng.EPI_RELU, mode=mode)
    assert eng.last_path().startswith("umma_pair_" + mode), eng.last_path()
    Ch = host(C)
    rows = [0, 1, 127, 128, 129, 255, 256, 383, 384, 2303, 2304, M - 2, M - 1]
    cols = [0, 1, 127, 128, 129, 255, 256, 1151, 1152, 2303, 2304, N - 2, N - 1]
    R = port.matmul_strided(An[rows], Bn)
    check(mode, Ch[rows], np.maximum(R + bn, 0), absmm(An[rows], Bn) + np.abs(bn), K, f"pair {layout} rows")
    Cc = port.matmul_strided(An, np.ascontiguousarray(Bn[:, cols]))
    check(mode, Ch[:, cols], np.maximum(Cc + bn[cols], 0), absmm(An, Bn[:, cols]) + np.abs(bn[cols]), K,
          f"pair {layout} cols")


@pytest.mark.parametrize("mode", ["tf32", "tf32x3"])
def test_pair_kernel_batched_bias_row(eng, port, mode):
    """Batched pair tiles (tile index walks batch, m, n) with a per-row bias."""
    Bt, M, N, K = 3, 1290, 1100, 200
    A = inputs.uniform((Bt, M, K), -1, 1, 95)
    B = inputs.uniform((Bt, K, N), -1, 1, 96)
    bm = inputs.uniform((M,), -1, 1, 97)
    C = torch.empty(Bt, M, N, device="cuda")
    eng.gemm(dev(A), dev(B), C, bias=dev(bm), epi=eng.EPI_BIAS_ROW, mode=mode)
    assert eng.last_path().startswith("umma_pair_" + mode), eng.last_path()
    Ch = host(C)
    rows = [0, 127, 128, 255, 256, 1023, 1024, 1279, 1280, M - 1]
    for b in range(Bt):
        R = port.matmul_strided(A[b][rows], B[b])
        check(mode, Ch[b][rows], R + bm[rows][:, None], absmm(A[b][rows], B[b]) + np.abs(bm[rows])[:, None], K,
              f"pair batch {b}")


def _bmm_grads_ref(port, A, B, dC):
    """Per-batch oracle gradients of C = bmm(A, B) (A, B may be numpy broadcast views)."""
    dA = np.stack([port.matmul_strided(dC[i], B[i].T) for i in range(A.shape[0])])
    dB = np.stack([port.matmul_strided(A[i].T, dC[i]) for i in range(A.shape[0])])
    return dA, dB


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("case", ["batched", "b_broadcast", "a_broadcast", "config3"])
def test_bmm_backward(eng, port, mode, case):
    """Batched NT/TN gradients through transposed 3-D views; a broadcast operand's gradient
    is the batch sum (one folded GEMM for B, per-batch GEMMs + ordered row sums for A)."""
    if case == "config3":
        A, B0 = inputs.config3()
        bt, M, K = A.shape
        N = B0.shape[2]
    else:
        bt, M, K, N = 6, 200, 48, 136
        A = inputs.uniform((1 if case == "a_broadcast" else bt, M, K), -1, 1, 120)
        B0 = inputs.uniform((1 if case in ("b_broadcast",) else bt, K, N), -1, 1, 121)
    dC = inputs.normal((bt, M, N), 1.0, 122)
    Ab = np.broadcast_to(A, (bt, M, K))
    Bb = np.broadcast_to(B0, (bt, K, N))
    Ad = dev(A).expand(bt, M, K) if A.shape[0] == 1 else dev(A)
    Bd = dev(B0).expand(bt, K, N) if B0.shape[0] == 1 else dev(B0)
    dA, dB = eng.bmm_backward(Ad, Bd, dev(dC), mode=mode)
    dA_ref, dB_ref = _bmm_grads_ref(port, Ab, Bb, dC)
    DA = absmm(dC, np.swapaxes(np.abs(Bb), 1, 2))
    DB = absmm(np.swapaxes(np.abs(Ab), 1, 2), dC)
    if A.shape[0] == 1:
        assert tuple(dA.shape) == (1, M, K)
        check(mode, host(dA)[0], dA_ref.astype(np.float64).sum(0), DA.sum(0), bt * N, f"{case} dA (summed)")
    else:
        check(mode, host(dA), dA_ref, DA, N, f"{case} dA")
    if B0.shape[0] == 1:
        assert tuple(dB.shape) == (1, K, N)
        check(mode, host(dB)[0], dB_ref.astype(np.float64).sum(0), DB.sum(0), bt * M, f"{case} dB (summed)")
    else:
        check(mode, host(dB), dB_ref, DB, M, f"{case} dB")


@pytest.mark.parametrize("mode", ["tf32", "tf32x3"])
def test_one_cta_wide_tiles_batched_short_rows(eng, port, mode):
    """Batched outputs with M <= 128 and enough 128x256 tiles to fill the GPU: too short for
    CTA pairs, too many tiles for the small-output path, so the one-CTA 256-wide kernel."""
    Bt, M, N, K = 40, 100, 1000, 72
    A = inputs.uniform((Bt, M, K), -1, 1, 140)
    B = inputs.uniform((Bt, K, N), -1, 1, 141)
    C = torch.empty(Bt, M, N, device="cuda")
    eng.gemm(dev(A), dev(B), C, mode=mode)
    path = eng.last_path()
    assert path.startswith(f"umma_{mode} bn=256"), path
    check(mode, host(C), port.bmm(A, B), absmm(A, B), K, "one-CTA bn=256 batched")


@pytest.mark.parametrize("mode", ["tf32x3", "tf32"])
def test_pair_kernel_streamk_remainder(eng, port, mode):
    """256 tiles of 256 x 256 over 74 clusters (3.46 rounds): in 3xTF32 the last 34 tiles
    are cut into equal k-ranges across all clusters (stream-K) and summed by the last of
    each tile's contributors; in TF32 they run whole. Full rows of the stream-K tiles
    (rows 6144..8191 hold them) and of whole tiles are checked."""
    M, K, N = 8192, 2048, 2048
    A = inputs.uniform((M, K), -1, 1, 301)
    B = inputs.uniform((K, N), -1, 1, 302)
    C = torch.full((M, N), float("nan"), device="cuda")
    eng.gemm(dev(A), dev(B), C, mode=mode)
    path = eng.last_path()
    assert path.startswith("umma_pair_" + mode), path
    assert ("streamk=34" in path) == (mode == "tf32x3"), path
    rows = [0, 255, 256, 4095, 6144, 6400, 6655, 7000, 7936, 8191]
    c = host(C)[rows]
    check(mode, c, port.matmul_strided(A[rows], B), absmm(A[rows], B), K, f"stream-K ({path})")
    # Run again: the arrival counters start from zero on every call and the result is
    # bit-identical (the pieces of a tile are summed in k order whoever arrives last).
    C2 = torch.full((M, N), float("nan"), device="cuda")
    eng.gemm(dev(A), dev(B), C2, mode=mode)
    assert torch.equal(C, C2)
    assert eng.device_status(reset=True) == 0


# ------------------------------------------------------------ epilogue store forms ---

def test_tma_store_epilogue_matches_register_stores(eng, port, tmp_path):
    """The epilogue writes C through TMA tensor stores (whole lines) unless
    MT_TMA_EPILOGUE=0 selects stores straight from registers. Both write the same
    accumulator values, so the outputs must agree bit for bit: ragged pair and one-CTA
    tiles, batched tiles with a row bias, config 3's broadcast bmm, and a C window whose
    surroundings must keep their sentinel. One process per setting (read once)."""
    import subprocess
    import sys
    script = os.path.join(os.path.dirname(__file__), "tma_store_cases.py")
    res = {}
    for flag in ("1", "0"):
        out = str(tmp_path / f"tma{flag}.npz")
        env = dict(os.environ, MT_TMA_EPILOGUE=flag)
        r = subprocess.run([sys.executable, script, out], env=env, capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
        res[flag] = np.load(out)
    tma, reg = res["1"], res["0"]
    names = [k for k in tma.files if not k.startswith("path_")]
    assert len(names) == 10
    for k in names:
        assert "tma_store" in str(tma["path_" + k]), (k, str(tma["path_" + k]))
        assert "tma_store" not in str(reg["path_" + k]), (k, str(reg["path_" + k]))
        assert tma[k].shape == reg[k].shape and np.array_equal(tma[k], reg[k]), k
    for mode in ("tf32", "tf32x3"):
        big = tma[f"window_{mode}"]
        M, N = 1030, 1000
        mask = np.ones_like(big, dtype=bool)
        mask[8:8 + M, 4:4 + N] = False
        assert np.all(big[mask] == 12345.0), mode
        A = inputs.uniform((M, 64), -1, 1, 199)
        B = inputs.uniform((64, N), -1, 1, 200)
        check(mode, big[8:8 + M, 4:4 + N], port.matmul(A, B), absmm(A, B), 64, f"window {mode}")


@pytest.mark.parametrize("layout", ["NN", "NT", "TN", "gen"])
def test_strict_small_grid_tiles_match_large_tiles(eng, port, layout):
    """Strict fp32 on fewer 128x128 tiles than SMs runs 64x64 tiles (4x the CTAs). Each
    output is the same FFMA chain in k order either way, so a small product equals, bit for
    bit, the top-left block of a large one over the same rows, columns and K; ragged
    edges, every operand layout, an unaligned view, and a bias + ReLU epilogue."""
    Mb, Nb, K = 4100, 1000, 301
    a = inputs.uniform((Mb, K + 1), -1, 1, 1701)
    b = inputs.uniform((K + 1, Nb), -1, 1, 1702)
    bias = inputs.uniform((Nb,), -1, 1, 1703)
    ad, bd = dev(a), dev(b)
    if layout == "gen":
        A, B = ad[:, 1:], bd[1:, :]                     # start 4 bytes in: no vector loads for A
    elif layout == "NT":
        bt = np.zeros((Nb, K + 3), np.float32)          # rows of 304: the K-contiguous vector path
        bt[:, :K] = b[:K].T
        A, B = ad[:, :K], dev(bt)[:, :K].t()
    elif layout == "TN":
        A, B = dev(np.ascontiguousarray(a[:, :K].T)).t(), bd[:K]
    else:
        A, B = ad[:, :K], bd[:K]
    Cb = torch.empty(Mb, Nb, device="cuda")
    eng.gemm(A, B, Cb, bias=dev(bias), epi=eng.EPI_BIAS_COL | eng.EPI_RELU, mode="strict")
    assert eng.last_path().startswith("simt_fp32") and "tile=64" not in eng.last_path(), eng.last_path()
    Ms, Ns = 300, 200
    Cs = torch.empty(Ms, Ns, device="cuda")
    eng.gemm(A[:Ms], B[:, :Ns], Cs, bias=dev(bias[:Ns]), epi=eng.EPI_BIAS_COL | eng.EPI_RELU, mode="strict")
    assert "tile=64" in eng.last_path(), eng.last_path()
    assert torch.equal(Cs, Cb[:Ms, :Ns])
    An, Bn = host(A[:Ms]), host(B[:, :Ns])
    ref = np.maximum(port.matmul_strided(np.ascontiguousarray(An), np.ascontiguousarray(Bn)) + bias[:Ns], 0)
    check("strict", host(Cs), ref, absmm(An, Bn) + np.abs(bias[:Ns]), K, f"small grid {layout}")
