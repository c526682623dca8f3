"""Generates tests/golden/golden_v1.npz from the reference's OWN CPU code.

Run in a container that has the reference checkout (the oracle Makefile compiles the
reference headers into oracle/_ref/libref_cpu.so first):

    python tests/golden/make_golden.py

Every output below is computed by the reference's routines (matmul / matmul_cpu_strided /
bmm steps / Linear + MatmulBackward / conv2d / conv2d_backward_*), on small seeded inputs
and on the inputs of the reference's own tests. The fixtures pin the C restatement in
oracle/mt_oracle.c (bit-exact) and give the GPU tests reference outputs that do not
depend on any code of this repository.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from minitensor_b200 import inputs  # noqa: E402


def seq(shape, start, step):
    """test/spatial_test.cpp:10-16 fill_sequential: start + i * step in float."""
    n = int(np.prod(shape))
    i = np.arange(n, dtype=np.float32)
    return (np.float32(start) + i * np.float32(step)).astype(np.float32).reshape(shape)


def bench_fill(shape):
    """test/benchmark.cpp:48-54 make_gpu_tensor: ((i*131) % 997) / 997."""
    n = int(np.prod(shape))
    i = np.arange(n, dtype=np.int64)
    return (((i * 131) % 997).astype(np.float32) / np.float32(997.0)).reshape(shape)


def main():
    oracle.build()
    R = oracle.Ref()
    g = {}

    # tensor_test.cpp:258-283 / :285-317 known answer.
    A = np.arange(1, 7, dtype=np.float32).reshape(2, 3)
    B = np.arange(7, 13, dtype=np.float32).reshape(3, 2)
    g["mm_known_A"], g["mm_known_B"], g["mm_known_C"] = A, B, R.matmul(A, B)

    # Random contiguous matmuls, including ragged and degenerate shapes.
    for i, (M, K, N) in enumerate([(37, 53, 29), (64, 64, 64), (1, 256, 1), (130, 70, 260), (5, 1, 7)]):
        A = inputs.uniform((M, K), -1, 1, 100 + i)
        B = inputs.uniform((K, N), -1, 1, 200 + i)
        g[f"mm{i}_A"], g[f"mm{i}_B"], g[f"mm{i}_C"] = A, B, R.matmul(A, B)

    # benchmark.cpp:696-725 self-check shapes with the benchmark's deterministic fill.
    for i, (M, K, N) in enumerate([(32, 32, 32), (1, 256, 1)]):
        A = bench_fill((M, K))
        B = bench_fill((K, N))
        g[f"bench{i}_A"], g[f"bench{i}_B"], g[f"bench{i}_C"] = A, B, R.matmul(A, B)

    # Transposed views (MatmulBackward layouts): ta -> A = As.T, tb -> B = Bs.T.
    for i, (M, K, N, ta, tb) in enumerate([(48, 80, 40, 0, 1), (48, 80, 40, 1, 0), (33, 17, 65, 1, 1)]):
        As = inputs.uniform((K, M) if ta else (M, K), -1, 1, 300 + i)
        Bs = inputs.uniform((N, K) if tb else (K, N), -1, 1, 400 + i)
        g[f"mmt{i}_As"], g[f"mmt{i}_Bs"] = As, Bs
        g[f"mmt{i}_meta"] = np.array([M, K, N, ta, tb], np.int64)
        g[f"mmt{i}_C"] = R.matmul_t(As, Bs, M, K, N, ta, tb)

    # Row slice (a contiguous view with a non-zero offset).
    A = inputs.uniform((40, 24), -1, 1, 500)
    B = inputs.uniform((24, 36), -1, 1, 501)
    g["rows_A"], g["rows_B"], g["rows_meta"] = A, B, np.array([7, 29], np.int64)
    g["rows_C"] = R.matmul_rowslice(A, B, 7, 29)

    # bmm with a broadcast (expand) operand and with a full batch.
    A = inputs.normal((4, 16, 8), 0.125, 600)
    B0 = inputs.normal((1, 8, 24), 0.125, 601)
    g["bmmb_A"], g["bmmb_B0"], g["bmmb_C"] = A, B0, R.bmm(A, B0, True)
    B = inputs.normal((4, 8, 24), 0.125, 602)
    g["bmm_A"], g["bmm_B"], g["bmm_C"] = A, B, R.bmm(A, B, False)

    # Linear forward + backward (W is [in,out]).
    X = inputs.normal((16, 32), 1.0, 700)
    W = inputs.normal((32, 24), float(np.sqrt(2.0 / 32)), 701)
    b = inputs.normal((1, 24), 0.1, 702)
    dY = inputs.normal((16, 24), 1.0, 703)
    Y, dX, dW = R.linear(X, W, b, dY)
    g.update(lin_X=X, lin_W=W, lin_b=b, lin_dY=dY, lin_Y=Y, lin_dX=dX, lin_dW=dW)

    # spatial_test.cpp:155-185 conv known answer.
    x = seq((1, 1, 3, 3), 1.0, 1.0)
    w = np.ones((1, 1, 2, 2), np.float32)
    bias = np.zeros((1,), np.float32)
    g["convk_x"], g["convk_w"], g["convk_b"] = x, w, bias
    g["convk_y"] = R.conv2d(x, w, bias, 1, 0)

    # spatial_test.cpp:209-230 device-equivalence inputs (stride 2, pad 1).
    x = seq((4, 3, 32, 32), 0.1, 0.01)
    w = seq((16, 3, 3, 3), -0.5, 0.02)
    bias = np.full((16,), 0.1, np.float32)
    g["conveq_x"], g["conveq_w"], g["conveq_b"] = x, w, bias
    g["conveq_y"] = R.conv2d(x, w, bias, 2, 1)

    # Forward + all three backward products on padded / strided shapes.
    for i, (N, C, H, W_, Co, k, s, p) in enumerate([(2, 3, 5, 5, 4, 3, 1, 0), (2, 4, 9, 9, 6, 3, 1, 1),
                                                     (3, 5, 11, 10, 7, 3, 2, 1), (2, 8, 8, 8, 16, 1, 1, 0)]):
        x = inputs.normal((N, C, H, W_), 1.0, 800 + i)
        w = inputs.normal((Co, C, k, k), float(np.sqrt(2.0 / (C * k * k))), 810 + i)
        bias = inputs.normal((Co,), 0.1, 820 + i)
        y = R.conv2d(x, w, bias, s, p)
        dy = inputs.normal(y.shape, 1.0, 830 + i)
        dx, dw, db = R.conv2d_backward(dy, x, w, s, p)
        g[f"conv{i}_meta"] = np.array([s, p], np.int64)
        g.update({f"conv{i}_x": x, f"conv{i}_w": w, f"conv{i}_b": bias, f"conv{i}_y": y,
                  f"conv{i}_dy": dy, f"conv{i}_dx": dx, f"conv{i}_dw": dw, f"conv{i}_db": db})

    out = os.path.join(HERE, "golden_v1.npz")
    np.savez_compressed(out, **g)
    print(out, len(g), "arrays", os.path.getsize(out), "bytes")


if __name__ == "__main__":
    main()
