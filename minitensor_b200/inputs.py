"""Seeded synthetic inputs for the five workload configurations.

Generator: MT19937 seeded like ``std::mt19937(seed)`` (numpy's legacy RandomState uses the
same init_genrand seeding). Uniform values restate libstdc++'s
``uniform_real_distribution<float>`` over ``generate_canonical<float>``: one 32-bit draw x,
u = float(x) / 2^32 (clamped below 1), value = u * (b - a) + a, all in float32 -- so they
are the values a C++ harness with the same seed would see. Normal values are those of
libstdc++'s ``normal_distribution<float>`` (the polar method, with the C library's logf),
drawn by the small C generator inputs_gen.c (libmtinputs.so), because the reference fills
its weights that way (include/Module.hpp:99-105 Linear, :226-232 Conv2D). No dataset is
involved: all inputs are synthetic, with the shapes and distributions of the
configurations below.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_LIB = None


def _gen():
    global _LIB
    if _LIB is None:
        from minitensor_b200 import build
        path = build.INPUTS_LIB
        if not os.path.exists(path):
            build.build_inputs()
        L = ctypes.CDLL(path)
        fp = ctypes.POINTER(ctypes.c_float)
        L.mtin_normal_f32.argtypes = [ctypes.c_uint32, ctypes.c_float, ctypes.c_float, fp, ctypes.c_size_t]
        L.mtin_normal_f32.restype = None
        _LIB = L
    return _LIB


def uniform(shape, lo: float, hi: float, seed: int) -> np.ndarray:
    n = int(np.prod(shape))
    rs = np.random.RandomState(seed)
    x = rs.randint(0, 2**32, size=n, dtype=np.uint64).astype(np.uint32)
    u = x.astype(np.float32) / np.float32(4294967296.0)
    u = np.where(u >= np.float32(1.0), np.nextafter(np.float32(1.0), np.float32(0.0)), u).astype(np.float32)
    v = u * (np.float32(hi) - np.float32(lo)) + np.float32(lo)
    return v.astype(np.float32).reshape(shape)


def normal(shape, std, seed: int, mean=0.0) -> np.ndarray:
    """normal_distribution<float>(mean, std) on mt19937(seed), row-major. `std` is rounded to
    float32 first, as the distribution's float parameter is."""
    out = np.empty(int(np.prod(shape)), np.float32)
    _gen().mtin_normal_f32(seed, float(np.float32(mean)), float(np.float32(std)),
                           out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), out.size)
    return out.reshape(shape)


def he_std_conv(fan_in: int) -> np.float32:
    """Conv2D's std: sqrt(T(2) / T(fan_in)) in float (include/Module.hpp:225-226)."""
    return np.sqrt(np.float32(2.0) / np.float32(fan_in))


def he_std_linear(in_features: int) -> np.float32:
    """Linear's std: std::sqrt(2.0 / in) in double, then the float parameter (Module.hpp:101)."""
    return np.float32(np.sqrt(2.0 / in_features))


# Configurations (BASELINE.json "configs", in order).
def config1():
    """C[512,512] = A[512,512] . B[512,512]; A, B ~ U[-1,1], seed 0 (A then B)."""
    ab = uniform((2, 512, 512), -1.0, 1.0, 0)
    return ab[0].copy(), ab[1].copy()


def config2():
    """Linear 1024 -> 4096, batch 256. X ~ N(0,1) seed 2; W [in,out] He-normal seed 42;
    bias 0; dY ~ N(0,1) seed 3."""
    X = normal((256, 1024), 1.0, 2)
    W = normal((1024, 4096), he_std_linear(1024), 42)
    b = np.zeros((1, 4096), np.float32)
    dY = normal((256, 4096), 1.0, 3)
    return X, W, b, dY


def config3():
    """A [64,512,64] ~ N(0,0.125) seed 4; B0 [1,64,512] ~ N(0,0.125) seed 5, expanded."""
    A = normal((64, 512, 64), 0.125, 4)
    B0 = normal((1, 64, 512), 0.125, 5)
    return A, B0


def config4():
    """x [32,64,56,56] ~ N(0,1) seed 6; W [64,64,3,3] He-normal seed 42 (the weights of the
    reference's first Conv2D<float>(64, 64, 3)); b 0; dY [32,64,56,56] ~ N(0,1) seed 7;
    stride 1, pad 1."""
    x = normal((32, 64, 56, 56), 1.0, 6)
    W = normal((64, 64, 3, 3), he_std_conv(576), 42)
    b = np.zeros((64,), np.float32)
    dY = normal((32, 64, 56, 56), 1.0, 7)
    return x, W, b, dY


def config5(n: int = 8192):
    """A, B [8192,8192] ~ U[-1,1], seed 1 (A then B)."""
    ab = uniform((2, n, n), -1.0, 1.0, 1)
    return ab[0], ab[1]
