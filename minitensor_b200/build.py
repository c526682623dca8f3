"""Builds libmtgemm.so in-tree for sm_100a (nvcc cross-compiles; no GPU needed).

    python -m minitensor_b200.build            # the engine library
    python -m minitensor_b200.build --verbose  # also prints ptxas register/smem usage
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libmtgemm.so")
# The reference checkout: $MT_REFERENCE_ROOT, else a "reference" directory beside the repo.
REF_ROOT = os.environ.get("MT_REFERENCE_ROOT",
                          os.path.join(os.path.dirname(ROOT), "reference"))

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[str]:
    return [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC)) if f.endswith(".cu")]


def deps() -> list[str]:
    out = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    out.append(os.path.join(INCLUDE, "mtgemm.h"))
    return out


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(d) <= t for d in deps())


INPUTS_SRC = os.path.join(PKG, "inputs_gen.c")
INPUTS_LIB = os.path.join(PKG, "libmtinputs.so")


def build_inputs(force: bool = False) -> str:
    """libmtinputs.so: the seeded synthetic-input generator (host C, no FMA contraction)."""
    if not force and os.path.exists(INPUTS_LIB) and os.path.getmtime(INPUTS_LIB) >= os.path.getmtime(INPUTS_SRC):
        return INPUTS_LIB
    subprocess.check_call(["gcc", "-O2", "-ffp-contract=off", "-fPIC", "-shared", "-o", INPUTS_LIB + ".tmp",
                           INPUTS_SRC, "-lm"])
    os.replace(INPUTS_LIB + ".tmp", INPUTS_LIB)
    return INPUTS_LIB


def build(verbose: bool = False, force: bool = False) -> str:
    build_inputs(force)
    if not force and up_to_date():
        return LIB
    cmd = [nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "--expt-relaxed-constexpr",
           "-Xcompiler", "-fPIC,-fvisibility=hidden", "-shared",
           "-I", INCLUDE, "-I", CSRC, "-o", LIB + ".tmp", *sources()]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.check_call(cmd)
    os.replace(LIB + ".tmp", LIB)
    return LIB


OVERLAY = os.path.join(PKG, "overlay")
DROPIN_OUT = os.path.join(OVERLAY, "_build")
DROPIN_BIN = os.path.join(DROPIN_OUT, "dropin_test")
# Symbols defined by gpu_ops_b200.cpp (the reference declares them at
# include/TensorOps.hpp:703-712); the reference object's own definitions are renamed.
OVERRIDDEN = ("matmul_gpu", "matmul_gpu_strided", "matmul_gpu_v2", "matmul_gpu_bk16", "conv2d_gpu",
              "conv2d_gpu_strided", "conv2d_backward_input_gpu", "conv2d_backward_weight_gpu",
              "conv2d_backward_bias_gpu")


def _run(cmd):
    subprocess.check_call(cmd)


def build_dropin(ref_root: str = REF_ROOT) -> str | None:
    """Builds overlay/_build/dropin_test: the reference's own dispatchers, autograd and
    modules (headers unmodified; src/gpu_ops.cpp compiled from where it lies) with the
    GEMM/conv entry points served by gpu_ops_b200.cpp + libmtgemm.so. Needs the reference
    checkout; returns None without it (the built binary travels with the other outputs)."""
    src = os.path.join(ref_root, "src", "gpu_ops.cpp")
    if not os.path.exists(src):
        return None
    build()
    os.makedirs(DROPIN_OUT, exist_ok=True)
    ref_inc = os.path.join(ref_root, "include")
    cuda_inc = os.path.join(os.path.dirname(os.path.dirname(nvcc())), "include")
    ref_obj = os.path.join(DROPIN_OUT, "ref_gpu_ops.o")
    if not os.path.exists(ref_obj) or os.path.getmtime(ref_obj) < os.path.getmtime(src):
        _run([nvcc(), "-x", "cu", "-std=c++20", "-DUSE_CUDA", *ARCH, "-O3", "-w", "-Xcompiler", "-fPIC",
              "-I", ref_inc, "-c", src, "-o", ref_obj])
    cxx = ["g++", "-std=c++20", "-O2", "-fPIC", "-DUSE_CUDA", "-I", ref_inc, "-I", INCLUDE, "-I", cuda_inc]
    ov_obj = os.path.join(DROPIN_OUT, "gpu_ops_b200.o")
    test_obj = os.path.join(DROPIN_OUT, "dropin_test.o")
    _run([*cxx, "-c", os.path.join(OVERLAY, "gpu_ops_b200.cpp"), "-o", ov_obj])
    _run([*cxx, "-c", os.path.join(OVERLAY, "dropin_test.cpp"), "-o", test_obj])
    # Rename the reference's definitions of the overridden entry points so that each
    # symbol has exactly one definition (the overlay's) in the link.
    defined = subprocess.check_output(["nm", "--defined-only", ov_obj], text=True).split("\n")
    syms = [ln.split()[-1] for ln in defined if ln.strip() and any(f"{len(n)}{n}I" in ln for n in OVERRIDDEN)]
    split_obj = os.path.join(DROPIN_OUT, "ref_gpu_ops_split.o")
    _run(["objcopy", *[f"--redefine-sym={s}={s}__reference_replaced" for s in syms], ref_obj, split_obj])
    _run([nvcc(), *ARCH, "-o", DROPIN_BIN, test_obj, ov_obj, split_obj, "-L", PKG, "-lmtgemm",
          "-Xlinker", "-rpath", "-Xlinker", "$ORIGIN/../.."])
    return DROPIN_BIN


REFGPU_SRC = os.path.join(ROOT, "baseline", "ref_gpu.cpp")
REFGPU_LIB = os.path.join(ROOT, "baseline", "_ref", "libref_gpu.so")


def build_refgpu(ref_root: str = REF_ROOT) -> str | None:
    """baseline/_ref/libref_gpu.so: the reference's own GPU kernels (src/gpu_ops.cpp compiled
    unmodified for sm_100a, its headers unmodified) behind the timing shim
    baseline/ref_gpu.cpp -- the same-hardware baseline bench.py reports. Needs the
    reference checkout; returns None without it (the built library travels)."""
    src = os.path.join(ref_root, "src", "gpu_ops.cpp")
    if not os.path.exists(src):
        return None
    os.makedirs(DROPIN_OUT, exist_ok=True)
    os.makedirs(os.path.dirname(REFGPU_LIB), exist_ok=True)
    ref_inc = os.path.join(ref_root, "include")
    cuda_inc = os.path.join(os.path.dirname(os.path.dirname(nvcc())), "include")
    ref_obj = os.path.join(DROPIN_OUT, "ref_gpu_ops.o")
    if not os.path.exists(ref_obj) or os.path.getmtime(ref_obj) < os.path.getmtime(src):
        _run([nvcc(), "-x", "cu", "-std=c++20", "-DUSE_CUDA", *ARCH, "-O3", "-w", "-Xcompiler", "-fPIC",
              "-I", ref_inc, "-c", src, "-o", ref_obj])
    shim_obj = os.path.join(DROPIN_OUT, "ref_gpu_shim.o")
    _run(["g++", "-std=c++20", "-O2", "-fPIC", "-DUSE_CUDA", "-I", ref_inc, "-I", cuda_inc, "-c", REFGPU_SRC,
          "-o", shim_obj])
    _run([nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", REFGPU_LIB, shim_obj, ref_obj])
    return REFGPU_LIB


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv, force=True))
    if "--dropin" in sys.argv:
        print(build_dropin())
        print(build_refgpu())
