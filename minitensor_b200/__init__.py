"""minitensor_b200 -- B200 (sm_100a) engine for miniTensor's fp32 GEMM path.

The kernels and the C ABI live in ``csrc/`` (built into ``libmtgemm.so``; the ABI is
declared in ``include/mtgemm.h``). ``engine`` mirrors the reference's GPU entry points on
top of it, ``sharded`` splits large GEMMs over several GPUs, ``inputs`` makes the seeded
synthetic workloads.
"""
from . import engine  # noqa: F401
from .engine import (  # noqa: F401
    bmm, bmm_gpu, gemm, linear_backward, linear_forward, linear_fwd_gpu, matmul, matmul_gpu,
    matmul_gpu_bk16, matmul_gpu_strided, matmul_gpu_v2,
)
