"""GPU tests of the sharded GEMM path.

On one GPU: the multi-destination epilogue (every tile stored to several buffers) and the
bounded cross-GPU flag barrier (a wait that runs out records status 6 and returns; the
context stays usable). On two or more GPUs (skipped otherwise): the fused column-sharded
GEMM + all-gather across real processes, checked against the CPU oracle.
"""
import ctypes
import datetime
import os
import socket

import numpy as np
import pytest
import torch

from minitensor_b200 import engine, inputs
from parity import absmm, check, dev, host

pytestmark = pytest.mark.gpu


def _multi(A, B, C, extras, mode):
    L = engine.lib()
    P = ctypes.POINTER(engine.MtTensor)
    L.mt_gemm_multi.argtypes = [P, P, P, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                ctypes.c_void_p]
    arr = (ctypes.c_void_p * max(1, len(extras)))(*[e.data_ptr() for e in extras])
    engine._check(L.mt_gemm_multi(ctypes.byref(engine.view(A)), ctypes.byref(engine.view(B)),
                                  ctypes.byref(engine.view(C)), arr, len(extras), None, 0, engine._mode(mode),
                                  engine._stream(None)))


@pytest.mark.parametrize("mode", ["tf32", "tf32x3", "strict"])
def test_multi_destination_epilogue(eng, port, mode):
    M, K, N = 384, 256, 640
    A = inputs.uniform((M, K), -1, 1, 71)
    B = inputs.uniform((K, N), -1, 1, 72)
    C = torch.empty(M, N, device="cuda")
    extras = [torch.full((M, N), -7.0, device="cuda") for _ in range(3)]
    _multi(dev(A), dev(B), C, extras, mode)
    ref = port.matmul(A, B)
    c = host(C)
    check(mode, c, ref, absmm(A, B), K, "local")
    for e in extras:
        assert np.array_equal(host(e), c)


@pytest.mark.parametrize("mode", ["tf32", "tf32x3"])
def test_multi_destination_epilogue_pair_kernel(eng, port, mode):
    """The CTA-pair kernel (>= 74 tiles of 256 x 256) writing every tile to 4 outputs."""
    M, K, N = 2304, 160, 2336
    A = inputs.uniform((M, K), -1, 1, 75)
    B = inputs.uniform((K, N), -1, 1, 76)
    C = torch.empty(M, N, device="cuda")
    extras = [torch.full((M, N), -7.0, device="cuda") for _ in range(3)]
    _multi(dev(A), dev(B), C, extras, mode)
    assert eng.last_path().startswith("umma_pair_" + mode), eng.last_path()
    c = host(C)
    rows = [0, 127, 128, 255, 256, 2047, 2048, M - 1]
    check(mode, c[rows], port.matmul_strided(A[rows], B), absmm(A[rows], B), K, "pair local")
    for e in extras:
        assert np.array_equal(host(e), c)


@pytest.mark.parametrize("mode", ["tf32x3", "tf32"])
def test_multi_destination_split_units(eng, port, mode):
    """A multi-destination GEMM with fewer than two rounds of pair tiles (96 tiles over 74
    clusters, as one rank's shard at 8 GPUs): whole tiles are cut into two k-halves handed
    out as separate units (split=2), and in 3xTF32 the remainder runs stream-K; every
    destination gets the same, correct C."""
    M, K, N = 4096, 1024, 1536
    A = inputs.uniform((M, K), -1, 1, 311)
    B = inputs.uniform((K, N), -1, 1, 312)
    C = torch.full((M, N), float("nan"), device="cuda")
    extras = [torch.full((M, N), -7.0, device="cuda") for _ in range(3)]
    _multi(dev(A), dev(B), C, extras, mode)
    path = eng.last_path()
    assert "split=2" in path and ("streamk=" in path) == (mode == "tf32x3"), path
    c = host(C)
    rows = [0, 255, 256, 2047, 2048, 3071, 3072, 3583, 3584, M - 1]
    check(mode, c[rows], port.matmul_strided(A[rows], B), absmm(A[rows], B), K, f"split units ({path})")
    for e in extras:
        assert np.array_equal(host(e), c)
    assert eng.device_status(reset=True) == 0


def test_multi_destination_ragged_columns_clipped(eng, port):
    """N = 2340 (not a multiple of 32): the last column block of each tile is partial and
    the TMA stores must clip it; every destination is a window of a wider buffer whose
    guard columns must stay untouched."""
    M, K, N = 2304, 96, 2340
    A = inputs.uniform((M, K), -1, 1, 77)
    B = inputs.uniform((K, N), -1, 1, 78)
    bufs = [torch.full((M, N + 12), 3.0, device="cuda") for _ in range(4)]
    views = [b[:, :N] for b in bufs]
    _multi(dev(A), dev(B), views[0], views[1:], "tf32x3")
    assert eng.last_path().startswith("umma_pair_tf32x3"), eng.last_path()
    c0 = host(views[0])
    rows = [0, 255, 256, 1151, M - 1]
    check("tf32x3", c0[rows], port.matmul_strided(A[rows], B), absmm(A[rows], B), K, "ragged local")
    for b, v in zip(bufs, views):
        assert np.array_equal(host(v), c0)
        assert np.all(host(b)[:, N:] == 3.0)


def test_column_shard_into_wide_buffers(eng, port):
    # The sharded layout on one GPU: 4 "ranks" write their column blocks into 4 full-width Cs.
    M, K, N, world = 256, 192, 512, 4
    A = inputs.uniform((M, K), -1, 1, 73)
    B = inputs.uniform((K, N), -1, 1, 74)
    Cs = [torch.zeros(M, N, device="cuda") for _ in range(world)]
    Ad = dev(A)
    for r in range(world):
        n0, n1 = N * r // world, N * (r + 1) // world
        Bs = dev(np.ascontiguousarray(B[:, n0:n1]))
        others = [Cs[d][:, n0:] for d in range(world) if d != r]   # element (0, n0) of each peer C
        _multi(Ad, Bs, Cs[r][:, n0:n1], others, "tf32x3")
    ref = port.matmul(A, B)
    for C in Cs:
        check("tf32x3", host(C), ref, absmm(A, B), K, "sharded layout")


@pytest.mark.parametrize("mode", ["tf32x3", "tf32", "strict"])
def test_batch_shard_into_full_buffers(eng, port, mode):
    """The batch-sharded layout on one GPU: 3 "ranks" each compute a block of a broadcast
    bmm (batch 7 cut 2/2/3, B broadcast with batch stride 0) and write it into all three
    full-size Cs through the 3-D multi-destination epilogue."""
    from minitensor_b200.sharded import shard_batches
    bt, M, K, N, world = 7, 320, 64, 288, 3
    A = inputs.uniform((bt, M, K), -1, 1, 91)
    B0 = inputs.uniform((1, K, N), -1, 1, 92)
    Cs = [torch.full((bt, M, N), -5.0, device="cuda") for _ in range(world)]
    Ad, Bd = dev(A), dev(B0)
    for r in range(world):
        b0, b1 = shard_batches(bt, world, r)
        others = [Cs[d][b0:] for d in range(world) if d != r]   # element (b0, 0, 0) of each peer C
        _multi(Ad[b0:b1], Bd.expand(b1 - b0, K, N), Cs[r][b0:b1], others, mode)
    ref = port.bmm(A, np.broadcast_to(B0, (bt, K, N)))
    for C in Cs:
        check(mode, host(C), ref, absmm(A, B0), K, "batch-sharded layout")


def test_peer_barrier_timeout_reports_status(eng):
    L = engine.lib()
    L.mt_peer_barrier.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_uint64,
                                  ctypes.c_void_p]
    assert engine.device_status(reset=True) == 0
    mine = torch.zeros(2, dtype=torch.int32, device="cuda")
    other = torch.zeros(2, dtype=torch.int32, device="cuda")    # "rank 1" never raises its flag
    arr = (ctypes.c_void_p * 2)(mine.data_ptr(), other.data_ptr())
    engine._check(L.mt_peer_barrier(arr, 0, 2, 1, int(0.2e9), engine._stream(None)))
    assert engine.device_status(reset=True) == 6
    assert host(other).tolist() == [1, 0]                       # our flag reached the peer array
    # The context is still usable.
    A = torch.ones(64, 64, device="cuda")
    C = torch.empty(64, 64, device="cuda")
    engine.gemm(A, A, C, mode="tf32x3")
    assert float(host(C)[0, 0]) == 64.0
    assert engine.device_status(reset=True) == 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _sharded_worker(rank, world, port, out, mode, shape=(1024, 1536, 512), gather=None):
    import torch.distributed as dist
    from minitensor_b200 import sharded
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    M, N, K = shape
    A = inputs.uniform((M, K), -1, 1, 81)
    B = inputs.uniform((K, N), -1, 1, 82)
    plan = sharded.ShardedGemm(M, N, K, rank, world, timeout_s=5.0, gather=gather)
    C = torch.zeros(M, N, device="cuda")
    for _ in range(2):   # twice: the second call reuses the IPC mappings and a new epoch
        plan.run(dev(A), dev(np.ascontiguousarray(B[:, plan.n0:plan.n1])), C, mode=mode)
    torch.cuda.synchronize()
    np.save(os.path.join(out, f"c{rank}.npy"), C.cpu().numpy())
    status = engine.device_status(reset=True)
    dist.barrier()
    plan.close()
    dist.destroy_process_group()
    assert status == 0, status


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode,shape,gather", [("tf32x3", (1024, 1536, 512), "epilogue"),
                                               ("strict", (1024, 1536, 512), "epilogue"),
                                               ("tf32", (2304, 4672, 128), "epilogue"),
                                               ("tf32x3", (2304, 4672, 128), "epilogue"),
                                               ("tf32x3", (1000, 1536, 512), "copy"),
                                               ("tf32", (2304, 4672, 128), "copy")])
def test_sharded_gemm_two_gpus(eng, port, tmp_path, mode, shape, gather):
    """Column shards on two GPUs, every rank ending with the full C. `epilogue`: the GEMM
    epilogue stores into the peers (the (2304, 4672, 128) cases give each rank >= 74 tiles
    of 256 x 256: the CTA-pair kernel); `copy`: row chunks pushed by the copy engines
    (M = 1000: a ragged last chunk)."""
    import torch.multiprocessing as mp
    world = 2
    mp.spawn(_sharded_worker, args=(world, _free_port(), str(tmp_path), mode, shape, gather), nprocs=world,
             join=True)
    M, N, K = shape
    A = inputs.uniform((M, K), -1, 1, 81)
    B = inputs.uniform((K, N), -1, 1, 82)
    rows = sorted(set([0, 127, 128, 255, 256, M // 2, M - 1]))
    ref = port.matmul_strided(A[rows], B)
    for r in range(world):
        check(mode, np.load(tmp_path / f"c{r}.npy")[rows], ref, absmm(A[rows], B), K, f"rank {r}")


def _bmm_worker(rank, world, port, out, mode, shape):
    import torch.distributed as dist
    from minitensor_b200 import sharded
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    bt, M, K, N = shape
    A = inputs.uniform((bt, M, K), -1, 1, 93)
    B0 = inputs.uniform((1, K, N), -1, 1, 94)
    plan = sharded.ShardedBmm(bt, M, N, K, rank, world, timeout_s=5.0)
    C = torch.zeros(bt, M, N, device="cuda")
    Ad = dev(np.ascontiguousarray(A[plan.b0:plan.b1]))
    Bd = dev(B0).expand(plan.b1 - plan.b0, K, N)
    for _ in range(2):   # the second call reuses the mappings with a new epoch
        plan.run(Ad, Bd, C, mode=mode)
    torch.cuda.synchronize()
    np.save(os.path.join(out, f"c{rank}.npy"), C.cpu().numpy())
    status = engine.device_status(reset=True)
    dist.barrier()
    plan.close()
    dist.destroy_process_group()
    assert status == 0, status


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode,shape", [("tf32x3", (64, 512, 64, 512)), ("tf32", (7, 300, 96, 520)),
                                        ("strict", (5, 256, 64, 256))])
def test_sharded_bmm_two_gpus(eng, port, tmp_path, mode, shape):
    """Batch shards of a broadcast bmm on two GPUs (config 3's shape, and uneven batches
    with ragged tiles): every rank ends with the whole C."""
    import torch.multiprocessing as mp
    world = 2
    mp.spawn(_bmm_worker, args=(world, _free_port(), str(tmp_path), mode, shape), nprocs=world, join=True)
    bt, M, K, N = shape
    A = inputs.uniform((bt, M, K), -1, 1, 93)
    B0 = inputs.uniform((1, K, N), -1, 1, 94)
    ref = port.bmm(A, np.broadcast_to(B0, (bt, K, N)))
    for r in range(world):
        check(mode, np.load(tmp_path / f"c{r}.npy"), ref, absmm(A, B0), K, f"rank {r}")
