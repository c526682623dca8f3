"""Column-sharded GEMM over the GPUs of one box (one process per GPU).

The reference is single-GPU (README.md:273). For the large-GEMM configuration the output
C = A.B is split by N-columns: rank r holds A and B[:, n0:n1] and computes C[:, n0:n1].
Every rank needs the whole C afterwards, so the shards must be all-gathered.

Product path (``ShardedGemm.run``): the GEMM and the all-gather are ONE kernel. Each
rank opens the other ranks' C buffers through CUDA IPC; the tcgen05 kernel's epilogue
stores each finished 128x256 tile into the local C and, over NVLink, into the same
columns of every peer's C while the next tile's main loop runs. A stream-ordered flag
barrier (bounded wait, device status on timeout) then makes all ranks' writes visible.

Baseline (``allgather_shards``): local GEMM into a shard buffer, then an NCCL (or gloo on
CPU) all-gather and a relayout into row-major C.

torch.distributed is only the plumbing: it exchanges IPC handles and runs the baseline.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import engine


def shard_columns(N: int, world: int, rank: int) -> tuple[int, int]:
    """Columns [n0, n1) of rank `rank`: near-equal contiguous blocks covering [0, N)."""
    return N * rank // world, N * (rank + 1) // world


class PeerTensor:
    """Device pointers to the same tensor on every rank (own pointer at index `rank`)."""

    def __init__(self, t: torch.Tensor, rank: int, world: int, group=None):
        L = engine.lib()
        self.t = t   # keep the local allocation alive while peers map it
        self.rank, self.world = rank, world
        h = (ctypes.c_char * 64)()
        off = ctypes.c_uint64(0)
        engine._check(L.mt_ipc_get_handle(t.data_ptr(), h, ctypes.byref(off)))
        mine = (bytes(h), off.value)
        allh = [None] * world
        dist.all_gather_object(allh, mine, group=group)
        self.ptrs = [0] * world
        self._opened = []
        for d, (hb, o) in enumerate(allh):
            if d == rank:
                self.ptrs[d] = t.data_ptr()
                continue
            p = ctypes.c_void_p()
            buf = (ctypes.c_char * 64).from_buffer_copy(hb)
            engine._check(L.mt_ipc_open(buf, o, ctypes.byref(p)))
            self.ptrs[d] = p.value
            self._opened.append((p.value, o))

    def close(self):
        L = engine.lib()
        for p, o in self._opened:
            L.mt_ipc_close(ctypes.c_void_p(p), o)
        self._opened = []


class ShardedGemm:
    """C[M,N] = A[M,K] . B[K,N] with B's columns sharded over `world` ranks; every rank
    ends with the full C. Call collectively (same order on every rank)."""

    def __init__(self, M: int, N: int, K: int, rank: int | None = None, world: int | None = None, group=None,
                 timeout_s: float = 10.0):
        self.M, self.N, self.K = M, N, K
        self.rank = dist.get_rank(group) if rank is None else rank
        self.world = dist.get_world_size(group) if world is None else world
        if self.world > 8:
            raise ValueError("at most 8 GPUs per sharded GEMM")
        self.group = group
        self.n0, self.n1 = shard_columns(N, self.world, self.rank)
        self.timeout_ns = int(timeout_s * 1e9)
        self.epoch = 0
        self.flags = torch.zeros(self.world, dtype=torch.int32, device="cuda")
        self._flag_peers = PeerTensor(self.flags, self.rank, self.world, group)
        self._flag_arr = (ctypes.c_void_p * self.world)(*self._flag_peers.ptrs)
        self._bound = {}

    def _peers(self, C: torch.Tensor) -> PeerTensor:
        key = (C.data_ptr(), C.numel())
        pt = self._bound.get(key)
        if pt is None:
            pt = PeerTensor(C, self.rank, self.world, self.group)
            self._bound[key] = pt
        return pt

    def run(self, A: torch.Tensor, B_shard: torch.Tensor, C: torch.Tensor, mode="tf32x3", stream=None):
        """A [M,K] and B_shard [K, n1-n0] on this GPU; C [M,N] row-major on every rank
        (the same C tensor across calls reuses the IPC mappings)."""
        if C.shape != (self.M, self.N) or not C.is_contiguous():
            raise ValueError("C must be a contiguous [M, N] tensor")
        if B_shard.shape != (self.K, self.n1 - self.n0) or A.shape != (self.M, self.K):
            raise ValueError("A must be [M, K] and B_shard [K, n1 - n0]")
        pt = self._peers(C)
        es = C.element_size()
        extra = [pt.ptrs[d] + self.n0 * es for d in range(self.world) if d != self.rank]
        arr = (ctypes.c_void_p * max(1, len(extra)))(*extra)
        Cv = C[:, self.n0:self.n1]
        s = engine._stream(stream)
        L = engine.lib()
        engine._check(L.mt_gemm_multi(ctypes.byref(engine.view(A)), ctypes.byref(engine.view(B_shard)),
                                      ctypes.byref(engine.view(Cv)), arr, len(extra), None, 0, engine._mode(mode), s))
        self.epoch += 1
        engine._check(L.mt_peer_barrier(self._flag_arr, self.rank, self.world, self.epoch, self.timeout_ns, s))

    def close(self):
        for pt in self._bound.values():
            pt.close()
        self._bound = {}
        self._flag_peers.close()


def allgather_shards(C_shard: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """Baseline reassembly: all-gather equal-width [M, N/world] shards (NCCL on GPU, gloo
    on CPU) and relayout the rank-blocked result into row-major [M, N]."""
    M, w = C_shard.shape
    parts = [torch.empty_like(C_shard) for _ in range(world)]
    dist.all_gather(parts, C_shard.contiguous(), group=group)
    return torch.cat(parts, dim=1)
