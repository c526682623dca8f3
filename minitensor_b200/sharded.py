"""Column-sharded GEMM over the GPUs of one box (one process per GPU).

The reference is single-GPU (README.md:273). For the large-GEMM configuration the output
C = A.B is split by N-columns: rank r holds A and B[:, n0:n1] and computes C[:, n0:n1].
Every rank needs the whole C afterwards, so the shards must be all-gathered.

Product path (``ShardedGemm.run``). Each rank opens the other ranks' C buffers through
CUDA IPC, then pushes its columns into every peer's C in one of two ways:

* ``gather="epilogue"`` (default): the GEMM and the all-gather are ONE kernel -- the
  tcgen05 epilogue hands each finished 32x32 block of a tile to the TMA engine, which
  stores it into the local C and, over NVLink, into the same columns of every peer's C,
  meant to run while the next tile's main loop runs. Measured on 8192^3, the gather is
  hidden on 2 ranks. On 4 and 8 ranks it adds about the time the received bytes take
  over the link (0.25-0.5 ms per step), so it is not hidden there.
* ``gather="copy"``: the GEMM runs in row chunks into the local C; after each chunk the
  copy engines push that chunk's columns to every peer (one 2-D copy per peer, each peer
  on its own stream) while the next chunk is computed. Slower here at every size (the
  shard rows are narrow strided runs: 4 KB at 8 ranks); kept as an option.

A stream-ordered flag barrier (bounded wait, device status on timeout) then makes all
ranks' writes visible. An optional host-side step gate (``PeerLiveness``) finds a peer
that left, died or fell behind before the next step is launched.

Baseline (``allgather_shards``): local GEMM into a shard buffer, then an NCCL (or gloo on
CPU) all-gather and a relayout into row-major C.

Batched matmuls (``ShardedBmm``) split the batch instead: rank r computes C[b0:b1] from
A[b0:b1] and its B batches (or the one broadcast B), and the same multi-destination
epilogue stores that contiguous block of batches into every rank's C.

torch.distributed is only the plumbing: it exchanges IPC handles and runs the baseline.
"""
from __future__ import annotations

import ctypes
import time
import warnings

import torch
import torch.distributed as dist

from . import engine


def shard_columns(N: int, world: int, rank: int) -> tuple[int, int]:
    """Columns [n0, n1) of rank `rank`: near-equal contiguous blocks covering [0, N)."""
    return N * rank // world, N * (rank + 1) // world


def shard_batches(batch: int, world: int, rank: int) -> tuple[int, int]:
    """Batches [b0, b1) of rank `rank`: near-equal contiguous blocks covering [0, batch)."""
    return batch * rank // world, batch * (rank + 1) // world


def row_chunks(M: int, chunks: int) -> list[tuple[int, int]]:
    """Row ranges [r0, r1) of the copy pipeline: `chunks` near-equal parts of [0, M) with
    boundaries on 256-row tiles (fewer parts when M has fewer tiles)."""
    tiles_m = (M + 255) // 256
    chunks = max(1, min(chunks, tiles_m))
    return [(256 * (tiles_m * c // chunks), min(M, 256 * (tiles_m * (c + 1) // chunks))) for c in range(chunks)]


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


class _PeerOutput:
    """What every sharded product shares: the ranks' output buffers mapped into each other
    (CUDA IPC, made once per distinct output tensor) and the bounded cross-GPU flag
    barrier that orders every rank's writes before the output is read."""

    def __init__(self, rank, world, group, timeout_s, liveness):
        self.liveness = liveness
        self.rank = dist.get_rank(group) if rank is None else rank
        self.world = dist.get_world_size(group) if world is None else world
        if self.world > 8:
            raise ValueError("at most 8 GPUs per sharded product")
        self.group = group
        self.timeout_ns = int(timeout_s * 1e9)
        self.epoch = 0
        self.flags = torch.zeros(self.world, dtype=torch.int32, device="cuda")
        self._flag_peers = PeerTensor(self.flags, self.rank, self.world, group)
        self._flag_arr = (ctypes.c_void_p * self.world)(*self._flag_peers.ptrs)
        self._bound = {}

    # Distinct C tensors kept mapped before the caller is warned (see _peers).
    MAX_BOUND_QUIET = 16

    def _peers(self, C: torch.Tensor) -> PeerTensor:
        """Peer pointers of C. Every distinct C stays mapped on every rank (and alive) until
        close(): unmapping earlier would need all ranks' in-flight steps to be finished."""
        key = (C.data_ptr(), C.numel())
        pt = self._bound.get(key)
        if pt is None:
            pt = PeerTensor(C, self.rank, self.world, self.group)
            self._bound[key] = pt
            if len(self._bound) == self.MAX_BOUND_QUIET + 1:
                warnings.warn(f"{type(self).__name__} keeps every distinct C tensor mapped on all ranks until "
                              "close(); pass the same C each step", RuntimeWarning, stacklevel=3)
        return pt

    def _barrier(self, s):
        self.epoch += 1
        engine._check(engine.lib().mt_peer_barrier(self._flag_arr, self.rank, self.world, self.epoch,
                                                   self.timeout_ns, s))

    def close(self):
        for pt in self._bound.values():
            pt.close()
        self._bound = {}
        self._flag_peers.close()


class ShardedGemm(_PeerOutput):
    """C[M,N] = A[M,K] . B[K,N] with B's columns sharded over `world` ranks; every rank
    ends with the full C. Call collectively (same order on every rank)."""

    def __init__(self, M: int, N: int, K: int, rank: int | None = None, world: int | None = None, group=None,
                 timeout_s: float = 10.0, gather: str | None = None, chunks: int | None = None,
                 liveness: "PeerLiveness | None" = None):
        super().__init__(rank, world, group, timeout_s, liveness)
        self.M, self.N, self.K = M, N, K
        self.n0, self.n1 = shard_columns(N, self.world, self.rank)
        if gather is None:
            gather = "epilogue"
        if gather not in ("epilogue", "copy"):
            raise ValueError("gather must be 'epilogue' or 'copy'")
        self.gather = gather
        # Row chunks for the copy pipeline: boundaries on 256-row tiles; fewer chunks when
        # the shard is narrow so that each chunk still has work for most SM pairs.
        if chunks is None:
            chunks = 4 if self.world <= 4 else 2
        self.row_chunks = row_chunks(M, chunks)
        self._copy_streams = [torch.cuda.Stream() for _ in range(self.world - 1)] if gather == "copy" else []

    def run(self, A: torch.Tensor, B_shard: torch.Tensor, C: torch.Tensor, mode="tf32x3", stream=None):
        """A [M,K] and B_shard [K, n1-n0] on this GPU; C [M,N] row-major on every rank.
        Pass the same C tensor each step: its IPC mappings are made once and reused, and
        each new C adds mappings that last until close()."""
        if C.shape != (self.M, self.N) or not C.is_contiguous():
            raise ValueError("C must be a contiguous [M, N] tensor")
        if B_shard.shape != (self.K, self.n1 - self.n0) or A.shape != (self.M, self.K):
            raise ValueError("A must be [M, K] and B_shard [K, n1 - n0]")
        if self.liveness is not None:
            self.liveness.step()   # raises PeerLost before anything is launched
        pt = self._peers(C)
        es = C.element_size()
        s = engine._stream(stream)
        L = engine.lib()
        if self.gather == "epilogue":
            extra = [pt.ptrs[d] + self.n0 * es for d in range(self.world) if d != self.rank]
            arr = (ctypes.c_void_p * max(1, len(extra)))(*extra)
            Cv = C[:, self.n0:self.n1]
            engine._check(L.mt_gemm_multi(ctypes.byref(engine.view(A)), ctypes.byref(engine.view(B_shard)),
                                          ctypes.byref(engine.view(Cv)), arr, len(extra), None, 0,
                                          engine._mode(mode), s))
        else:
            main = torch.cuda.current_stream() if stream is None else stream
            if not isinstance(main, torch.cuda.Stream):
                main = torch.cuda.ExternalStream(int(main))
            peers = [d for d in range(self.world) if d != self.rank]
            pitch, width = self.N * es, (self.n1 - self.n0) * es
            for r0, r1 in self.row_chunks:
                engine.gemm(A[r0:r1], B_shard, C[r0:r1, self.n0:self.n1], mode=mode, stream=main)
                ev = torch.cuda.Event()
                ev.record(main)
                off = (r0 * self.N + self.n0) * es
                for cs, d in zip(self._copy_streams, peers):
                    cs.wait_event(ev)
                    engine._check(L.mt_copy_rows_async(pt.ptrs[d] + off, pitch, pt.ptrs[self.rank] + off, pitch,
                                                       width, r1 - r0, cs.cuda_stream))
            for cs in self._copy_streams:
                ev = torch.cuda.Event()
                ev.record(cs)
                main.wait_event(ev)
        self._barrier(s)


class ShardedBmm(_PeerOutput):
    """C[b] = A[b] . B[b] for b in [0, batch) with the batch split over `world` ranks
    (include/TensorOps.hpp:933-991 is the single-GPU bmm this shards); every rank ends with
    the full C [batch, M, N]. Rank r computes batches [b0, b1) = shard_batches(batch, world,
    r) and its multi-destination epilogue stores them into every rank's C, whose block of
    those batches is contiguous, so nothing is relaid out. Call collectively."""

    def __init__(self, batch: int, M: int, N: int, K: int, rank: int | None = None, world: int | None = None,
                 group=None, timeout_s: float = 10.0, liveness: "PeerLiveness | None" = None):
        super().__init__(rank, world, group, timeout_s, liveness)
        self.batch, self.M, self.N, self.K = batch, M, N, K
        self.b0, self.b1 = shard_batches(batch, self.world, self.rank)

    def run(self, A_shard: torch.Tensor, B_shard: torch.Tensor, C: torch.Tensor, mode="tf32x3", stream=None):
        """A_shard [b1-b0, M, K] and B_shard [b1-b0, K, N] (any views: B may be a broadcast
        operand expanded with batch stride 0) on this GPU; C [batch, M, N] contiguous on
        every rank. Pass the same C each step (its IPC mappings are made once)."""
        nb = self.b1 - self.b0
        if C.shape != (self.batch, self.M, self.N) or not C.is_contiguous():
            raise ValueError("C must be a contiguous [batch, M, N] tensor")
        if A_shard.shape != (nb, self.M, self.K) or B_shard.shape != (nb, self.K, self.N):
            raise ValueError("A_shard must be [b1-b0, M, K] and B_shard [b1-b0, K, N]")
        if self.liveness is not None:
            self.liveness.step()
        pt = self._peers(C)
        s = engine._stream(stream)
        if nb > 0:
            off = self.b0 * self.M * self.N * C.element_size()
            extra = [pt.ptrs[d] + off for d in range(self.world) if d != self.rank]
            arr = (ctypes.c_void_p * max(1, len(extra)))(*extra)
            engine._check(engine.lib().mt_gemm_multi(ctypes.byref(engine.view(A_shard)),
                                                     ctypes.byref(engine.view(B_shard)),
                                                     ctypes.byref(engine.view(C[self.b0:self.b1])), arr, len(extra),
                                                     None, 0, engine._mode(mode), s))
        self._barrier(s)


class PeerLost(RuntimeError):
    """A peer rank left, aborted or missed a step deadline; no further step may launch."""


class PeerLiveness:
    """Host-side step gate over the process group's key-value store.

    Before step e every rank publishes ``ready/e/<rank>`` and waits, polling, until all
    peers have published theirs. A rank that leaves between steps (``leave()``), dies, or
    is slower than ``timeout_s`` is therefore noticed on the host BEFORE the next launch,
    so no kernel is started that would write into, or wait on, a departed peer's memory.
    A rank that gives up marks itself ``gone/<rank>`` so that late peers stop too instead
    of launching a step nobody else joins. One store round trip per peer per step: meant
    for eager steps, not for inside a captured graph (the gate runs at capture time only).
    """

    def __init__(self, rank: int, world: int, store=None, timeout_s: float = 10.0,
                 prefix: str = "mt_live", poll_s: float = 0.002):
        if store is None:
            store = dist.distributed_c10d._get_default_store()
        self.rank, self.world, self.store = rank, world, store
        self.timeout_s, self.poll_s, self.prefix = timeout_s, poll_s, prefix
        self.epoch = 0

    def _gone(self, r: int) -> str:
        return f"{self.prefix}/gone/{r}"

    def _ready(self, e: int, r: int) -> str:
        return f"{self.prefix}/ready/{e}/{r}"

    def gone_peers(self) -> list[int]:
        return [r for r in range(self.world) if r != self.rank and self.store.check([self._gone(r)])]

    def step(self) -> int:
        """Gate for the next step. Returns its epoch; raises PeerLost (and marks this rank
        gone) if a peer has left or does not arrive within the timeout."""
        self.epoch += 1
        e = self.epoch
        self.store.set(self._ready(e, self.rank), b"1")
        waiting = [r for r in range(self.world) if r != self.rank]
        deadline = time.monotonic() + self.timeout_s
        while True:
            gone = self.gone_peers()
            if gone:
                self._give_up()
                raise PeerLost(f"rank {self.rank}: peer(s) {gone} left before step {e}")
            waiting = [r for r in waiting if not self.store.check([self._ready(e, r)])]
            if not waiting:
                # Every peer has published step e, so each has left gate e - 1 and no longer
                # reads this rank's key of that step: drop it (the store stays bounded).
                if e > 1:
                    try:
                        self.store.delete_key(self._ready(e - 1, self.rank))
                    except Exception:   # a store without deletion: the keys just remain
                        pass
                return e
            if time.monotonic() > deadline:
                self._give_up()
                raise PeerLost(f"rank {self.rank}: peer(s) {waiting} missed step {e} "
                               f"within {self.timeout_s:g} s")
            time.sleep(self.poll_s)

    def leave(self) -> None:
        """Announce a departure between steps (call after this rank's stream is idle)."""
        self._give_up()

    def _give_up(self) -> None:
        self.store.set(self._gone(self.rank), b"1")


def allgather_shards(C_shard: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """Baseline reassembly: all-gather equal-width [M, N/world] shards (NCCL on GPU, gloo
    on CPU) and relayout the rank-blocked result into row-major [M, N]."""
    M, w = C_shard.shape
    parts = [torch.empty_like(C_shard) for _ in range(world)]
    dist.all_gather(parts, C_shard.contiguous(), group=group)
    return torch.cat(parts, dim=1)


def allgather_batch_shards(C_block: torch.Tensor, batch: int, world: int, group=None) -> torch.Tensor:
    """Baseline reassembly of a batch-sharded bmm: all-gather every rank's block of batches
    (NCCL on GPU, gloo on CPU; blocks padded to the largest so the collective sees equal
    sizes) into [batch, M, N]. Each block is contiguous in the result: no relayout."""
    M, N = C_block.shape[1], C_block.shape[2]
    width = (batch + world - 1) // world
    pad = torch.zeros((width, M, N), dtype=C_block.dtype, device=C_block.device)
    pad[:C_block.shape[0]] = C_block
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    blocks = []
    for r, part in enumerate(parts):
        b0, b1 = shard_batches(batch, world, r)
        blocks.append(part[:b1 - b0])
    return torch.cat(blocks, dim=0)

