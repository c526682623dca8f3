"""CPU tests of the multi-GPU host logic with world_size-2 gloo process groups: the column
shard plan, the baseline all-gather reassembly, and failure detection (a rank that dies
before the collective makes the survivor's collective fail within its timeout, never hang).
"""
import datetime
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from minitensor_b200.sharded import allgather_batch_shards, allgather_shards, shard_batches, shard_columns


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_plan_covers_columns():
    for N in (1, 7, 8, 8192, 1000):
        for world in (1, 2, 3, 4, 8):
            cols = []
            for r in range(world):
                n0, n1 = shard_columns(N, world, r)
                assert 0 <= n0 <= n1 <= N
                cols.extend(range(n0, n1))
            assert cols == list(range(N))


def test_batch_shard_plan_covers_batches():
    for batch in (1, 2, 7, 64, 65):
        for world in (1, 2, 3, 4, 8):
            got = []
            for r in range(world):
                b0, b1 = shard_batches(batch, world, r)
                assert 0 <= b0 <= b1 <= batch and b1 - b0 in (batch // world, batch // world + 1)
                got.extend(range(b0, b1))
            assert got == list(range(batch))


def _batch_gather_worker(rank, world, port, out, batch):
    # Each rank computes its block of a broadcast bmm (config 3's shape, batch cut
    # unevenly) and the baseline all-gather reassembles [batch, M, N] on every rank.
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    rs = np.random.RandomState(1)
    A = rs.standard_normal((batch, 6, 4)).astype(np.float32)
    B0 = rs.standard_normal((1, 4, 5)).astype(np.float32)
    b0, b1 = shard_batches(batch, world, rank)
    block = torch.from_numpy(np.matmul(A[b0:b1], B0))
    C = allgather_batch_shards(block, batch, world)
    np.save(os.path.join(out, f"c{rank}.npy"), C.numpy())
    np.save(os.path.join(out, "ref.npy"), np.matmul(A, B0))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,batch", [(2, 7), (3, 64)])
def test_batch_allgather_reassembly_gloo(tmp_path, world, batch):
    mp.spawn(_batch_gather_worker, args=(world, free_port(), str(tmp_path), batch), nprocs=world, join=True)
    ref = np.load(tmp_path / "ref.npy")
    for r in range(world):
        assert np.array_equal(np.load(tmp_path / f"c{r}.npy"), ref)


def _gather_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    rs = np.random.RandomState(0)
    A = rs.standard_normal((12, 5)).astype(np.float32)
    B = rs.standard_normal((5, 8)).astype(np.float32)
    n0, n1 = shard_columns(8, world, rank)
    C_shard = torch.from_numpy(A @ B[:, n0:n1])
    C = allgather_shards(C_shard, world)
    np.save(os.path.join(out, f"c{rank}.npy"), C.numpy())
    np.save(os.path.join(out, "ref.npy"), A @ B)
    dist.barrier()
    dist.destroy_process_group()


def test_allgather_reassembly_gloo(tmp_path):
    mp.spawn(_gather_worker, args=(2, free_port(), str(tmp_path)), nprocs=2, join=True)
    ref = np.load(tmp_path / "ref.npy")
    for r in range(2):
        assert np.array_equal(np.load(tmp_path / f"c{r}.npy"), ref)


def _dying_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        # This rank fails on the host before its collective (between steps).
        os._exit(3)
    t0 = time.time()
    try:
        allgather_shards(torch.ones(4, 2), world)
        status = "completed"
    except Exception as e:  # gloo reports the lost peer / timeout as an error
        status = f"error:{type(e).__name__}"
    with open(os.path.join(out, "survivor.txt"), "w") as f:
        f.write(f"{status} {time.time() - t0:.2f}")
    os._exit(0)


def test_dead_rank_is_detected_not_hung(tmp_path):
    ctx = mp.get_context("spawn")
    port = free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung past the process-group timeout"
    status, secs = open(tmp_path / "survivor.txt").read().split()
    assert status.startswith("error"), status
    assert float(secs) < 30


def test_row_chunks_cover_rows_on_tile_boundaries():
    from minitensor_b200.sharded import row_chunks
    for M, chunks in [(8192, 4), (8192, 2), (1000, 4), (300, 4), (256, 3), (1, 4), (8192, 1)]:
        parts = row_chunks(M, chunks)
        assert parts[0][0] == 0 and parts[-1][1] == M
        for (a0, a1), (b0, b1) in zip(parts, parts[1:]):
            assert a1 == b0
        assert all(r0 < r1 for r0, r1 in parts)
        assert all(r0 % 256 == 0 for r0, _ in parts)
        assert len(parts) == min(chunks, (M + 255) // 256)


# --- host-side step gate (PeerLiveness): a departed or late peer is found before a launch ---

def _live_worker(rank, world, port, out, scenario, timeout_s):
    from minitensor_b200.sharded import PeerLiveness, PeerLost
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    gate = PeerLiveness(rank, world, timeout_s=timeout_s)
    log = []
    try:
        log.append(f"step{gate.step()}")
        dist.barrier()   # stands for the end-of-step device barrier: step 1 finished everywhere
        if rank == 1 and scenario == "leave":
            gate.leave()
            log.append("left")
            raise SystemExit
        if rank == 1 and scenario == "die":
            with open(os.path.join(out, "r1.txt"), "w") as f:
                f.write(" ".join(log + ["died"]))
            os._exit(3)
        if rank == 1 and scenario == "late":
            time.sleep(3 * timeout_s)
        if scenario == "ok":
            log.append(f"step{gate.step()}")
            dist.barrier()
            # Keys of finished steps are dropped: only the latest step's remain.
            stale = [k for k in (gate._ready(1, 0), gate._ready(1, 1)) if gate.store.check([k])]
            log.append(f"stale{len(stale)}")
        for _ in range(2):
            t0 = time.monotonic()
            try:
                log.append(f"step{gate.step()}")
            except PeerLost:
                log.append(f"lost@{time.monotonic() - t0:.2f}")
                break
    except SystemExit:
        pass
    with open(os.path.join(out, f"r{rank}.txt"), "w") as f:
        f.write(" ".join(log))
    # Rank 0 hosts the store: keep it up until the peer has written its result.
    if rank == 0:
        t0 = time.monotonic()
        while not os.path.exists(os.path.join(out, "r1.txt")) and time.monotonic() - t0 < 30:
            time.sleep(0.05)
    os._exit(0)


def _run_live(tmp_path, scenario, timeout_s=1.0):
    ctx = mp.get_context("spawn")
    port = free_port()
    procs = [ctx.Process(target=_live_worker, args=(r, 2, port, str(tmp_path), scenario, timeout_s))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung in the step gate"
    return [open(tmp_path / f"r{r}.txt").read().split() for r in range(2)]


def _lost_after(entry):
    assert entry.startswith("lost@"), entry
    return float(entry[5:])


def test_liveness_gate_all_ranks_step_together(tmp_path):
    r0, r1 = _run_live(tmp_path, "ok")
    assert r0 == r1 == ["step1", "step2", "stale0", "step3", "step4"]


def test_liveness_peer_that_leaves_is_seen_before_next_step(tmp_path):
    r0, r1 = _run_live(tmp_path, "leave", timeout_s=5.0)
    assert r1 == ["step1", "left"]
    assert r0[0] == "step1" and len(r0) == 2
    assert _lost_after(r0[1]) < 2.0   # announced departure: no need to wait out the timeout


def test_liveness_dead_peer_bounded_by_timeout(tmp_path):
    r0, r1 = _run_live(tmp_path, "die", timeout_s=1.0)
    assert r1 == ["step1", "died"]
    assert r0[0] == "step1"
    assert 0.9 <= _lost_after(r0[1]) < 5.0


def test_liveness_late_peer_stops_too(tmp_path):
    # Rank 0 gives up after the timeout and marks itself gone; the late rank then finds
    # that mark at once instead of launching a step that nobody else joins.
    r0, r1 = _run_live(tmp_path, "late", timeout_s=1.0)
    assert r0[0] == r1[0] == "step1"
    assert 0.9 <= _lost_after(r0[1]) < 5.0
    assert _lost_after(r1[1]) < 1.0


def _late_collective_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=2))
    if rank == 1:
        time.sleep(6)   # delayed past the group timeout, between steps
    t0 = time.time()
    try:
        allgather_shards(torch.ones(4, 2), world)
        status = "completed"
    except Exception as e:
        status = f"error:{type(e).__name__}"
    with open(os.path.join(out, f"r{rank}.txt"), "w") as f:
        f.write(f"{status} {time.time() - t0:.2f}")
    os._exit(0)


def test_rank_delayed_past_timeout_fails_collective_not_hangs(tmp_path):
    ctx = mp.get_context("spawn")
    port = free_port()
    procs = [ctx.Process(target=_late_collective_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung past the process-group timeout"
    status, secs = open(tmp_path / "r0.txt").read().split()
    assert status.startswith("error"), status
    assert float(secs) < 20
