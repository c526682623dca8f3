"""CPU tests of the CTA-pair kernel's work schedule (whole tiles round-robin, then the
stream-K remainder), restated from minitensor_b200/csrc/umma_gemm2.cuh (Sched) and
mt_api.cu (pair_streamk_plan). The kernel's correctness rests on three properties that
are pure integer arithmetic, checked here over many shapes:

1. every (tile, k-block) is done by exactly one cluster;
2. the pieces of a cut tile carry seg = 0 .. nseg-1 in k order, each exactly once, and
   every piece agrees on nseg (the last-arriver count and the partial slots depend on it);
3. nseg never exceeds the partial slots the host allocates (sk_maxseg).
"""
import itertools

import pytest


def slot_of(tile, sk_dp, S, maxseg, t0):
    """umma::sk_slot: S slots per split whole tile, maxseg per stream-K tile."""
    return (tile - t0) * S if tile < sk_dp else (sk_dp - t0) * S + (tile - sk_dp) * maxseg


def plan(num_tiles, clusters, kblocks, split_dp=False, gate=False):
    """(sk_dp, S, slots) as pair_streamk_plan sets them. gate=False: the stream-K remainder
    whenever it fits (the schedule properties are tested on every shape); gate=True: only
    where the host enables it (3xTF32 with more than 5% of the last round idle)."""
    S = 2 if split_dp and kblocks >= 16 else 1
    units = num_tiles * S
    sk_dp, maxseg = num_tiles, 0
    rounds_up = (units + clusters - 1) // clusters if clusters > 0 else 0
    worth_it = (rounds_up * clusters - units) / units > 0.05 if units else False
    if clusters > 0 and units > clusters and (worth_it or not gate):
        dp = (units // clusters) * clusters // S
        rem = num_tiles - dp
        W = rem * kblocks
        if rem > 0 and W >= 8 * clusters:
            sk_dp = dp
            minr = W // clusters
            maxseg = (kblocks + minr - 1) // minr + 1
    if S == 1 and sk_dp == num_tiles:
        return num_tiles, 1, 0          # nothing is cut: no partial slots
    return sk_dp, S, maxseg


def items(num_tiles, sk_dp, kblocks, c, C, S=1):
    """The Sched sequence of cluster c of C: (tile, kb0, kb1, seg, nseg)."""
    out = []
    u = c
    while u < sk_dp * S:
        t, sp = divmod(u, S)
        out.append((t, kblocks * sp // S, kblocks * (sp + 1) // S, sp, S))
        u += C
    W = (num_tiles - sk_dp) * kblocks
    if W == 0:
        return out
    x, hi = W * c // C, W * (c + 1) // C

    def owner(y):
        return ((y + 1) * C + W - 1) // W - 1

    while x < hi:
        t = x // kblocks
        kb0 = x - t * kblocks
        kb1 = min(kblocks, kb0 + (hi - x))
        cf = owner(t * kblocks)
        nseg = owner(t * kblocks + kblocks - 1) - cf + 1
        out.append((sk_dp + t, kb0, kb1, c - cf, nseg))
        x += kb1 - kb0
    return out


def check_schedule(num_tiles, C, kblocks, split_dp=False):
    sk_dp, S, slots = plan(num_tiles, C, kblocks, split_dp)
    covered = {}
    pieces = {}
    for c in range(C):
        for tile, kb0, kb1, seg, nseg in items(num_tiles, sk_dp, kblocks, c, C, S):
            assert 0 <= kb0 < kb1 <= kblocks
            for kb in range(kb0, kb1):
                assert (tile, kb) not in covered, (tile, kb)
                covered[(tile, kb)] = c
            pieces.setdefault(tile, []).append((kb0, kb1, seg, nseg, c))
    assert len(covered) == num_tiles * kblocks
    # Partial slots: every piece of every cut tile gets its own slot, inside the allocation.
    t0 = 0 if S > 1 else sk_dp
    nslots = (sk_dp - t0) * S + (num_tiles - sk_dp) * slots
    used = set()
    for tile, ps in pieces.items():
        if len(ps) > 1:
            for p in ps:
                slot = slot_of(tile, sk_dp, S, slots, t0) + p[2]
                assert 0 <= slot < nslots and slot not in used, (tile, p, slot, nslots)
                used.add(slot)
    for tile, ps in pieces.items():
        ps.sort()
        nsegs = {p[3] for p in ps}
        assert len(nsegs) == 1 and nsegs.pop() == len(ps), (tile, ps)
        assert [p[2] for p in ps] == list(range(len(ps))), (tile, ps)   # seg in k order
        if len(ps) > 1:
            assert len(ps) <= (S if tile < sk_dp else slots), (tile, len(ps), slots)
            if tile >= sk_dp:
                clusters = [p[4] for p in ps]
                assert clusters == list(range(clusters[0], clusters[0] + len(ps)))   # consecutive clusters
            else:
                assert S > 1 and len(ps) == S
    return sk_dp, S, slots


def test_config5_shards():
    # 8192^3 over 1, 2, 4, 8 GPUs with 74 clusters: 256 x 256 tiles, K = 8192 -> 256 k-blocks.
    for tiles in (1024, 512, 256, 128):
        sk_dp, S, slots = check_schedule(tiles, 74, 256)
        assert S == 1 and sk_dp == tiles - tiles % 74 and slots >= 2
    assert plan(256, 74, 256) == (222, 1, 4)
    # Where the host turns it on: the 4- and 8-GPU shards (3.46 / 1.73 rounds), not one GPU's
    # 13.8 rounds or two GPUs' 6.9.
    assert plan(1024, 74, 256, gate=True)[0] == 1024 and plan(512, 74, 256, gate=True)[0] == 512
    assert plan(256, 74, 256, gate=True)[0] == 222 and plan(128, 74, 256, split_dp=True, gate=True)[0] == 111
    # The 8-GPU shard with peers: whole tiles in two halves, 3 rounds of halves, then stream-K.
    sk_dp, S, slots = check_schedule(128, 74, 256, split_dp=True)
    assert (sk_dp, S) == (111, 2) and slots >= 2


def test_off_when_ranges_would_be_short_or_rounds_are_whole():
    assert plan(148, 74, 256) == (148, 1, 0)       # whole rounds
    assert plan(90, 74, 5) == (90, 1, 0)           # 16 x 5 k-blocks < 8 per cluster
    assert plan(60, 74, 256) == (60, 1, 0)         # fewer tiles than clusters: not a pair launch
    assert plan(128, 74, 8, split_dp=True)[1] == 1   # halves need 8 k-blocks each
    check_schedule(90, 74, 5)


@pytest.mark.parametrize("C", [1, 2, 3, 7, 37, 74])
@pytest.mark.parametrize("split_dp", [False, True])
def test_many_shapes(C, split_dp):
    for tiles, kblocks in itertools.product([C + 1, 2 * C - 1, 3 * C + 2, 5 * C + C // 2 + 1],
                                            [1, 2, 7, 8, 9, 16, 31, 64, 256]):
        check_schedule(tiles, C, kblocks, split_dp)
