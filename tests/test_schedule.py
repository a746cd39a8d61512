"""The GEMM's work schedule without a GPU.

The plan (which tiles are spread over the SM pairs by K-step ranges) comes from
the library itself through mpk_gemm_plan, on a host without a GPU the device is
taken to have 148 SMs.  The per-cluster walk over work units is the kernel's
(UnitWalk in mix_precision_kernel_b200/csrc/gemm.cu), restated here so that its
invariants can be checked over many shapes: every K-step of every tile is
computed exactly once, a tile split over several clusters is finished by exactly
one owner that waits only for clusters with a lower logical index (which started
earlier, so the wait always ends), each cluster stores at most one partial and
stores it in its first unit, and every cluster's work is balanced."""
import itertools

import pytest

PAIR_M, BN, BK = 256, 256, 64


def walk(c, nclusters, tiles, kb, sk_tiles, sk_clusters):
    """Units of logical cluster c: (tile, kb0, kb1, kind, first_contrib)."""
    units = []
    sk_iters = sk_tiles * kb
    start = lambda i: i * sk_iters // sk_clusters
    lo, hi = (start(c), start(c + 1)) if c < sk_clusters else (0, 0)
    while hi > lo:
        t = (hi - 1) // kb
        t0 = t * kb
        b = max(lo, t0)
        kb0, kb1 = b - t0, hi - t0
        kind = "contrib" if kb1 < kb else ("owner" if kb0 > 0 else "whole")
        first = c
        if kind == "owner":
            first = c - 1
            while first > 0 and start(first) > t0:
                first -= 1
        units.append((t, kb0, kb1, kind, first))
        hi = b
    item = sk_tiles + c
    while item < tiles:
        units.append((item, 0, kb, "whole", c))
        item += nclusters
    return units


def check_walk(tiles, kb, sk_tiles, sk_clusters, nclusters):
    cover = {}
    per_cluster = []
    for c in range(nclusters):
        us = walk(c, nclusters, tiles, kb, sk_tiles, sk_clusters)
        per_cluster.append(sum(u[2] - u[1] for u in us))
        contribs = [i for i, u in enumerate(us) if u[3] == "contrib"]
        assert contribs in ([], [0]), (c, us)  # at most one partial, in the first unit
        for t, kb0, kb1, kind, first in us:
            assert 0 <= kb0 < kb1 <= kb
            for k in range(kb0, kb1):
                assert (t, k) not in cover
                cover[(t, k)] = (c, kind, first)
    assert len(cover) == tiles * kb
    # owners: exactly one per split tile, contributors are exactly the clusters first..owner-1
    for t in range(tiles):
        kinds = {cover[(t, k)] for k in range(kb)}
        clusters = sorted({x[0] for x in kinds})
        if len(clusters) == 1:
            assert all(x[1] == "whole" for x in kinds)
            continue
        owner = clusters[-1]
        assert all(x[1] == "owner" for x in kinds if x[0] == owner)
        assert all(x[1] == "contrib" for x in kinds if x[0] != owner)
        first = next(x[2] for x in kinds if x[0] == owner)
        assert clusters == list(range(first, owner + 1))
        assert cover[(t, kb - 1)][0] == owner
    # balance: stream-K ranges differ by at most one K-step
    sk = [min(per_cluster[c], 10**9) for c in range(min(sk_clusters, nclusters))]
    return per_cluster


def test_walk_invariants_exhaustive():
    for tiles, kb, csk in itertools.product(range(1, 40), (1, 2, 3, 7, 8, 64), (1, 2, 5, 13, 74)):
        for sk_tiles in {tiles, tiles % 7, min(tiles, 3)}:
            if sk_tiles == 0 or csk > sk_tiles * kb:
                continue
            nclusters = max(csk, min(74, tiles))
            check_walk(tiles, kb, sk_tiles, csk, nclusters)


@pytest.mark.parametrize("M,N,K", [(512, 12288, 4096), (128, 4096, 4096), (4096, 12288, 4096),
                                   (2048, 3584, 8192), (16384, 2048, 2048), (4096, 4096, 4096)])
def test_library_plan_walks_cleanly(mpk_lib, M, N, K):
    tiles, sk_tiles, sk_pairs = mpk_lib.gemm_plan(M, N, K)
    assert tiles == -(-M // PAIR_M) * -(-N // BN)
    kb = -(-K // BK)
    if sk_tiles:
        nclusters = max(sk_pairs, min(74, tiles))
        work = check_walk(tiles, kb, sk_tiles, sk_pairs, nclusters)
        # no cluster does more than the balanced share plus one K-step of the spread tiles
        waves = (tiles - sk_tiles) // 74
        assert max(work) <= waves * kb + -(-sk_tiles * kb // sk_pairs)


def test_plan_of_the_scaling_shapes(mpk_lib):
    """On 74 SM pairs: the dense projection on 4 GPUs (1024 rows each) has 192
    tiles, 2 full waves + 44; those 44 tiles' 2816 K-steps go to all 74 pairs.  The
    wide shape on 8 GPUs (3584 columns each): 1 wave of 128 K-steps + 38.  Products
    with no full wave, more than three, fewer than 128 whole K-steps per pair (the
    dense projection on 8 GPUs: 1 wave of 64), a last wave over 85 % full, whole
    waves only, or a spread that would leave under 8 K-steps per pair keep whole
    tiles."""
    assert mpk_lib.gemm_plan(1024, 12288, 4096) == (192, 44, 74)
    assert mpk_lib.gemm_plan(512, 12288, 4096) == (96, 0, 0)
    assert mpk_lib.gemm_plan(2048, 3584, 8192) == (112, 38, 74)
    assert mpk_lib.gemm_plan(128, 4096, 4096) == (16, 0, 0)       # no full wave
    assert mpk_lib.gemm_plan(4096, 12288, 4096) == (768, 0, 0)    # ten waves
    assert mpk_lib.gemm_plan(16384, 2048, 2048) == (512, 0, 0)    # last wave 68/74 full
    assert mpk_lib.gemm_plan(512, 512, 512) == (4, 0, 0)          # 32 K-steps: 4 per pair at most
    assert mpk_lib.gemm_plan(256, 256 * 74, 4096) == (74, 0, 0)   # one full wave
    prev = mpk_lib.set_gemm_schedule(mpk_lib.SCHEDULE_TILES)
    try:
        assert mpk_lib.gemm_plan(1024, 12288, 4096) == (192, 0, 0)
        mpk_lib.set_gemm_schedule(mpk_lib.SCHEDULE_STREAM_K)
        assert mpk_lib.gemm_plan(512, 512, 512) == (4, 4, 32)
    finally:
        mpk_lib.set_gemm_schedule(prev)
    assert mpk_lib.gemm_schedule() == prev


def test_workspace_size_includes_the_partials(mpk_lib):
    M, N, K = 1024, 12288, 4096
    base = M * K * 2
    size = mpk_lib.gemm_workspace_size(M, N, K)
    assert size >= base + 74 * 2 * 128 * 256 * 4
    prev = mpk_lib.set_gemm_schedule(mpk_lib.SCHEDULE_TILES)
    try:
        assert mpk_lib.gemm_workspace_size(M, N, K) == base
    finally:
        mpk_lib.set_gemm_schedule(prev)


def test_unknown_schedule_is_rejected(mpk_lib):
    with pytest.raises(mpk_lib.MpkError) as e:
        mpk_lib.set_gemm_schedule(7)
    assert e.value.status == mpk_lib.MPK_ERR_INVALID_VALUE
