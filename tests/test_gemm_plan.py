"""K3's launch plan on the host (zest_plan_gemm, no GPU): the tile order and
the stream-K split the launch makes for the configs' shapes, and the split's
invariants for any shape: the runs cover every (tile, k-block) once, every
tile cut into runs is finished by one pair that collects the partials of the
pairs before it, and the partial-sum workspace (160 CTA slots) suffices."""
import os
import sys

import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(__file__)), "ggml-xdna_b200"))
import zest_b200 as Z  # noqa: E402
from zest_b200.gemm_case import SHAPES  # noqa: E402

pytestmark = pytest.mark.skipif(any(os.environ.get(v) for v in ("ZEST_GEMM_SK", "ZEST_GEMM_BN", "ZEST_GEMM_PAIR",
                                                                  "ZEST_GEMM_RASTER")),
                                 reason="a tuning variable overrides the default plan")

SMS = 148
PAIRS = SMS // 2

# measured per launch on a B200 (device time, whole tiles -> stream-K): split
# where a quarter of the pair-slots sit idle at K >= 4096, or at K >= 8192
# with a full wave; whole tiles elsewhere
SPLIT = {"C3 o", "C3 down", "C2 down", "C5 m1024 down", "C4 m2048 down"}


@pytest.mark.parametrize("name", list(SHAPES))
def test_stream_k_where_it_measured_faster(name):
    M, Ns, K = SHAPES[name]
    p = Z.plan_gemm(M, K, Ns, SMS)
    assert p["pair_kernel"] == 1 and p["tile_n"] == 256 and p["k_blocks"] == K // 64
    assert p["tiles"] == (M + 255) // 256 * sum((N + 255) // 256 for N in Ns)
    assert bool(p["stream_k"]) == (name in SPLIT), p


def test_tile_order_keeps_the_reread_operand_in_l2():
    # rows: B (N x K) <= 60 MB and the smaller, read from L2 by every wave
    assert Z.plan_gemm(8192, 9728, [2560], SMS)["raster"] == 1
    # columns: A <= 60 MB (C1: A 5 MB, B 50 MB)
    assert Z.plan_gemm(1024, 2560, [9728], SMS)["raster"] == 2
    # groups of 8 tile rows: neither fits (C4 down: A 71 MB, B 178 MB)
    assert Z.plan_gemm(2048, 17408, [5120], SMS)["raster"] == 0


def test_rows_of_one_tile_take_the_one_cta_kernel():
    p = Z.plan_gemm(100, 512, [768, 300], SMS)
    assert p["pair_kernel"] == 0 and p["stream_k"] == 0
    assert p["tiles_m"] == 1 and p["tiles_n"] == 3 + 2 and p["ctas"] == 3


def test_small_launch_uses_only_the_pairs_it_needs():
    p = Z.plan_gemm(2048, 10752, [2048], SMS)  # 64 tiles, one partial wave, left whole
    assert p["stream_k"] == 0 and p["ctas"] == 2 * 64


def walk(p, pair):
    """The runs pair `pair` makes, in order: (tile, kb0, kb1). The device's
    unit_iter: the last run of its stream-K stretch, then its whole tiles,
    then the rest of the stretch from its end back to its start."""
    nk, q = p["k_blocks"], p["run_k_blocks"]
    end = p["split_tiles"] * nk
    u0 = min(pair * q, end)
    u1 = min(u0 + q, end)
    runs = []

    def take():
        nonlocal u1
        st = (u1 - 1) // nk
        start = max(u0, st * nk)
        runs.append((p["whole_tiles"] + st, start - st * nk, u1 - st * nk))
        u1 = start

    if u1 > u0:
        take()
    t = pair
    while t < p["whole_tiles"]:
        runs.append((t, 0, nk))
        t += PAIRS
    while u1 > u0:
        take()
    return runs


@pytest.mark.parametrize("M,N,K", [(2048, 2560, 4096), (1024, 2048, 10752), (8192, 2560, 9728), (2048, 5120, 17408),
                                   (3000, 700, 8192), (1024, 9728, 2560), (4096, 1000, 12800)])
def test_split_covers_every_unit_once_and_finishers_wait_only_on_first_runs(M, N, K):
    p = Z.plan_gemm(M, K, [N], SMS)
    if not p["stream_k"]:
        assert p["whole_tiles"] == p["tiles"] and p["split_tiles"] == 0
        return
    nk = p["k_blocks"]
    assert p["whole_tiles"] + p["split_tiles"] == p["tiles"] and p["whole_tiles"] % PAIRS == 0
    assert 2 * PAIRS <= 160, "a workspace slot per CTA"
    seen = {}
    first_run = {}
    for pair in range(PAIRS):
        runs = walk(p, pair)
        for i, (t, k0, k1) in enumerate(runs):
            assert 0 <= k0 < k1 <= nk
            for kb in range(k0, k1):
                assert (t, kb) not in seen, "a unit computed twice"
                seen[(t, kb)] = pair
            if k1 < nk:  # stops inside a tile: leaves a partial
                assert i == 0, "a partial comes from a pair's first run"
                first_run[pair] = t
    assert len(seen) == p["tiles"] * nk, "every (tile, k-block) computed"
    for t in range(p["whole_tiles"], p["tiles"]):
        owners = sorted({seen[(t, kb)] for kb in range(nk)})
        finisher = seen[(t, nk - 1)]
        assert finisher == owners[-1], "the pair with the tile's last k-block finishes it"
        for j in owners[:-1]:
            assert first_run.get(j) == t, "the finisher waits only on first runs"


def test_plan_refuses_bad_calls():
    for args in [(0, 512, [64]), (128, 0, [64]), (256, 512, []), (256, 512, [64] * 5), (256, 512, [0])]:
        with pytest.raises(Z.ZestError, match="zest_plan_gemm"):
            Z.plan_gemm(*args, sms=SMS)
