"""The N>1 host logic on CPU: world_size-2 gloo ranks, each multiplying its
slab of weight rows (the oracle stands in for the GPU kernels), then the
all-gather of slab outputs rebuilds the full row-major product on every rank."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from zest_b200.shard import shard_rows, slab_width


def test_shards_cover_rows_exactly():
    for N in (1, 127, 128, 1024, 2560, 9728, 17408):
        for world in (1, 2, 4, 8):
            spans = [shard_rows(N, world, r) for r in range(world)]
            covered = []
            for lo, n in spans:
                covered.extend(range(lo, lo + n))
            assert covered == list(range(N)), (N, world)
            assert all(lo % 128 == 0 for lo, n in spans if n)
            assert slab_width(N, world) == max(n for _, n in spans)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, q, wire_bf16: bool = False):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "ggml-xdna_b200")]
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    from oracle import oracle as O
    from zest_b200.shard import gather_slabs, shard_rows, slab_width

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        M, N, K = 64, 1000, 256
        raw = O.quantize(O.Q8_0, O.weights_f32(N, K, 1))
        W = O.dequant(O.Q8_0, raw, N, K)
        X = O.activations(M, K, 2)
        lo, n = shard_rows(N, world, rank)
        w = slab_width(N, world)
        slab = torch.zeros((M, w), dtype=torch.float32)
        rounded = O.round_bf16 if wire_bf16 else (lambda a: a)  # the GEMM's default bf16-rounded output
        if n:
            slab[:, :n] = torch.from_numpy(rounded(O.mul_mat(W[lo:lo + n], X)))
        full = torch.full((M, N), float("nan"))
        gather_slabs(slab, full, world, N, wire=torch.bfloat16 if wire_bf16 else None)
        want = rounded(O.mul_mat(W, X))
        q.put((rank, bool(np.array_equal(full.numpy(), want))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("wire_bf16", [False, True])
def test_gather_rebuilds_row_major_product_gloo(wire_bf16):
    # with bf16-rounded results, bf16 slabs on the wire rebuild them exactly
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q, wire_bf16)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    results = dict(q.get(timeout=10) for _ in range(world))
    assert all(p.exitcode == 0 for p in procs)
    assert results == {0: True, 1: True}


def test_k_shards_cover_columns_exactly():
    from zest_b200.shard import shard_cols
    for K in (64, 2560, 9728, 17408):
        for world in (1, 2, 4, 8):
            spans = [shard_cols(K, world, r) for r in range(world)]
            covered = []
            for k0, k in spans:
                covered.extend(range(k0, k0 + k))
            assert covered == list(range(K)), (K, world)
            assert all(k0 % 64 == 0 and k % 64 == 0 for k0, k in spans if k)


def _tp_rank(rank: int, world: int, port: int, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "ggml-xdna_b200")]
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    from oracle import oracle as O
    from zest_b200.shard import all_reduce_rows, shard_cols

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        # the down projection of a tensor-parallel FFN: each rank holds a column
        # slab of the input (the N-sharded SwiGLU) and the same slab of the
        # weight; the row chunks of the partial products are all-reduced one by one
        M, N, K, chunk = 96, 320, 1024, 32
        W = O.dequant(O.Q8_0, O.quantize(O.Q8_0, O.weights_f32(N, K, 3)), N, K)
        X = O.activations(M, K, 4)
        k0, k = shard_cols(K, world, rank)
        part = torch.from_numpy(O.mul_mat(W[:, k0:k0 + k], X[:, k0:k0 + k]))
        works = [all_reduce_rows(part, r0, min(chunk, M - r0)) for r0 in range(0, M, chunk)]
        for w in works:
            w.wait()
        want = O.mul_mat(W, X)
        err = float(np.max(np.abs(part.numpy() - want)) / np.max(np.abs(want)))
        q.put((rank, err < 1e-5))
    finally:
        dist.destroy_process_group()


def test_k_sharded_partials_sum_to_the_product_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    results = dict(q.get(timeout=10) for _ in range(world))
    assert all(p.exitcode == 0 for p in procs)
    assert results == {0: True, 1: True}


def _any_rank_rank(rank: int, world: int, port: int, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "ggml-xdna_b200")]
    from datetime import timedelta

    import torch.distributed as dist

    from zest_b200.shard import any_rank

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        # a failure seen by rank 1 alone sends every rank down the error path,
        # and after it every rank still meets the next collective
        seen = [any_rank(False), any_rank(rank == 1), any_rank(True)]
        dist.barrier()
        q.put((rank, seen))
    finally:
        dist.destroy_process_group()


def test_ranks_take_an_error_path_together_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_any_rank_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    results = dict(q.get(timeout=10) for _ in range(world))
    assert all(p.exitcode == 0 for p in procs)
    assert results == {0: [False, True, True], 1: [False, True, True]}


def test_any_rank_without_a_process_group():
    from zest_b200.shard import any_rank
    assert any_rank(True) is True and any_rank(False) is False
