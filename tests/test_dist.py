"""Multi-rank host logic on CPU: two gloo ranks run the same aggregation
code that bench.py and the sharded CLI run over NCCL on GPUs."""
import os
import socket

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

from mlpgemm import dist_util as DU  # noqa: E402
from mlpgemm.shard import shard_plan  # noqa: E402


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # each rank "timed" a different total; the job time is the slowest
        total = 10.0 + 5.0 * rank
        mx = DU.reduce_max(dist, total, "cpu")
        ok = DU.reduce_all(dist, rank != 1 or True, "cpu")
        bad = DU.reduce_all(dist, rank == 0, "cpu")     # one rank failed its check
        rate = DU.weak_scaling_rate(2.0 * 4096 ** 3, world, 100, mx)
        out[rank] = (mx, ok, bad, rate)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_aggregate():
    world = 2
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(world, _free_port(), out), nprocs=world, join=True)
    for r in range(world):
        mx, ok, bad, rate = out[r]
        assert mx == 15.0
        assert ok is True and bad is False
        assert rate == pytest.approx(2.0 * 4096 ** 3 * 2 * 100 / 0.015 / 1e12)


def _rows_reduce_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        def measure(key):
            if key == "a":                      # both ranks fine: the job takes the slower
                return 1.0 + rank, True, 1e-4 * (rank + 1)
            if key == "b" and rank == 1:        # this rank's run fails outright
                raise RuntimeError("boom on rank 1\nsecond line")
            if key == "c" and rank == 0:        # this rank's parity check fails
                return 0.5, False, 0.25
            return 0.5, True, 0.0
        out[rank] = DU.reduce_rows(dist, "cpu", ["a", "b", "c", "d"], measure)
        dist.barrier()   # every rank reached here: no collective was skipped
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_reduce_rows_with_a_failing_rank():
    # the per-dtype rows of bench.py's sharded suite: one all-reduce per row
    # on every rank, even where one rank's run raised or failed its check
    world = 2
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_rows_reduce_worker, args=(world, _free_port(), out), nprocs=world, join=True)
    inf = float("inf")
    for r in range(world):
        a, b, c, d = out[r]
        assert a == (2.0, 2e-4, True, "")
        assert b[:3] == (inf, inf, False)
        assert b[3] == ("boom on rank 1" if r == 1 else "")
        assert c[:3] == (0.5, inf, False) and c[3] == ""
        assert d == (0.5, 0.0, True, "")


def test_shard_plan_covers_columns():
    for M in (4096, 11008, 1000, 33):
        for G in (1, 2, 4, 8):
            plan = shard_plan(M, G)
            assert len(plan) == G
            assert sum(w for _, w in plan) == M
            pos = 0
            for m0, w in plan:
                assert m0 == pos or w == 0
                pos = m0 + w
                if G > 1 and w and m0 + w < M:
                    assert w % 32 == 0
    assert shard_plan(11008, 8) == [(i * 1376, 1376) for i in range(8)]


def test_pipeline_row_chunks():
    from mlpgemm.shard import row_chunks
    for N in (1, 100, 128, 129, 2048, 4096, 1000):
        for c in (1, 2, 4, 8):
            parts = row_chunks(N, c)
            assert parts[0][0] == 0 and parts[-1][1] == N
            assert all(a < b for a, b in parts)
            assert all(parts[i][1] == parts[i + 1][0] for i in range(len(parts) - 1))
            assert all((b - a) % 128 == 0 for a, b in parts[:-1])
            assert len(parts) <= max(1, c)
    assert row_chunks(2048, 4) == [(0, 512), (512, 1024), (1024, 1536), (1536, 2048)]


def test_strong_scaling_rate():
    assert DU.strong_scaling_rate(2.0, 1.0) == pytest.approx(2e-9)


def test_row_blocks_cover_rows():
    from mlpgemm.shard import row_blocks
    for N in (1, 7, 16, 100, 128, 300, 1000, 2048, 4096):
        for G in (1, 2, 4, 8):
            for c in (1, 2, 4):
                ch, rounds, blocks = row_blocks(N, G, c)
                assert len(blocks) == G and all(len(b) == rounds for b in blocks)
                seen = []
                for g in range(G):
                    for k, (r0, h) in enumerate(blocks[g]):
                        assert 0 <= h <= ch
                        if h:   # a block sits at its own rows of the round
                            assert r0 == k * G * ch + g * ch
                            seen += range(r0, r0 + h)
                assert sorted(seen) == list(range(N))
                if ch > 128:
                    assert ch % 128 == 0
                if rounds > 1:
                    assert ch >= 128
    assert row_blocks(2048, 8, 1)[:2] == (256, 1)
    assert row_blocks(2048, 2, 4)[:2] == (256, 4)
    assert row_blocks(2048, 8, 4)[:2] == (128, 2)


def _rows_worker(rank, world, port, out):
    """Each rank computes its block-cyclic rows of Y = X @ W and gathers the
    rounds in place; the result must be X @ W with no permute."""
    from mlpgemm.shard import gather_round, row_blocks
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        res = {}
        for N, chunks in ((300, 1), (1024, 4), (5, 1), (1000, 2)):
            g = torch.Generator().manual_seed(N)
            X = torch.randint(-8, 8, (N, 24), generator=g, dtype=torch.int64)
            W = torch.randint(-8, 8, (24, 40), generator=g, dtype=torch.int64)
            ch, rounds, blocks = row_blocks(N, world, chunks)
            Y = torch.zeros(rounds * world * ch, 40, dtype=torch.int64)
            for c, (r0, h) in enumerate(blocks[rank]):
                if h:
                    Y[c * world * ch + rank * ch:c * world * ch + rank * ch + h] = X[r0:r0 + h] @ W
                gather_round(dist, Y, c, world, rank, ch)
            res[(N, chunks)] = bool(torch.equal(Y[:N], X @ W))
        out[rank] = res
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_row_shard_gather_in_place():
    world = 2
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_rows_worker, args=(world, _free_port(), out), nprocs=world, join=True)
    for r in range(world):
        assert all(out[r].values()), out[r]


def test_rank_rows_block_cyclic_with_padding():
    import numpy as np
    from mlpgemm.shard import _rank_rows, row_blocks
    N, row_bytes = 1000, 6
    # 16-bit values, distinct per row, seen as rows of 2 * row_bytes bytes
    X = (np.arange(N)[:, None] * 7 + np.arange(row_bytes)[None, :]).astype(np.uint16).view(np.uint8)
    rb = 2 * row_bytes
    for world, chunks in ((2, 2), (4, 1), (3, 2)):
        ch, rounds, blocks = row_blocks(N, world, chunks)
        for g in range(world):
            out = _rank_rows(X, rb, blocks[g], ch).reshape(rounds, ch, rb)
            for c, (r0, h) in enumerate(blocks[g]):
                assert np.array_equal(out[c, :h], X.reshape(N, rb)[r0:r0 + h])
                assert not out[c, h:].any()   # zero past N
