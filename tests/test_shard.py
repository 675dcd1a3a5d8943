"""Host-side logic of the M-row sharding (no GPU): partitions and the weight broadcast,
including two gloo ranks on CPU."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tensorforge_b200.shard import all_partitions, broadcast_weights, row_partition


@pytest.mark.parametrize("m", [0, 1, 7, 8, 1000, 131072, 131073])
@pytest.mark.parametrize("n", [1, 2, 3, 4, 8])
def test_partition_covers_rows_once(m, n):
    parts = all_partitions(m, n)
    assert parts[0][0] == 0 and parts[-1][1] == m
    for (a0, a1), (b0, _) in zip(parts, parts[1:]):
        assert a1 == b0 and a0 <= a1
    sizes = [r1 - r0 for r0, r1 in parts]
    assert max(sizes) - min(sizes) <= 1


def test_partition_matches_survey_formula():
    # cfg4: M = 131072 over 8 GPUs -> 16384 rows each; rank r starts at floor(r M / n).
    assert all_partitions(131072, 8) == [(r * 16384, (r + 1) * 16384) for r in range(8)]
    assert row_partition(10, 3, 1) == (3, 6)


@pytest.mark.parametrize("bad", [(10, 0, 0), (10, 2, 2), (-1, 2, 0), (10, 2, -1)])
def test_partition_rejects_bad_requests(bad):
    with pytest.raises(ValueError):
        row_partition(*bad)


def test_broadcast_is_noop_without_process_group():
    w, b = torch.ones(3, 4), torch.zeros(4)
    ws = broadcast_weights(w, b)
    assert ws.weight is w and ws.bias is b


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, m, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        k, n = 6, 5
        w = torch.arange(k * n, dtype=torch.float32).reshape(k, n) if rank == 0 else torch.full((k, n), -1.0)
        b = torch.arange(n, dtype=torch.float32) * 0.5 if rank == 0 else torch.full((n,), -1.0)
        ws = broadcast_weights(w, b, src=0)
        ok_w = bool(torch.equal(ws.weight, torch.arange(k * n, dtype=torch.float32).reshape(k, n)))
        ok_b = bool(torch.equal(ws.bias, torch.arange(n, dtype=torch.float32) * 0.5))
        r0, r1 = row_partition(m, world, rank)
        got = [None] * world
        dist.all_gather_object(got, (r0, r1))
        results[rank] = (ok_w, ok_b, got)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_broadcast_and_partition():
    world, m = 2, 1001
    port = _free_port()
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        procs = [ctx.Process(target=_rank_main, args=(r, world, port, m, results)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
        res = dict(results)
    assert set(res) == {0, 1}
    for rank in range(world):
        ok_w, ok_b, parts = res[rank]
        assert ok_w and ok_b
        assert parts == all_partitions(m, world)
