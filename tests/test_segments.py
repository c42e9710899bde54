"""Host logic of the batched-segment multi-GPU mode on CPU: the static
partition, micro-batching, and the ordered gather over a 2-rank gloo process
group (no GPU: the engine is replaced by a deterministic stand-in)."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from qwenasr_b200 import segments


@pytest.mark.parametrize("n,world", [(64, 1), (64, 2), (64, 8), (7, 3), (3, 8), (0, 2)])
def test_partition_is_even_and_complete(n, world):
    ranges = [segments.segment_range(n, r, world) for r in range(world)]
    flat = [s for r in ranges for s in r]
    assert flat == list(range(n))
    sizes = [len(r) for r in ranges]
    assert max(sizes) - min(sizes) <= 1


def test_partition_rejects_bad_requests():
    with pytest.raises(ValueError):
        segments.segment_range(8, 2, 2)
    with pytest.raises(ValueError):
        segments.segment_range(8, 0, 0)


def _fake_decode(segs):
    # stand-in for decode_batch: ids that encode (segment, step)
    return [[1000 * s + k for k in range(3)] for s in segs]


def test_micro_batches_cover_rank_share():
    res = segments.run_rank(_fake_decode, 20, 8, rank=1, world=3)
    assert sorted(res) == list(segments.segment_range(20, 1, 3))
    assert res[7] == [7000, 7001, 7002]


def test_single_process_gather():
    res = segments.run_rank(_fake_decode, 5, 2, 0, 1)
    out = segments.gather_in_order(res, 5)
    assert out == [[1000 * s + k for k in range(3)] for s in range(5)]
    with pytest.raises(RuntimeError, match="missing"):
        segments.gather_in_order({0: [1]}, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        local = segments.run_rank(_fake_decode, n, 4, rank, world)
        out = segments.gather_in_order(local, n, dist)
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_gather_in_segment_order():
    world, n = 2, 13
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got[1] is None
    assert got[0] == [[1000 * s + k for k in range(3)] for s in range(n)]
