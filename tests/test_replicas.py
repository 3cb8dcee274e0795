"""Host logic of the data-parallel replicas (no GPU): batch slicing, concurrent replica runs
against fake models, and the one-process-per-rank group over ``gloo`` with world size 2 (the
barrier and the max-over-ranks timing reduction that ``bench.py`` uses under torchrun)."""

from __future__ import annotations

import os
import socket
import threading

import numpy as np
import pytest

from mgc_cuda.replicas import ReplicaGroup, ReplicaSet, shard


@pytest.mark.parametrize("total,world", [(0, 1), (7, 1), (8, 2), (9, 2), (3, 4), (256, 8), (1001, 3)])
def test_shard_covers_every_row_once(total: int, world: int) -> None:
    seen = []
    for rank in range(world):
        start, count = shard(total, world, rank)
        seen.extend(range(start, start + count))
    assert seen == list(range(total))
    counts = [shard(total, world, r)[1] for r in range(world)]
    assert max(counts) - min(counts) <= 1


def test_shard_rejects_bad_ranks() -> None:
    with pytest.raises(ValueError):
        shard(8, 2, 2)
    with pytest.raises(ValueError):
        shard(8, 0, 0)
    with pytest.raises(ValueError):
        shard(-1, 2, 0)


class _FakeModel:
    """Doubles its input and records the thread it ran on."""

    def __init__(self, tag: float) -> None:
        self.tag = tag
        self.threads: list[int] = []
        self.closed = False

    def run(self, feeds):  # noqa: ANN001, ANN201
        self.threads.append(threading.get_ident())
        x = feeds["x"]
        return {"y": x * 2.0, "who": np.full((x.shape[0], 1), self.tag, np.float32)}

    def close(self) -> None:
        self.closed = True


def test_replica_set_splits_and_concatenates_in_device_order() -> None:
    models = [_FakeModel(float(i)) for i in range(4)]
    rs = ReplicaSet(models)
    x = np.arange(8 * 3, dtype=np.float32).reshape(8, 3)
    out = rs.run({"x": x})
    np.testing.assert_array_equal(out["y"], x * 2.0)
    np.testing.assert_array_equal(out["who"][:, 0], [0, 0, 1, 1, 2, 2, 3, 3])
    assert all(len(m.threads) == 1 for m in models)
    rs.close()
    assert all(m.closed for m in models)


def test_replica_set_refuses_a_batch_that_does_not_split() -> None:
    rs = ReplicaSet([_FakeModel(0.0), _FakeModel(1.0)])
    with pytest.raises(ValueError, match="does not split"):
        rs.run({"x": np.zeros((3, 2), np.float32)})
    rs.close()


def test_single_process_group_is_a_no_op(monkeypatch: pytest.MonkeyPatch) -> None:
    monkeypatch.setenv("WORLD_SIZE", "1")
    monkeypatch.setenv("RANK", "0")
    g = ReplicaGroup(backend="gloo")
    g.barrier()
    assert g.max(3.5) == 3.5
    g.close()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return int(s.getsockname()[1])


def _rank_main(rank: int, world: int, port: int, q) -> None:  # noqa: ANN001
    os.environ.update({"WORLD_SIZE": str(world), "RANK": str(rank), "LOCAL_RANK": str(rank),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    try:
        g = ReplicaGroup(backend="gloo", timeout_s=30)
        start, count = shard(256, g.world, g.rank)
        g.barrier()
        slowest = g.max(10.0 + g.rank)  # per-rank "elapsed ms"
        g.close()
        q.put((rank, start, count, slowest))
    except Exception as exc:  # pragma: no cover - reported through the queue
        q.put((rank, "error", repr(exc), None))


def test_two_rank_group_over_gloo() -> None:
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results == [(0, 0, 128, 11.0), (1, 128, 128, 11.0)]
