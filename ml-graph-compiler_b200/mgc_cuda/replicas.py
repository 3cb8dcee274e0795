"""Data-parallel replicas: the multi-GPU form of the cuda target.

Inference over a batch has no exchange step, so nothing is sharded inside a graph: every GPU holds
a whole replica (its own arena, resident weights and CUDA Graph) and runs its own slice of the
batch. The reference runs one compiled model per host process; its latency harness starts one
worker process per measurement cell (``benchmarks/latency.py:112-150``). Two ways to run replicas
here:

* one process per GPU (``torchrun``): ``shard(total, world, rank)`` names each rank's rows and
  ``ReplicaGroup`` holds the process group that is used only for the barrier around a timed
  region and the max-over-ranks reduction of its elapsed time — no collective touches the data;
* several GPUs from one process: ``ReplicaSet`` splits every input along axis 0, runs each
  replica from its own host thread (the C ABI releases the GIL), and concatenates the outputs in
  device order.
"""

from __future__ import annotations

import datetime
import os
from collections.abc import Callable, Mapping, Sequence
from concurrent.futures import ThreadPoolExecutor
from typing import Any, Protocol

import numpy as np


def shard(total: int, world: int, rank: int) -> tuple[int, int]:
    """(first row, row count) of ``rank``'s contiguous slice of ``total`` rows over ``world``
    ranks; the first ``total % world`` ranks take one extra row."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if total < 0:
        raise ValueError(f"negative row count {total}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


class _Runnable(Protocol):
    def run(self, feeds: Mapping[str, np.ndarray]) -> dict[str, np.ndarray]: ...


class ReplicaSet:
    """Equal-batch replicas of one model on several devices of this process.

    Every replica is compiled for the same per-device batch, so a call's batch must be that
    batch times the number of replicas; each replica gets one contiguous slice."""

    def __init__(self, models: Sequence[_Runnable], batch_axis: int = 0) -> None:
        if not models:
            raise ValueError("a ReplicaSet needs at least one model")
        self.models = list(models)
        self.batch_axis = batch_axis
        self._pool = ThreadPoolExecutor(max_workers=len(self.models))

    @classmethod
    def compile(cls, build: Callable[[int], Any], per_device_batch: int, devices: Sequence[int],
                **compile_kwargs: Any) -> ReplicaSet:
        """``build(batch)`` returns an optimised, scheduled reference graph for ``batch`` rows;
        one copy is lowered and loaded on each device."""
        from mgc_cuda.runtime import compile_graph

        return cls([compile_graph(build(per_device_batch), device=d, **compile_kwargs) for d in devices])

    def split(self, feeds: Mapping[str, np.ndarray]) -> list[dict[str, np.ndarray]]:
        """Each replica's feeds: every input cut into ``len(models)`` equal slices on the batch axis."""
        n = len(self.models)
        parts: list[dict[str, np.ndarray]] = [{} for _ in range(n)]
        for name, value in feeds.items():
            a = np.asarray(value)
            rows = a.shape[self.batch_axis]
            if rows % n:
                raise ValueError(f"input {name!r}: batch {rows} does not split over {n} replicas")
            for r in range(n):
                start, count = shard(rows, n, r)
                index = [slice(None)] * a.ndim
                index[self.batch_axis] = slice(start, start + count)
                parts[r][name] = np.ascontiguousarray(a[tuple(index)])
        return parts

    def run(self, feeds: Mapping[str, np.ndarray]) -> dict[str, np.ndarray]:
        """Run all replicas concurrently and concatenate their outputs in device order."""
        parts = self.split(feeds)
        results = list(self._pool.map(lambda mp: mp[0].run(mp[1]), zip(self.models, parts)))
        return {name: np.concatenate([r[name] for r in results], axis=self.batch_axis) for name in results[0]}

    def close(self) -> None:
        self._pool.shutdown(wait=True)
        for m in self.models:
            close = getattr(m, "close", None)
            if close is not None:
                close()


class ReplicaGroup:
    """The process group of a one-process-per-GPU run, read from the torchrun environment
    (``WORLD_SIZE``, ``RANK``, ``LOCAL_RANK``). With one process no group is created. The group
    carries only the barrier around a timed region and ``max`` of a per-rank timing; it is made
    with a short timeout so ranks that lose a peer end with an error instead of waiting."""

    def __init__(self, backend: str = "nccl", timeout_s: float = 300.0) -> None:
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.backend = backend
        self._dist: Any = None
        if self.world > 1:
            import torch
            import torch.distributed as dist

            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            kwargs: dict[str, Any] = {"timeout": datetime.timedelta(seconds=timeout_s)}
            if backend == "nccl":
                kwargs["device_id"] = torch.device("cuda", self.local_rank)
            dist.init_process_group(backend, **kwargs)
            self._dist = dist

    def _device(self) -> str:
        return f"cuda:{self.local_rank}" if self.backend == "nccl" else "cpu"

    def barrier(self) -> None:
        """Synchronise this GPU (when the backend is NCCL) and then every rank."""
        if self.backend == "nccl":
            import torch

            torch.cuda.synchronize()
        if self._dist is not None:
            self._dist.barrier()
            if self.backend == "nccl":
                import torch

                torch.cuda.synchronize()

    def max(self, value: float) -> float:
        """The largest ``value`` over all ranks (the job's time is its slowest rank's)."""
        if self._dist is None:
            return float(value)
        import torch

        t = torch.tensor([float(value)], dtype=torch.float64, device=self._device())
        self._dist.all_reduce(t, op=self._dist.ReduceOp.MAX)
        return float(t.item())

    def close(self) -> None:
        if self._dist is not None:
            self._dist.barrier()
            self._dist.destroy_process_group()
            self._dist = None
