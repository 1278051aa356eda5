"""Request-batch data parallelism over GPU replicas (host side).

The layer path has no exchange step: every GPU holds its own weights, arena,
CUDA graph and head, and recognizes its own contiguous slice of the lines
(replicas only, no collective on the data path). This module holds the host
logic around that:

* `shard`: the contiguous slice of a batch a replica owns;
* `ReplicaPool`: one host thread per replica, as the reference's workers
  drive their devices (recognition_worker.cpp:700-746), with failure
  detection: a replica that raises, or that does not finish within the
  deadline, is reported by index while the others' results are kept;
* `max_over_ranks`, `tokens_digest`, `all_equal_over_ranks`: the
  torch.distributed helpers bench.py uses (timing is the max over ranks;
  decoded tokens are compared across replicas by digest).
"""

from __future__ import annotations

import hashlib
import threading
import time
from dataclasses import dataclass, field
from typing import Any, Callable, Sequence

import numpy as np


def shard(total: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of rank's contiguous slice; sizes differ by at most one
    (the first total % world ranks take one more)."""
    if world < 1 or not 0 <= rank < world or total < 0:
        raise ValueError(f"bad shard request total={total} rank={rank} world={world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


@dataclass
class ReplicaFailure:
    replica: int
    kind: str  # "error" or "timeout"
    message: str


@dataclass
class PoolResult:
    outputs: list[Any]  # per replica; None where the replica failed
    failures: list[ReplicaFailure] = field(default_factory=list)

    @property
    def ok(self) -> bool:
        return not self.failures


class ReplicaPool:
    """Runs `work(replica, start, stop)` for every replica on its own host
    thread and waits at most `deadline_s` for all of them.

    A replica that raises is reported as "error" with its message; one that
    is still running at the deadline is reported as "timeout" (its thread is
    left to finish or hang on its own: a host thread cannot be killed, and
    the device work it drives is bounded by its kernels' own wait limits).
    Results of the replicas that finished are returned either way.
    """

    def __init__(self, replicas: int, deadline_s: float = 60.0):
        if replicas < 1:
            raise ValueError("replicas must be >= 1")
        self.replicas = replicas
        self.deadline_s = deadline_s

    def run(self, total: int, work: Callable[[int, int, int], Any]) -> PoolResult:
        outputs: list[Any] = [None] * self.replicas
        errors: dict[int, str] = {}
        done = [threading.Event() for _ in range(self.replicas)]

        def body(i: int) -> None:
            start, stop = shard(total, i, self.replicas)
            try:
                outputs[i] = work(i, start, stop)
            except BaseException as e:  # noqa: BLE001 - reported, not swallowed
                errors[i] = f"{type(e).__name__}: {e}"
            finally:
                done[i].set()

        threads = [threading.Thread(target=body, args=(i,), daemon=True, name=f"replica-{i}")
                   for i in range(self.replicas)]
        for t in threads:
            t.start()
        end = time.monotonic() + self.deadline_s
        for ev in done:
            ev.wait(max(0.0, end - time.monotonic()))
        failures = []
        for i in range(self.replicas):
            if not done[i].is_set():
                failures.append(ReplicaFailure(i, "timeout", f"replica {i} did not finish within "
                                                             f"{self.deadline_s:g} s"))
                outputs[i] = None
            elif i in errors:
                failures.append(ReplicaFailure(i, "error", errors[i]))
                outputs[i] = None
        return PoolResult(outputs, failures)


def concat_tokens(parts: Sequence[tuple[np.ndarray, np.ndarray, np.ndarray]]):
    """Joins per-replica (ids [n,T], lengths [n], scores [n]) in replica order."""
    ids = np.concatenate([p[0] for p in parts], axis=0)
    lens = np.concatenate([p[1] for p in parts], axis=0)
    scores = np.concatenate([p[2] for p in parts], axis=0)
    return ids, lens, scores


def tokens_digest(ids: np.ndarray, lens: np.ndarray, scores: np.ndarray) -> str:
    """SHA-256 over the decoded lines (kept ids only, lengths, score bits)."""
    h = hashlib.sha256()
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    lens = np.ascontiguousarray(lens, dtype=np.int32)
    for row, n in zip(ids, lens):
        h.update(row[:n].tobytes())
    h.update(lens.tobytes())
    h.update(np.ascontiguousarray(scores, dtype=np.float32).tobytes())
    return h.hexdigest()


def max_over_ranks(value: float, device=None) -> float:
    """Max of a float over all ranks of the default process group (the
    value itself without one)."""
    import torch
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def all_equal_over_ranks(digest: str) -> bool:
    """True when every rank passed the same digest (collective call)."""
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return True
    got: list[Any] = [None] * dist.get_world_size()
    dist.all_gather_object(got, digest)
    return all(g == got[0] for g in got)
