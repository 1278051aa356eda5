"""Host side of the replicas-only multi-GPU path (ppocr_b200/replicas.py),
on CPU: contiguous sharding, the per-replica thread pool with failure
detection (a replica that raises, one that hangs), and the torch.distributed
helpers bench.py uses, over world_size-2 `gloo` process groups. The work of a
replica is the CTC collapse of its shard (oracle C restatement), so a sharded
run must reproduce the single-replica result bit for bit."""

import ctypes
import datetime
import os
import socket
import threading
from pathlib import Path

import numpy as np
import pytest
import torch.multiprocessing as mp

from helpers import rng

REPO = Path(__file__).resolve().parents[1]


def _collapse(lib, ids, probs, T):
    lines = ids.shape[0]
    o_ids = np.empty((lines, T), np.int32)
    o_len = np.empty(lines, np.int32)
    o_sc = np.empty(lines, np.float32)
    ids = np.ascontiguousarray(ids, np.int32)
    probs = np.ascontiguousarray(probs, np.float32)
    lib.oracle_ctc_collapse(ids.ctypes.data, probs.ctypes.data, lines, T, 0, o_ids.ctypes.data,
                            o_len.ctypes.data, o_sc.ctypes.data)
    return o_ids, o_len, o_sc


def _frames(seed, lines, T=40):
    r = rng(seed)
    ids = r.integers(0, 6, (lines, T)).astype(np.int32)
    probs = r.random((lines, T)).astype(np.float32)
    return ids, probs


@pytest.mark.parametrize("total", [0, 1, 7, 512, 513])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shard_partitions_contiguously(total, world):
    from ppocr_b200.replicas import shard

    spans = [shard(total, r, world) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == total
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1


def test_shard_rejects_bad_requests():
    from ppocr_b200.replicas import shard

    for args in [(10, 2, 2), (10, -1, 2), (10, 0, 0), (-1, 0, 1)]:
        with pytest.raises(ValueError):
            shard(*args)


def test_pool_matches_single_replica(oracle_c):
    from ppocr_b200.replicas import ReplicaPool, concat_tokens, tokens_digest

    ids, probs = _frames(90, 301)
    want = _collapse(oracle_c, ids, probs, 40)
    res = ReplicaPool(4, deadline_s=30).run(301, lambda i, a, b: _collapse(oracle_c, ids[a:b], probs[a:b], 40))
    assert res.ok
    got = concat_tokens(res.outputs)
    for g, w in zip(got, want):
        assert np.array_equal(g, w)
    assert tokens_digest(*got) == tokens_digest(*want)


def test_pool_reports_failing_replica_and_keeps_the_others(oracle_c):
    from ppocr_b200.replicas import ReplicaPool

    ids, probs = _frames(91, 64)

    def work(i, a, b):
        if i == 1:
            raise RuntimeError("device lost")
        return _collapse(oracle_c, ids[a:b], probs[a:b], 40)

    res = ReplicaPool(3, deadline_s=30).run(64, work)
    assert [(f.replica, f.kind) for f in res.failures] == [(1, "error")]
    assert "device lost" in res.failures[0].message
    assert res.outputs[1] is None
    want = _collapse(oracle_c, ids, probs, 40)
    for i in (0, 2):
        from ppocr_b200.replicas import shard

        a, b = shard(64, i, 3)
        assert np.array_equal(res.outputs[i][0], want[0][a:b])


def test_pool_reports_hung_replica_within_deadline(oracle_c):
    from ppocr_b200.replicas import ReplicaPool

    ids, probs = _frames(92, 40)
    release = threading.Event()

    def work(i, a, b):
        if i == 2:
            release.wait(30)  # hangs until the test lets it go
        return _collapse(oracle_c, ids[a:b], probs[a:b], 40)

    try:
        res = ReplicaPool(4, deadline_s=0.5).run(40, work)
    finally:
        release.set()
    assert [(f.replica, f.kind) for f in res.failures] == [(2, "timeout")]
    assert all(res.outputs[i] is not None for i in (0, 1, 3))


# ----------------------------------------------------- gloo, world_size 2
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=20):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _oracle_lib():
    lib = ctypes.CDLL(str(REPO / "oracle" / "_build" / "liboracle.so"))
    P = ctypes.c_void_p
    lib.oracle_ctc_collapse.argtypes = [P, P, ctypes.c_long, ctypes.c_int, ctypes.c_int, P, P, P]
    return lib


def _rank_sharded(rank, world, port, out_dir):
    import sys

    sys.path.insert(0, str(REPO / "ppocrv6-native-server_b200"))
    import torch.distributed as dist

    from ppocr_b200.replicas import all_equal_over_ranks, max_over_ranks, shard, tokens_digest

    _init(rank, world, port)
    lib = _oracle_lib()
    ids, probs = _frames(93, 130)
    a, b = shard(130, rank, world)
    part = _collapse(lib, ids[a:b], probs[a:b], 40)
    gathered = [None] * world
    dist.all_gather_object(gathered, part)
    m = max_over_ranks(float(rank + 1))
    same = all_equal_over_ranks(tokens_digest(*_collapse(lib, ids, probs, 40)))
    if rank == 0:
        np.savez(Path(out_dir) / "r0.npz", ids=np.concatenate([g[0] for g in gathered]),
                 lens=np.concatenate([g[1] for g in gathered]), sc=np.concatenate([g[2] for g in gathered]),
                 m=np.array([m]), same=np.array([same]))
    dist.destroy_process_group()


def test_gloo_two_ranks_shard_and_gather(tmp_path, oracle_c):
    port = _free_port()
    mp.start_processes(_rank_sharded, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn", join=True)
    got = np.load(tmp_path / "r0.npz")
    ids, probs = _frames(93, 130)
    want = _collapse(oracle_c, ids, probs, 40)
    assert np.array_equal(got["ids"], want[0])
    assert np.array_equal(got["lens"], want[1])
    assert np.array_equal(got["sc"], want[2])
    assert got["m"][0] == 2.0 and bool(got["same"][0])


def _rank_one_leaves(rank, world, port, out_dir):
    import sys

    sys.path.insert(0, str(REPO / "ppocrv6-native-server_b200"))
    import torch.distributed as dist

    from ppocr_b200.replicas import max_over_ranks

    _init(rank, world, port, timeout_s=5)
    max_over_ranks(1.0)  # step 1: both ranks take part
    if rank == 1:
        os._exit(0)  # leaves between steps, nothing in flight
    try:
        max_over_ranks(2.0)  # step 2: the peer is gone
        outcome = "no error"
    except Exception as e:  # noqa: BLE001 - the detection under test
        outcome = f"detected: {type(e).__name__}"
    (Path(out_dir) / "r0.txt").write_text(outcome)
    os._exit(0)


def test_gloo_rank_that_leaves_is_detected_by_the_next_collective(tmp_path):
    port = _free_port()
    ctx = mp.start_processes(_rank_one_leaves, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn",
                             join=False)
    for p in ctx.processes:
        p.join(60)
    assert all(not p.is_alive() for p in ctx.processes)
    assert (tmp_path / "r0.txt").read_text().startswith("detected")
