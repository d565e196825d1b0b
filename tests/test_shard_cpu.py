"""Batch sharding across ranks, tested with world_size-2 gloo process groups on CPU.

The scan itself is replaced by the oracle on each rank's rows (no GPU): the
tests check the split, the output assembly order, and that a failure on one
rank (a status flag or a host exception) reaches every rank before any rank
waits in the gather.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from saccade_v1_b200.shard import ShardFailure, gather_batch, run_sharded, shard_rows


def test_shard_rows_cover_the_batch():
    for batch in (0, 1, 7, 64, 65):
        for world in (1, 2, 3, 8):
            shards = [shard_rows(batch, world, r) for r in range(world)]
            assert shards[0].begin == 0 and shards[-1].end == batch
            for a, b in zip(shards, shards[1:]):
                assert a.end == b.begin
            assert max(s.size for s in shards) - min(s.size for s in shards) <= 1
            assert all(s.rows == max(x.size for x in shards) for s in shards)
    with pytest.raises(ValueError):
        shard_rows(4, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(batch):
    from oracle.oracle import Shape, random_case
    return random_case(Shape(batch, 9, 6, 4, 1, 1, True), 0x5eed0900)


def _scan_rows(k, begin, end):
    from oracle import oracle
    L, D, N = k.shape.length, k.shape.channels, k.shape.state
    sub = oracle.Case(oracle.Shape(end - begin, L, D, N, 1, 1, True), k.u.reshape(-1, L * D)[begin:end],
                      k.delta.reshape(-1, L * D)[begin:end], k.a, k.b.reshape(-1, L * N)[begin:end],
                      k.c.reshape(-1, L)[begin:end], k.d)
    return oracle.run(sub).reshape(end - begin, L, D)


def _worker(rank, world, port, batch, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        k = _case(batch)

        def scan_shard(shard):
            if mode == "raise" and rank == 1:
                raise RuntimeError("host-side failure on rank 1")
            y = torch.from_numpy(_scan_rows(k, shard.begin, shard.end))
            flags = 0x200 if (mode == "flag" and rank == 1) else 0
            return y, flags

        try:
            y = run_sharded(scan_shard, batch)
            q.put((rank, "ok", y.numpy()))
        except ShardFailure as e:
            q.put((rank, "failure", str(e)))
    finally:
        dist.destroy_process_group()


def _spawn(batch, mode, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, batch, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return sorted(out, key=lambda x: x[0])


@pytest.mark.parametrize("batch", [4, 5])
def test_two_ranks_assemble_the_full_output(batch):
    results = _spawn(batch, "ok")
    want = _scan_rows(_case(batch), 0, batch)
    for rank, status, y in results:
        assert status == "ok"
        assert np.array_equal(y, want), rank


@pytest.mark.parametrize("mode", ["flag", "raise"])
def test_failure_on_one_rank_reaches_every_rank(mode):
    results = _spawn(4, mode)
    assert [r[1] for r in results] == ["failure", "failure"]


def test_gather_batch_rejects_wrong_shard():
    from saccade_v1_b200.shard import Shard
    with pytest.raises(ValueError):
        gather_batch(torch.zeros(3, 2), Shard(0, 2, 0, 2, 2), 4)


def test_c_abi_shard_rows_matches_python_split():
    """sacc_shard_rows (include/sacc_shard.h) splits rows exactly as shard.shard_rows."""
    import ctypes

    from saccade_v1_b200 import _lib
    from saccade_v1_b200.shard import shard_rows
    L = _lib.load()
    r0, n = ctypes.c_uint64(0), ctypes.c_uint64(0)
    for total in (0, 1, 7, 64, 65, 511, 4096):
        for world in (1, 2, 3, 4, 8):
            for rank in range(world):
                assert L.sacc_shard_rows(total, world, rank, ctypes.byref(r0), ctypes.byref(n)) == _lib.SACC_OK
                s = shard_rows(total, world, rank)
                assert (r0.value, r0.value + n.value) == (s.begin, s.end), (total, world, rank)
    assert L.sacc_shard_rows(8, 2, 2, ctypes.byref(r0), ctypes.byref(n)) == _lib.SACC_EINVAL
    assert "rank must be in [0, world)" in _lib.last_error()
