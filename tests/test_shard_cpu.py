"""Sequence sharding of a batch over ranks (host logic), with world_size-2 gloo process groups on
the CPU: the partition, the gathered result against a single-process run, and a failing rank."""
import multiprocessing as mp
import os
import socket
import sys

import numpy as np
import pytest

from gten_b200.shard import generate_sharded, shard_range

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


class FakeModel:
    """Deterministic stand-in for Model.generate_batch: id = f(prompt row, step)."""

    def generate_batch(self, prompts, n_gen):
        p = np.asarray(prompts, np.int64)
        base = (p.sum(axis=1) * 7 + p[:, 0]) % 32000
        return ((base[:, None] + 31 * np.arange(n_gen)[None, :]) % 32000).astype(np.int32)


class FailingModel(FakeModel):
    def generate_batch(self, prompts, n_gen):
        raise RuntimeError("injected failure on this rank")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, batch, n_gen, fail_rank, q):
    sys.path.insert(0, os.path.join(ROOT, "nanochatllms.cpp_b200"))
    import datetime

    import torch.distributed as dist

    from gten_b200.shard import generate_sharded as gen
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
        prompts = np.random.default_rng(5).integers(0, 32000, (batch, 9)).astype(np.int32)
        model = FailingModel() if rank == fail_rank else FakeModel()
        out = gen(model, prompts, n_gen)
        q.put((rank, "ok", None if out is None else out.tolist()))
    except Exception as ex:  # reported to the parent, which checks who failed and how
        q.put((rank, "error", type(ex).__name__))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def _run(world, batch, n_gen, fail_rank=-1, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, batch, n_gen, fail_rank, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            r, status, payload = q.get(timeout=timeout)
            results[r] = (status, payload)
    finally:
        for p in procs:
            p.join(timeout=10)
            if p.is_alive():
                p.kill()
    return results


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shard_range_partitions(world):
    for n in range(0, 71):
        ranges = [shard_range(n, world, r) for r in range(world)]
        pos = 0
        for start, count in ranges:
            assert start == pos and count >= 0
            pos += count
        assert pos == n
        sizes = [c for _, c in ranges]
        assert max(sizes) - min(sizes) <= 1


def test_shard_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)
    with pytest.raises(ValueError):
        shard_range(-1, 2, 0)


@pytest.mark.parametrize("batch", [1, 2, 11])
def test_generate_sharded_gloo_matches_single_process(batch):
    n_gen = 6
    res = _run(2, batch, n_gen)
    assert res[0][0] == "ok" and res[1] == ("ok", None)
    prompts = np.random.default_rng(5).integers(0, 32000, (batch, 9)).astype(np.int32)
    want = FakeModel().generate_batch(prompts, n_gen)
    assert np.array_equal(np.array(res[0][1], np.int32), want)


def test_generate_sharded_failing_rank_does_not_hang():
    """Rank 1 raises inside its shard; rank 0's gather ends with an error (the peer is gone or the
    group's 10 s timeout expires) instead of waiting for good."""
    res = _run(2, 4, 3, fail_rank=1, timeout=90)
    assert res[1] == ("error", "RuntimeError")
    assert res[0][0] == "error"
