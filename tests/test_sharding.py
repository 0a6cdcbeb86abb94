"""Multi-rank host logic on CPU: balanced shards cover every unit once, and the assembling
all-gather (gloo, world_size 2 and 3) rebuilds exactly the unsharded result, uneven shards
included.  Each rank computes its shard with the oracle, as a GPU rank would with the kernels."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT  # noqa: F401  (sets sys.path)
from lightning_core_b200.sharding import assemble, shard_range


@pytest.mark.parametrize("total,world", [(128, 1), (128, 2), (128, 8), (7, 3), (2, 4), (0, 2), (8192, 8)])
def test_shard_ranges_partition(total, world):
    seen = []
    sizes = []
    for r in range(world):
        lo, hi = shard_range(total, r, world)
        seen.extend(range(lo, hi))
        sizes.append(hi - lo)
    assert seen == list(range(total))
    assert max(sizes) - min(sizes) <= 1
    assert sizes[0] == max(sizes)


def test_shard_range_rejects_bad_args():
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)
    with pytest.raises(ValueError):
        shard_range(10, 0, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, units, q, k, v, a, b, out_dir):
    from oracle import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        P = O.port()
        lo, hi = shard_range(units, rank, world)
        att = P.attention_units(q[lo:hi], k[lo:hi], v[lo:hi], causal=True, threads=1) if hi > lo else \
            np.zeros((0,) + q.shape[1:], np.float32)
        full_att = assemble(torch.from_numpy(att), units, rank, world)
        rlo, rhi = shard_range(a.shape[0], rank, world)
        c = P.matmul(np.ascontiguousarray(a[rlo:rhi]), b) if rhi > rlo else np.zeros((0, b.shape[1]), np.float32)
        full_c = assemble(torch.from_numpy(c), a.shape[0], rank, world)
        np.save(os.path.join(out_dir, f"att_{rank}.npy"), full_att.numpy())
        np.save(os.path.join(out_dir, f"c_{rank}.npy"), full_c.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_sharded_step_matches_unsharded(tmp_path, world):
    rng = np.random.default_rng(world)
    units = 5
    q, k, v = (rng.standard_normal((units, 33, 16)).astype(np.float32) for _ in range(3))
    a = rng.uniform(-1, 1, (11, 24)).astype(np.float32)
    b = rng.uniform(-1, 1, (24, 9)).astype(np.float32)
    mp.start_processes(_worker, args=(world, _free_port(), units, q, k, v, a, b, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    from oracle import oracle as O

    P = O.port()
    want_att = P.attention_units(q, k, v, causal=True, threads=1)
    want_c = P.matmul(a, b)
    for r in range(world):
        np.testing.assert_array_equal(np.load(tmp_path / f"att_{r}.npy"), want_att)
        np.testing.assert_array_equal(np.load(tmp_path / f"c_{r}.npy"), want_c)


def test_library_shard_range_matches(lc):
    """lcShardRange (the split the library's sharded entry points use) == the harness split."""
    for total in (0, 1, 7, 128, 8192, 3136):
        for world in (1, 2, 3, 4, 8):
            for r in range(world):
                assert lc.shard_range(total, r, world) == shard_range(total, r, world)
    with pytest.raises(ValueError):
        lc.shard_range(10, 2, 2)


def _failing_worker(rank, world, port, out_dir, bad_rank):
    import datetime

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    status = "ok"
    try:
        if rank == bad_rank:
            raise RuntimeError("injected failure before the gather")
        local = torch.full((shard_range(6, rank, world)[1] - shard_range(6, rank, world)[0], 4), float(rank))
        assemble(local, 6, rank, world)
    except RuntimeError as exc:  # the failed peer surfaces as an error in the collective
        status = f"error: {type(exc).__name__}"
        if rank == bad_rank:
            with open(os.path.join(out_dir, f"status_{rank}.txt"), "w") as f:
                f.write(status)
            raise
    with open(os.path.join(out_dir, f"status_{rank}.txt"), "w") as f:
        f.write(status)


def test_rank_failure_surfaces_as_error_not_hang(tmp_path):
    """A rank that fails before the assembling all-gather: every other rank's collective ends with
    an error (closed connection or the 10 s process-group timeout), nobody hangs."""
    import time

    world, bad = 3, 1
    t0 = time.time()
    with pytest.raises(Exception):
        mp.start_processes(_failing_worker, args=(world, _free_port(), str(tmp_path), bad), nprocs=world, join=True,
                           start_method="spawn")
    # the survivors finish on their own (join re-raised the bad rank's error first)
    deadline = time.time() + 60
    while time.time() < deadline and not all((tmp_path / f"status_{r}.txt").exists() for r in range(world)):
        time.sleep(0.2)
    assert time.time() - t0 < 90
    for r in range(world):
        status = (tmp_path / f"status_{r}.txt").read_text()
        assert status.startswith("error"), (r, status)
