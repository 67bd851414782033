"""Multi-process (world size 2, gloo on CPU) coverage of the N>1 path: chains
are sharded across ranks with no data-path collective, and a rank that fails
is detected by the others through a short process-group timeout."""
from __future__ import annotations

import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from bayes_ssm.sharding import chain_shard, shard_sizes


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    g = torch.Generator().manual_seed(0)
    n, t, d, m = 11, 9, 8, 8
    k = torch.nn.functional.normalize(torch.randn(n, t, d, generator=g), dim=-1)
    q = torch.nn.functional.normalize(torch.randn(n, t, d, generator=g), dim=-1)
    v = torch.randn(n, t, m, generator=g)
    a = torch.sigmoid(torch.randn(n, t, d, generator=g) + 2)
    p = torch.full((n, t), 0.02)
    r = torch.full((n, t), 0.5)
    return k, v, q, a, p, r


def _sharded_worker(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    import bayes_ssm
    k, v, q, a, p, r = _inputs()
    sl = chain_shard(k.shape[0], world, rank)
    y, _, _ = bayes_ssm.bayesian_layer(k[sl], v[sl], q[sl], transition_diagonals=a[sl],
                                       process_variances=p[sl], observation_variances=r[sl],
                                       chunk_length=4)
    # gather only to check the result; the data path itself has no collective
    sizes = shard_sizes(k.shape[0], world)
    buf = torch.zeros(max(sizes), *y.shape[1:])
    buf[: y.shape[0]] = y
    gathered = [torch.zeros_like(buf) for _ in range(world)]
    dist.all_gather(gathered, buf)
    t = torch.tensor([float(rank + 1)])
    dist.all_reduce(t, op=dist.ReduceOp.MAX)  # bench.py's max-over-ranks timing
    if rank == 0:
        full = torch.cat([g[:s] for g, s in zip(gathered, sizes)])
        torch.save({"y": full, "tmax": float(t)}, out_path)
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_chains_equal_unsharded(tmp_path):
    import bayes_ssm
    out = tmp_path / "y.pt"
    mp.spawn(_sharded_worker, args=(2, _free_port(), str(out)), nprocs=2, join=True)
    got = torch.load(out)
    k, v, q, a, p, r = _inputs()
    want, _, _ = bayes_ssm.bayesian_layer(k, v, q, transition_diagonals=a, process_variances=p,
                                          observation_variances=r, chunk_length=4)
    assert torch.equal(got["y"], want)
    assert got["tmax"] == 2.0


def _failing_worker(rank, world, port, flag_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    if rank == 1:
        # leaves between steps, with no collective in flight
        dist.destroy_process_group()
        os._exit(0)
    try:
        dist.barrier()
        outcome = "no error"
    except Exception as exc:  # the survivor must see an error, not hang
        outcome = type(exc).__name__
    with open(flag_path, "w") as f:
        f.write(outcome)
    os._exit(0)


def test_dead_rank_is_detected_by_timeout(tmp_path):
    flag = tmp_path / "flag.txt"
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, str(flag))) for r in range(2)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=90)
        assert not pr.is_alive(), "a rank hung instead of timing out"
    assert flag.read_text() != "no error"


def test_chain_shard_partition():
    for n in (0, 1, 7, 16384):
        for world in (1, 2, 3, 8):
            parts = [chain_shard(n, world, r) for r in range(world)]
            assert parts[0].start == 0 and parts[-1].stop == n
            assert all(a.stop == b.start for a, b in zip(parts, parts[1:]))
            sizes = shard_sizes(n, world)
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        chain_shard(4, 2, 2)
