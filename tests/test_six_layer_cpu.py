"""CPU: the six-layer hybrid LM (BASELINE config 5's model) -- its parameter
count and names at the reference's sizes, a training step on a small
instance, and a world-size-2 gloo DDP step whose ranks end with identical
parameters (the gradient all-reduce is the only collective)."""
from __future__ import annotations

import os
import socket
from datetime import timedelta

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from bayes_ssm.six_layer import SixLayerLM, make_optimizer, parameter_count, train_step

SMALL = dict(vocab_size=96, width=64, heads=8, kv_heads=2, mlp_width=96, chunk_length=4, dtype=torch.float32)


def test_reference_size_and_layout():
    m = SixLayerLM(device="meta")
    # example/results/gb300_6layer_bayes_paper_d8_fused.json: "parameters": 101942304
    assert parameter_count(m) == 101_942_304
    kinds = [type(b.mixer).__name__ for b in m.blocks]
    assert kinds == ["BayesianMixer", "BayesianMixer", "GQAAttention", "BayesianMixer", "BayesianMixer",
                     "GQAAttention"]
    names = set(dict(m.named_parameters()))
    for key in ("embedding.weight", "final_norm.weight", "blocks.0.mixer.qkv_proj.weight",
                "blocks.2.mixer.k_proj.weight", "blocks.5.ffn.down.weight"):
        assert key in names


def test_training_step_reduces_loss():
    torch.manual_seed(0)
    m = SixLayerLM(**SMALL)
    opt = make_optimizer(m, lr=3e-3)
    g = torch.Generator().manual_seed(1)
    tok = torch.randint(SMALL["vocab_size"], (2, 13), generator=g)
    losses = [float(train_step(m, opt, tok[:, :-1], tok[:, 1:], vocab_size=SMALL["vocab_size"]))
              for _ in range(6)]
    assert all(torch.isfinite(torch.tensor(losses)))
    assert losses[-1] < losses[0]
    # the tied head: logits are FP32 and use the embedding matrix
    logits = m(tok[:, :-1])
    assert logits.dtype == torch.float32 and logits.shape == (2, 12, SMALL["vocab_size"])


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ddp_worker(rank, world, port, out_path):
    from torch.nn.parallel import DistributedDataParallel as DDP
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    torch.manual_seed(0)  # identical initialisation on every rank
    m = SixLayerLM(**SMALL)
    ddp = DDP(m, broadcast_buffers=False, gradient_as_bucket_view=True, bucket_cap_mb=1)
    opt = make_optimizer(ddp, lr=1e-3)
    g = torch.Generator().manual_seed(10 + rank)  # a different batch per rank
    tok = torch.randint(SMALL["vocab_size"], (2, 9), generator=g)
    train_step(ddp, opt, tok[:, :-1], tok[:, 1:], vocab_size=SMALL["vocab_size"])
    flat = torch.cat([p.detach().reshape(-1) for p in m.parameters()])
    gathered = [torch.zeros_like(flat) for _ in range(world)]
    dist.all_gather(gathered, flat)
    if rank == 0:
        torch.save({"params": gathered, "tok0": tok}, out_path)
    dist.barrier()
    dist.destroy_process_group()


def test_ddp_step_keeps_ranks_identical(tmp_path):
    out = tmp_path / "p.pt"
    mp.spawn(_ddp_worker, args=(2, _free_port(), str(out)), nprocs=2, join=True)
    got = torch.load(out)
    p0, p1 = got["params"]
    assert torch.equal(p0, p1)
    # and the step moved the parameters (averaged gradients were applied)
    torch.manual_seed(0)
    init = torch.cat([p.detach().reshape(-1) for p in SixLayerLM(**SMALL).parameters()])
    assert not torch.equal(p0, init)
