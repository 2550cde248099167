"""The benchmark's sampled parity check (bench.checked_step) on CPU, driven by the reference's
own optimizer: at world size 1 and over two gloo ranks the check must find no mismatch (its
torch recomputation is the reference's op sequence), and a one-ulp error planted in the
reference's master after its step must be found at that position."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench
from oracle import stage_ref

SHAPES = [(64, 33), (1000,), (7,), (3, 5000), (1,)]


def _reference():
    if not stage_ref.stage():
        pytest.skip("the reference optimizer is not staged (no checkout here)")
    cls, kind = bench._reference_class()
    assert kind == "reference"
    return cls


def _setup(cls, rank: int, world: int):
    g = torch.Generator().manual_seed(5)
    params = [torch.nn.Parameter((torch.randn(s, generator=g) * 0.02).to(torch.bfloat16)) for s in SHAPES]
    opt = cls([{"params": params, "lr": 1e-3}], rank=rank, world_size=world, weight_decay=0.01)
    gs = torch.Generator().manual_seed(9)
    for i in range(len(SHAPES)):
        m = torch.randn(SHAPES[i], generator=gs) * 1e-3
        v = (torch.randn(SHAPES[i], generator=gs) * 1e-5).abs()
        if i in opt.param_steps:
            opt.exp_avg[i].copy_(m)
            opt.exp_avg_sq[i].copy_(v)
            opt.param_steps[i] = 100
    gg = torch.Generator().manual_seed(100 + rank)
    inputs = [(torch.randn(s, generator=gg) * 0.05).to(torch.bfloat16) for s in SHAPES]
    return params, opt, inputs


def test_world1_reference_has_no_mismatch():
    cls = _reference()
    params, opt, inputs = _setup(cls, 0, 1)
    out = bench.checked_step(opt, params, inputs, [int(np.prod(s)) for s in SHAPES], per_rank=3000)
    assert out["mismatches"] == 0, out
    assert out["max_ulp"] == 0 and out["norm"]["ok"], out
    assert out["checked_positions"] > 2000


def test_planted_master_error_is_found():
    cls = _reference()

    class Planted(cls):
        def step(self):
            super().step()
            m = self.master[0].view(-1)  # tensor 0's first element is always sampled
            m[0:1].view(torch.int32).add_(1)  # one ulp, after the update

    params, opt, inputs = _setup(Planted, 0, 1)
    out = bench.checked_step(opt, params, inputs, [int(np.prod(s)) for s in SHAPES], per_rank=500)
    assert out["fields"]["master"] == 1 and out["max_ulp"] == 1, out


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cls, _ = bench._reference_class()
        params, opt, inputs = _setup(cls, rank, world)
        out = bench.checked_step(opt, params, inputs, [int(np.prod(s)) for s in SHAPES], per_rank=2000)
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_world2_gloo_reference_has_no_mismatch():
    _reference()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in (0, 1):
        assert res[r]["mismatches"] == 0, res[r]
        assert res[r]["norm"]["ok"], res[r]
    assert res[0]["fields"] == res[1]["fields"]
