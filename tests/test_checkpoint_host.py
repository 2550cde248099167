"""Shard files of the optimizer-state checkpoint (host logic, no GPU): one file per rank
under <dir>/optimizer/, written atomically, read back by the same rank and world size."""
import os

import pytest
import torch

from hybridagent_b200 import checkpoint


class FakeOptimizer:
    def __init__(self, rank, world, value):
        self.rank, self.world = rank, world
        self.state = {"format": "x", "value": torch.full((4,), float(value))}
        self.loaded = None

    def state_dict(self):
        return self.state

    def load_state_dict(self, state):
        self.loaded = state


def test_each_rank_writes_and_reads_its_own_shard(tmp_path):
    for r in range(3):
        path = checkpoint.save_optimizer_state(FakeOptimizer(r, 3, r + 1), tmp_path)
        assert path == os.path.join(tmp_path, "optimizer", f"rank{r}-of3.pt")
    assert sorted(os.listdir(tmp_path / "optimizer")) == ["rank0-of3.pt", "rank1-of3.pt", "rank2-of3.pt"]
    opt = FakeOptimizer(1, 3, 0)
    checkpoint.load_optimizer_state(opt, tmp_path)
    assert torch.equal(opt.loaded["value"], torch.full((4,), 2.0))


def test_missing_shard_for_another_world_size(tmp_path):
    checkpoint.save_optimizer_state(FakeOptimizer(0, 2, 1), tmp_path)
    with pytest.raises(FileNotFoundError, match="rank 0 of 4"):
        checkpoint.load_optimizer_state(FakeOptimizer(0, 4, 0), tmp_path)
