"""Sharded optimizer-state checkpoints on disk.

The reference saves the model only (hybrid_rl/policy.py:97-102, called on rank 0 at
hybrid_rl/train.py:353-362), so an interrupted HybridRL run restarts with fresh AdamW
moments.  Here every rank writes its own shard of the optimizer state into the same
checkpoint directory, next to the model files:

    <checkpoint-dir>/optimizer/rank{r}-of{W}.pt

Each shard is ``ZeroOneAdamW.state_dict()`` (fp32 master / exp_avg / exp_avg_sq and the
step counts of the rank's owned tensors, plus the owner map and sizes that identify the
layout), written to a temporary file and renamed, so a crash never leaves a partial
shard under the final name.  Loading into an optimizer built over the same parameters,
rank and world size resumes bit-identically.  Unlike the model save, every rank calls
these functions.
"""
from __future__ import annotations

import os

import torch

SUBDIR = "optimizer"


def shard_path(directory: str | os.PathLike, rank: int, world: int) -> str:
    return os.path.join(os.fspath(directory), SUBDIR, f"rank{rank}-of{world}.pt")


def save_optimizer_state(optimizer, directory: str | os.PathLike) -> str:
    """Writes this rank's shard under ``directory``; returns its path."""
    path = shard_path(directory, optimizer.rank, optimizer.world)
    os.makedirs(os.path.dirname(path), exist_ok=True)
    tmp = f"{path}.tmp-{os.getpid()}"
    torch.save(optimizer.state_dict(), tmp)
    os.replace(tmp, path)
    return path


def load_optimizer_state(optimizer, directory: str | os.PathLike) -> None:
    """Loads this rank's shard from ``directory`` (raises if it is missing or was written
    for another rank, world size or parameter layout)."""
    path = shard_path(directory, optimizer.rank, optimizer.world)
    if not os.path.exists(path):
        raise FileNotFoundError(f"no optimizer shard for rank {optimizer.rank} of {optimizer.world} at {path}")
    state = torch.load(path, map_location="cpu", weights_only=False)
    optimizer.load_state_dict(state)
