"""Seeded inputs of the golden parity cases.

Shared by ``make_golden.py`` (which runs the unmodified reference optimizer on them, in
this build container only) and by the tests (which rebuild the same inputs from the same
seeds and compare against the stored outputs).  Everything here is plain numpy so the
inputs do not depend on torch's random number generators.

Value distributions follow the parity configurations of the optimizer benchmark:
params ~N(0, 0.02); grads ~N(0, sigma) fresh every step; optional pre-loaded state
master ~N(0, 0.02), m ~N(0, 1e-5), v ~|N(0, 1e-8)| at step 100; shapes are small stand-ins
for the transformer matrices / vectors of the benchmark models, with ragged sizes.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

F32, BF16, F16 = 0, 1, 2
DTYPE_NAMES = {F32: "float32", BF16: "bfloat16", F16: "float16"}


def rne_bf16(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round to nearest even (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def rne_f16(x: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def from_f32(x: np.ndarray, dtype: int) -> np.ndarray:
    if dtype == F32:
        return np.ascontiguousarray(x, dtype=np.float32)
    return rne_bf16(x) if dtype == BF16 else rne_f16(x)


def to_f32(a: np.ndarray, dtype: int) -> np.ndarray:
    if dtype == F32:
        return a.astype(np.float32)
    if dtype == BF16:
        return (a.astype(np.uint32) << 16).view(np.float32)
    return a.view(np.float16).astype(np.float32)


@dataclass
class Case:
    name: str
    case_id: int
    shapes: list[tuple[int, ...]]
    dtype: int
    steps: int
    world: int = 1
    lr: float = 1e-6
    betas: tuple[float, float] = (0.9, 0.999)
    eps: float = 1e-8
    weight_decay: float = 0.01
    max_norm: float = 1.0
    grad_sigma: float = 1e-4
    preload_state: bool = False      # master/m/v/step as in the bf16 benchmark configs
    target_norm: float | None = None  # rescale every step's grads to this global norm
    # (step, rank, tensor) -> None: the gradient is absent; "zero": all-zero gradient;
    # "inf" / "nan": one element replaced
    overrides: dict = field(default_factory=dict)
    call_step_after_nonfinite: bool = True
    # store per-tensor SHA-256 digests and seeded sample positions instead of whole arrays
    # (full-size configurations whose arrays would not belong in the repository)
    digest: bool = False

    @property
    def numels(self) -> list[int]:
        return [int(np.prod(s)) for s in self.shapes]

    def rng(self, *key: int) -> np.random.Generator:
        return np.random.default_rng([self.case_id, *key])

    def initial_params_f32(self) -> list[np.ndarray]:
        return [(self.rng(0, 0, i).standard_normal(n) * 0.02).astype(np.float32) for i, n in enumerate(self.numels)]

    def initial_params(self) -> list[np.ndarray]:
        """Parameter values as the dtype's bit patterns (fp32 values for F32)."""
        return [from_f32(p, self.dtype) for p in self.initial_params_f32()]

    def preload(self, i: int) -> tuple[np.ndarray, np.ndarray, np.ndarray, int]:
        """(master, m, v, step) written into the reference's state after construction."""
        n = self.numels[i]
        r = self.rng(1, 0, i)
        master = (r.standard_normal(n) * 0.02).astype(np.float32)
        m = (r.standard_normal(n) * 1e-5).astype(np.float32)
        v = np.abs(r.standard_normal(n) * 1e-8).astype(np.float32)
        return master, m, v, 100

    def grads(self, step: int, rank: int) -> list[np.ndarray | None]:
        """This rank's gradients for one step, as dtype bit patterns (fp32 for F32)."""
        raw = [(self.rng(2 + step, rank, i).standard_normal(n) * self.grad_sigma).astype(np.float32)
               for i, n in enumerate(self.numels)]
        if self.target_norm is not None:
            total = np.sqrt(sum(float(np.sum(g.astype(np.float64) ** 2)) for g in raw))
            k = self.target_norm / (total * np.sqrt(self.world))
            raw = [(g * k).astype(np.float32) for g in raw]
        out: list[np.ndarray | None] = []
        for i, g in enumerate(raw):
            kind = self.overrides.get((step, rank, i))
            if kind is None and (step, -1, i) in self.overrides:
                kind = self.overrides[(step, -1, i)]
            if kind == "none":
                out.append(None)
                continue
            if kind == "zero":
                g = np.zeros_like(g)
            elif kind == "inf":
                g = g.copy()
                g[len(g) // 3] = np.inf
            elif kind == "nan":
                g = g.copy()
                g[len(g) // 2] = np.nan
            out.append(from_f32(g, self.dtype) if self.dtype != F32 else g)
        return out


_SMALL = [(32, 64)] * 4 + [(64, 32)] * 2 + [(512,)] * 2 + [(96, 40), (13,), (1,), (257,)]

CASES = [
    Case("cfg1_fp32", 1, _SMALL, F32, steps=10, grad_sigma=1e-2),
    Case("fp32_big_lr", 2, _SMALL, F32, steps=5, grad_sigma=1e-3, lr=1e-3, weight_decay=0.1),
    Case("bf16_preloaded", 3, _SMALL, BF16, steps=3, preload_state=True),
    Case("bf16_clip", 4, _SMALL, BF16, steps=3, preload_state=True, target_norm=4.0),
    Case("bf16_big_lr_clip", 5, _SMALL, BF16, steps=4, lr=1e-3, grad_sigma=1e-2),
    Case("f16_clip", 6, _SMALL, F16, steps=3, grad_sigma=1e-2),
    Case("bf16_sparse", 7, _SMALL, BF16, steps=3, grad_sigma=1e-2,
         overrides={(0, -1, 1): "none", (1, -1, 1): "none", (1, -1, 5): "none", (0, -1, 2): "zero",
                    (1, -1, 2): "zero", (2, -1, 8): "zero"}),
    Case("bf16_inf", 8, _SMALL, BF16, steps=2, grad_sigma=1e-2, overrides={(1, -1, 3): "inf"}),
    Case("bf16_nan", 9, _SMALL, BF16, steps=2, grad_sigma=1e-2, overrides={(1, -1, 6): "nan"}),
    Case("bf16_world2", 10, _SMALL, BF16, steps=3, world=2, grad_sigma=1e-2,
         overrides={(0, 1, 3): "none", (1, 0, 4): "none", (1, -1, 9): "none", (2, 0, 0): "zero"}),
    Case("fp32_world2", 11, _SMALL, F32, steps=3, world=2, grad_sigma=1e-2, preload_state=True),
    # rank 1 alone holds a +inf at step 1: every rank must see a non-finite norm and skip
    Case("bf16_world2_inf", 12, _SMALL, BF16, steps=3, world=2, grad_sigma=1e-2, overrides={(1, 1, 5): "inf"},
         call_step_after_nonfinite=False),
]

# BASELINE configuration 1 at its real shapes: 48 x (256, 512), 8 x (1024, 256), 8 x (65536,),
# fp32, grads ~N(0, 1e-3) fresh every step, lr 1e-6, wd 0.01, clip 1.0, 10 steps (the global norm
# is ~2.99, so every step clips)
CONFIG1 = [(256, 512)] * 48 + [(1024, 256)] * 8 + [(65536,)] * 8
DIGEST_CASES = [Case("cfg1_full", 13, CONFIG1, F32, steps=10, grad_sigma=1e-3, digest=True)]

CASES_BY_NAME = {c.name: c for c in CASES + DIGEST_CASES}

SAMPLES = 50_000


def sample_positions(case: Case) -> tuple[np.ndarray, np.ndarray]:
    """(tensor, offset) of the sampled elements of a digest case: SAMPLES seeded positions
    over the whole parameter list plus every tensor's first and last element."""
    bounds = np.concatenate([[0], np.cumsum(case.numels)]).astype(np.int64)
    flat = np.random.default_rng([case.case_id, 99]).integers(0, int(bounds[-1]), size=SAMPLES)
    flat = np.unique(np.concatenate([flat, bounds[:-1], bounds[1:] - 1]))
    tensor = np.searchsorted(bounds, flat, side="right") - 1
    return tensor.astype(np.int64), (flat - bounds[tensor]).astype(np.int64)


def digest(a: np.ndarray) -> str:
    """SHA-256 of an array's little-endian bytes (fp32 values, or 16-bit patterns)."""
    import hashlib
    return hashlib.sha256(np.ascontiguousarray(a).reshape(-1).tobytes()).hexdigest()
