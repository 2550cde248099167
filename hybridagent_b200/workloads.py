"""Parameter sets of the optimizer-step benchmark configurations (shapes only).

Each function returns the trainable tensors' shapes in module order (per layer:
attention projections, MLP / experts, norm vectors; then embeddings and the final norm),
standing in for the real checkpoints: the optimizer step only sees shapes and values,
and values are synthetic (seeded) in the benchmark and tests.
"""
from __future__ import annotations

import math

Shape = tuple[int, ...]


def _dense(hidden: int, layers: int, q_heads: int, kv_heads: int, head_dim: int, inter: int, vocab: int, *,
           tied: bool, norms_per_layer: int) -> list[Shape]:
    out: list[Shape] = []
    for _ in range(layers):
        out += [(q_heads * head_dim, hidden), (kv_heads * head_dim, hidden), (kv_heads * head_dim, hidden),
                (hidden, q_heads * head_dim)]
        out += [(inter, hidden), (inter, hidden), (hidden, inter)]
        out += [(hidden,)] * norms_per_layer + [(head_dim,), (head_dim,)]
    out.append((vocab, hidden))
    out.append((hidden,))
    if not tied:
        out.append((vocab, hidden))
    return out


def qwen3_8b() -> list[Shape]:
    """hidden 4096, 36 layers, 32 q / 8 kv heads of 128, SwiGLU 12288, vocab 151936, untied."""
    return _dense(4096, 36, 32, 8, 128, 12288, 151936, tied=False, norms_per_layer=2)


def gemma_12b() -> list[Shape]:
    """hidden 3840, 48 layers, 16 q / 8 kv heads of 256, GeGLU 15360, vocab 262144, tied,
    pre/post norms around attention and MLP."""
    return _dense(3840, 48, 16, 8, 256, 15360, 262144, tied=True, norms_per_layer=4)


def qwen3_14b() -> list[Shape]:
    """hidden 5120, 40 layers, 40 q / 8 kv heads of 128, intermediate 17408, vocab 151936."""
    return _dense(5120, 40, 40, 8, 128, 17408, 151936, tied=False, norms_per_layer=2)


def moe_26b_a4b(experts: int = 128) -> list[Shape]:
    """hidden 2816, 30 layers, 128 experts of gate/up/down 2816x704 per layer, router
    2816x128, 16 q / 8 kv heads of 256, vocab 262144 tied; one tensor per expert matrix."""
    out: list[Shape] = []
    for _ in range(30):
        out += [(4096, 2816), (2048, 2816), (2048, 2816), (2816, 4096), (experts, 2816)]
        for _ in range(experts):
            out += [(704, 2816), (704, 2816), (2816, 704)]
        out += [(2816,)] * 4 + [(256,), (256,)]
    out += [(262144, 2816), (2816,)]
    return out


def config1_cpu() -> list[Shape]:
    """48 matrices 256x512, 8 matrices 1024x256, 8 vectors of 65536 (8,912,896 params)."""
    return [(256, 512)] * 48 + [(1024, 256)] * 8 + [(65536,)] * 8


WORKLOADS = {
    "qwen3_8b": qwen3_8b,
    "gemma_12b": gemma_12b,
    "qwen3_14b": qwen3_14b,
    "moe_26b_a4b": moe_26b_a4b,
    "config1_cpu": config1_cpu,
}


def numels(shapes: list[Shape]) -> list[int]:
    return [math.prod(s) for s in shapes]


def truncated(shapes: list[Shape], max_params: int) -> list[Shape]:
    """Leading tensors of a parameter set holding at most ``max_params`` elements (a
    bounded sample of the same distribution of shapes)."""
    out, total = [], 0
    for s in shapes:
        n = math.prod(s)
        if total + n > max_params and out:
            break
        out.append(s)
        total += n
    return out
