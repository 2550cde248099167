"""Writes tests/golden/<case>.npz by running the UNMODIFIED reference optimizer
(hybrid_rl.optimizer.ZeroOneAdamW from the HybridAgent checkout) on the seeded inputs of
``cases.py``, on CPU, at world size 1 in-process and at world size 2 over gloo.

Run in the build container, where the reference checkout exists:

    python tests/golden/make_golden.py --reference <path to the HybridAgent checkout> [--only <case>]

The fixtures are committed; nothing on the GPU machines runs this script.

Each step follows the caller order of hybrid_rl/train.py:248-295: zero_grad, set grads,
all_reduce_grads, clip_grad_norm(max_norm), step.  Stored per case: the norm returned by
every step, the final parameter of every tensor (dtype bit patterns), the owner's final
master / exp_avg / exp_avg_sq / param_steps, and the owner map.  Full-size cases
(``digest=True``: BASELINE configuration 1 at its real shapes) store instead the SHA-256 of
every final array and the values at seeded sample positions (``cases.sample_positions``).
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from cases import BF16, CASES, DIGEST_CASES, F16, F32, digest, sample_positions  # noqa: E402

TORCH_DTYPE = {F32: torch.float32, BF16: torch.bfloat16, F16: torch.float16}


def to_torch(a: np.ndarray, dtype: int) -> torch.Tensor:
    if dtype == F32:
        return torch.from_numpy(a.copy())
    return torch.from_numpy(a.view(np.int16).copy()).view(TORCH_DTYPE[dtype])


def to_numpy(t: torch.Tensor, dtype: int) -> np.ndarray:
    t = t.detach().contiguous().reshape(-1)
    if dtype == F32:
        return t.numpy().copy()
    return t.view(torch.int16).numpy().view(np.uint16).copy()


def run_case(case, rank: int, world: int, reference: str) -> dict:
    sys.path.insert(0, reference)
    from hybrid_rl.optimizer import ZeroOneAdamW

    torch.set_num_threads(1)
    params = [torch.nn.Parameter(to_torch(p, case.dtype).reshape(s))
              for p, s in zip(case.initial_params(), case.shapes)]
    opt = ZeroOneAdamW([{"params": params, "lr": case.lr}], rank=rank, world_size=world, betas=case.betas,
                       eps=case.eps, weight_decay=case.weight_decay)
    if case.preload_state:
        for i in opt.master:
            master, m, v, step = case.preload(i)
            opt.master[i].copy_(torch.from_numpy(master).reshape(case.shapes[i]))
            opt.exp_avg[i].copy_(torch.from_numpy(m).reshape(case.shapes[i]))
            opt.exp_avg_sq[i].copy_(torch.from_numpy(v).reshape(case.shapes[i]))
            opt.param_steps[i] = step
            if not opt.master_is_parameter[i]:
                params[i].data.copy_(opt.master[i].to(params[i].dtype))
        if world > 1:
            for i, p in enumerate(params):
                dist.broadcast(p.data, src=opt.owner[i])
    norms = []
    for step in range(case.steps):
        opt.zero_grad(set_to_none=True)
        for p, g in zip(params, case.grads(step, rank)):
            p.grad = None if g is None else to_torch(g, case.dtype).reshape(p.shape)
        opt.all_reduce_grads()
        norm = opt.clip_grad_norm(case.max_norm)
        norms.append(norm)
        if np.isfinite(norm) or case.call_step_after_nonfinite:
            opt.step()
    out = {"norms": np.array(norms, np.float64), "owner": np.array(opt.owner, np.int32)}
    for i, p in enumerate(params):
        out[f"param_{i}"] = to_numpy(p.data, case.dtype)
    for i in opt.master:
        out[f"master_{i}"] = opt.master[i].reshape(-1).numpy().copy()
        out[f"exp_avg_{i}"] = opt.exp_avg[i].reshape(-1).numpy().copy()
        out[f"exp_avg_sq_{i}"] = opt.exp_avg_sq[i].reshape(-1).numpy().copy()
        out[f"param_steps_{i}"] = np.array(opt.param_steps[i], np.int64)
    return out


def _worker(rank: int, world: int, case, reference: str, port: int, queue) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        queue.put((rank, run_case(case, rank, world, reference)))
    finally:
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="HybridAgent checkout containing hybrid_rl/")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    for k, case in enumerate(CASES + DIGEST_CASES):
        if args.only and case.name != args.only:
            continue
        if case.world == 1:
            out = run_case(case, 0, 1, args.reference)
        else:
            ctx = mp.get_context("spawn")
            q = ctx.Queue()
            procs = [ctx.Process(target=_worker, args=(r, case.world, case, args.reference, 29610 + k, q))
                     for r in range(case.world)]
            for p in procs:
                p.start()
            results = dict(q.get() for _ in procs)
            for p in procs:
                p.join()
                assert p.exitcode == 0
            out = {}
            for r in range(case.world):
                for key, val in results[r].items():
                    if key.startswith(("master_", "exp_avg", "param_steps_")) or key not in out:
                        out[key] = val
                    elif key.startswith("param_"):
                        assert np.array_equal(out[key], val), "ranks disagree on " + key
                    elif key == "norms":
                        assert np.array_equal(out[key], val, equal_nan=True), "ranks disagree on norms"
        if case.digest:  # full-size case: digests of every final array and the sampled elements
            full, out = out, {"norms": out["norms"], "owner": out["owner"]}
            tensor, offset = sample_positions(case)
            for key in ("param", "master", "exp_avg", "exp_avg_sq"):
                out[f"sha256_{key}"] = np.array([digest(full[f"{key}_{i}"]) for i in range(len(case.shapes))])
                out[f"sample_{key}"] = np.array([full[f"{key}_{t}"][o] for t, o in zip(tensor, offset)])
            out["param_steps"] = np.array([int(full[f"param_steps_{i}"]) for i in range(len(case.shapes))])
        out["meta"] = np.array(json.dumps({"case": case.name, "torch": torch.__version__,
                                           "cpu_capability": torch.backends.cpu.get_cpu_capability()}))
        path = os.path.join(HERE, f"{case.name}.npz")
        np.savez_compressed(path, **out)
        print(f"{case.name}: norms={out['norms'].tolist()} -> {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
