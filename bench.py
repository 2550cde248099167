"""ZeRO-1 AdamW step benchmark (HybridAgent's hybrid_rl/optimizer.py step, B200 build).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload qwen3_8b] [--impl ours|reference]

One step is the reference trainer's optimizer sequence over one batch of gradients
(hybrid_rl/train.py:287-295): the caller's gradients land in ``p.grad``,
``all_reduce_grads()``, ``clip_grad_norm(1.0)``, ``step()``.  The workload is the
Qwen3-8B-shaped parameter set (8.19 B parameters in 399 tensors, bf16 params / grads,
fp32 master / m / v, state pre-loaded at step 100), synthetic seeded values, the whole
model sharded ZeRO-1 over N GPUs (strong scaling: the model is fixed as N grows).

Printed (rank 0, one JSON line):
  value        whole-job Gparams/s = parameters / device step time (max over ranks), all
               inputs resident in HBM (131 GB at N=1, far larger than the 126 MB L2, so no
               flush between steps);
  e2e          the same through the public API with the step's gradients copied from
               pinned host memory each step (H2D inside the timed region, on a copy
               stream into a second gradient set so that step k+1's copy overlaps step
               k's optimizer) and the norm read back (D2H);
  roofline     N=1: the fused AdamW kernel's algorithmic bytes (26 B per owned parameter plus
               the stored bf16 groups, or 28 B with full writes) over its CUDA-event
               duration on the launch stream, against the measured HBM copy peak; traffic =
               ncu DRAM bytes per parameter from the committed record of that write mode.
               N>1: the longest phase (push or update + all-gather) with the resource that
               binds it, NVLink against the probed link peak (profiles/nvlink_peak.json)
               and the nominal 900 GB/s; every phase in ``roofline_fused``;
  parity       one more step after timing, checked at ~100,000 seeded positions per rank
               against torch's CUDA kernels running the reference's op sequence;
  cpu_baseline the reference's own optimizer (staged unmodified by oracle/stage_ref.py) on
               this host's CPU cores (N=1, rank 0), on a bounded sample of the same
               parameter set (configuration 1: the whole of it);
  clocks       nvidia-smi samples taken during the timed region;
  iteration_with_backward
               N > 1, after the above: forward + backward + optimizer per iteration with
               gradient landing off and on the copy engines (measure_landing, the ``--landing``
               synthetic backward over ``--tokens`` tokens), on a second optimizer built once
               the timed one is released.
``--impl reference`` times only that CPU implementation (rank 0; other ranks exit), for the
steps and warm-up it prints, plus BASELINE configuration 1 whole (``config1``).
``--probe-links`` (N > 1) measures NVLink bandwidth between the GPUs instead.

``--landing`` measures gradient landing instead and prints its own JSON line: a synthetic
forward + backward whose weight gradients are GEMMs over ``--tokens`` tokens (one ``linear``
per matrix, a dot product per vector) followed by the optimizer sequence, with landing off and
on (same optimizer).  N > 1: the early pushes of the exchange, receive window sized for two
rounds so the whole exchange can start during backward; N = 1: the norm's square sums taken as
the gradients land.  Per variant the forward + backward time, the optimizer time left after
backward, and their sum, max over ranks.
"""
from __future__ import annotations

import argparse
import contextlib
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

ALGO_BYTES_ADAMW = {"bf16": 28, "f16": 28, "f32": 28}   # per owned parameter, per AdamW launch
ALGO_BYTES_SUMSQ = {"bf16": 2, "f16": 2, "f32": 4}
FALLBACK_HBM_GBS = 6650.0
RECIPE_NVLINK_GBS = 770.0   # the pool's published peer-copy figure, used only where no probe of ours exists
NOMINAL_NVLINK_GBS = 900.0  # NVLink 5, per direction per GPU
# ncu DRAM bytes per parameter of one update launch: full writes of the bf16 copy, and writes of
# the changed groups only
TRAFFIC_PROFILES = {"full": os.path.join(ROOT, "profiles", "adamw_kernel_qwen3_8b.json"),
                    "changed groups": os.path.join(ROOT, "profiles", "adamw_delta_kernel_qwen3_8b.json")}
LINK_PROFILE = os.path.join(ROOT, "profiles", "nvlink_peak.json")


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="qwen3_8b")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--e2e-steps", type=int, default=4)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-sample-params", type=int, default=200_000_000)
    ap.add_argument("--max-params", type=int, default=0, help="truncate the parameter set (smoke / profiling)")
    ap.add_argument("--landing", action="store_true", help="measure gradient landing")
    ap.add_argument("--no-landing", action="store_true", help="N > 1: leave out the iteration_with_backward "
                    "measurement of the step's JSON line")
    ap.add_argument("--tokens", type=int, default=2048, help="tokens of the --landing synthetic backward")
    ap.add_argument("--probe-links", action="store_true", help="measure NVLink bandwidth between the N GPUs")
    ap.add_argument("--probe-bytes", type=int, default=2 << 30, help="--probe-links: bytes each rank moves")
    ap.add_argument("--parity-per-rank", type=int, default=100_000,
                    help="sampled positions per rank of the checked step after timing (0: no check)")
    ap.add_argument("--land-ctas", default="0,64", help="--landing: comma-separated CTA caps to measure, of "
                    "the early pushes at N > 1 (0: copy engines), of the square sums at N = 1 (0: one per chunk)")
    return ap.parse_args()


# ---------------------------------------------------------------- CPU baseline / reference arm
def _reference_class():
    """The reference's own ``ZeroOneAdamW`` staged unmodified under oracle/_ref by
    oracle/stage_ref.py (kind "reference"), else the op-for-op restatement of its world-1
    path in oracle/torch_ops.py (kind "port")."""
    from oracle import stage_ref
    if stage_ref.staged() is not None:
        if stage_ref.OUT not in sys.path:
            sys.path.insert(0, stage_ref.OUT)
        from hybrid_rl.optimizer import ZeroOneAdamW
        return ZeroOneAdamW, "reference"
    return None, "port"


def _world1_gloo() -> None:
    """A world-size-1 gloo process group, as the north star's CPU baseline specifies (at world 1
    the reference issues no collective: optimizer.py:99, 152, 168, 192)."""
    import torch.distributed as dist
    if not dist.is_initialized():
        dist.init_process_group("gloo", store=dist.HashStore(), rank=0, world_size=1)


def reference_cpu(shapes, dtype, *, lr: float, grad_sigma: float, preload: bool, steps: int, warmup: int,
                  fresh_grads: bool, seed: int = 7) -> dict:
    """Times the reference optimizer on CPU tensors at world size 1: per step the caller's
    gradients are set (outside the timed region) and ``all_reduce_grads() +
    clip_grad_norm(1.0) + step()`` is timed (hybrid_rl/train.py:287-295), every host thread.
    ``preload``: m ~N(0,1e-5), v ~|N(0,1e-8)|, step 100 (the GPU arm's state)."""
    import torch

    from oracle.torch_ops import TorchZeroOneW1

    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)  # every host core (torchrun would leave 1)
    cls, kind = _reference_class()
    n = sum(math.prod(s) for s in shapes)
    g = torch.Generator().manual_seed(seed)
    params = [torch.nn.Parameter((torch.randn(s, generator=g) * 0.02).to(dtype)) for s in shapes]
    if cls is not None:
        _world1_gloo()
        opt = cls([{"params": params, "lr": lr}], rank=0, world_size=1, betas=(0.9, 0.999), eps=1e-8,
                  weight_decay=0.01)
        state = [(opt.exp_avg[i], opt.exp_avg_sq[i]) for i in range(len(shapes))]
    else:
        opt = TorchZeroOneW1([p.data for p in params], lr, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
        state = list(zip(opt.exp_avg, opt.exp_avg_sq))
    if preload:
        for i, (m, v) in enumerate(state):
            m.normal_(0, 1e-5, generator=g)
            v.normal_(0, 1e-8, generator=g).abs_()
            if cls is not None:
                opt.param_steps[i] = 100
            else:
                opt.steps[i] = 100

    def grads():
        return [(torch.randn(s, generator=g) * grad_sigma).to(dtype) for s in shapes]

    base = grads()
    times, norms = [], []
    for k in range(warmup + steps):
        fresh = grads() if fresh_grads else [x.clone() for x in base]  # the clip scales gradients in place
        if cls is not None:
            opt.zero_grad(set_to_none=True)
            for p, x in zip(params, fresh):
                p.grad = x
            t0 = time.perf_counter()
            opt.all_reduce_grads()
            norm = opt.clip_grad_norm(1.0)
            opt.step()
        else:
            t0 = time.perf_counter()
            norm = opt.step(fresh, 1.0)
        dt = time.perf_counter() - t0
        if k >= warmup:
            times.append(dt)
            norms.append(norm)
    sec = sum(times) / len(times)
    return {"value": round(n / sec / 1e9, 4), "unit": "Gparams/s", "cores": torch.get_num_threads(),
            "kind": kind, "ms_per_step": round(sec * 1e3, 3), "steps": steps, "warmup": warmup, "params": n,
            "tensors": len(shapes), "last_norm": norms[-1] if norms else None,
            "impl": ("hybrid_rl.optimizer.ZeroOneAdamW (unmodified, staged by oracle/stage_ref.py), world size 1 "
                     "over gloo" if kind == "reference" else "oracle/torch_ops.py restatement (reference not staged)"),
            "host": f"torch {torch.__version__} CPU, {cores} host CPUs visible, {torch.get_num_threads()} threads"}


def cpu_sample(workload: str, sample_params: int, steps: int, warmup: int) -> dict:
    """The reference on CPU over the leading tensors of the GPU arm's parameter set (bf16
    parameters and gradients, fp32 state pre-loaded at step 100, the same gradients every step)."""
    import torch

    from hybridagent_b200 import workloads
    shapes = workloads.truncated(workloads.WORKLOADS[workload](), sample_params)
    out = reference_cpu(shapes, torch.bfloat16, lr=1e-6, grad_sigma=1e-4, preload=True, steps=steps,
                        warmup=warmup, fresh_grads=False)
    out["sample"] = (f"leading {out['tensors']} tensors of {workload} ({out['params']} params), bf16 params/grads, "
                     f"fp32 state at step 100; mean of {steps} timed steps after {warmup} warm-up; {out['host']}")
    return out


def cpu_config1(steps: int = 9, warmup: int = 1) -> dict:
    """BASELINE configuration 1 on the reference: 64 fp32 tensors (48 x 256x512, 8 x 1024x256,
    8 x 65536; 8,912,896 params), params ~N(0,0.02), fresh grads ~N(0,1e-3) every step, m = v =
    0, lr 1e-6, wd 0.01, clip 1.0, 10 steps of which the first is not timed."""
    import torch

    from hybridagent_b200 import workloads
    out = reference_cpu(workloads.config1_cpu(), torch.float32, lr=1e-6, grad_sigma=1e-3, preload=False,
                        steps=steps, warmup=warmup, fresh_grads=True, seed=11)
    out["sample"] = (f"BASELINE config 1 in full: {out['params']} fp32 params in 64 tensors, fresh grads each step, "
                     f"{warmup + steps} steps, the first untimed; {out['host']}")
    return out


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # one CPU measurement per job, on rank 0
    steps, warmup = max(args.steps, 1), max(args.warmup, 0)
    base = cpu_sample(args.workload, args.cpu_sample_params, steps=steps, warmup=warmup)
    cfg1 = cpu_config1()
    out = {"metric": "ZeRO-1 AdamW step Gparams/s", "value": base["value"], "unit": "Gparams/s",
           "impl": "reference", "n_gpus": args.gpus, "steps": steps, "warmup": warmup,
           "ms_per_step": base["ms_per_step"], "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
           "dtype": "fp32", "data": "synthetic",
           "config": {"workload": args.workload, "sample": base["sample"], "params_timed": base["params"]},
           "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample", "impl")},
           "config1": {k: cfg1[k] for k in ("value", "unit", "ms_per_step", "cores", "kind", "steps", "warmup",
                                            "params", "sample", "last_norm")},
           "e2e": {"value": base["value"], "unit": "Gparams/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


# ---------------------------------------------------------------- sampled parity (after the timed region)
class SampledParity:
    """A checked optimizer step over seeded sample positions of the whole parameter set.

    Run once, after timing.  Every rank copies to the host-visible gather its gradients at
    every sampled position and, at the positions of the tensors it owns, master / exp_avg /
    exp_avg_sq and the step count before the step, its reduced gradient after
    ``all_reduce_grads``, and its state after ``step``; every rank also copies its bf16
    parameters afterwards.  Rank 0 then recomputes the step at those positions with torch's
    own CUDA kernels running the reference's op sequence (hybrid_rl/optimizer.py:151-191):
    the owner's sum of the W ranks' gradients (fp32 adds in rank order, one rounding to the
    gradient dtype: exact at W <= 2, the build's documented reduction at W > 2; the
    reference's ``dist.reduce`` rounds per hop in NCCL's own order), the clip factor of this
    step's norm (optimizer.py:156-159), the update and the bf16 copy; every rank's parameter
    must equal the owner's.  The norm itself is checked against an independent fp64 sum of
    the reduced gradients.  Nothing here is timed."""

    def __init__(self, numels: list[int], per_rank: int, world: int, seed: int, dev):
        import numpy as np
        import torch
        rng = np.random.default_rng(seed)
        bounds = np.concatenate([[0], np.cumsum(numels)]).astype(np.int64)
        flat = rng.integers(0, int(bounds[-1]), size=per_rank * world, dtype=np.int64)
        # every tensor's first and last element as well (ragged tails, 1-element tensors)
        flat = np.unique(np.concatenate([flat, bounds[:-1], bounds[1:] - 1]))
        tensor = np.searchsorted(bounds, flat, side="right") - 1
        offset = flat - bounds[tensor]
        self.tensor = tensor
        self.k = len(flat)
        self.groups = []
        for i in np.unique(tensor):
            sel = tensor == i
            self.groups.append((int(i), torch.from_numpy(offset[sel]).to(dev)))
        self.dev = dev
        self.world = world

    def take(self, get, dtype):
        """Values at every sample position of the tensors ``get(i)`` returns (zeros where it
        returns None), concatenated in position order."""
        import torch
        parts = []
        for i, idx in self.groups:
            t = get(i)
            parts.append(torch.zeros(len(idx), dtype=dtype, device=self.dev) if t is None
                         else t.detach().reshape(-1)[idx].to(dtype))
        return torch.cat(parts)

    def gather(self, x):
        """[world, k] of every rank's x (raw bits travel unchanged)."""
        import torch
        import torch.distributed as dist
        if self.world == 1:
            return x[None]
        raw = x.contiguous().view(torch.uint8)  # bytes: NCCL moves them untouched
        out = torch.empty((self.world, raw.numel()), dtype=torch.uint8, device=self.dev)
        dist.all_gather_into_tensor(out.view(-1), raw)
        return out.view(x.dtype)


def _ordered_bits(x):
    """fp32 bit patterns mapped to integers that order like the values (ulp distances)."""
    import torch
    b = x.view(torch.int32).to(torch.int64)
    return torch.where(b < 0, -(b & 0x7FFFFFFF), b)


def checked_step(opt, params, inputs, numels, per_rank: int, max_norm: float = 1.0) -> dict:
    """One optimizer step with the sampled parity check; returns the bench line's
    ``parity`` object (on every rank; rank 0's is printed)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    world, dev = opt.world, params[0].device
    sync = torch.cuda.synchronize if dev.type == "cuda" else (lambda: None)
    sp = SampledParity(numels, per_rank, world, seed=20261202, dev=dev)
    gdt = params[0].dtype  # the benchmark's sets have one parameter dtype
    bits = torch.int16 if params[0].element_size() == 2 else torch.int32
    owner = torch.as_tensor(np.asarray(opt.owner)[sp.tensor], device=dev)
    owned = set(opt.param_steps)
    mine = lambda d: (lambda i: d[i] if i in owned else None)  # noqa: E731

    for p, g in zip(params, inputs):
        p.grad = g
    sync()
    g_pre = sp.gather(sp.take(lambda i: params[i].grad, gdt))
    st_pre = [sp.gather(sp.take(mine(d), torch.float32)) for d in (opt.master, opt.exp_avg, opt.exp_avg_sq)]
    steps = torch.zeros(len(params), dtype=torch.int64, device=dev)
    for i in owned:
        steps[i] = opt.param_steps[i]
    if world > 1:
        dist.all_reduce(steps)
    opt.all_reduce_grads()
    g_red = sp.gather(sp.take(mine({i: params[i].grad for i in owned}), gdt))
    # independent norm: fp64 sum of the squares of this rank's reduced gradients, all ranks
    acc = torch.zeros((), dtype=torch.float64, device=dev)
    for i in owned:
        g = params[i].grad
        if g is not None:
            for part in g.reshape(-1).split(1 << 26):
                acc += part.double().square().sum()
    if world > 1:
        dist.all_reduce(acc)
    norm = opt.clip_grad_norm(max_norm)
    p_pre = sp.take(lambda i: params[i].detach(), gdt)
    opt.step()
    sync()
    st_post = [sp.gather(sp.take(mine(d), torch.float32)) for d in (opt.master, opt.exp_avg, opt.exp_avg_sq)]
    p_post = sp.gather(sp.take(lambda i: params[i].detach(), gdt))

    # --- expected values, torch CUDA kernels, the reference's op sequence
    sel = owner[None]
    pick = lambda a: a.gather(0, sel)[0]  # noqa: E731  the owner's row at every position
    acc32 = g_pre[0].float()
    for r in range(1, world):
        acc32 = acc32 + g_pre[r].float()
    g_exp = acc32.to(gdt)
    red_bad = int((pick(g_red).view(bits) != g_exp.view(bits)).sum())
    exact = math.sqrt(float(acc))
    g_clip = g_exp.clone()
    if max_norm > 0 and norm > max_norm:
        g_clip.mul_(float(max_norm) / (norm + 1e-6))  # optimizer.py:156-159 (bf16 in place)
    master, m, v = (pick(a).clone() for a in st_pre)
    t_all = steps[torch.as_tensor(sp.tensor, device=dev)] + 1
    lr = torch.as_tensor(np.asarray(opt.lrs, dtype=np.float64)[sp.tensor], device=dev)
    b1, b2 = opt.betas
    for t in torch.unique(t_all).tolist():
        for lr_v in torch.unique(lr[t_all == t]).tolist():
            s = (t_all == t) & (lr == lr_v)
            gradient = g_clip[s].float()
            ms, ma, va = master[s], m[s], v[s]
            c1, c2 = 1.0 - b1 ** t, 1.0 - b2 ** t
            if opt.weight_decay:
                ms.mul_(1.0 - lr_v * opt.weight_decay)
            ma.mul_(b1).add_(gradient, alpha=1.0 - b1)
            va.mul_(b2).addcmul_(gradient, gradient, value=1.0 - b2)
            den = (va / c2).sqrt().add_(opt.eps)
            ms.addcdiv_(ma / c1, den, value=-lr_v)
            master[s], m[s], v[s] = ms, ma, va
    p_exp = master.to(gdt)
    fields = {"reduced_grad": red_bad}
    max_ulp = 0
    for name, got, want in (("master", pick(st_post[0]), master), ("exp_avg", pick(st_post[1]), m),
                            ("exp_avg_sq", pick(st_post[2]), v)):
        d = (_ordered_bits(got) - _ordered_bits(want)).abs()
        fields[name] = int((d != 0).sum())
        max_ulp = max(max_ulp, int(d.max()))
    fields["param_every_rank"] = int((p_post.view(bits) != p_exp.view(bits)[None]).sum())
    rel = abs(norm - exact) / exact if exact else abs(norm)
    changed = float((p_post[0].view(bits) != p_pre.view(bits)).double().mean())
    return {"changed_param_fraction": changed, "checked_positions": sp.k, "checked_values": sp.k * (4 + world), "mismatches": sum(fields.values()),
            "max_ulp": max_ulp, "fields": fields,
            "norm": {"returned": norm, "fp64_of_reduced": exact, "rel_err": rel, "ok": bool(rel <= 1e-6)},
            "reduction": "exact (W<=2)" if world <= 2 else f"fp32 rank-order sum rounded once to {str(gdt)[6:]}",
            "checker": "torch CUDA ops running the reference's op sequence at seeded positions (plus every "
                       "tensor's first and last element), after the timed region"}


# ---------------------------------------------------------------- GPU helpers
class PhaseTimer:
    """CUDA events around the optimizer's kernel launches, on the launching stream."""

    def __init__(self):
        self.enabled = False
        self._open = {}
        self.pairs: dict[str, list] = {}

    def begin(self, name):
        if self.enabled:
            import torch
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._open[name] = e

    def end(self, name):
        if self.enabled and name in self._open:
            import torch
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self.pairs.setdefault(name, []).append((self._open.pop(name), e))

    def per_step_ms(self, steps: int) -> dict[str, float]:
        """Total time of each phase over the timed region divided by the steps (phases that
        run several times a step, like the exchange rounds, add up)."""
        return {k: sum(a.elapsed_time(b) for a, b in v) / steps for k, v in self.pairs.items()}


class ClockSampler:
    """nvidia-smi samples (every 200 ms) for the duration of the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices: list[int]):
        self.gpus = set(gpu_indices)
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        self.file.flush()
        rows = []
        with open(self.file.name) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9 or not parts[0].isdigit() or int(parts[0]) not in self.gpus:
                    continue
                try:
                    rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[5:9]))
                except ValueError:
                    continue
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for _, _, _, flags in rows for k, v in enumerate(flags) if v.lower() == "active"})
        loaded = [r for r in rows if r[2] > 200.0] or rows  # samples under load (power above idle)
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows), "samples_under_load": len(loaded),
                "power_w_max": max(r[2] for r in rows)}


def measured_hbm_peak() -> tuple[float, str]:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic_per_param(mode: str) -> tuple[float | None, str | None]:
    """DRAM bytes per owned parameter of one AdamW launch writing the parameter copies in
    ``mode``, from the committed ncu record, and the record's path."""
    path = TRAFFIC_PROFILES[mode]
    try:
        with open(path) as f:
            return float(json.load(f)["traffic_bytes_per_param"]), os.path.relpath(path, ROOT)
    except (OSError, KeyError, ValueError):
        return None, None


def phase_roofline(how: str, ms: float, hbm_bytes: float, link_bytes: float, hbm_peak: float,
                   link_peak: float) -> dict:
    """One phase of a multi-GPU step against both of its resources: the target time is the
    slower of its HBM bytes at the HBM peak and its NVLink bytes at the link peak (GB/s), the
    resource that sets it is the bound, and ``frac`` = target / measured."""
    t_hbm, t_link = hbm_bytes / (hbm_peak * 1e9), link_bytes / (link_peak * 1e9)
    gbs = link_bytes / (ms * 1e-3) / 1e9
    return {"how": how, "bound": "nvlink" if t_link >= t_hbm else "hbm", "measured_ms": round(ms, 3),
            "target_ms": round(max(t_hbm, t_link) * 1e3, 3), "frac": round(max(t_hbm, t_link) * 1e3 / ms, 4),
            "nvlink_bytes": int(link_bytes), "hbm_bytes": int(hbm_bytes), "link_gbs_achieved": round(gbs, 1),
            "hbm_gbs_achieved": round(hbm_bytes / (ms * 1e-3) / 1e9, 1), "frac_of_link_peak": round(gbs / link_peak, 4),
            "frac_of_nominal_link": round(gbs / NOMINAL_NVLINK_GBS, 4)}


def measured_link_peak(world: int) -> tuple[float, str]:
    """Per-direction NVLink bandwidth at this world size: the best pattern of the committed
    ``bench.py --probe-links`` record at that size (or the nearest size probed), else the
    pool's published peer-copy figure."""
    try:
        with open(LINK_PROFILE) as f:
            by_world = json.load(f)["by_world"]
    except (OSError, KeyError, ValueError):
        return RECIPE_NVLINK_GBS, "recipe figure (no probe record)"
    sizes = sorted(int(k) for k in by_world)
    if not sizes:
        return RECIPE_NVLINK_GBS, "recipe figure (no probe record)"
    w = min(sizes, key=lambda s: (abs(s - world), -s))
    best = max(by_world[str(w)].items(), key=lambda kv: kv[1])
    return float(best[1]), f"measured: profiles/nvlink_peak.json, world {w}, {best[0]}"


def run_ours(args) -> None:
    import numpy as np
    import torch
    import torch.distributed as dist

    from hybridagent_b200 import ZeroOneAdamW, workloads

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)

    shapes = workloads.WORKLOADS[args.workload]()
    if args.max_params:
        shapes = workloads.truncated(shapes, args.max_params)
    numels = [math.prod(s) for s in shapes]
    n_params = sum(numels)

    # BASELINE config 1 is fp32 throughout with grads ~N(0,1e-3) and fresh state; the model-shaped
    # sets are bf16 with grads ~N(0,1e-4) and state pre-loaded at step 100
    fp32_set = args.workload == "config1_cpu"
    pdt = torch.float32 if fp32_set else torch.bfloat16
    # parameters (identical on every rank), ~N(0, 0.02)
    gen = torch.Generator(device=dev).manual_seed(1234)
    params = [torch.nn.Parameter((torch.randn(s, device=dev, generator=gen) * 0.02).to(pdt)) for s in shapes]
    opt = ZeroOneAdamW([{"params": params, "lr": 1e-6}], rank=rank, world_size=world, betas=(0.9, 0.999), eps=1e-8,
                       weight_decay=0.01)
    if not fp32_set:  # state pre-loaded at step 100: m ~N(0,1e-5), v ~|N(0,1e-8)|
        gs = torch.Generator(device=dev).manual_seed(99 + rank)
        for i in opt.param_steps:
            opt.exp_avg[i].normal_(0, 1e-5, generator=gs)
            opt.exp_avg_sq[i].normal_(0, 1e-8, generator=gs).abs_()
            opt.param_steps[i] = 100
    # this rank's gradients of the whole model (different per rank)
    gg = torch.Generator(device=dev).manual_seed(555 + rank)
    sigma = 1e-3 if fp32_set else 1e-4
    inputs = [(torch.randn(s, device=dev, generator=gg) * sigma).to(pdt) for s in shapes]
    owned = list(opt.param_steps)
    owned_params = sum(numels[i] for i in owned)
    torch.cuda.synchronize()

    def one_step():
        for p, g in zip(params, inputs):
            p.grad = g
        opt.all_reduce_grads()
        norm = opt.clip_grad_norm(1.0)
        opt.step()
        return norm

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(max(args.warmup, 3)):
        one_step()
    warmup = max(args.warmup, 3)
    timer = PhaseTimer()
    opt.timer = timer
    barrier()
    launches0 = opt.launches
    sampler = ClockSampler([local] if world == 1 else list(range(world))) if rank == 0 else contextlib.nullcontext()
    with sampler as clocks:
        barrier()
        start = torch.cuda.Event(enable_timing=True)
        stop = torch.cuda.Event(enable_timing=True)
        timer.enabled = True
        start.record()
        for _ in range(args.steps):
            norm = one_step()
        stop.record()
        barrier()
        timer.enabled = False
    launches = opt.launches - launches0
    writes = opt.write_stats()  # how the last timed update wrote the parameter copies
    ms = start.elapsed_time(stop) / args.steps
    phases = timer.per_step_ms(args.steps)
    t = torch.tensor([ms, phases.get("adamw", 0.0)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t[0])
    clock = clocks.summary() if rank == 0 else None

    # ---- end to end: gradients from pinned host memory each step, norm read back
    e2e = None
    if not args.no_e2e:
        pool_elems = min(max(numels), 1 << 31)
        host = torch.empty(pool_elems, dtype=pdt, pin_memory=True)
        host.copy_(inputs[int(np.argmax(numels))].reshape(-1)[:pool_elems].cpu())
        h2d_bytes = inputs[0].element_size() * n_params
        d2h_bytes = 8 * len(opt._classes)

        # double-buffered inputs: step k+1's gradients cross PCIe on a copy stream while step
        # k's optimizer runs (a data loader's prefetch); every step's copy and its norm read-back
        # are inside the timed region
        try:
            spare = [torch.empty_like(g) for g in inputs]
            bufs = [inputs, spare]
            how = "double-buffered: the next step's copy overlaps this step's optimizer"
        except torch.OutOfMemoryError:
            spare = None
            bufs = [inputs, inputs]
            how = "single-buffered (no room for a second gradient set)"
        copy_stream = torch.cuda.Stream(device=dev)
        copied = [torch.cuda.Event(), torch.cuda.Event()]
        used = [torch.cuda.Event(), torch.cuda.Event()]

        def h2d(slot):
            copy_stream.wait_event(used[slot])  # the step that read this set has finished
            with torch.cuda.stream(copy_stream):
                for g, n in zip(bufs[slot], numels):
                    g.view(-1).copy_(host[:n], non_blocking=True)
            copied[slot].record(copy_stream)

        def e2e_run(steps):
            main = torch.cuda.current_stream()
            for ev in used:
                ev.record(main)
            h2d(0)
            for k in range(steps):
                slot = k % 2 if spare is not None else 0
                main.wait_event(copied[slot])
                if k + 1 < steps and spare is not None:
                    h2d(1 - slot)
                for p, g in zip(params, bufs[slot]):
                    p.grad = g
                opt.all_reduce_grads()
                opt.clip_grad_norm(1.0)  # reads the norm back to the host
                opt.step()
                used[slot].record(main)
                if spare is None and k + 1 < steps:
                    h2d(0)

        e2e_run(2)
        barrier()
        t0 = time.perf_counter()
        e2e_run(args.e2e_steps)
        torch.cuda.synchronize()
        e2e_ms = (time.perf_counter() - t0) * 1e3 / args.e2e_steps
        te = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_ms = float(te[0])
        e2e = {"value": round(n_params / (e2e_ms * 1e-3) / 1e9, 3), "unit": "Gparams/s", "ms_per_step": round(e2e_ms, 3),
               "h2d_bytes_per_step": h2d_bytes, "d2h_bytes_per_step": d2h_bytes,
               "bound": "PCIe: the host-to-device copy of the step's gradients" if world == 1 else
                        f"the host: all {world} ranks copy the whole model's gradients out of one host's pinned "
                        "memory at once",
               "how": f"host wall clock over {args.e2e_steps} steps; every step copies all gradients from pinned host "
                      f"memory (per-tensor cudaMemcpyAsync, {how}) and reads the norm back in clip_grad_norm"}
        del spare, bufs

    # ---- one more step, checked at sampled positions against torch's CUDA kernels (not timed)
    parity = None
    if args.parity_per_rank > 0:
        parity = checked_step(opt, params, inputs, numels, args.parity_per_rank)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # BASELINE configuration 1 runs whole on the CPU; the model-shaped sets as a bounded sample
        base = (cpu_config1() if fp32_set else
                cpu_sample(args.workload, args.cpu_sample_params, steps=4, warmup=1))
        cpu = {k: base[k] for k in ("value", "unit", "cores", "kind", "sample", "impl", "ms_per_step")}

    # ---- the whole iteration at N > 1: a synthetic backward + the optimizer, gradient landing off
    # and on, on a second optimizer built once this one is released (not part of the timed step)
    landing = None
    if world > 1 and not args.no_landing and not fp32_set:
        from types import SimpleNamespace
        barrier()
        info = SimpleNamespace(comm_mode=opt.comm_mode, push_streams=opt.push_streams, push_ctas=opt.push_ctas,
                               gather_mode=opt.gather_mode, tail_split=opt.tail_split)
        opt.close()
        opt = info
        params = inputs = None
        import gc
        gc.collect()
        torch.cuda.empty_cache()
        try:
            landing = measure_landing(args, shapes, dev, rank, world, [0], min(args.steps, 5))
        except Exception as e:  # noqa: BLE001 -- an extra measurement after the timed region: its
            # failure (out of memory, where every rank allocates the same sizes and all raise
            # together) is reported in the line instead of losing the line
            landing = {"error": f"{type(e).__name__}: {(str(e).splitlines() or [''])[0]}"}

    if rank != 0:
        if world > 1:
            dist.barrier()
            if landing is None:
                opt.close()
            dist.destroy_process_group()
        return
    peak, peak_kind = measured_hbm_peak()
    adamw_ms = phases.get("adamw")
    # the update reads grad + master/m/v and writes master/m/v (26 B per owned param); the bf16 copy
    # costs 2 B per param when written in full, else 8 B per stored 4-element group (the groups of
    # every 32-byte sector that holds a changed value)
    delta = writes["mode"] == "changed groups"
    algo = (26 * owned_params + 8 * writes["changed_groups"]) if delta else ALGO_BYTES_ADAMW["bf16"] * owned_params
    achieved = algo / (adamw_ms * 1e-3) / 1e9 if adamw_ms else None
    tpp, tpp_src = profiled_traffic_per_param(writes["mode"])
    hbm_roof = {"bound": "hbm", "kernel": f"adamw_kernel<{'f32' if fp32_set else 'bf16'}>" +
                (" (changed groups of the bf16 copy)" if delta else ""),
                "param_writes": writes,
                "achieved": None if achieved is None else round(achieved, 1),
                "peak": peak, "unit": "GB/s",
                "frac": None if achieved is None else round(achieved / peak, 4),
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                else "fallback 6.65 TB/s",
                "algorithmic_bytes_per_launch": algo,
                "traffic": None if tpp is None else round(tpp * owned_params),
                "traffic_source": None if tpp is None else f"ncu dram__bytes_read+write per parameter of one launch "
                f"({tpp_src}), times this launch's parameters"}
    roofline, nvlink = hbm_roof, None
    if world > 1 and opt.comm_mode == "p2p":
        # per phase: its HBM bytes and the bytes it moves over NVLink per GPU; the phase is bound by
        # whichever takes longer at its measured peak, and the roofline line names the longest
        # phase with that resource.  push: this rank's gradients of the other ranks' tensors
        # ((W-1)/W of 2 B/param).  adamw: the update (its algorithmic HBM bytes, `algo`) and the
        # parameter all-gather: 2 B x (W-1) per owned param with full writes, or only the stored
        # groups (the update kernel's own count) with changed-sector writes
        link, link_src = measured_link_peak(world)
        foreign = n_params - owned_params
        push_how = ("copy engines, one stream per peer" if opt.push_streams < 0 else
                    f"copy engines on {opt.push_streams} streams + gather_kernel" if opt.push_streams > 0 else
                    f"gather_capped_kernel peer stores on {opt.push_ctas} CTAs" if opt.push_ctas > 0 else
                    "gather_kernel peer stores, one CTA per chunk")
        if opt.gather_mode == "ce":
            gather_how, moved = "adamw_kernel<bf16> in parts + copy-engine all-gather", 1.0
        elif delta:
            gather_how = "adamw_kernel<bf16, PEERS, DELTA>: stores of the changed 4-element groups, fused"
            moved = writes["changed_groups"] / max(writes["groups"], 1)
        else:
            gather_how, moved = "adamw_kernel<bf16, PEERS>: every group stored into every peer, fused", 1.0
        adamw_link = int(2 * owned_params * (world - 1) * moved)
        nvlink = {"link_peak_gbs": link, "link_peak_source": link_src, "nominal_gbs": NOMINAL_NVLINK_GBS,
                  "all_gather_fraction_moved": round(moved, 6)}
        # HBM: push -- read every gradient, write this rank's own pieces and receive the peers'
        # (~2 B/param each way); adamw -- 28 B per owned param plus the peers' parameter stores landing here
        for name, how, link_bytes, hbm_bytes in (("push", push_how, 2 * foreign, 4 * n_params),
                                                 ("adamw", gather_how, adamw_link, algo + int(2 * foreign * moved))):
            ms_phase = phases.get(name)
            if ms_phase:
                nvlink[name] = phase_roofline(how, ms_phase, hbm_bytes, link_bytes, peak, link)
        dom = max((k for k in ("push", "adamw") if k in nvlink), key=lambda k: nvlink[k]["measured_ms"], default=None)
        if dom is not None and nvlink[dom]["bound"] == "nvlink":
            d = nvlink[dom]
            roofline = {"bound": "nvlink", "kernel": d["how"], "phase": dom, "achieved": d["link_gbs_achieved"],
                        "peak": link, "unit": "GB/s", "frac": d["frac_of_link_peak"],
                        "frac_of_nominal": d["frac_of_nominal_link"], "peak_source": link_src,
                        "algorithmic_bytes_per_launch": d["nvlink_bytes"], "traffic": None,
                        "traffic_source": "NVLink bytes are algorithmic; ncu's NVLink counters were not readable "
                                          "on this pool", "hbm_adamw": hbm_roof}
        elif dom is not None:
            roofline = dict(hbm_roof, phase=dom)
    out = {
        "metric": "ZeRO-1 AdamW step Gparams/s",
        "value": round(n_params / (ms_max * 1e-3) / 1e9, 3),
        "unit": "Gparams/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": warmup,
        "ms_per_step": round(ms_max, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "fp32",
        "data": "synthetic",
        "config": {"workload": args.workload, "params": n_params, "tensors": len(shapes),
                   "param_dtype": "fp32" if fp32_set else "bf16", "state_dtype": "fp32",
                   "parallelism": f"zero1_dp{world}",
                   "push": push_how if world > 1 and nvlink else None,
                   "all_gather": gather_how if world > 1 and nvlink else None,
                   "tail_split": opt.tail_split if world > 1 and nvlink else None,
                   "l2": f"inputs larger than L2: {(n_params * 16) / 1e9 / world:.1f} GB of grads+state per GPU "
                         "per step vs 126 MB L2, no flush"},
        "roofline": roofline,
        "phases_ms": {k: round(v, 4) for k, v in phases.items()},
        "comm_mode": opt.comm_mode,
        "roofline_fused": nvlink,
        "last_norm": norm,
        "parity": parity,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "clocks": clock,
        "gpu_launches": launches,
        "iteration_with_backward": landing,
    }
    print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        if landing is None:
            opt.close()
        dist.destroy_process_group()


def measure_landing(args, shapes, dev, rank: int, world: int, caps: list[int], steps: int) -> dict:
    """Forward + backward + optimizer iterations with gradient landing off and on, on a fresh
    optimizer built with ``land_grads=True`` (N > 1: the early pushes of the exchange, receive
    window sized for two rounds; N = 1: the norm's square sums taken as the gradients land).
    The synthetic backward: one ``linear`` per matrix over ``args.tokens`` tokens, a dot product
    per vector.  Per variant the forward + backward time, the optimizer time left after
    backward, and their sum, CUDA events, mean over ``steps``, max over ranks."""
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F

    from hybridagent_b200 import ZeroOneAdamW

    n_params = sum(math.prod(s) for s in shapes)
    window = 2 * n_params + (256 << 20) if world > 1 else 0  # every piece may be pushed as it lands
    saved = os.environ.get("HYBRIDAGENT_B200_RECV_BYTES")
    if world > 1:
        os.environ["HYBRIDAGENT_B200_RECV_BYTES"] = str(window)
    gen = torch.Generator(device=dev).manual_seed(1234)
    params = [torch.nn.Parameter((torch.randn(s, device=dev, generator=gen) * 0.02).to(torch.bfloat16))
              for s in shapes]
    try:
        opt = ZeroOneAdamW([{"params": params, "lr": 1e-6}], rank=rank, world_size=world, weight_decay=0.01,
                           land_grads=True)
    finally:
        if saved is None:
            os.environ.pop("HYBRIDAGENT_B200_RECV_BYTES", None)
        else:
            os.environ["HYBRIDAGENT_B200_RECV_BYTES"] = saved
    gx = torch.Generator(device=dev).manual_seed(777 + rank)
    T = args.tokens
    dims_in = sorted({s[1] for s in shapes if len(s) == 2})
    dims_out = max(s[0] for s in shapes if len(s) == 2)
    x = {d: (torch.randn(T, d, device=dev, generator=gx) * 0.02).to(torch.bfloat16) for d in dims_in}
    r = (torch.randn(T, dims_out, device=dev, generator=gx) * 1e-3).to(torch.bfloat16)
    v = {s[0]: (torch.randn(s[0], device=dev, generator=gx) * 1e-3).to(torch.bfloat16)
         for s in shapes if len(s) == 1}

    def fwd_bwd():
        terms = []
        for p in params:
            if p.dim() == 2:
                terms.append((F.linear(x[p.shape[1]], p) * r[:, :p.shape[0]]).sum())
            else:
                terms.append((p * v[p.shape[0]]).sum())
        torch.autograd.backward(terms)

    def one(ev):
        opt.zero_grad(set_to_none=True)
        ev[0].record()
        fwd_bwd()
        ev[1].record()
        opt.all_reduce_grads()
        opt.clip_grad_norm(1.0)
        opt.step()
        ev[2].record()

    warm = max(args.warmup, 3)
    out = {}
    for variant in ["off"] + [f"on_ctas{n}" for n in caps]:
        opt.landing_enabled = variant != "off"
        if opt.landing_enabled:  # N > 1: CTAs of the early pushes; N = 1: of the square sums
            opt.land_ctas = int(variant[len("on_ctas"):])
        launches0 = opt.land_launches if world > 1 else opt.land_norm_steps
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
        for _ in range(warm):
            one([torch.cuda.Event(enable_timing=True) for _ in range(3)])
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        for ev in evs:
            one(ev)
        torch.cuda.synchronize()
        fb = sum(e[0].elapsed_time(e[1]) for e in evs) / len(evs)
        st = sum(e[1].elapsed_time(e[2]) for e in evs) / len(evs)
        t = torch.tensor([fb, st, fb + st], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out[variant] = {"fwd_bwd_ms": round(float(t[0]), 3), "step_after_backward_ms": round(float(t[1]), 3),
                        "total_ms": round(float(t[2]), 3)}
        if world > 1:
            out[variant]["early_push_calls_per_step"] = (opt.land_launches - launches0) // (len(evs) + warm)
        else:
            out[variant]["landed_norm_steps"] = f"{opt.land_norm_steps - launches0}/{len(evs) + warm}"
    comm_mode = opt.comm_mode
    if world > 1:
        dist.barrier()
    opt.close()
    best = min((k for k in out if k != "off"), key=lambda k: out[k]["total_ms"])
    return {"variants": out, "best": best, "saved_ms": round(out["off"]["total_ms"] - out[best]["total_ms"], 3),
            "steps": steps, "warmup": warm, "tokens": T, "recv_window_bytes": window, "comm_mode": comm_mode}


def run_landing(args) -> None:
    """``--landing``: prints measure_landing's result for the workload as its own JSON line."""
    import torch
    import torch.distributed as dist

    from hybridagent_b200 import workloads

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    shapes = workloads.WORKLOADS[args.workload]()
    if args.max_params:
        shapes = workloads.truncated(shapes, args.max_params)
    res = measure_landing(args, shapes, dev, rank, world, [int(x) for x in args.land_ctas.split(",")], args.steps)
    if rank == 0:
        out, best = res["variants"], res["best"]
        line = {"metric": "fwd_bwd_plus_step_ms", "value": out[best]["total_ms"], "unit": "ms", "n_gpus": world,
                "steps": args.steps, "warmup": res["warmup"], "higher_is_better": False, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": args.workload, "params": sum(math.prod(s) for s in shapes),
                           "tensors": len(shapes), "tokens": res["tokens"],
                           "recv_window_bytes": res["recv_window_bytes"],
                           "comm_mode": res["comm_mode"], "parallelism": f"zero1-dp{world}"},
                "landing": out, "best": best, "saved_ms": res["saved_ms"]}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_probe_links(args) -> None:
    """NVLink per-direction bandwidth between this node's GPUs, measured the ways the step
    moves data (one JSON line from rank 0; the figures behind the link roofline).

    Every rank moves ``--probe-bytes`` at once (all ranks together, CUDA events on every
    stream used, max over ranks, best of ``--steps``), into IPC-mapped buffers of its peers:
      ce_one_peer   one cudaMemcpyAsync to the next rank (ring);
      ce_all_peers  1/(W-1) of the bytes to every peer, one copy-engine stream per peer;
      ce_pull_all   the same bytes read from every peer by the copy engines;
      sm_one_peer   the library's copy kernel (ha_gather) storing to the next rank;
      sm_all_peers  the copy kernel storing 1/(W-1) to every peer (one launch, chunks interleaved);
      sm_pull_all   the copy kernel loading 1/(W-1) from every peer into local memory.
    Plain loads, stores and copies only (no TMA, no multicast)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from hybridagent_b200 import _lib, layout
    from hybridagent_b200.p2p import DeviceBuffer, PeerMap

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world < 2 or world != args.gpus:
        raise SystemExit("--probe-links needs --gpus N > 1 under torchrun")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    total = args.probe_bytes // (2 * (world - 1) * 256) * (2 * (world - 1) * 256)  # whole 16-byte vectors per peer
    per_peer = total // (world - 1)
    src = DeviceBuffer(total // 2, torch.bfloat16, dev)
    src.tensor.view(torch.int16).copy_(torch.arange(total // 2, device=dev, dtype=torch.int32).to(torch.int16))
    recv = DeviceBuffer(world * total // 2, torch.bfloat16, dev)  # region r: what rank r sent here
    pm = PeerMap({"src": src, "recv": recv}, rank, world)
    if not pm.ok:
        raise SystemExit(f"peer mapping failed: {pm.error}")
    nxt = (rank + 1) % world
    peers = [(rank + 1 + j) % world for j in range(world - 1)]
    streams = [torch.cuda.Stream(device=dev) for _ in peers]
    main = torch.cuda.current_stream()

    def entries(kind: str) -> list[tuple[int, int, int]]:
        """(src address, dst address, bytes) of this rank's copies for a pattern."""
        if kind == "one":
            return [(src.ptr, pm.bases["recv"][nxt] + rank * total, total)]
        if kind == "push":
            return [(src.ptr + j * per_peer, pm.bases["recv"][q] + rank * total + j * per_peer, per_peer)
                    for j, q in enumerate(peers)]
        # pull: peer q's slice j of its source into region q of this rank's own buffer
        return [(pm.bases["src"][q] + j * per_peer, recv.ptr + q * total + j * per_peer, per_peer)
                for j, q in enumerate(peers)]

    def table(ents):
        t = np.zeros(len(ents), dtype=_lib.COPY_DTYPE)
        for k, (a, b, n) in enumerate(ents):
            t[k]["src"], t[k]["dst"], t[k]["numel"] = a, b, n // 2
        return t

    def run_ce(ents):
        ready = torch.cuda.Event()
        ready.record(main)
        for st, e in zip(streams, ents):
            st.wait_event(ready)
            _lib.call("ha_copy_async", _lib.np_ptr(table([e])), 1, 2, st.cuda_stream)
        for st in streams[:len(ents)]:
            main.wait_stream(st)

    sm_tabs = {}

    def run_sm(kind):
        if kind not in sm_tabs:
            ents = entries(kind)
            t = table(ents)
            counts = t["numel"].astype(np.int64)
            ch = layout.interleaved_chunks(np.arange(len(ents)), np.arange(len(ents)), counts, 0, len(ents),
                                           _lib.HA_ADAMW_CHUNK)
            sm_tabs[kind] = (torch.from_numpy(t.view(np.uint8).copy()).to(dev),
                             torch.from_numpy(ch.view(np.uint8).copy()).to(dev), len(ch))
        t, ch, n = sm_tabs[kind]
        _lib.call("ha_gather", t.data_ptr(), ch.data_ptr(), n, _lib.HA_ADAMW_CHUNK, 2, main.cuda_stream)

    patterns = {"ce_one_peer": lambda: run_ce(entries("one")), "ce_all_peers": lambda: run_ce(entries("push")),
                "ce_pull_all": lambda: run_ce(entries("pull")), "sm_one_peer": lambda: run_sm("one"),
                "sm_all_peers": lambda: run_sm("push"), "sm_pull_all": lambda: run_sm("pull")}
    results = {}
    for name, fn in patterns.items():
        best = None
        for it in range(max(args.warmup, 1) + max(args.steps, 1)):
            dist.barrier()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(main)
            fn()
            b.record(main)
            torch.cuda.synchronize()
            t = torch.tensor([a.elapsed_time(b)], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            if it >= max(args.warmup, 1):
                best = float(t) if best is None else min(best, float(t))
        results[name] = {"ms": round(best, 4), "gbs_per_direction": round(total / (best * 1e-3) / 1e9, 1)}
    # the last pattern wrote region q of this rank's buffer from peer q's source: check the bytes
    dist.barrier()
    got, want = recv.tensor.view(torch.int16), src.tensor.view(torch.int16)
    ok = all(torch.equal(got[q * total // 2 + j * per_peer // 2:q * total // 2 + (j + 1) * per_peer // 2],
                         want[j * per_peer // 2:(j + 1) * per_peer // 2]) for j, q in enumerate(peers))
    flag = torch.tensor([0 if ok else 1], device=dev)
    dist.all_reduce(flag)
    if rank == 0:
        print(json.dumps({"probe": "nvlink", "n_gpus": world, "bytes_per_rank": total, "steps": args.steps,
                          "warmup": args.warmup, "data_ok": int(flag) == 0, "results": results,
                          "how": "every rank at once, CUDA events on the launching stream (copy streams joined), "
                                 "max over ranks, best of the timed repetitions; bytes = this rank's egress "
                                 "(ingress for the pulls)"}), flush=True)
    dist.barrier()
    torch.cuda.synchronize()
    pm.close()
    dist.barrier()
    dist.destroy_process_group()


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.probe_links:
        run_probe_links(args)
    elif args.landing:
        run_landing(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
