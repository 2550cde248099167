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
  roofline     the fused AdamW kernel: 28 algorithmic bytes per owned parameter over its
               CUDA-event duration on the launch stream, against the measured HBM copy
               peak; traffic = ncu DRAM bytes per launch from the committed profile;
  cpu_baseline the reference's op sequence on this host's CPU cores (N=1, rank 0), on a
               bounded sample of the same parameter set;
  clocks       nvidia-smi samples taken during the timed region.
``--impl reference`` times only that CPU implementation (rank 0; other ranks exit).

``--landing`` (N > 1) measures gradient landing instead and prints its own JSON line: a
synthetic forward + backward whose weight gradients are GEMMs over ``--tokens`` tokens
(one ``linear`` per matrix, a dot product per vector) followed by the optimizer sequence,
with the early pushes off and on (same optimizer, receive window sized for two rounds so
the whole exchange can start during backward); per variant the forward + backward time,
the optimizer time left after backward, and their sum, max over ranks.
"""
from __future__ import annotations

import argparse
import contextlib
import datetime
import json
import math
import os
import re
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
NVLINK_GBS = 770.0  # measured peer copy per direction on this pool's B200s (the NVLink roofline reference)
TRAFFIC_PROFILE = os.path.join(ROOT, "profiles", "adamw_kernel_qwen3_8b.md")


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
    ap.add_argument("--landing", action="store_true", help="measure gradient landing (N > 1)")
    ap.add_argument("--tokens", type=int, default=2048, help="tokens of the --landing synthetic backward")
    ap.add_argument("--land-ctas", default="0,64", help="--landing: comma-separated CTA caps of the early "
                    "pushes to measure (0: copy engines)")
    return ap.parse_args()


# ---------------------------------------------------------------- CPU baseline (reference op sequence)
def cpu_baseline(workload: str, sample_params: int, steps: int = 4, warmup: int = 1) -> dict:
    """The reference's per-tensor eager op sequence (hybrid_rl/optimizer.py:148-191, as
    restated op for op in oracle/torch_ops.py) on CPU tensors over the leading tensors of
    the parameter set, bf16 params / grads with fp32 state at step 100, all host threads."""
    import torch

    from hybridagent_b200 import workloads
    from oracle.torch_ops import TorchZeroOneW1

    torch.set_num_threads(len(os.sched_getaffinity(0)))  # every host core (torchrun would leave 1)
    shapes = workloads.truncated(workloads.WORKLOADS[workload](), sample_params)
    n = sum(math.prod(s) for s in shapes)
    g = torch.Generator().manual_seed(7)
    params = [(torch.randn(s, generator=g) * 0.02).to(torch.bfloat16) for s in shapes]
    opt = TorchZeroOneW1(params, 1e-6, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
    for i, s in enumerate(shapes):
        opt.exp_avg[i].normal_(0, 1e-5, generator=g)
        opt.exp_avg_sq[i].normal_(0, 1e-8, generator=g).abs_()
        opt.steps[i] = 100
    grads = [(torch.randn(s, generator=g) * 1e-4).to(torch.bfloat16) for s in shapes]
    times = []
    for k in range(warmup + steps):
        fresh = [x.clone() for x in grads]  # the step clips its gradients in place
        t0 = time.perf_counter()
        opt.step(fresh, 1.0)
        dt = time.perf_counter() - t0
        if k >= warmup:
            times.append(dt)
    sec = statistics.median(times)
    return {"value": round(n / sec / 1e9, 4), "unit": "Gparams/s", "cores": torch.get_num_threads(),
            "kind": "port", "ms_per_step": round(sec * 1e3, 2),
            "sample": f"leading {len(shapes)} tensors of {workload} ({n} params), bf16 params/grads, fp32 state; "
                      f"median of {steps} steps after {warmup} warm-up; torch {torch.__version__} CPU, "
                      f"{len(os.sched_getaffinity(0))} host CPUs visible"}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # one CPU measurement per job, on rank 0
    base = cpu_baseline(args.workload, args.cpu_sample_params, steps=min(max(args.steps, 1), 4), warmup=1)
    out = {"metric": "ZeRO-1 AdamW step Gparams/s", "value": base["value"], "unit": "Gparams/s",
           "impl": "reference", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": base["ms_per_step"], "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
           "dtype": "fp32", "data": "synthetic",
           "config": {"workload": args.workload, "sample": base["sample"]},
           "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
           "e2e": {"value": base["value"], "unit": "Gparams/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


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


def profiled_traffic_per_param() -> float | None:
    """DRAM bytes per owned parameter of one AdamW launch, from the committed ncu summary."""
    try:
        text = open(TRAFFIC_PROFILE).read()
    except OSError:
        return None
    m = re.search(r"traffic_bytes_per_param:\s*([0-9.]+)", text)
    return float(m.group(1)) if m else None


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

    # parameters (identical on every rank), bf16, ~N(0, 0.02)
    gen = torch.Generator(device=dev).manual_seed(1234)
    params = [torch.nn.Parameter((torch.randn(s, device=dev, generator=gen) * 0.02).to(torch.bfloat16))
              for s in shapes]
    opt = ZeroOneAdamW([{"params": params, "lr": 1e-6}], rank=rank, world_size=world, betas=(0.9, 0.999), eps=1e-8,
                       weight_decay=0.01)
    # state pre-loaded at step 100: m ~N(0,1e-5), v ~|N(0,1e-8)|
    gs = torch.Generator(device=dev).manual_seed(99 + rank)
    for i in opt.param_steps:
        opt.exp_avg[i].normal_(0, 1e-5, generator=gs)
        opt.exp_avg_sq[i].normal_(0, 1e-8, generator=gs).abs_()
        opt.param_steps[i] = 100
    # this rank's gradients of the whole model, ~N(0, 1e-4) bf16 (different per rank)
    gg = torch.Generator(device=dev).manual_seed(555 + rank)
    inputs = [(torch.randn(s, device=dev, generator=gg) * 1e-4).to(torch.bfloat16) for s in shapes]
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
        host = torch.empty(pool_elems, dtype=torch.bfloat16, pin_memory=True)
        host.copy_(inputs[int(np.argmax(numels))].reshape(-1)[:pool_elems].cpu())
        h2d_bytes = 2 * n_params
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
               "how": f"host wall clock over {args.e2e_steps} steps; every step copies all gradients from pinned host "
                      f"memory (per-tensor cudaMemcpyAsync, {how}) and reads the norm back in clip_grad_norm"}
        del spare, bufs

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.workload, args.cpu_sample_params)

    if rank != 0:
        if world > 1:
            dist.barrier()
            opt.close()
            dist.destroy_process_group()
        return
    peak, peak_kind = measured_hbm_peak()
    adamw_ms = phases.get("adamw")
    algo = ALGO_BYTES_ADAMW["bf16"] * owned_params
    achieved = algo / (adamw_ms * 1e-3) / 1e9 if adamw_ms else None
    tpp = profiled_traffic_per_param()
    nvlink = None
    if world > 1 and opt.comm_mode == "p2p":
        # fused compute + collective kernels: target time = max(HBM bytes / HBM peak, NVLink bytes / link)
        foreign = n_params - owned_params  # gradients this rank sends, parameters it receives
        push_link = 2 * foreign
        adamw_link = 2 * owned_params * (world - 1)
        nvlink = {}
        for name, link_bytes, hbm_bytes in (("push", push_link, 4 * n_params),
                                            ("adamw", adamw_link, algo + 2 * foreign)):
            ms_phase = phases.get(name)
            if not ms_phase:
                continue
            target = max(hbm_bytes / (peak * 1e9), link_bytes / (NVLINK_GBS * 1e9)) * 1e3
            nvlink[name] = {"measured_ms": round(ms_phase, 3), "target_ms": round(target, 3),
                            "frac": round(target / ms_phase, 4), "nvlink_bytes": link_bytes, "hbm_bytes": hbm_bytes,
                            "link_gbs_achieved": round(link_bytes / (ms_phase * 1e-3) / 1e9, 1)}
        nvlink["link_peak"] = f"{NVLINK_GBS} GB/s per direction (measured peer copy)"
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
                   "param_dtype": "bf16", "state_dtype": "fp32", "parallelism": f"zero1_dp{world}",
                   "l2": f"inputs larger than L2: {(n_params * 16) / 1e9 / world:.0f} GB of grads+state per GPU "
                         "per step vs 126 MB L2, no flush"},
        "roofline": {"bound": "hbm", "kernel": "adamw_kernel<bf16>",
                     "achieved": None if achieved is None else round(achieved, 1),
                     "peak": peak, "unit": "GB/s",
                     "frac": None if achieved is None else round(achieved / peak, 4),
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                     else "fallback 6.65 TB/s",
                     "algorithmic_bytes_per_launch": algo,
                     "traffic": None if tpp is None else round(tpp * owned_params),
                     "traffic_source": None if tpp is None else "ncu dram__bytes_read+write per launch, "
                     "profiles/adamw_kernel_qwen3_8b.md, scaled to this launch's parameters"},
        "phases_ms": {k: round(v, 4) for k, v in phases.items()},
        "comm_mode": opt.comm_mode,
        "roofline_fused": nvlink,
        "last_norm": norm,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "clocks": clock,
        "gpu_launches": launches,
    }
    print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        opt.close()
        dist.destroy_process_group()


def run_landing(args) -> None:
    """Gradient landing: forward + backward + optimizer step, early pushes off vs on."""
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F

    from hybridagent_b200 import ZeroOneAdamW, workloads

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus or world < 2:
        raise SystemExit("--landing needs --gpus N > 1 under torchrun")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    shapes = workloads.WORKLOADS[args.workload]()
    if args.max_params:
        shapes = workloads.truncated(shapes, args.max_params)
    n_params = sum(math.prod(s) for s in shapes)
    # a receive window of two rounds: every piece may be pushed while its gradient lands
    os.environ["HYBRIDAGENT_B200_RECV_BYTES"] = str(2 * n_params + (256 << 20))
    gen = torch.Generator(device=dev).manual_seed(1234)
    params = [torch.nn.Parameter((torch.randn(s, device=dev, generator=gen) * 0.02).to(torch.bfloat16))
              for s in shapes]
    opt = ZeroOneAdamW([{"params": params, "lr": 1e-6}], rank=rank, world_size=world, weight_decay=0.01,
                       land_grads=True)
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

    out = {}
    caps = [int(x) for x in args.land_ctas.split(",")]
    for variant in ["off"] + [f"on_ctas{n}" for n in caps]:
        opt.landing_enabled = variant != "off"
        if opt.landing_enabled:
            opt.land_ctas = int(variant[len("on_ctas"):])
        launches0 = opt.land_launches
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
        for _ in range(max(args.warmup, 3)):
            one([torch.cuda.Event(enable_timing=True) for _ in range(3)])
        dist.barrier()
        torch.cuda.synchronize()
        for ev in evs:
            one(ev)
        torch.cuda.synchronize()
        fb = sum(e[0].elapsed_time(e[1]) for e in evs) / len(evs)
        st = sum(e[1].elapsed_time(e[2]) for e in evs) / len(evs)
        t = torch.tensor([fb, st, fb + st], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out[variant] = {"fwd_bwd_ms": round(float(t[0]), 3), "step_after_backward_ms": round(float(t[1]), 3),
                        "total_ms": round(float(t[2]), 3),
                        "early_push_calls_per_step": (opt.land_launches - launches0) // (len(evs) + max(args.warmup, 3))}
    best = min((k for k in out if k != "off"), key=lambda k: out[k]["total_ms"])
    if rank == 0:
        line = {"metric": "fwd_bwd_plus_step_ms", "value": out[best]["total_ms"], "unit": "ms", "n_gpus": world,
                "steps": args.steps, "warmup": max(args.warmup, 3), "higher_is_better": False, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": args.workload, "params": n_params, "tensors": len(shapes), "tokens": T,
                           "recv_window_bytes": int(os.environ["HYBRIDAGENT_B200_RECV_BYTES"]),
                           "comm_mode": opt.comm_mode, "parallelism": f"zero1-dp{world}"},
                "landing": out, "best": best,
                "saved_ms": round(out["off"]["total_ms"] - out[best]["total_ms"], 3)}
        print(json.dumps(line), flush=True)
    dist.barrier()
    opt.close()
    dist.destroy_process_group()


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.landing:
        run_landing(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
