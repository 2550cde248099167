"""One rank of the multi-GPU parity run (launched by tests/test_multi_gpu.py through
torchrun).  Drives hybridagent_b200.ZeroOneAdamW at world size N over NCCL on a golden
case and writes this rank's results for the test to compare."""
from __future__ import annotations

import datetime
import math
import os
import pickle
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.dirname(HERE), HERE, os.path.join(HERE, "golden")]


def peer_delay(out_dir: str) -> None:
    """Both ranks take one step; then rank 1 stalls on the host (a 12 s sleep, nothing of
    its in flight) while rank 0 starts the next step.  Rank 0's first collective must end
    in CommFailure after the 5 s watchdog timeout, before any of its kernels reads or
    writes rank 1's memory; rank 1, resuming, learns of the failure on the host (rank 0's
    result file) and launches nothing.  Progress lines and periodic stack dumps go to files
    for diagnosis."""
    import faulthandler
    import time

    import torch
    import torch.distributed as dist

    from cases import CASES_BY_NAME
    from helpers import to_torch
    from hybridagent_b200 import ZeroOneAdamW
    from hybridagent_b200.comm import CommFailure

    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    log = open(os.path.join(out_dir, f"rank{rank}.log"), "w", buffering=1)
    faulthandler.dump_traceback_later(20, repeat=True, file=log)
    t_start = time.monotonic()

    def note(msg):
        log.write(f"{time.monotonic() - t_start:8.3f} {msg}\n")

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    case = CASES_BY_NAME["bf16_world2"]
    params = [torch.nn.Parameter(to_torch(p, case.dtype, s, dev)) for p, s in zip(case.initial_params(), case.shapes)]
    opt = ZeroOneAdamW([{"params": params, "lr": case.lr}], rank=rank, world_size=world, comm_timeout_s=5.0)
    note(f"built, mode {opt.comm_mode}")

    def step(s):
        opt.zero_grad(set_to_none=True)
        for p, g, shape in zip(params, case.grads(s, rank), case.shapes):
            p.grad = None if g is None else to_torch(g, case.dtype, shape, dev)
        note(f"step {s}: all_reduce_grads")
        opt.all_reduce_grads()
        note(f"step {s}: clip_grad_norm")
        opt.clip_grad_norm(case.max_norm)
        note(f"step {s}: step")
        opt.step()

    step(0)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    note("step 0 done on both ranks")
    result = {"rank": rank, "mode": opt.comm_mode}
    if rank == 1:
        time.sleep(12.0)  # host-injected stall, nothing in flight
        note("resuming after the stall")
        if os.path.exists(os.path.join(out_dir, "rank0.pkl")):
            # rank 0 already gave up on this exchange: learn it on the host and launch nothing
            result["error"] = "peer reported CommFailure before this rank's next launch"
            result["elapsed"] = 0.0
            note(f"result {result}")
            with open(os.path.join(out_dir, f"rank{rank}.pkl"), "wb") as f:
                pickle.dump(result, f)
            faulthandler.cancel_dump_traceback_later()
            log.close()
            os._exit(0)
    t0 = time.monotonic()
    try:
        step(1)
        torch.cuda.synchronize()
        result["error"] = None
    except CommFailure as e:
        result["error"] = str(e)
    result["elapsed"] = time.monotonic() - t0
    note(f"result {result}")
    with open(os.path.join(out_dir, f"rank{rank}.pkl"), "wb") as f:
        pickle.dump(result, f)
    faulthandler.cancel_dump_traceback_later()
    log.close()
    os._exit(0)  # the communicator is aborted: skip collective teardown


def mixed(out_dir: str) -> None:
    """bf16, fp32 and fp16 parameters in one optimizer at world size W (three dtype classes,
    each with its own exchange rounds), three steps; writes this rank's results."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from helpers import Z, to_numpy, to_torch
    from hybridagent_b200 import ZeroOneAdamW

    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    spec = mixed_spec()
    rng = np.random.default_rng(3)
    init = [Z.narrow((rng.standard_normal(int(np.prod(s))) * 0.02).astype(np.float32), d) for s, d in spec]
    params = [torch.nn.Parameter(to_torch(b, d, s, dev)) for b, (s, d) in zip(init, spec)]
    opt = ZeroOneAdamW([{"params": params[:4], "lr": 1e-3}, {"params": params[4:], "lr": 3e-4}], rank=rank,
                       world_size=world, weight_decay=0.05)
    norms = []
    for step in range(3):
        opt.zero_grad(set_to_none=True)
        for p, g, (s, d) in zip(params, mixed_grads(step, rank), spec):
            p.grad = None if g is None else to_torch(g, d, s, dev)
        opt.all_reduce_grads()
        norms.append(opt.clip_grad_norm(1.0))
        opt.step()
    torch.cuda.synchronize()
    result = {"rank": rank, "norms": norms, "owner": opt.owner, "mode": opt.comm_mode,
              "params": [to_numpy(p.data, d) for p, (_, d) in zip(params, spec)],
              "state": {i: (to_numpy(opt.master[i], 0), to_numpy(opt.exp_avg[i], 0), to_numpy(opt.exp_avg_sq[i], 0),
                            opt.param_steps[i]) for i in opt.param_steps}}
    with open(os.path.join(out_dir, f"rank{rank}.pkl"), "wb") as f:
        pickle.dump(result, f)
    dist.barrier()
    opt.close()
    dist.destroy_process_group()


def mixed_spec():
    from helpers import Z
    # one fp16 tensor: the other rank's fp16 segment is empty
    return [((64, 96), Z.BF16), ((33,), Z.F32), ((1000,), Z.BF16), ((48, 16), Z.F32), ((40, 24), Z.F16),
            ((4097,), Z.BF16), ((7,), Z.BF16), ((256, 64), Z.F32)]


def mixed_grads(step, rank):
    """Rank-dependent gradients; tensor 2 is absent on rank 1 at step 1."""
    import numpy as np

    from helpers import Z
    rng = np.random.default_rng([11, step, rank])
    out = []
    for k, (s, d) in enumerate(mixed_spec()):
        g = Z.narrow((rng.standard_normal(int(np.prod(s))) * 0.05).astype(np.float32), d)
        out.append(None if (k == 2 and step == 1 and rank == 1) else g)
    return out


def main(name: str, out_dir: str) -> None:
    import torch
    import torch.distributed as dist

    from cases import CASES_BY_NAME
    from helpers import to_numpy, to_torch
    from hybridagent_b200 import ZeroOneAdamW

    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    case = CASES_BY_NAME[name]
    # gradient landing: the gradients come out of two backward passes that each contribute
    # half of them (exact in binary floating point), so every landed gradient is pushed
    # early twice and the second push must win
    landing = os.environ.get("WORKER_LANDING") == "1"
    params = [torch.nn.Parameter(to_torch(p, case.dtype, s, dev)) for p, s in zip(case.initial_params(), case.shapes)]
    opt = ZeroOneAdamW([{"params": params, "lr": case.lr}], rank=rank, world_size=world, betas=case.betas,
                       eps=case.eps, weight_decay=case.weight_decay, land_grads=landing)
    assert opt.landing_enabled == (landing and opt.comm_mode == "p2p")
    if case.preload_state:
        for i in opt.param_steps:
            master, m, v, step = case.preload(i)
            opt.master[i].copy_(torch.from_numpy(master).reshape(case.shapes[i]))
            opt.exp_avg[i].copy_(torch.from_numpy(m).reshape(case.shapes[i]))
            opt.exp_avg_sq[i].copy_(torch.from_numpy(v).reshape(case.shapes[i]))
            opt.param_steps[i] = step
            if not opt.master_is_parameter[i]:
                params[i].data.copy_(opt.master[i].to(params[i].dtype))
        for i, p in enumerate(params):  # owners publish their copies, as make_golden.py does
            dist.broadcast(p.data, src=opt.owner[i])
    norms, grads_seen = [], []
    for s in range(case.steps):
        opt.zero_grad(set_to_none=True)
        if landing:
            half = [None if g is None else to_torch(g, case.dtype, shape, dev) * 0.5
                    for g, shape in zip(case.grads(s, rank), case.shapes)]
            for _ in range(2):
                terms = [(p * h).sum() for p, h in zip(params, half) if h is not None]
                if terms:
                    torch.autograd.backward(terms)
        else:
            for p, g, shape in zip(params, case.grads(s, rank), case.shapes):
                p.grad = None if g is None else to_torch(g, case.dtype, shape, dev)
        if os.environ.get("WORKER_DIRTY") == "1" and s == 1 and rank == world - 1:
            # this rank overwrites its copy of a tensor another rank owns: the next step must
            # restore the owner's values everywhere (the reference's broadcast does)
            j = next(i for i in range(len(params)) if opt.owner[i] != rank)
            with torch.no_grad():
                params[j].copy_(torch.zeros_like(params[j]))
        opt.all_reduce_grads()
        grads_seen.append({i: None if p.grad is None else to_numpy(p.grad, case.dtype) for i, p in enumerate(params)})
        n = opt.clip_grad_norm(case.max_norm)
        norms.append(n)
        if math.isfinite(n) or case.call_step_after_nonfinite:
            opt.step()
    torch.cuda.synchronize()
    result = {
        "rank": rank, "norms": norms, "owner": opt.owner, "mode": opt.comm_mode, "land_launches": opt.land_launches,
        "dense_steps": opt.dense_steps,
        "params": [to_numpy(p.data, case.dtype) for p in params],
        "state": {i: (to_numpy(opt.master[i], 0), to_numpy(opt.exp_avg[i], 0), to_numpy(opt.exp_avg_sq[i], 0),
                      opt.param_steps[i]) for i in opt.param_steps},
        "grads": grads_seen,
    }
    with open(os.path.join(out_dir, f"rank{rank}.pkl"), "wb") as f:
        pickle.dump(result, f)
    dist.barrier()
    opt.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    if sys.argv[1] == "peer_delay":
        peer_delay(sys.argv[2])
    elif sys.argv[1] == "mixed":
        mixed(sys.argv[2])
    else:
        main(sys.argv[1], sys.argv[2])
