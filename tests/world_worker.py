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
    params = [torch.nn.Parameter(to_torch(p, case.dtype, s, dev)) for p, s in zip(case.initial_params(), case.shapes)]
    opt = ZeroOneAdamW([{"params": params, "lr": case.lr}], rank=rank, world_size=world, betas=case.betas,
                       eps=case.eps, weight_decay=case.weight_decay)
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
        for p, g, shape in zip(params, case.grads(s, rank), case.shapes):
            p.grad = None if g is None else to_torch(g, case.dtype, shape, dev)
        opt.all_reduce_grads()
        grads_seen.append({i: None if p.grad is None else to_numpy(p.grad, case.dtype) for i, p in enumerate(params)})
        n = opt.clip_grad_norm(case.max_norm)
        norms.append(n)
        if math.isfinite(n) or case.call_step_after_nonfinite:
            opt.step()
    torch.cuda.synchronize()
    result = {
        "rank": rank, "norms": norms, "owner": opt.owner, "mode": opt.comm_mode,
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
    main(sys.argv[1], sys.argv[2])
