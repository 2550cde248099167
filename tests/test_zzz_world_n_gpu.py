"""The optimizer at world size 4 and 8 (each skipped without that many GPUs), p2p mode, over
the bf16_world2 golden case's shapes and seeded gradients on W ranks, with a 16 KiB receive
window (several exchange rounds), by the push kernel and by the copy engines (two balanced
streams, or one stream per peer with the parameter all-gather by the copy engines too).

At W > 2 no two reductions round alike, so the reference is the oracle's W-rank run with the
owner's reduction: fp32 sums in rank order, rounded once (``reduce_grads(round_once=True)``,
the same check ``tests/test_world2_gloo.py`` runs on CPU ranks).  Norms within 1e-6 and
replayed; states and parameters bit for bit; every rank holds the same parameters.  This file
runs last so that nothing else waits on it.
"""
import os
import pickle
import subprocess
import sys

import numpy as np
import pytest

from cases import CASES_BY_NAME
from helpers import Z, assert_bits_equal

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _gpus() -> int:
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.parametrize("push", ["kernel", "copyengine", "peer_cegather"])
@pytest.mark.parametrize("world", [4, 8])
def test_world_n_p2p_matches_round_once_oracle(world, push, tmp_path):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    name = "bf16_world2"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", HYBRIDAGENT_B200_COMM="p2p", HYBRIDAGENT_B200_RECV_BYTES="16384",
               HYBRIDAGENT_B200_PUSH_STREAMS={"kernel": "0", "copyengine": "2", "peer_cegather": "peer"}[push])
    if push == "peer_cegather":  # one copy-engine stream per peer; all-gather by the copy engines in parts
        env.update(HYBRIDAGENT_B200_GATHER="ce", HYBRIDAGENT_B200_GATHER_PART_BYTES="4096")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={29800 + world}",
           os.path.join(HERE, "world_worker.py"), name, str(tmp_path)]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    res = [pickle.load(open(tmp_path / f"rank{r}.pkl", "rb")) for r in range(world)]
    assert all(r["mode"] == "p2p" for r in res)
    norms = res[0]["norms"]
    assert all(r["norms"] == norms for r in res)
    case = CASES_BY_NAME[name]
    ora = Z.OracleZeroOne(case.initial_params(), [case.dtype] * len(case.shapes), [case.lr] * len(case.shapes),
                          world=world, betas=case.betas, eps=case.eps, weight_decay=case.weight_decay)
    assert ora.owner == res[0]["owner"]
    for s in range(case.steps):
        ora.reduce_grads([case.grads(s, r) for r in range(world)], round_once=True)
        assert Z.isclose_norm(norms[s], Z.norm_from_sumsq(ora.sumsq()), 1e-6), s
        ora.clip_grad_norm(case.max_norm, norm=norms[s])
        ora.step()
    for i in range(len(case.shapes)):
        for r in range(1, world):
            assert np.array_equal(res[0]["params"][i].view(np.uint8), res[r]["params"][i].view(np.uint8)), (i, r)
        assert_bits_equal(res[0]["params"][i], ora.params[i], f"param[{i}]")
        master, m, v, steps = res[ora.owner[i]]["state"][i]
        om, oea, oeas, osteps = ora.tensor_state(i)
        assert steps == osteps
        assert_bits_equal(master, om, f"master[{i}]")
        assert_bits_equal(m, oea, f"exp_avg[{i}]")
        assert_bits_equal(v, oeas, f"exp_avg_sq[{i}]")
