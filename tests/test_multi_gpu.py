"""The optimizer at world size 2 on two GPUs (skipped with fewer GPUs), in both
communication modes: p2p (gradients pushed into the owners' buffers over NVLink, summed by
the owner; parameters stored into every peer by the update kernel, or sent by the copy
engines part by part as the update finishes them) and nccl (local pack, NCCL reduce-scatter
and all-gather).

Each rank runs tests/world_worker.py under torchrun on a world-size-2 golden case.  At
world size 2 every reduction's sums have one rounding whatever the algorithm, so the
owners' reduced gradients, norms and states can be held bit for bit to the oracle (torch-
CUDA form, replaying this run's norms) and to the reference's own gloo run within the
parity criterion.  The parameters must agree bit for bit across ranks.
"""
import os
import pickle
import subprocess
import sys

import numpy as np
import pytest

from cases import CASES_BY_NAME
from helpers import Z, assert_bits_equal, assert_state_close, golden, lr_exception, oracle_replay

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _gpus() -> int:
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("mode", ["p2p", "p2p_rounds", "nccl", "p2p_landing", "p2p_rounds_landing",
                                  "p2p_landing_copyengine", "p2p_cepush", "p2p_rounds_cepush", "p2p_cegather",
                                  "p2p_rounds_peerpush_cegather", "p2p_dirty", "p2p_rounds_cappedpush",
                                  "p2p_rounds_tailsplit_landing"])
@pytest.mark.parametrize("name", ["bf16_world2", "fp32_world2", "bf16_world2_inf"])
def test_world2_matches_oracle_and_reference(name, mode, tmp_path):
    """*_landing*: gradients produced by two backward passes and pushed while they land
    (early pushes in 4 KiB buckets, by the capped kernel or the copy engines), the exchange
    pushing only the rest."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", HYBRIDAGENT_B200_COMM=mode.split("_")[0])
    if "rounds" in mode:  # a 16 KiB receive window: ~9 exchange rounds of 1024 elements
        env["HYBRIDAGENT_B200_RECV_BYTES"] = "16384"
    # the peer-bound pieces by the copy engines on 2 streams (the world-2 default: *_cepush and
    # the landing modes) or by the push kernel (p2p, p2p_rounds)
    env["HYBRIDAGENT_B200_PUSH_STREAMS"] = ("peer" if "peerpush" in mode else
                                            "2" if ("cepush" in mode or "landing" in mode) else "0")
    if "tailsplit" in mode:  # the last of the ~9 rounds cut into 3 more of halving length
        env["HYBRIDAGENT_B200_TAIL_SPLIT"] = "3"
    if "cappedpush" in mode:  # the push kernel on a 3-CTA grid walking each round's chunk list
        env["HYBRIDAGENT_B200_PUSH_CTAS"] = "3"
    if mode == "p2p_dirty":  # rank 1 zeroes its copy of a tensor rank 0 owns before step 1
        env["WORKER_DIRTY"] = "1"
    if "cegather" in mode:  # the update in one-chunk parts, each sent to the peer by the copy engines
        env.update(HYBRIDAGENT_B200_GATHER="ce", HYBRIDAGENT_B200_GATHER_PART_BYTES="4096")
    if "landing" in mode:
        env.update(WORKER_LANDING="1", HYBRIDAGENT_B200_LAND_BUCKET_BYTES="4096",
                   HYBRIDAGENT_B200_LAND_CTAS="0" if "copyengine" in mode else "3")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29731",
           os.path.join(HERE, "world_worker.py"), name, str(tmp_path)]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    res = [pickle.load(open(tmp_path / f"rank{r}.pkl", "rb")) for r in range(2)]
    case = CASES_BY_NAME[name]
    g = golden(name)
    assert res[0]["mode"] == res[1]["mode"] == mode.split("_")[0]
    assert res[0]["norms"] == res[1]["norms"]
    assert res[0]["owner"] == g["owner"].tolist()
    if "landing" in mode:
        assert all(r["land_launches"] > 0 for r in res)
    if mode == "p2p_dirty":  # the step after the write is a full one on every rank, then changed groups again
        assert all(r["dense_steps"] == res[0]["dense_steps"] for r in res)
        assert res[0]["dense_steps"] >= 1
    for s, (mine, ref) in enumerate(zip(res[0]["norms"], g["norms"].tolist())):
        assert Z.isclose_norm(mine, ref, 1e-6), (s, mine, ref)
    ora, _ = oracle_replay(case, Z.FORM_TORCH_CUDA, norms=res[0]["norms"])
    for i in range(len(case.shapes)):
        assert np.array_equal(res[0]["params"][i].view(np.uint8), res[1]["params"][i].view(np.uint8)), i
        assert_bits_equal(res[0]["params"][i], ora.params[i], f"param[{i}]")
        owner = res[0]["owner"][i]
        master, m, v, steps = res[owner]["state"][i]
        om, oea, oeas, osteps = ora.tensor_state(i)
        assert steps == osteps == int(g[f"param_steps_{i}"])
        assert_bits_equal(master, om, f"master[{i}]")
        assert_bits_equal(m, oea, f"exp_avg[{i}]")
        assert_bits_equal(v, oeas, f"exp_avg_sq[{i}]")
        assert_state_close(master, g[f"master_{i}"], f"ref master[{i}]", lr_ulps=lr_exception(case))
        # after all_reduce_grads only the owner holds a gradient
        other = 1 - owner
        assert res[other]["grads"][-1][i] is None


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_stalled_peer_raises_comm_failure(tmp_path):
    """Rank 1 stalls on the host between steps (12 s) while rank 0's next collective waits:
    the communicator watchdog (5 s timeout) aborts it and the step raises CommFailure on
    rank 0 instead of hanging; rank 1 learns of it on the host before its next launch.  The
    failure is injected on the host only; no rank dies with memory mapped by another."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "20", "150", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29733",
           os.path.join(HERE, "world_worker.py"), "peer_delay", str(tmp_path)]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True)
    logs = "".join(f"--- rank{r}.log\n" + (tmp_path / f"rank{r}.log").read_text()
                   for r in range(2) if (tmp_path / f"rank{r}.log").exists())
    assert proc.returncode == 0, logs + proc.stdout[-4000:] + proc.stderr[-6000:]
    r0 = pickle.load(open(tmp_path / "rank0.pkl", "rb"))
    r1 = pickle.load(open(tmp_path / "rank1.pkl", "rb"))
    assert r0["mode"] == r1["mode"] == "p2p"
    assert r0["error"] is not None and "did not complete within 5 s" in r0["error"], logs
    assert 5.0 <= r0["elapsed"] < 60.0, logs
    assert r1["error"] == "peer reported CommFailure before this rank's next launch", logs


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("mode", ["p2p", "p2p_rounds", "nccl"])
def test_world2_mixed_dtype_classes(mode, tmp_path):
    """bf16 + fp32 + fp16 parameters in one optimizer (three dtype classes, each exchanged
    in its own rounds; the single fp16 tensor leaves one rank an empty fp16 segment), a tensor
    absent on one rank: bit for bit against the oracle."""
    sys.path.insert(0, HERE)
    from world_worker import mixed_grads, mixed_spec
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", HYBRIDAGENT_B200_COMM=mode.split("_")[0])
    if mode == "p2p_rounds":
        env["HYBRIDAGENT_B200_RECV_BYTES"] = "4096"
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29735",
           os.path.join(HERE, "world_worker.py"), "mixed", str(tmp_path)]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    res = [pickle.load(open(tmp_path / f"rank{r}.pkl", "rb")) for r in range(2)]
    assert res[0]["mode"] == res[1]["mode"] == mode.split("_")[0]
    assert res[0]["norms"] == res[1]["norms"]
    spec = mixed_spec()
    rng = np.random.default_rng(3)
    init = [Z.narrow((rng.standard_normal(int(np.prod(s))) * 0.02).astype(np.float32), d) for s, d in spec]
    ora = Z.OracleZeroOne(init, [d for _, d in spec], [1e-3] * 4 + [3e-4] * 4, world=2, weight_decay=0.05)
    assert ora.owner == res[0]["owner"]
    for step in range(3):
        ora.reduce_grads([mixed_grads(step, r) for r in range(2)])
        mine = Z.norm_from_sumsq(ora.sumsq())
        assert Z.isclose_norm(res[0]["norms"][step], mine, 1e-6), (step, res[0]["norms"][step], mine)
        ora.clip_grad_norm(1.0, norm=res[0]["norms"][step])
        ora.step()
    for i, (_, d) in enumerate(spec):
        assert np.array_equal(res[0]["params"][i].view(np.uint8), res[1]["params"][i].view(np.uint8)), i
        assert_bits_equal(res[0]["params"][i], ora.params[i], f"param[{i}]")
        master, m, v, steps = res[ora.owner[i]]["state"][i]
        om, oea, oeas, osteps = ora.tensor_state(i)
        assert steps == osteps
        assert_bits_equal(master, om, f"master[{i}]")
        assert_bits_equal(m, oea, f"exp_avg[{i}]")
        assert_bits_equal(v, oeas, f"exp_avg_sq[{i}]")
