"""World size 2 on CPU over gloo: the host logic of the multi-rank path.

Two gloo ranks each build the product's shard plan (hybridagent_b200.layout) and run the
owner-major data flow the CUDA path runs -- local gradients packed into the plan's slots
(zeros for missing ones), used mask MAX, SUM reduce-scatter of the packed buffer, norm
over owned gradients, clip + update of the owned slots, all-gather of the parameter
buffer -- with the oracle doing the arithmetic.  The result must equal the reference's
own world-size-2 run (golden vectors written over gloo by make_golden.py): the plan keeps
the reference's owners and reproduces its reduction exactly (a 2-operand bf16 / fp32 sum
has one rounding whatever the algorithm).
"""
import os
import socket

import numpy as np
import pytest

from cases import CASES_BY_NAME


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, name, queue):
    import sys
    sys.path[:0] = [os.path.dirname(os.path.dirname(os.path.abspath(__file__))), os.path.dirname(__file__),
                    os.path.join(os.path.dirname(__file__), "golden")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch
    import torch.distributed as dist

    from cases import CASES_BY_NAME as C
    from hybridagent_b200 import layout
    from hybridagent_b200._lib import HA_BF16, HA_F32
    from oracle import zero1 as Z

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        case = C[name]
        code = HA_BF16 if case.dtype == Z.BF16 else HA_F32
        numels = case.numels
        plan = layout.plan(numels, [code] * len(numels), world)
        plans = [None] * world
        dist.all_gather_object(plans, (plan.owner, plan.classes[0].offset, plan.classes[0].seg_len))
        assert all(p == plans[0] for p in plans)
        (cls,) = plan.classes
        seg = cls.seg_len
        tdt = torch.bfloat16 if case.dtype == Z.BF16 else torch.float32
        npdt = np.uint16 if case.dtype == Z.BF16 else np.float32

        def as_torch(a):
            return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16) if npdt == np.uint16 \
                else torch.from_numpy(a.copy())

        def as_np(t):
            return t.view(torch.int16).numpy().view(np.uint16).copy() if npdt == np.uint16 else t.numpy().copy()

        # packed parameters (identical on all ranks) and this rank's owned state
        params = np.zeros(world * seg, npdt)
        init = case.initial_params()
        for i in cls.indices:
            start = plan.owner[i] * seg + cls.offset[i]
            params[start:start + numels[i]] = init[i]
        owned = cls.owned(plan.owner, rank)
        state = {}
        for i in owned:
            master = Z.widen(init[i], case.dtype).copy()
            m = np.zeros(numels[i], np.float32)
            v = np.zeros(numels[i], np.float32)
            steps = 0
            if case.preload_state:
                master, m, v, steps = case.preload(i)
                master, m, v = master.copy(), m.copy(), v.copy()
                start = rank * seg + cls.offset[i]
                params[start:start + numels[i]] = Z.narrow(master, case.dtype, Z.FORM_TORCH_CUDA)
            state[i] = [master, m, v, steps]
        if case.preload_state:  # owners publish their copies (the all-gather)
            buf = as_torch(params)
            parts = [torch.empty(seg, dtype=tdt) for _ in range(world)]
            dist.all_gather(parts, buf[rank * seg:(rank + 1) * seg].clone())
            params = as_np(torch.cat(parts))
        norms = []
        for s in range(case.steps):
            grads = case.grads(s, rank)
            used = torch.tensor([g is not None for g in grads], dtype=torch.uint8)
            dist.all_reduce(used, op=dist.ReduceOp.MAX)
            packed = np.zeros(world * seg, npdt)
            for i in cls.indices:
                if grads[i] is not None:
                    start = plan.owner[i] * seg + cls.offset[i]
                    packed[start:start + numels[i]] = grads[i]
            t = as_torch(packed)
            dist.all_reduce(t, op=dist.ReduceOp.SUM)  # gloo has no reduce_scatter; keep own segment
            own = as_np(t)[rank * seg:(rank + 1) * seg]
            mine = {i: own[cls.offset[i]:cls.offset[i] + numels[i]].copy() for i in owned if used[i]}
            total = torch.tensor([sum(Z.sumsq(g, case.dtype) for g in mine.values())], dtype=torch.float64)
            dist.all_reduce(total)
            norm = Z.norm_from_sumsq(float(total))
            norms.append(norm)
            scale = Z.clip_scale_for(norm, case.max_norm)
            for i, g in mine.items():
                st = state[i]
                st[3] += 1
                start = rank * seg + cls.offset[i]
                if case.dtype == Z.F32:
                    Z.adamw_tensor(Z.FORM_TORCH_CUDA, g, case.dtype, st[0], st[1], st[2], None, case.dtype,
                                   lr=case.lr, beta1=case.betas[0], beta2=case.betas[1], eps=case.eps,
                                   weight_decay=case.weight_decay, step=st[3], clip_scale=scale)
                    params[start:start + numels[i]] = st[0]
                else:
                    p = params[start:start + numels[i]].copy()
                    Z.adamw_tensor(Z.FORM_TORCH_CUDA, g, case.dtype, st[0], st[1], st[2], p, case.dtype,
                                   lr=case.lr, beta1=case.betas[0], beta2=case.betas[1], eps=case.eps,
                                   weight_decay=case.weight_decay, step=st[3], clip_scale=scale)
                    params[start:start + numels[i]] = p
            parts = [torch.empty(seg, dtype=tdt) for _ in range(world)]
            dist.all_gather(parts, as_torch(params[rank * seg:(rank + 1) * seg].copy()))
            params = as_np(torch.cat(parts))
        final = {i: params[plan.owner[i] * seg + cls.offset[i]:plan.owner[i] * seg + cls.offset[i] + numels[i]]
                 for i in cls.indices}
        queue.put((rank, norms, final, {i: (st[0], st[1], st[2], st[3]) for i, st in state.items()}, plan.owner))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("name", ["bf16_world2", "fp32_world2"])
def test_world2_host_path_matches_reference(name):
    import torch.multiprocessing as mp

    from helpers import Z, assert_bits_equal, assert_state_close, golden

    case = CASES_BY_NAME[name]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, name, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        rank, norms, final, state, owner = q.get(timeout=300)
        results[rank] = (norms, final, state, owner)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    g = golden(name)
    assert results[0][0] == results[1][0]  # every rank sees the same norm (same skip decision)
    for s, (mine, ref) in enumerate(zip(results[0][0], g["norms"].tolist())):
        assert Z.isclose_norm(mine, ref, 1e-6), (s, mine, ref)
    assert results[0][3] == g["owner"].tolist()
    for i in range(len(case.shapes)):
        a, b = results[0][1][i], results[1][1][i]
        assert np.array_equal(a.view(np.uint8), b.view(np.uint8)), f"ranks disagree on param {i}"
        owner = int(g["owner"][i])
        master, m, v, steps = results[owner][2][i]
        assert steps == int(g[f"param_steps_{i}"])
        assert_bits_equal(m, g[f"exp_avg_{i}"], f"exp_avg[{i}]")
        assert_state_close(v, g[f"exp_avg_sq_{i}"], f"exp_avg_sq[{i}]")
        assert_state_close(master, g[f"master_{i}"], f"master[{i}]")
        if case.dtype == Z.BF16:
            assert_bits_equal(Z.narrow(master, Z.BF16), a, f"param[{i}]")


def _rank_main_p2p(rank, world, port, name, queue, tail=0):
    """The p2p data flow: in rounds (layout.exchange_pieces, a small round size so slots
    straddle rounds), each rank pushes each piece of its gradients to the address the
    product computes (half round % 2 of the owner's receive window, region <rank>), the
    owner adds the regions of the round in rank order into its reduced gradients, clips and
    updates its slots, and each new parameter is stored at layout.peer_deltas offsets into
    every peer's packed parameters.  Device memories are simulated as numpy arrays at fake
    base addresses; the stores that cross ranks travel through gloo."""
    import sys
    sys.path[:0] = [os.path.dirname(os.path.dirname(os.path.abspath(__file__))), os.path.dirname(__file__),
                    os.path.join(os.path.dirname(__file__), "golden")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch
    import torch.distributed as dist

    from cases import CASES_BY_NAME as C
    from hybridagent_b200 import layout
    from hybridagent_b200._lib import HA_BF16, HA_F32
    from oracle import zero1 as Z

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        case = C[name]
        code = HA_BF16 if case.dtype == Z.BF16 else HA_F32
        numels = case.numels
        plan = layout.plan(numels, [code] * len(numels), world)
        (cls,) = plan.classes
        seg = cls.seg_len
        npdt = np.uint16 if case.dtype == Z.BF16 else np.float32
        esz = np.dtype(npdt).itemsize
        SPACE = 1 << 40
        S = 64 * max(2, 40 // world)  # small rounds: slots straddle rounds, both window halves are used
        recv_bases = [(r + 1) * SPACE for r in range(world)]               # each rank's receive window
        param_bases = [(r + 1) * SPACE + SPACE // 2 for r in range(world)]  # each rank's packed params
        pieces = layout.exchange_pieces(cls, plan.owner, numels, S, tail)
        assert pieces.n_rounds > 4
        deltas = layout.peer_deltas(param_bases, rank)
        peers = [r for r in range(world) if r != rank]

        def exchange(images):
            """images[r]: this rank's stores into rank r's memory."""
            everyone = [None] * world
            dist.all_gather_object(everyone, images)
            return [everyone[s][rank] for s in range(world)]

        params = np.zeros(world * seg, npdt)
        init = case.initial_params()
        for i in cls.indices:
            start = plan.owner[i] * seg + cls.offset[i]
            params[start:start + numels[i]] = init[i]
        owned = cls.owned(plan.owner, rank)
        state = {i: [Z.widen(init[i], case.dtype).copy(), np.zeros(numels[i], np.float32),
                     np.zeros(numels[i], np.float32), 0] for i in owned}
        window = np.zeros(2 * world * S, npdt)  # this rank's double-buffered receive window
        own = np.zeros(max(cls.own_len[rank], 1), npdt)
        norms = []
        for s in range(case.steps):
            grads = case.grads(s, rank)
            used = torch.tensor([g is not None for g in grads], dtype=torch.uint8)
            dist.all_reduce(used, op=dist.ReduceOp.MAX)
            for k in range(pieces.n_rounds):
                # push round k: each piece at the address the product computes for it
                images = [dict() for _ in range(world)]
                for j in np.nonzero(pieces.round == k)[0]:
                    t = int(pieces.tensor[j])
                    o, so, c = int(pieces.owner[j]), int(pieces.src_off[j]), int(pieces.count[j])
                    addr = recv_bases[o] + ((k % 2) * world * S + rank * S + int(pieces.dst_off[j])) * esz
                    elem = (addr - recv_bases[o]) // esz
                    assert (k % 2) * world * S + rank * S <= elem and elem + c <= (k % 2) * world * S + (rank + 1) * S
                    if t < 0:  # a gap between slots: zeros
                        images[o][elem] = np.zeros(c, npdt)
                        continue
                    i = cls.indices[t]
                    g = grads[i] if grads[i] is not None and used[i] else np.zeros(numels[i], npdt)
                    images[o][elem] = g[so:so + c]
                for img in exchange(images):
                    for elem, g in img.items():
                        window[elem:elem + len(g)] = g
                # owner: add the regions of this half in rank order, round once
                count = pieces.own_counts(cls, rank)[k]
                half = (k % 2) * world * S
                acc = Z.widen(window[half:half + count].copy(), case.dtype)
                for r in range(1, world):
                    acc = acc + Z.widen(window[half + r * S:half + r * S + count], case.dtype)
                b = int(pieces.bounds[k])
                own[b:b + count] = Z.narrow(acc, case.dtype) if case.dtype != Z.F32 else acc
            mine = {i: own[cls.offset[i]:cls.offset[i] + numels[i]].copy() for i in owned if used[i]}
            # like the product's fused sums: the whole reduced region, gaps included (all zero)
            total = torch.tensor([Z.sumsq(own[:cls.own_len[rank]].copy(), case.dtype)], dtype=torch.float64)
            dist.all_reduce(total)
            norm = Z.norm_from_sumsq(float(total))
            norms.append(norm)
            scale = Z.clip_scale_for(norm, case.max_norm)
            images = [dict() for _ in range(world)]
            for i, g in mine.items():
                st = state[i]
                st[3] += 1
                start = rank * seg + cls.offset[i]
                p = None if case.dtype == Z.F32 else params[start:start + numels[i]].copy()
                Z.adamw_tensor(Z.FORM_TORCH_CUDA, g, case.dtype, st[0], st[1], st[2], p, case.dtype, lr=case.lr,
                               beta1=case.betas[0], beta2=case.betas[1], eps=case.eps,
                               weight_decay=case.weight_decay, step=st[3], clip_scale=scale)
                new = st[0] if p is None else p
                params[start:start + numels[i]] = new
                local_addr = param_bases[rank] + start * esz
                for q, d in zip(peers, deltas):  # the fused all-gather: same element on every peer
                    elem = (local_addr + d - param_bases[q]) // esz
                    assert elem == start
                    images[q][elem] = new.copy()
            for img in exchange(images):
                for elem, v in img.items():
                    params[elem:elem + len(v)] = v
        final = {i: params[plan.owner[i] * seg + cls.offset[i]:plan.owner[i] * seg + cls.offset[i] + numels[i]]
                 for i in cls.indices}
        queue.put((rank, norms, final, {i: tuple(st) for i, st in state.items()}, plan.owner))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("name,tail", [("bf16_world2", 0), ("bf16_world2", 2)])
def test_world2_p2p_host_path_matches_reference(name, tail):
    import torch.multiprocessing as mp

    from helpers import Z, assert_bits_equal, assert_state_close, golden

    case = CASES_BY_NAME[name]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main_p2p, args=(r, 2, port, name, q, tail)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        rank, norms, final, state, owner = q.get(timeout=300)
        results[rank] = (norms, final, state, owner)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    g = golden(name)
    assert results[0][0] == results[1][0]
    for s, (mine, ref) in enumerate(zip(results[0][0], g["norms"].tolist())):
        assert Z.isclose_norm(mine, ref, 1e-6), (s, mine, ref)
    for i in range(len(case.shapes)):
        a, b = results[0][1][i], results[1][1][i]
        assert np.array_equal(a.view(np.uint8), b.view(np.uint8)), f"ranks disagree on param {i}"
        owner = int(g["owner"][i])
        master, m, v, steps = results[owner][2][i]
        assert steps == int(g[f"param_steps_{i}"])
        assert_bits_equal(m, g[f"exp_avg_{i}"], f"exp_avg[{i}]")
        assert_state_close(v, g[f"exp_avg_sq_{i}"], f"exp_avg_sq[{i}]")
        assert_state_close(master, g[f"master_{i}"], f"master[{i}]")
        assert_bits_equal(Z.narrow(master, Z.BF16), a, f"param[{i}]")


@pytest.mark.parametrize("world,tail", [(3, 0), (4, 0), (3, 3)])
def test_p2p_host_path_beyond_two_ranks_matches_oracle(world, tail):
    """The p2p data flow at W = 3 and 4 (gloo ranks on CPU; the GPU tests run W = 2 only):
    the product's piece layout, window addresses, rounds and peer offsets with the owner
    summing every rank's region in fp32 and rounding once, against the oracle's W-rank run
    with that reduction -- norms within 1e-6, states and parameters bit for bit."""
    import torch.multiprocessing as mp

    from helpers import Z, assert_bits_equal

    name = "bf16_world2"  # its shapes, value distributions and absent gradients, over W ranks
    case = CASES_BY_NAME[name]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main_p2p, args=(r, world, port, name, q, tail)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        rank, norms, final, state, owner = q.get(timeout=300)
        results[rank] = (norms, final, state, owner)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    norms = results[0][0]
    assert all(results[r][0] == norms for r in range(world))
    ora = Z.OracleZeroOne(case.initial_params(), [case.dtype] * len(case.shapes), [case.lr] * len(case.shapes),
                          world=world, betas=case.betas, eps=case.eps, weight_decay=case.weight_decay)
    assert ora.owner == results[0][3]
    for s in range(case.steps):
        ora.reduce_grads([case.grads(s, r) for r in range(world)], round_once=True)
        assert Z.isclose_norm(norms[s], Z.norm_from_sumsq(ora.sumsq()), 1e-6), s
        ora.clip_grad_norm(case.max_norm, norm=norms[s])
        ora.step()
    for i in range(len(case.shapes)):
        for r in range(1, world):
            assert np.array_equal(results[0][1][i].view(np.uint8), results[r][1][i].view(np.uint8)), (i, r)
        assert_bits_equal(results[0][1][i], ora.params[i], f"param[{i}]")
        master, m, v, steps = results[ora.owner[i]][2][i]
        om, oea, oeas, osteps = ora.tensor_state(i)
        assert steps == osteps
        assert_bits_equal(master, om, f"master[{i}]")
        assert_bits_equal(m, oea, f"exp_avg[{i}]")
        assert_bits_equal(v, oeas, f"exp_avg_sq[{i}]")
