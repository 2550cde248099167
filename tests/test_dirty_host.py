"""Host-side detection of parameters and masters written behind the optimizer's back (no GPU):
the versions torch keeps for every tensor decide which tensors the next step must write in
full instead of by changed groups."""
from types import SimpleNamespace

import numpy as np
import torch

from hybridagent_b200.optimizer import ZeroOneAdamW


def _stub(n=4):
    params = [torch.nn.Parameter(torch.zeros(8)) for _ in range(n)]
    masters = [torch.zeros(16), None]
    stub = SimpleNamespace(params=params, _force_dirty=np.zeros(n, dtype=bool),
                           _classes=[SimpleNamespace(master_buf=masters[0], owned=[0, 2]),
                                     SimpleNamespace(master_buf=masters[1], owned=[1, 3])])
    stub._param_versions = lambda: ZeroOneAdamW._param_versions(stub)
    stub._master_versions = lambda: ZeroOneAdamW._master_versions(stub)
    stub._seen_params = stub._param_versions()
    stub._seen_masters = stub._master_versions()
    return stub, params, masters


def test_nothing_written_nothing_dirty():
    stub, _, _ = _stub()
    assert not ZeroOneAdamW._detect_dirty(stub).any()


def test_in_place_parameter_write_is_dirty_once():
    stub, params, _ = _stub()
    with torch.no_grad():
        params[3].copy_(torch.ones(8))  # e.g. a model's load_state_dict
    assert ZeroOneAdamW._detect_dirty(stub).tolist() == [False, False, False, True]
    assert not ZeroOneAdamW._detect_dirty(stub).any()  # recorded: clean until written again


def test_rebound_parameter_is_dirty():
    stub, params, _ = _stub()
    params[1].data = torch.ones(8)
    assert ZeroOneAdamW._detect_dirty(stub).tolist() == [False, True, False, False]


def test_master_write_dirties_the_class_owned_tensors():
    stub, _, masters = _stub()
    masters[0][4:8].add_(1.0)  # a view of the packed master buffer, as optimizer.master[i] is
    assert ZeroOneAdamW._detect_dirty(stub).tolist() == [True, False, True, False]


def test_marked_tensors_are_dirty_once():
    stub, params, _ = _stub()
    params[2].data.fill_(5.0)  # through .data: torch keeps no version of it
    assert not ZeroOneAdamW._detect_dirty(stub).any()
    ZeroOneAdamW.mark_parameters_dirty(stub, [2])
    assert ZeroOneAdamW._detect_dirty(stub).tolist() == [False, False, True, False]
    assert not ZeroOneAdamW._detect_dirty(stub).any()
    ZeroOneAdamW.mark_parameters_dirty(stub)
    assert ZeroOneAdamW._detect_dirty(stub).all()
