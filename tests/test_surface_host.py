"""The constructor's argument errors on the host (no GPU): the same exception types and
messages as the reference's ZeroOneAdamW (hybrid_rl/optimizer.py:30-33, 43-44) for the same
bad arguments, compared with the reference itself where its files are staged; and parameters
off the GPU are refused loudly (there is no CPU path)."""
import pytest
import torch

from hybridagent_b200 import ZeroOneAdamW
from oracle import stage_ref


def _params(n=2, requires_grad=True):
    return [torch.nn.Parameter(torch.zeros(3, 4), requires_grad=requires_grad) for _ in range(n)]


BAD = [
    ("betas out of range", dict(param_groups=lambda: [{"params": _params(), "lr": 1e-3}], rank=0, world_size=1,
                                betas=(0.9, 1.0))),
    ("betas of three", dict(param_groups=lambda: [{"params": _params(), "lr": 1e-3}], rank=0, world_size=1,
                            betas=(0.9, 0.99, 0.5))),
    ("negative beta", dict(param_groups=lambda: [{"params": _params(), "lr": 1e-3}], rank=0, world_size=1,
                           betas=(-0.1, 0.99))),
    ("rank beyond world", dict(param_groups=lambda: [{"params": _params(), "lr": 1e-3}], rank=2, world_size=2)),
    ("world zero", dict(param_groups=lambda: [{"params": _params(), "lr": 1e-3}], rank=0, world_size=0)),
    ("no trainable parameters", dict(param_groups=lambda: [{"params": _params(requires_grad=False), "lr": 1e-3}],
                                     rank=0, world_size=1)),
    ("empty groups", dict(param_groups=lambda: [], rank=0, world_size=1)),
]


def _call(cls, kw):
    kw = dict(kw)
    groups = kw.pop("param_groups")()
    with pytest.raises(Exception) as info:
        cls(groups, **kw)
    return type(info.value), str(info.value)


@pytest.mark.parametrize("name,kw", BAD, ids=[b[0] for b in BAD])
def test_argument_errors(name, kw):
    ours = _call(ZeroOneAdamW, kw)
    assert ours[0] is ValueError, ours
    if stage_ref.stage():
        import sys
        if stage_ref.OUT not in sys.path:
            sys.path.insert(0, stage_ref.OUT)
        from hybrid_rl.optimizer import ZeroOneAdamW as Reference
        assert _call(Reference, kw) == ours


def test_duplicate_and_frozen_parameters_are_skipped_before_the_device_check():
    p = _params(1)[0]
    frozen = _params(1, requires_grad=False)[0]
    # the same parameter twice and a frozen one: deduplicated and skipped (optimizer.py:36-42), then
    # refused because it is on the CPU
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        ZeroOneAdamW([{"params": [p, frozen], "lr": 1e-3}, {"params": [p], "lr": 1e-4}], rank=0, world_size=1)


def test_8bit_is_refused():
    with pytest.raises(NotImplementedError, match="use_8bit"):
        ZeroOneAdamW([{"params": _params(), "lr": 1e-3}], rank=0, world_size=1, use_8bit=True)
