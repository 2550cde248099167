"""World-size-1 gradient landing's bookkeeping on the host (no GPU): clip_grad_norm may add the
square sums taken while the gradients landed only if every owned gradient present now landed
exactly once and is the same tensor, unmodified (torch's version counter), as when it was
summed; anything else sends it back to the full pass."""
from types import SimpleNamespace

import torch

from hybridagent_b200.optimizer import ZeroOneAdamW


def _stub(n=3):
    params = [SimpleNamespace(grad=torch.ones(4 + k)) for k in range(n)]
    stub = SimpleNamespace(_lland=True, _lland_valid=True, _lland_slots=1, params=params,
                           _classes=[SimpleNamespace(owned=list(range(n)))],
                           _lland_seen={i: (p.grad, p.grad._version) for i, p in enumerate(params)})
    return stub


def _ready(stub):
    return ZeroOneAdamW._lland_ready(stub)


def test_every_gradient_landed_once_unchanged():
    assert _ready(_stub())


def test_gradient_modified_in_place_after_landing():
    stub = _stub()
    stub.params[1].grad.mul_(1.0)  # same values, but torch counts the write
    assert not _ready(stub)


def test_gradient_replaced_after_landing():
    stub = _stub()
    stub.params[2].grad = stub.params[2].grad.clone()
    assert not _ready(stub)


def test_gradient_that_never_landed():
    stub = _stub()
    del stub._lland_seen[0]
    assert not _ready(stub)


def test_landed_gradient_since_set_to_none():
    stub = _stub()
    stub.params[0].grad = None  # summed, then dropped: its square sum must not count
    assert not _ready(stub)


def test_absent_gradient_that_never_landed_is_fine():
    stub = _stub()
    stub.params[0].grad = None
    del stub._lland_seen[0]
    assert _ready(stub)


def test_invalidated_or_empty_step():
    stub = _stub()
    stub._lland_valid = False  # landed twice, out of arena room, or clipped in place
    assert not _ready(stub)
    stub = _stub()
    stub._lland_slots = 0  # nothing was summed
    assert not _ready(stub)
    stub = _stub()
    stub._lland = False  # landing not set up
    assert not _ready(stub)


def test_unusable_landings_invalidate_without_touching_the_gpu():
    # a gradient that is absent, not owned by a dtype class, or strided cannot be summed from
    # its landing; the hook marks the step invalid before it would queue anything
    for grad, class_of in ((None, {0: 0}), (torch.ones(4), {}), (torch.ones(4, 4).t(), {0: 0})):
        stub = SimpleNamespace(_lland_valid=True, _lland_class_of=class_of, _lland_pending=[])
        ZeroOneAdamW._lland_on_landed(stub, 0, SimpleNamespace(grad=grad))
        assert stub._lland_valid is False and stub._lland_pending == []
