"""Host-side bookkeeping of gradient landing (no GPU): what the post-accumulate-grad hook
records and forgets."""


def test_landing_hook_forgets_a_push_when_the_gradient_changes_unpushed():
    """A gradient accumulated again while landing is off (in place: same tensor object) must
    not keep the earlier early push: the hook drops it, so the exchange sends it whole."""
    from types import SimpleNamespace

    from hybridagent_b200.optimizer import ZeroOneAdamW
    grad = object()
    for enabled, ok in ((False, True), (True, False)):
        stub = SimpleNamespace(landing_enabled=enabled, _land_ok=ok, _landed={3: (grad, 0), 4: (grad, 0)})
        ZeroOneAdamW._on_landed(stub, 3, SimpleNamespace(grad=grad))
        assert stub._landed == {4: (grad, 0)}
