"""Checkpoints (neural/checkpoint.rs): the known answers of
neural/tests/checkpoint_tests.rs on host parameters, and on the device a
training run resumed from a snapshot of its parameters and Adam state that
continues the uninterrupted run bitwise."""
import numpy as np
import pytest

import oracle
from poorgrad_b200 import checkpoint, neural
from poorgrad_b200.graph import Tape, filled
from poorgrad_b200.plan import Request


def model(t, fill):
    # checkpoint_tests.rs:10-24
    full = lambda shape: np.full(shape, fill, np.float32)
    return (neural.Sequential()
            .then(neural.Linear(t, full((2, 3)), full(3)))
            .then(neural.Activation(neural.Activation.TANH))
            .then(neural.Linear(t, full((3, 1)), full(1))))


def test_positional_checkpoints_round_trip(built):
    # checkpoint_tests.rs:26-57
    t = Tape()
    trained = model(t, 0.5)
    out = trained.express(t.leaf(filled((1, 2), 1.0)))
    net = t.into_network()
    params = net.parameters()
    payloads = checkpoint.snapshot(params, trained)
    assert len(payloads) == 4
    t2 = Tape()
    fresh = model(t2, 0.0)
    out2 = fresh.express(t2.leaf(filled((1, 2), 1.0)))
    net2 = t2.into_network()
    restored = checkpoint.restore(net2.parameters(), fresh, payloads)
    a = oracle.run(net.compile(Request([out])), params)[out.index]
    b = oracle.run(net2.compile(Request([out2])), restored)[out2.index]
    assert a.tobytes() == b.tobytes()


def test_positional_restore_rejects_a_count_mismatch(built):
    # checkpoint_tests.rs:59-65
    t = Tape()
    module = model(t, 0.0)
    params = t.into_network().parameters()
    with pytest.raises(AssertionError, match="payloads but the module has"):
        checkpoint.restore(params, module, [np.ones((2, 3), np.float32)])


def test_named_checkpoints_round_trip(built):
    # checkpoint_tests.rs:67-82
    t = Tape()
    trained = model(t, 0.25)
    entries = checkpoint.named_snapshot(t.into_network().parameters(), trained)
    assert [path for path, _ in entries] == ["0.weights", "0.bias", "2.weights", "2.bias"]
    t2 = Tape()
    fresh = model(t2, 0.0)
    restored = checkpoint.named_restore(t2.into_network().parameters(), fresh, entries)
    assert checkpoint.snapshot(restored, fresh)[0].reshape(-1).tolist() == [0.25] * 6


def test_named_restore_rejects_missing_entries(built):
    # checkpoint_tests.rs:84-94
    t = Tape()
    module = model(t, 0.5)
    params = t.into_network().parameters()
    entries = checkpoint.named_snapshot(params, module)
    del entries[2]
    with pytest.raises(AssertionError, match="missing entries for: 2.weights"):
        checkpoint.named_restore(params, module, entries)


def test_named_restore_rejects_unexpected_entries(built):
    # checkpoint_tests.rs:96-110
    t = Tape()
    first = model(t, 0.5)
    second = neural.Sequential().then(
        neural.Linear(t, np.full((2, 3), 0.5, np.float32), np.full(3, 0.5, np.float32)))
    params = t.into_network().parameters()
    entries = checkpoint.named_snapshot(params, first)
    with pytest.raises(AssertionError, match="no parameter matches"):
        checkpoint.named_restore(params, second, entries)


def test_tied_parameters_restore_once(built):
    # checkpoint_tests.rs:112-145: one table under two paths
    class Tied:
        def __init__(self, table):
            self.table = table

        def visit(self, v):
            v.enter("embedding")
            v.parameter("weights", self.table)
            v.leave()
            v.enter("head")
            v.parameter("weights", self.table)
            v.leave()

    t = Tape()
    table = t.parameter(filled((2, 2), 0.5))
    module = Tied(table)
    params = t.into_network().parameters()
    entries = checkpoint.named_snapshot(params, module)
    assert [p for p, _ in entries] == ["embedding.weights", "head.weights"]
    restored = checkpoint.named_restore(params, module, entries)
    assert checkpoint.snapshot(restored, module)[0].reshape(-1).tolist() == [0.5] * 4


@pytest.mark.gpu
def test_a_resumed_device_run_continues_bitwise(device):
    # five Adam steps uninterrupted, against three steps, a snapshot of the
    # device parameters and optimizer state, a fresh plan restored from it,
    # and two more steps
    from poorgrad_b200 import backend, configs
    w = configs.char_mlp(batch=256)
    opt = w.optimizer

    def session(params):
        plan = backend.DevicePlan(w.columns)
        dp = backend.DeviceParameters(plan, params)
        o = backend.Optimizer(plan, dp, backend.ADAM, zip(w.params, w.grads), opt["lr"],
                              opt.get("beta1", 0.9), opt.get("beta2", 0.999),
                              opt.get("eps", 1e-8))
        return plan, dp, o

    module = _StateModule(w.params)
    plan, dp, o = session(w.network.parameters())
    for step in range(5):
        plan.forward(dp, w.feeds(step), sync=True)
    uninterrupted = checkpoint.snapshot(dp, module)

    plan, dp, o = session(w.network.parameters())
    for step in range(3):
        plan.forward(dp, w.feeds(step), sync=True)
    saved = checkpoint.named_snapshot(dp, module)
    saved_state = o.state_snapshot()
    del plan, dp, o

    plan, dp, o = session([np.zeros_like(p) for p in w.network.parameters()])
    checkpoint.named_restore(dp, module, saved)
    o.state_restore(saved_state)
    for step in range(3, 5):
        plan.forward(dp, w.feeds(step), sync=True)
    resumed = checkpoint.snapshot(dp, module)
    for a, b in zip(uninterrupted, resumed):
        assert a.tobytes() == b.tobytes()


class _StateModule:
    """Announces a workload's parameters by position, as a module would."""

    def __init__(self, symbols):
        self.symbols = list(symbols)

    def visit(self, v):
        for i, s in enumerate(self.symbols):
            v.enter(i)
            v.parameter("value", s)
            v.leave()
