"""Engine-backward plans (`Request::backward`, `Run::backward`,
engine/run.rs:229-318) on the device: the reverse scan runs inside the plan
and its parameter gradients agree with the recorded-gradient plan of the same
graph (`Tape::differentiate`), which the reference pins bitwise to the engine
(graph/tests/differentiate_tests.rs:520); here both are checked against the
oracle's run of the recorded-gradient columns and the oracle's own reverse
scan."""
import numpy as np
import pytest

import oracle
from poorgrad_b200 import backend, neural
from poorgrad_b200.graph import Tape, tensor, selection
from poorgrad_b200.plan import Request


def _graph(batch=64):
    t = Tape()
    rng = np.random.default_rng(3)
    x = t.input(tensor((batch, 24), rng.uniform(-1, 1, (batch, 24))))
    y = t.input(selection(rng.integers(0, 7, batch), 7))
    l1 = neural.Linear(t, rng.uniform(-0.3, 0.3, (24, 32)).astype(np.float32), np.zeros(32, np.float32))
    ln = neural.LayerNorm(t, 32)
    l2 = neural.Linear(t, rng.uniform(-0.3, 0.3, (32, 7)).astype(np.float32), np.zeros(7, np.float32))
    h = ln.express(l1.express(x)).tanh()
    loss = neural.cross_entropy(l2.express(h.relu()), y)
    params = l1.parameters() + ln.parameters() + l2.parameters()
    return t, loss, params


def test_backward_columns_lower_on_the_host(built):
    t, loss, params = _graph()
    cols = t.into_network().compile(Request([loss]).backward())
    text = backend.lower_describe(cols)
    assert "gemm3xtf32" in text
    backend.nvrtc_check(cols)


@pytest.mark.gpu
def test_engine_backward_matches_the_recorded_gradients(device):
    t, loss, params = _graph()
    n_forward = len(t)
    recorded = t.differentiate(loss, params)
    net = t.into_network()
    engine = net.compile(Request([loss]).backward())
    ref = oracle.run(net.compile(Request([loss] + recorded)), net.parameters(),
                     read=[g.index for g in recorded])
    scan = oracle.backward(engine, net.parameters(), loss, params)
    plan = backend.DevicePlan(engine)
    dp = backend.DeviceParameters(plan, net.parameters())
    plan.forward(dp, sync=True)
    for p, g in zip(params, recorded):
        got = plan.gradient(loss, p)
        np.testing.assert_allclose(got, ref[g.index], rtol=1e-4, atol=1e-6)
    for p, e in zip(params, scan):
        np.testing.assert_allclose(plan.gradient(loss, p), e, rtol=1e-4, atol=1e-6)
    assert n_forward < len(t)
