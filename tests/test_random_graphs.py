"""Seeded random recorded graphs through the whole path.  Each graph draws a
chain of the reference's operations (elementwise arithmetic and
transcendentals, axis broadcasts and reductions, matmul, transposes, views,
log-softmax and log-sum-exp, gather) over a few parameters, sums it into a
scalar loss and records its gradients with `Tape::differentiate`.  On the CPU
each plan is lowered (fusion groups, register-held row values, arena
planning and their host-side checks) and its generated source compiled by
NVRTC; on the device it runs against the oracle."""
import numpy as np
import pytest

import oracle
from poorgrad_b200 import backend
from poorgrad_b200.graph import BF16, Tape, selection, tensor
from poorgrad_b200.plan import Request

SEEDS = list(range(24))


def random_graph(seed, element=0):
    rng = np.random.default_rng(seed)
    rows = int(rng.choice([4, 64, 96]))
    cols = int(rng.choice([8, 32, 48]))
    t = Tape(element)
    params = [t.parameter(tensor((rows, cols), rng.uniform(-1, 1, rows * cols))),
              t.parameter(tensor((cols,), rng.uniform(-1, 1, cols))),
              t.parameter(tensor((cols, cols), rng.uniform(-0.5, 0.5, cols * cols)))]
    x, bias, w = params
    values = [x]
    for _ in range(int(rng.integers(4, 10))):
        v = values[int(rng.integers(len(values)))]
        kind = int(rng.integers(12))
        if kind == 0:
            v = v + values[int(rng.integers(len(values)))]
        elif kind == 1:
            v = v * values[int(rng.integers(len(values)))]
        elif kind == 2:
            v = v.tanh()
        elif kind == 3:
            v = (v * v.literal(tensor((rows, cols), np.full(rows * cols, 0.5)))).exp()
        elif kind == 4:
            v = v + bias.broadcast_along(0, v)
        elif kind == 5:
            v = v.matmul(w)
        elif kind == 6:
            s = v.sum_along(1)
            v = v - s.broadcast_along(1, v)
        elif kind == 7:
            v = v.log_softmax(1)
        elif kind == 8:
            l = v.logsumexp(1)
            v = v * l.broadcast_along(1, v)
        elif kind == 9:
            v = v.transpose().transpose() - v.relu()
        elif kind == 10:
            c = v.sum_along(0)
            v = v * c.broadcast_along(0, v).tanh()
        else:
            idx = rng.integers(0, rows, rows)
            v = v.gather(t.input(selection(idx.tolist(), rows)))
        values.append(v)
    loss = sum((v.sum() for v in values[1:]), values[0].sum())
    grads = t.differentiate(loss, params)
    net = t.into_network()
    return net, net.compile(Request([loss] + grads)), loss, grads


@pytest.mark.parametrize("seed", SEEDS)
def test_random_graph_lowers_and_compiles(built, seed):
    net, cols, loss, grads = random_graph(seed)
    text = backend.lower_describe(cols)
    assert "arena" in text
    backend.nvrtc_check(cols)
    out = oracle.run(cols, net.parameters(), read=[loss] + grads)
    assert np.isfinite(out[loss.index]).all()


@pytest.mark.parametrize("seed", SEEDS[:8])
def test_random_bf16_graph_lowers_with_rounding_and_compiles(built, seed):
    net, cols, loss, grads = random_graph(seed, BF16)
    text = backend.lower_describe(cols, with_source=True)
    assert text.count("tb_rb(") > 1  # beyond the prelude's definition
    backend.nvrtc_check(cols)
    out = oracle.run(cols, net.parameters(), read=[loss] + grads)
    for v in out.values():
        assert oracle.round_bf16(v).tobytes() == v.tobytes()


@pytest.mark.gpu
@pytest.mark.parametrize("seed", SEEDS)
def test_random_graph_on_the_device(device, seed):
    net, cols, loss, grads = random_graph(seed)
    params = net.parameters()
    ref = oracle.run(cols, params, read=[loss] + grads)
    plan = backend.DevicePlan(cols)
    dp = backend.DeviceParameters(plan, params)
    plan.forward(dp, sync=True)
    scale = max(1.0, abs(float(ref[loss.index])))
    np.testing.assert_allclose(plan.of(loss), ref[loss.index], rtol=1e-4, atol=1e-5 * scale)
    for g in grads:
        r = ref[g.index]
        tol = 1e-4 * max(1.0, float(np.abs(r).max()))
        np.testing.assert_allclose(plan.of(g), r, rtol=1e-4, atol=tol)
