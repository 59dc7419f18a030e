"""The closure contract of graph/tests/differentiate_tests.rs:11-28: the
gradients `Tape::differentiate` records (host mirror, run as a plan by the
oracle) reproduce the engine's own reverse scan (`Run::backward`, restated
in the oracle) bitwise, for every function, with the same seed, masking and
accumulation order.  Plus the higher-order and masking cases of the same
file."""
import math

import numpy as np
import pytest

import oracle
from poorgrad_b200.graph import Tape, filled, selection, tensor
from poorgrad_b200.plan import Request


def varied(shape, seed):
    # differentiate_tests.rs:30-41
    n = int(np.prod(shape)) if shape else 1
    return tensor(shape, [((i * 7 + seed * 3) % 11) * 0.375 - 1.5 for i in range(n)])


def closes(build):
    t = Tape()
    loss, wrt = build(t)
    recorded = t.differentiate(loss, wrt)
    net = t.into_network()
    cols = net.compile(Request([loss] + recorded))
    params = net.parameters()
    got = oracle.run(cols, params, read=recorded)
    engine = oracle.backward(cols, params, loss, wrt)
    for g, e in zip(recorded, engine):
        assert got[g.index].shape == e.shape
        assert got[g.index].tobytes() == e.tobytes(), (got[g.index], e)
    return engine


P = lambda t, shape, seed: t.parameter(varied(shape, seed))
L = lambda t, shape, seed: t.leaf(varied(shape, seed))

CASES = {
    # differentiate_tests.rs:43-369, one entry per function
    "add": lambda t: (lambda a, b: ((a + b).sum(), [a, b]))(P(t, (2, 3), 1), P(t, (2, 3), 2)),
    "sub": lambda t: (lambda a, b: ((a - b).sum(), [a, b]))(P(t, (2, 3), 1), P(t, (2, 3), 2)),
    "mul": lambda t: (lambda a, b: ((a * b).sum(), [a, b]))(P(t, (2, 3), 1), P(t, (2, 3), 2)),
    "div": lambda t: (lambda a, b: ((a / b).sum(), [a, b]))(
        P(t, (2, 3), 1), t.parameter(tensor((2, 3), [v * 0.5 + 1.0 for v in range(6)]))),
    "neg": lambda t: (lambda a: ((-a).sum(), [a]))(P(t, (4,), 1)),
    "tanh": lambda t: (lambda a: (a.tanh().sum(), [a]))(P(t, (4,), 1)),
    "exp": lambda t: (lambda a: (a.exp().sum(), [a]))(P(t, (4,), 1)),
    "ln": lambda t: (lambda a: (a.ln().sum(), [a]))(
        t.parameter(tensor((4,), [v * 0.75 for v in range(1, 5)]))),
    "sqrt": lambda t: (lambda a: (a.sqrt().sum(), [a]))(
        t.parameter(tensor((4,), [v * 1.25 for v in range(1, 5)]))),
    "powf": lambda t: (lambda a, b: (a.powf(b).sum(), [a, b]))(
        t.parameter(tensor((3,), [v * 0.5 + 0.25 for v in range(1, 4)])),
        t.parameter(tensor((3,), [2.0, 0.5, 3.0]))),
    "maximum": lambda t: (lambda a, b: (a.maximum(b).sum(), [a, b]))(
        P(t, (2, 3), 1), P(t, (2, 3), 2)),
    "relu": lambda t: (lambda a: (a.relu().sum(), [a]))(P(t, (2, 3), 1)),
    "step": lambda t: (lambda a: ((a.step(t.leaf(filled((2, 3), 0.0))) * a).sum(), [a]))(
        P(t, (2, 3), 1)),
    "matmul": lambda t: (lambda a, b: (a.matmul(b).sum(), [a, b]))(P(t, (2, 3), 1), P(t, (3, 4), 2)),
    "batched_matmul": lambda t: (lambda a, b: (a.matmul(b).sum(), [a, b]))(
        P(t, (2, 2, 3), 1), P(t, (2, 3, 4), 2)),
    "transpose": lambda t: (lambda a: ((a.transpose() * L(t, (3, 2), 2)).sum(), [a]))(P(t, (2, 3), 1)),
    "sum": lambda t: (lambda a: (a.sum(), [a]))(P(t, (2, 3), 1)),
    "sum_along": lambda t: (lambda a: ((a.sum_along(0) * L(t, (3,), 2)).sum(), [a]))(P(t, (2, 3), 1)),
    "broadcast_like": lambda t: (lambda a, r: ((a.broadcast_like(r) * r).sum(), [a]))(
        t.parameter(filled((), 1.25)), L(t, (2, 3), 2)),
    "broadcast_along": lambda t: (lambda a, r: ((a.broadcast_along(0, r) * r).sum(), [a]))(
        P(t, (3,), 1), L(t, (2, 3), 2)),
    "reshape": lambda t: (lambda a: ((a.reshape((6,)) * L(t, (6,), 2)).sum(), [a]))(P(t, (2, 3), 1)),
    "permute": lambda t: (lambda a: ((a.permute([2, 0, 1]) * L(t, (4, 2, 3), 2)).sum(), [a]))(
        P(t, (2, 3, 4), 1)),
    "narrow": lambda t: (lambda a: ((a.narrow(1, 1, 3) * L(t, (2, 3), 2)).sum(), [a]))(P(t, (2, 5), 1)),
    "pad": lambda t: (lambda a: ((a.pad(1, 2, 6) * L(t, (2, 6), 2)).sum(), [a]))(P(t, (2, 3), 1)),
    "unfold": lambda t: (lambda a: ((a.unfold(0, 3, 2, 1) * L(t, (3, 3), 2)).sum(), [a]))(P(t, (8,), 1)),
    "fold": lambda t: (lambda a: ((a.fold(0, 3, 2, 1, 8) * L(t, (8,), 2)).sum(), [a]))(P(t, (3, 3), 1)),
    "gather": lambda t: (lambda a: ((a.gather(t.input(selection([0, 2, 0], 3))) * L(t, (3, 2), 2))
                                    .sum(), [a]))(P(t, (3, 2), 1)),
    "scatter": lambda t: (lambda a: ((a.scatter(t.input(selection([0, 2, 0], 3)), 3)
                                      * L(t, (3, 2), 2)).sum(), [a]))(P(t, (3, 2), 1)),
    "log_softmax": lambda t: (lambda a: ((a.log_softmax(1) * L(t, (2, 4), 2)).sum(), [a]))(
        P(t, (2, 4), 1)),
    "logsumexp": lambda t: (lambda a: ((a.logsumexp(1) * L(t, (2,), 2)).sum(), [a]))(P(t, (2, 4), 1)),
    # differentiate_tests.rs:371-379
    "fan_out": lambda t: (lambda a: ((a * a).sum() + a.tanh().sum() + (-a).sum(), [a]))(
        P(t, (2, 3), 1)),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_recorded_gradients_close_bitwise_against_the_engine(built, name):
    closes(CASES[name])


def test_a_composed_loss_closes_through_a_plan(built):
    # differentiate_tests.rs:381-410: a dense model with a fed input
    def build(t):
        x = t.input(varied((2, 3), 1))
        w = P(t, (3, 2), 2)
        b = P(t, (2,), 3)
        logits = x.matmul(w) + b.broadcast_along(0, x.matmul(w))
        return logits.tanh().sum(), [w, b]
    closes(build)


def test_non_ancestors_answer_zeros(built):
    # differentiate_tests.rs:412-422
    (g,) = closes(lambda t: (P(t, (2,), 1).sum(), [P(t, (3,), 2)]))
    assert g.tolist() == [0.0, 0.0, 0.0]


def test_singular_disconnected_expressions_stay_masked(built):
    # differentiate_tests.rs:424-436
    def build(t):
        a = P(t, (2,), 1)
        zero = t.leaf(filled((2,), 0.0))
        _ = zero / zero
        return a.sum(), [a]
    (g,) = closes(build)
    assert g.tolist() == [1.0, 1.0]


def test_differentiate_rejects_non_scalar_losses(built):
    # differentiate_tests.rs:438-444
    t = Tape()
    a = P(t, (2,), 1)
    with pytest.raises(AssertionError, match="scalar loss"):
        t.differentiate(a + a, [a])


def second(build):
    t = Tape()
    x, loss = build(t)
    (first,) = t.differentiate(loss, [x])
    (g2,) = t.differentiate(first.sum(), [x])
    net = t.into_network()
    return oracle.run(net.compile(Request([g2])), net.parameters())[g2.index]


def test_second_derivative_of_a_cubic_is_exact(built):
    # differentiate_tests.rs:446-462
    def build(t):
        x = t.parameter(tensor((3,), [0.5, -1.25, 2.0]))
        return x, (x * x * x).sum()
    assert second(build).tolist() == [6.0 * v for v in (0.5, -1.25, 2.0)]


def test_second_derivative_of_tanh_matches_finite_differences(built):
    # differentiate_tests.rs:464-480 (f32 here: tolerance 1e-5)
    probe = 0.65

    def build(t):
        x = t.parameter(tensor((1,), [probe]))
        return x, x.tanh().sum()
    step = 1e-6
    d = lambda v: 1.0 - math.tanh(v) ** 2
    expected = (d(probe + step) - d(probe - step)) / (2 * step)
    assert abs(float(second(build)[0]) - expected) < 1e-5


def test_relu_hessians_are_exact_zeros(built):
    # differentiate_tests.rs:482-495
    def build(t):
        x = t.parameter(tensor((3,), [-2.0, 0.5, 3.0]))
        return x, x.relu().sum()
    assert second(build).tolist() == [0.0, 0.0, 0.0]


def test_tape_growth_stays_a_small_constant(built):
    # differentiate_tests.rs:497-518
    t = Tape()
    x = t.input(varied((4, 3), 1))
    w = P(t, (3, 4), 2)
    logits = x.matmul(w).tanh().matmul(P(t, (4, 2), 3))
    loss = logits.log_softmax(1).sum()
    before = len(t)
    t.differentiate(loss, [w])
    assert len(t) - before <= before * 6


def test_batched_matmul_matches_the_head_loop_bitwise(built):
    # differentiate_tests.rs:186-233, through the engine's reverse scan
    t = Tape()
    a, b = P(t, (2, 3, 4), 1), P(t, (2, 4, 5), 2)
    product = a.matmul(b)
    loss = product.sum()
    net = t.into_network()
    cols = net.compile(Request([loss, product]))
    batched = oracle.run(cols, net.parameters(), read=[product])[product.index]
    ga, gb = oracle.backward(cols, net.parameters(), loss, [a, b])

    t2 = Tape()
    a2, b2 = P(t2, (2, 3, 4), 1), P(t2, (2, 4, 5), 2)
    heads = [a2.narrow(0, h, 1).reshape((3, 4)).matmul(b2.narrow(0, h, 1).reshape((4, 5)))
             for h in range(2)]
    loss2 = heads[0].sum() + heads[1].sum()
    net2 = t2.into_network()
    cols2 = net2.compile(Request([loss2] + heads))
    out = oracle.run(cols2, net2.parameters(), read=heads)
    ga2, gb2 = oracle.backward(cols2, net2.parameters(), loss2, [a2, b2])
    assert batched.reshape(-1).tobytes() == np.concatenate(
        [out[h.index].reshape(-1) for h in heads]).tobytes()
    assert ga.tobytes() == ga2.tobytes() and gb.tobytes() == gb2.tobytes()


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(CASES))
def test_engine_backward_plans_on_the_device_follow_the_engine_scan(device, name):
    # `Request::backward` lowered on the device (the reverse scan appended as
    # nodes) against the oracle's scan of the same graph
    from poorgrad_b200 import backend
    t = Tape()
    loss, wrt = CASES[name](t)
    net = t.into_network()
    cols = net.compile(Request([loss]).backward())
    params = net.parameters()
    engine = oracle.backward(cols, params, loss, wrt)
    plan = backend.DevicePlan(cols)
    dp = backend.DeviceParameters(plan, params)
    plan.forward(dp, sync=True)
    for p, e in zip(wrt, engine):
        np.testing.assert_allclose(plan.gradient(loss, p), e, rtol=1e-5, atol=1e-6)


def test_a_recorded_training_loop_matches_the_engine_bitwise(built):
    # differentiate_tests.rs:519-587: twelve SGD generations through the
    # engine's reverse scan and through the recorded-gradient plan agree bit
    # for bit
    def build(t):
        x = t.input(varied((4, 3), 1))
        w = P(t, (3, 4), 2)
        b = P(t, (4,), 3)
        product = x.matmul(w)
        hidden = (product + b.broadcast_along(0, product)).tanh()
        head = P(t, (4, 2), 4)
        return x, [w, b, head], hidden.matmul(head).log_softmax(1).sum()

    te = Tape()
    xe, pe, le = build(te)
    ne = te.into_network()
    engine_cols = ne.compile(Request([le]).backward())
    tr = Tape()
    xr, pr, lr = build(tr)
    grads = tr.differentiate(lr, pr)
    nr = tr.into_network()
    recorded_cols = nr.compile(Request([lr] + grads))
    es, rs = ne.parameters(), nr.parameters()
    rate = np.float32(0.05)
    for step in range(12):
        batch = varied((4, 3), 10 + step).to_numpy().astype(np.float32)
        eg = oracle.backward(engine_cols, es, le, pe, {xe: batch})
        out = oracle.run(recorded_cols, rs, {xr: batch}, read=grads)
        es = [(p - g.reshape(-1) * rate).astype(np.float32) for p, g in zip(es, eg)]
        rs = [(p - out[g.index].reshape(-1) * rate).astype(np.float32) for p, g in zip(rs, grads)]
        for a, b in zip(es, rs):
            assert a.tobytes() == b.tobytes(), f"step {step}"
