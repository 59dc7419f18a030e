"""The plan contract of engine/tests/plan_tests.rs:9-162 through the device
plan: values agree with the interpreter (the oracle), what the roots cannot
observe is not computed, only readable values can be read, `observe` makes an
interior readable, forward-only plans refuse backward, feeds bind, liveness
frees nothing early, and one plan serves every training step."""
import numpy as np
import pytest

import oracle
from poorgrad_b200 import backend
from poorgrad_b200.graph import Tape, filled, tensor
from poorgrad_b200.plan import Request


def device_run(t, request, feeds=None):
    net = t.into_network()
    cols = net.compile(request)
    plan = backend.DevicePlan(cols)
    dp = backend.DeviceParameters(plan, net.parameters())
    plan.forward(dp, feeds, sync=True)
    return net, cols, plan


def test_unobservable_values_are_not_wanted(built):
    # plan_tests.rs:24-36 on the compiled columns
    t = Tape()
    x = t.leaf(filled((), 2.0))
    wanted = x * x
    unwanted = x + x
    cols = t.into_network().compile(Request([wanted]))
    assert cols.wanted[wanted.index] and not cols.wanted[unwanted.index]


@pytest.mark.gpu
def test_plan_forward_matches_the_interpreter(device):
    # plan_tests.rs:8-22 (tanh: CUDA's tanhf against glibc, relative 4e-6)
    t = Tape()
    x = t.leaf(tensor((2, 2), [1.0, 2.0, 3.0, 4.0]))
    y = t.leaf(tensor((2, 2), [0.5, -0.5, 1.5, -1.5]))
    target = ((x.matmul(y) + x).tanh() * y).sum()
    net, cols, plan = device_run(t, Request([target]))
    ref = oracle.run(cols, net.parameters())[target.index]
    np.testing.assert_allclose(plan.of(target), ref, rtol=4e-6)


@pytest.mark.gpu
def test_plan_skips_what_the_targets_cannot_observe(device):
    # plan_tests.rs:24-36
    t = Tape()
    x = t.leaf(filled((), 2.0))
    wanted = x * x
    _ = x + x
    _, _, plan = device_run(t, Request([wanted]))
    assert float(plan.of(wanted)) == 4.0


@pytest.mark.gpu
def test_reads_outside_the_readable_set_are_rejected(device):
    # plan_tests.rs:38-53
    t = Tape()
    x = t.leaf(filled((), 2.0))
    wanted = x * x
    interior = x * x * x
    target = interior + wanted
    _, _, plan = device_run(t, Request([target]))
    assert float(plan.of(target)) == 12.0
    with pytest.raises(backend.BackendError, match="not a readable value"):
        plan.of(interior)


@pytest.mark.gpu
def test_observe_makes_an_interior_value_readable(device):
    # plan_tests.rs:55-69
    t = Tape()
    x = t.leaf(filled((), 2.0))
    interior = x * x
    target = interior + x
    _, _, plan = device_run(t, Request([target], observe=[interior]))
    assert float(plan.of(target)) == 6.0
    assert float(plan.of(interior)) == 4.0


@pytest.mark.gpu
def test_forward_only_plans_refuse_backward(device):
    # plan_tests.rs:71-81
    t = Tape()
    x = t.parameter(filled((), 2.0))
    target = x * x
    _, _, plan = device_run(t, Request([target]))
    with pytest.raises(backend.BackendError, match="compile with backward set"):
        plan.gradient(target, x)


@pytest.mark.gpu
def test_liveness_frees_only_after_the_last_consumer(device):
    # plan_tests.rs:132-149: a diamond
    t = Tape()
    x = t.leaf(tensor((2,), [1.5, -2.5]))
    shared = x.tanh()
    early = shared * x
    late = (shared + early).sum()
    net, cols, plan = device_run(t, Request([late]))
    ref = oracle.run(cols, net.parameters())[late.index]
    np.testing.assert_allclose(plan.of(late), ref, rtol=4e-6)


@pytest.mark.gpu
def test_plan_forward_binds_feeds(device):
    # plan_tests.rs:151-162
    t = Tape()
    x = t.input(tensor((2,), [0.0, 0.0]))
    doubled = x * x.literal(tensor((2,), [2.0, 2.0]))
    _, _, plan = device_run(t, Request([doubled]), {x: np.array([4.0, 5.0], np.float32)})
    assert plan.of(doubled).tolist() == [8.0, 10.0]


@pytest.mark.gpu
def test_one_plan_serves_every_training_step(device):
    # plan_tests.rs:103-130: an engine-backward plan, five SGD steps taken
    # on the host from the device gradient, the loss equal to the
    # interpreter's at every step
    t = Tape()
    w = t.parameter(tensor((2,), [0.0, 0.0]))
    x = t.leaf(tensor((2,), [3.0, 2.0]))
    y = t.leaf(tensor((2,), [15.0, -6.0]))
    error = w * x - y
    loss = (error * error).sum()
    net = t.into_network()
    cols = net.compile(Request([loss]).backward())
    plan = backend.DevicePlan(cols)
    params = net.parameters()
    dp = backend.DeviceParameters(plan, params)
    for _ in range(5):
        plan.forward(dp, sync=True)
        ref = oracle.run(cols, params, read=[loss])[loss.index]
        (ref_grad,) = oracle.backward(cols, params, loss, [w])
        assert plan.of(loss).tobytes() == ref.tobytes()
        grad = plan.gradient(loss, w)
        assert grad.tobytes() == ref_grad.tobytes()
        params = [(params[0] - grad * np.float32(0.05)).astype(np.float32)]
        dp.upload(params)
    assert params[0][0] > 1.0


def engine_backward_on_device(t, loss, wrt, rtol):
    net = t.into_network()
    cols = net.compile(Request([loss]).backward())
    params = net.parameters()
    ref_loss = oracle.run(cols, params, read=[loss])[loss.index]
    ref = oracle.backward(cols, params, loss, wrt)
    plan = backend.DevicePlan(cols)
    dp = backend.DeviceParameters(plan, params)
    plan.forward(dp, sync=True)
    np.testing.assert_allclose(plan.of(loss), ref_loss, rtol=rtol)
    for p, r in zip(wrt, ref):
        np.testing.assert_allclose(plan.gradient(loss, p), r, rtol=rtol, atol=1e-7)


@pytest.mark.gpu
def test_training_liveness_on_a_convnet(device):
    # plan_tests.rs:235-290: conv, relu, pool, flatten, dense, cross-entropy;
    # what the derivative rules read is retained by the device plan
    from poorgrad_b200 import neural
    from poorgrad_b200.graph import selection
    t = Tape()
    x = t.leaf(tensor((2, 1, 4, 4), [v / 16.0 - 1.0 for v in range(32)]))
    w = t.parameter(tensor((2, 1, 3, 3), [v / 32.0 - 0.25 for v in range(18)]))
    b = t.parameter(tensor((2,), [0.1, -0.1]))
    head = t.parameter(tensor((8, 3), [v / 48.0 - 0.25 for v in range(24)]))
    targets = t.leaf(selection([1, 2], 3))
    pooled = neural.max_pool(neural.conv2d(x, w, b, 1, 1).relu(), 2, 2)
    loss = neural.cross_entropy(pooled.reshape((2, 8)).matmul(head), targets)
    engine_backward_on_device(t, loss, [w, b, head], rtol=2e-5)


@pytest.mark.gpu
def test_training_liveness_on_every_value_reader(device):
    # plan_tests.rs:292-326: mul, tanh, exp, ln, sqrt, powf, div, relu,
    # maximum with fan-out
    t = Tape()
    w = t.parameter(filled((), 0.7))
    x = t.leaf(filled((), 1.3))
    product = w * x
    squashed = product.tanh()
    grown = squashed.exp()
    loss = (squashed + grown + grown.ln() + grown.sqrt() + product.powf(x) + grown / product
            + product.relu() + product.maximum(x)) * product
    engine_backward_on_device(t, loss, [w], rtol=1e-5)


@pytest.mark.gpu
def test_training_liveness_retains_the_gather_selection(device):
    # plan_tests.rs:328-353: gather's backward scatters by the selection
    from poorgrad_b200.graph import selection
    t = Tape()
    table = t.parameter(tensor((4, 2), [v * 0.5 for v in range(8)]))
    sel = t.input(selection([2, 0, 3], 4))
    loss = table.gather(sel).sum()
    engine_backward_on_device(t, loss, [table], rtol=0)


def _product_tape():
    # plan_tests.rs:541-591: a 32 x 32 x 32 product
    t = Tape()
    a = t.parameter(tensor((32, 32), [(v % 37) * 0.21 - 3.7 for v in range(1024)]))
    b = t.parameter(tensor((32, 32), [(v % 29) * 0.17 - 2.3 for v in range(1024)]))
    return t, a, b


def test_the_numerics_posture_is_a_value_on_the_plan(built):
    # the posture travels with the columns; the lowering marks which plans
    # are bit-identical to the interpreter (only those run under Exact)
    from poorgrad_b200.plan import EXACT, FAST
    t, a, b = _product_tape()
    product = a.matmul(b)
    arithmetic = a * b + a
    net = t.into_network()
    assert net.compile(Request([product])).numerics == FAST
    exact = net.compile(Request([product]).numerics(EXACT))
    assert exact.numerics == EXACT
    assert "exact 0" in backend.lower_describe(exact)
    assert "exact 1" in backend.lower_describe(net.compile(Request([arithmetic]).numerics(EXACT)))


@pytest.mark.gpu
def test_exact_posture_declines_or_reproduces_the_interpreter(device):
    # Exact: a plan holding the tensor-core product declines (the
    # reference's `None`, Fidelity::meets); a plan of plain arithmetic runs
    # and equals the interpreter bitwise.  Fast: the product stays within
    # the 1e-4 envelope of the serial in-order product.
    from poorgrad_b200.plan import EXACT
    t, a, b = _product_tape()
    product = a.matmul(b)
    arithmetic = a * b + a
    net = t.into_network()
    params = net.parameters()
    with pytest.raises(backend.BackendError) as declined:
        backend.DevicePlan(net.compile(Request([product]).numerics(EXACT)))
    assert declined.value.code == 5 and "not bit-identical" in str(declined.value)
    exact = net.compile(Request([arithmetic]).numerics(EXACT))
    plan = backend.DevicePlan(exact)
    dp = backend.DeviceParameters(plan, params)
    plan.forward(dp, sync=True)
    assert plan.of(arithmetic).tobytes() == oracle.run(exact, params)[arithmetic.index].tobytes()
    fast = net.compile(Request([product]))
    plan = backend.DevicePlan(fast)
    dp = backend.DeviceParameters(plan, params)
    plan.forward(dp, sync=True)
    serial = oracle.run(fast, params)[product.index]
    got = plan.of(product)
    assert np.all(np.abs(got - serial) <= 1e-4 * np.maximum(np.abs(serial), 1.0))
