"""BatchNorm as the reference composes it (neural/batch_norm.rs:104-177):
the known answers of neural/tests/batch_norm_tests.rs on the oracle, and the
inference form fed with changing running statistics on the device."""
import numpy as np
import pytest

import oracle
from poorgrad_b200 import backend, neural
from poorgrad_b200.graph import Tape, filled, tensor
from poorgrad_b200.plan import Request


def run(t, roots, feeds=None):
    net = t.into_network()
    return oracle.run(net.compile(Request(roots)), net.parameters(), feeds)


def test_express_standardizes_every_feature():
    # batch_norm_tests.rs:55-83
    t = Tape()
    norm = neural.BatchNorm(t, 2, epsilon=0.0)
    out, mean, var = norm.express(t.leaf(tensor((2, 2), [1.0, 2.0, 3.0, 6.0])))
    assert out.shape == (2, 2) and mean.shape == (2,) and var.shape == (2,)
    got = run(t, [out, mean, var])
    assert got[mean.index].tolist() == [2.0, 4.0]
    assert got[var.index].tolist() == [1.0, 4.0]
    assert got[out.index].reshape(-1).tolist() == [-1.0, -1.0, 1.0, 1.0]


def test_express_applies_the_learned_affine():
    # batch_norm_tests.rs:85-101
    t = Tape()
    norm = neural.BatchNorm(t, 2, epsilon=0.0, scale=[2.0, 3.0], shift=[10.0, 20.0])
    out, _, _ = norm.express(t.leaf(tensor((2, 2), [1.0, 2.0, 3.0, 6.0])))
    assert run(t, [out])[out.index].reshape(-1).tolist() == [8.0, 17.0, 12.0, 23.0]


def test_epsilon_keeps_a_constant_feature_finite():
    # batch_norm_tests.rs:103-121
    t = Tape()
    norm = neural.BatchNorm(t, 1, epsilon=4.0)
    out, _, _ = norm.express(t.leaf(tensor((2, 1), [5.0, 5.0])))
    assert run(t, [out])[out.index].reshape(-1).tolist() == [0.0, 0.0]


def test_express_records_tensor_granularity():
    # batch_norm_tests.rs:123-140: sixteen computed nodes and two count
    # literals, whatever the batch and feature sizes
    for shape in ((3, 2), (64, 17)):
        t = Tape()
        norm = neural.BatchNorm(t, shape[1], epsilon=0.0)
        x = t.leaf(filled(shape, 1.0))
        before = len(t)
        norm.express(x)
        assert len(t) == before + 18


def test_express_rejects_mismatched_features():
    # batch_norm_tests.rs:189-200
    t = Tape()
    norm = neural.BatchNorm(t, 2)
    with pytest.raises(AssertionError, match="disagree on features"):
        norm.express(t.leaf(filled((2, 3), 1.0)))


def test_gradients_flow_through_the_batch_statistics():
    # batch_norm_tests.rs:202-236: input gradient [3/16, -3/16]; the scale
    # sees the normalized value, the shift the seed
    t = Tape()
    norm = neural.BatchNorm(t, 1, epsilon=3.0)
    x = t.parameter(tensor((2, 1), [3.0, 1.0]))
    out, _, _ = norm.express(x)
    target = out.narrow(0, 0, 1).sum()
    gx, gs, gb = t.differentiate(target, [x, norm.scale, norm.shift])
    got = run(t, [gx, gs, gb])
    assert np.allclose(got[gx.index].reshape(-1), [0.1875, -0.1875], atol=1e-6)
    assert got[gs.index].tolist() == [0.5]
    assert got[gb.index].tolist() == [1.0]


def fed_statistics(batch, features):
    t = Tape()
    norm = neural.BatchNorm(t, features, epsilon=0.0)
    x = t.input(filled((batch, features), 0.0))
    mean = t.input(filled((features,), 0.0))
    var = t.input(filled((features,), 1.0))
    out = norm.express_with(x, mean, var)
    net = t.into_network()
    return net, net.compile(Request([out])), x, mean, var, out


def test_express_with_normalizes_by_the_fed_statistics():
    # batch_norm_tests.rs:142-187: two runs of one recorded expression
    net, cols, x, mean, var, out = fed_statistics(1, 2)
    for m, v, expect in (([1.0, 4.0], [4.0, 16.0], [1.0, 1.0]),
                         ([3.0, 0.0], [1.0, 4.0], [0.0, 4.0])):
        feeds = {x: np.array([[3.0, 8.0]], np.float32), mean: np.array(m, np.float32),
                 var: np.array(v, np.float32)}
        got = oracle.run(cols, net.parameters(), feeds)
        assert got[out.index].reshape(-1).tolist() == expect


@pytest.mark.gpu
def test_express_with_on_the_device_follows_each_feed(device):
    batch, features = 1024, 96
    net, cols, x, mean, var, out = fed_statistics(batch, features)
    plan = backend.DevicePlan(cols)
    dp = backend.DeviceParameters(plan, net.parameters())
    rng = np.random.default_rng(9)
    for _ in range(3):
        feeds = {x: rng.normal(size=(batch, features)).astype(np.float32),
                 mean: rng.normal(size=features).astype(np.float32),
                 var: rng.uniform(0.5, 2.0, features).astype(np.float32)}
        ref = oracle.run(cols, net.parameters(), feeds)
        plan.forward(dp, feeds, sync=True)
        # subtract, sqrt, divide, multiply, add: correctly rounded on both sides
        assert plan.of(out).tobytes() == ref[out.index].tobytes()


@pytest.mark.gpu
def test_training_statistics_on_the_device_are_bitwise_the_recorded_formula(device):
    # training mode over a mini-batch (batch-norm's BatchNormTraining pattern,
    # payload/tensor.rs:802-851): the mean and the biased variance are column
    # folds over at most 256 rows, which the device runs as one serial fold
    # per feature from the first row -- the reference's order -- so the
    # statistics and the normalized output equal the oracle bit for bit; the
    # gradients through them carry the tolerance of their reassociated sums
    batch, features = 64, 4096
    t = Tape()
    rng = np.random.default_rng(3)
    x = t.parameter(tensor((batch, features), rng.normal(size=(batch, features)).astype(np.float32)))
    bn = neural.BatchNorm(t, features, scale=rng.uniform(0.5, 1.5, features),
                          shift=rng.normal(size=features))
    out, mean, var = bn.express(x)
    loss = (out * out).sum()
    grads = t.differentiate(loss, [x] + bn.parameters())
    net = t.into_network()
    cols = net.compile(Request([out, mean, var] + grads))
    ref = oracle.run(cols, net.parameters())
    plan = backend.DevicePlan(cols)
    dp = backend.DeviceParameters(plan, net.parameters())
    plan.forward(dp, sync=True)
    for v in (mean, var, out):
        assert plan.of(v).tobytes() == ref[v.index].tobytes()
    for g in grads:
        r = ref[g.index]
        np.testing.assert_allclose(plan.of(g), r, rtol=1e-4, atol=1e-5 * (np.abs(r).max() + 1e-30))
