"""The graph composites (graph/composite.rs: abs, softmax, mean_along,
broadcast_to, concat, stack) on the oracle, pinned on the known answers of
graph/tests/composite_tests.rs.  Gradients come from the oracle's restatement
of the engine's reverse scan (`Run::backward`); values that are exact in the
reference are exact here too; f64 tolerances become f32 ones."""
import math

import numpy as np
import pytest

import oracle
from poorgrad_b200.graph import Tape, concat, stack, tensor
from poorgrad_b200.plan import Request


def run(t, roots, grads_of=None, loss=None):
    net = t.into_network()
    cols = net.compile(Request(list(roots) + ([loss] if loss is not None else [])).backward())
    out = oracle.run(cols, net.parameters())
    grads = oracle.backward(cols, net.parameters(), loss, grads_of) if grads_of else []
    return out, grads


def test_abs_composes_from_maximum(built):
    # composite_tests.rs:3-17
    t = Tape()
    x = t.leaf(tensor((3,), [-2.0, 0.0, 3.0]))
    m = x.abs()
    out, (g,) = run(t, [m], [x], m.sum())
    assert out[m.index].tolist() == [2.0, 0.0, 3.0]
    assert g.tolist() == [-1.0, 1.0, 1.0]


def test_softmax_matches_the_probabilities(built):
    # composite_tests.rs:19-46
    for row, expected in (([0.0, math.log(3.0)], [0.25, 0.75]), ([1000.0, 1000.0], [0.5, 0.5])):
        t = Tape()
        p = t.leaf(tensor((1, 2), row)).softmax(1)
        out, _ = run(t, [p])
        assert np.allclose(out[p.index].reshape(-1), expected, atol=1e-6)


def test_logsumexp_reduces_like_a_smooth_maximum(built):
    # composite_tests.rs:48-79, 186-200
    t = Tape()
    x = t.leaf(tensor((2, 2), [0.0, math.log(3.0), 1000.0, 1000.0]))
    r = x.logsumexp(1)
    assert r.shape == (2,)
    out, (g,) = run(t, [r], [x], r.sum())
    v = out[r.index]
    assert abs(v[0] - math.log(4.0)) < 1e-6
    assert abs(v[1] - (1000.0 + math.log(2.0))) < 1e-3
    assert np.allclose(g[0], [0.25, 0.75], atol=1e-6)
    # at 1000 the f32 normalizer carries an ulp of 6e-5 into exp(x - out)
    assert np.allclose(g[1], [0.5, 0.5], atol=1e-4)


def test_mean_along_divides_by_the_axis_extent(built):
    # composite_tests.rs:81-105
    t = Tape()
    x = t.leaf(tensor((2, 3), [1.0, 2.0, 3.0, 4.0, 5.0, 6.0]))
    m = x.mean_along(0)
    assert m.shape == (3,)
    out, (g,) = run(t, [m], [x], m.sum())
    assert out[m.index].tolist() == [2.5, 3.5, 4.5]
    assert g.reshape(-1).tolist() == [0.5] * 6
    t = Tape()
    with pytest.raises(AssertionError, match="out of rank"):
        t.leaf(tensor((2,), [1.0, 2.0])).mean_along(1)


@pytest.mark.parametrize("source,values,target,expected,grad", [
    # composite_tests.rs:107-176
    ((3,), [1.0, 2.0, 3.0], (2, 3), [1.0, 2.0, 3.0] * 2, [2.0] * 3),
    ((2, 1, 2), [1.0, 2.0, 3.0, 4.0], (2, 3, 2),
     [1.0, 2.0, 1.0, 2.0, 1.0, 2.0, 3.0, 4.0, 3.0, 4.0, 3.0, 4.0], [3.0] * 4),
    ((1, 3), [1.0, 2.0, 3.0], (2, 2, 3), [1.0, 2.0, 3.0] * 4, [4.0] * 3),
    ((2, 2), [1.0, 2.0, 3.0, 4.0], (2, 2), [1.0, 2.0, 3.0, 4.0], [1.0] * 4),
    ((1,), [2.5], (2, 3), [2.5] * 6, [6.0]),
])
def test_broadcast_to(built, source, values, target, expected, grad):
    t = Tape()
    x = t.leaf(tensor(source, values))
    b = x.broadcast_to(target)
    assert b.shape == target
    out, (g,) = run(t, [b], [x], b.sum())
    assert out[b.index].reshape(-1).tolist() == expected
    assert g.reshape(-1).tolist() == grad


def test_broadcast_to_rejects_an_incompatible_axis(built):
    # composite_tests.rs:178-184
    t = Tape()
    with pytest.raises(AssertionError, match="cannot align"):
        t.leaf(tensor((3,), [1.0, 2.0, 3.0])).broadcast_to((2, 4))


def test_concat_joins_values(built):
    # composite_tests.rs:202-255
    t = Tape()
    top = t.leaf(tensor((2, 2), [1.0, 2.0, 3.0, 4.0]))
    bottom = t.leaf(tensor((1, 2), [5.0, 6.0]))
    joined = concat([top, bottom], 0)
    assert joined.shape == (3, 2)
    w = t.leaf(tensor((3, 2), [1.0, 2.0, 3.0, 4.0, 5.0, 6.0]))
    out, (gt, gb) = run(t, [joined], [top, bottom], (joined * w).sum())
    assert out[joined.index].reshape(-1).tolist() == [1.0, 2.0, 3.0, 4.0, 5.0, 6.0]
    assert gt.reshape(-1).tolist() == [1.0, 2.0, 3.0, 4.0]
    assert gb.reshape(-1).tolist() == [5.0, 6.0]
    t = Tape()
    left = t.leaf(tensor((2, 1), [1.0, 4.0]))
    right = t.leaf(tensor((2, 2), [2.0, 3.0, 5.0, 6.0]))
    joined = concat([left, right], 1)
    single = concat([left], 0)
    out, _ = run(t, [joined, single])
    assert out[joined.index].reshape(-1).tolist() == [1.0, 2.0, 3.0, 4.0, 5.0, 6.0]
    assert out[single.index].reshape(-1).tolist() == [1.0, 4.0]


def test_concat_rejects_bad_axes_and_shapes(built):
    # composite_tests.rs:257-271
    t = Tape()
    x = t.leaf(tensor((2,), [1.0, 2.0]))
    with pytest.raises(AssertionError, match="out of rank"):
        concat([x, x], 1)
    a = t.leaf(tensor((2, 2), [1.0] * 4))
    b = t.leaf(tensor((2, 3), [1.0] * 6))
    with pytest.raises(AssertionError, match="equal shapes off the axis"):
        concat([a, b], 0)


def test_stack_lifts_values_onto_a_new_axis(built):
    # composite_tests.rs:273-300
    t = Tape()
    first = t.leaf(tensor((3,), [1.0, 2.0, 3.0]))
    second = t.leaf(tensor((3,), [4.0, 5.0, 6.0]))
    rows = stack([first, second], 0)
    columns = stack([first, second], 1)
    assert rows.shape == (2, 3) and columns.shape == (3, 2)
    out, (g1, g2) = run(t, [rows, columns], [first, second], rows.sum())
    assert out[rows.index].reshape(-1).tolist() == [1.0, 2.0, 3.0, 4.0, 5.0, 6.0]
    assert out[columns.index].reshape(-1).tolist() == [1.0, 4.0, 2.0, 5.0, 3.0, 6.0]
    assert g1.tolist() == [1.0] * 3 and g2.tolist() == [1.0] * 3


def test_masked_softmax_composes_with_a_broadcast_mask(built):
    # composite_tests.rs:302-330
    t = Tape()
    scores = t.leaf(tensor((2, 3), [1.0, 1.0, 9.0, 2.0, 2.0, 9.0]))
    mask = t.leaf(tensor((3,), [0.0, 0.0, -np.inf]))
    p = (scores + mask.broadcast_to((2, 3))).softmax(1)
    out, (g,) = run(t, [p], [scores], p.narrow(1, 0, 1).sum())
    assert np.allclose(out[p.index].reshape(-1), [0.5, 0.5, 0.0, 0.5, 0.5, 0.0], atol=1e-6)
    assert np.allclose(g.reshape(-1), [0.25, -0.25, 0.0, 0.25, -0.25, 0.0], atol=1e-6)


def test_attention_heads_compose_with_a_loop_and_concat(built):
    # composite_tests.rs:332-372
    t = Tape()
    causal = t.leaf(tensor((2, 2), [0.0, -np.inf, 0.0, 0.0]))
    heads, leaves = [], []
    for seed in range(2):
        shift = float(seed)
        q = t.leaf(tensor((2, 2), [shift, 1.0, 0.0, 1.0]))
        k = t.leaf(tensor((2, 2), [1.0, 0.0, shift, 1.0]))
        v = t.leaf(tensor((2, 2), [1.0 + shift, 2.0, 3.0, 4.0 + shift]))
        heads.append((q.matmul(k.transpose()) + causal).softmax(1).matmul(v))
        leaves += [q, v]
    output = concat(heads, 1)
    assert output.shape == (2, 4)
    out, grads = run(t, [output], leaves, output.sum())
    assert np.allclose(out[output.index].reshape(-1)[:4], [1.0, 2.0, 2.0, 2.0], atol=1e-6)
    for g in grads[0::2]:
        assert np.any(g != 0.0)


@pytest.mark.gpu
def test_composites_on_the_device(device):
    # the same compositions in one engine-backward plan on the device,
    # against the oracle's values and reverse scan
    from poorgrad_b200 import backend
    rng = np.random.default_rng(4)
    t = Tape()
    a = t.parameter(tensor((2, 1, 8), rng.uniform(-1, 1, 16)))
    b = t.parameter(tensor((8,), rng.uniform(-1, 1, 8)))
    s = t.parameter(tensor((4, 8), rng.uniform(-2, 2, 32)))
    mask = t.leaf(tensor((8,), [0.0] * 6 + [-np.inf] * 2))
    grid = a.broadcast_to((2, 4, 8)) + b.broadcast_to((2, 4, 8))
    probs = (s + mask.broadcast_to((4, 8))).softmax(1)
    joined = concat([grid.reshape((8, 8)), probs.abs()], 0)
    stacked = stack([probs, s.mean_along(0).broadcast_to((4, 8))], 0)
    loss = (joined.tanh().sum() + stacked.logsumexp(2).sum())
    net = t.into_network()
    cols = net.compile(Request([loss, joined, stacked]).backward())
    params = net.parameters()
    ref = oracle.run(cols, params)
    grads = oracle.backward(cols, params, loss, [a, b, s])
    plan = backend.DevicePlan(cols)
    dp = backend.DeviceParameters(plan, params)
    plan.forward(dp, sync=True)
    for v in (joined, stacked, loss):
        np.testing.assert_allclose(plan.of(v), ref[v.index], rtol=4e-6, atol=1e-7)
    for p, g in zip((a, b, s), grads):
        np.testing.assert_allclose(plan.gradient(loss, p), g, rtol=1e-5, atol=1e-6)
