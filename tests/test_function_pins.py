"""The per-function known answers of the reference's rule tests
(function/tests/*_tests.rs), recorded as small graphs and differentiated with
Tape::differentiate: the oracle must give the stated values, and the lowered
device program, run on the host by the kernel emulator, must give the
oracle's bits (within a few ulp where a transcendental is involved)."""
import math

import numpy as np
import pytest

import kernel_emulator
import oracle
from poorgrad_b200.graph import Tape, filled, tensor
from poorgrad_b200.plan import Request


def both(t, roots):
    net = t.into_network()
    cols = net.compile(Request(roots))
    ref = oracle.run(cols, net.parameters())
    dev = kernel_emulator.run_program(cols, net.parameters())
    return ref, dev


def seeded(t, y, seed):
    # loss = sum(y * seed): the cotangent reaching y is `seed`
    return (y * t.leaf(filled(list(y.shape), seed))).sum()


def values(out, v):
    return np.asarray(out[v.index], np.float64).reshape(-1).tolist()


def test_add_hands_one_cotangent_per_operand(built):
    # add_tests.rs: forward 2 + 3 = 5, backward (1.5, 1.5)
    t = Tape()
    a, b = t.parameter(tensor([1], [2.0])), t.parameter(tensor([1], [3.0]))
    y = a + b
    ga, gb = t.differentiate(seeded(t, y, 1.5), [a, b])
    ref, dev = both(t, [y, ga, gb])
    assert values(ref, y) == [5.0] and values(ref, ga) == [1.5] and values(ref, gb) == [1.5]
    for v in (y, ga, gb):
        assert dev[v.index].tobytes() == ref[v.index].tobytes()


@pytest.mark.parametrize("left,right,expect", [
    (2.0, 3.0, (0.0, 1.5)),   # maximum_tests.rs: the gradient goes to the winner
    (2.0, 2.0, (1.5, 0.0)),   # maximum_tests.rs: ties go to the left operand
])
def test_maximum_hands_the_gradient_to_the_winner(built, left, right, expect):
    t = Tape()
    a, b = t.parameter(tensor([1], [left])), t.parameter(tensor([1], [right])),
    y = a.maximum(b)
    ga, gb = t.differentiate(seeded(t, y, 1.5), [a, b])
    ref, dev = both(t, [y, ga, gb])
    assert values(ref, y) == [max(left, right)]
    assert (values(ref, ga)[0], values(ref, gb)[0]) == expect
    for v in (y, ga, gb):
        assert dev[v.index].tobytes() == ref[v.index].tobytes()


def test_relu_stops_where_the_operand_is_negative(built):
    # relu_tests.rs: relu(-2) = 0 with no gradient, relu(2) = 2 passing 1.5
    t = Tape()
    x = t.parameter(tensor([2], [-2.0, 2.0]))
    y = x.relu()
    (g,) = t.differentiate(seeded(t, y, 1.5), [x])
    ref, dev = both(t, [y, g])
    assert values(ref, y) == [0.0, 2.0] and values(ref, g) == [0.0, 1.5]
    for v in (y, g):
        assert dev[v.index].tobytes() == ref[v.index].tobytes()


def test_step_is_the_left_biased_indicator_and_carries_no_gradient(built):
    # step_tests.rs: step([-1, 0, 0.5, 2], [0, 0, 1, 1]) = [0, 1, 0, 1] (ties
    # answer one); both operands are data, so d(x * step(x, t))/dx = step
    t = Tape()
    x = t.parameter(tensor([4], [-1.0, 0.0, 0.5, 2.0]))
    thr = t.parameter(tensor([4], [0.0, 0.0, 1.0, 1.0]))
    s = x.step(thr)
    gx, gt = t.differentiate((x * s).sum(), [x, thr])
    ref, dev = both(t, [s, gx, gt])
    assert values(ref, s) == [0.0, 1.0, 0.0, 1.0]
    assert values(ref, gx) == [0.0, 1.0, 0.0, 1.0]
    assert values(ref, gt) == [0.0, 0.0, 0.0, 0.0]
    for v in (s, gx, gt):
        assert dev[v.index].tobytes() == ref[v.index].tobytes()


def test_sqrt_divides_by_twice_the_output(built):
    # sqrt_tests.rs: sqrt(9) = 3; the cotangent 6 becomes 6 / (2 * 3) = 1
    t = Tape()
    x = t.parameter(tensor([1], [9.0]))
    y = x.sqrt()
    (g,) = t.differentiate(seeded(t, y, 6.0), [x])
    ref, dev = both(t, [y, g])
    assert values(ref, y) == [3.0] and values(ref, g) == [1.0]
    for v in (y, g):
        assert dev[v.index].tobytes() == ref[v.index].tobytes()


def test_powf_routes_the_power_and_exponential_rules(built):
    # powf_tests.rs: 2^3 = 8, d/dx = 3 * 2^2 = 12, d/dy = 8 ln 2; a negative
    # base keeps d/dx = y x^(y-1) = -4 and has no real d/dy (NaN)
    t = Tape()
    x = t.parameter(tensor([2], [2.0, -2.0]))
    e = t.parameter(tensor([2], [3.0, 2.0]))
    y = x.powf(e)
    gx, ge = t.differentiate(y.sum(), [x, e])
    ref, dev = both(t, [y, gx, ge])
    assert values(ref, y) == [8.0, 4.0]
    assert values(ref, gx) == [12.0, -4.0]
    g1 = values(ref, ge)
    assert math.isclose(g1[0], 8.0 * math.log(2.0), rel_tol=1e-6) and math.isnan(g1[1])
    for v in (y, gx):
        assert dev[v.index].tobytes() == ref[v.index].tobytes()
    d = dev[ge.index].reshape(-1)
    assert math.isclose(float(d[0]), g1[0], rel_tol=4e-6) and math.isnan(float(d[1]))


def test_scatter_accumulates_repeated_rows_and_gathers_back(built):
    # scatter_tests.rs: rows [1,2],[3,4],[5,6] scattered by [0, 2, 0] into 3
    # rows give [6,8],[0,0],[3,4]; the backward gathers the seed by the same
    # selection, each source row reading its own target row back
    from poorgrad_b200.graph import selection
    t = Tape()
    g = t.parameter(tensor([3, 2], [1, 2, 3, 4, 5, 6]))
    sel = t.leaf(selection([0, 2, 0], 3))
    y = g.scatter(sel, 3)
    seed = t.leaf(tensor([3, 2], [1, 2, 3, 4, 5, 6]))
    (gg,) = t.differentiate((y * seed).sum(), [g])
    ref, dev = both(t, [y, gg])
    assert values(ref, y) == [6.0, 8.0, 0.0, 0.0, 3.0, 4.0]
    assert values(ref, gg) == [1.0, 2.0, 5.0, 6.0, 1.0, 2.0]
    for v in (y, gg):
        assert dev[v.index].tobytes() == ref[v.index].tobytes()


def test_fold_sums_overlapping_windows_and_unfolds_back(built):
    # fold_tests.rs: an eight-element axis unfolded by size 3, step 2 (three
    # windows) folds back with the overlaps summed; the backward unfolds the
    # seed by the same parameters
    t = Tape()
    x = t.parameter(tensor([8], list(range(1, 9))))
    w = x.unfold(0, 3, 2, 1)
    y = w.fold(0, 3, 2, 1, 8)
    seed = t.leaf(tensor([8], [0.5 * v for v in range(8)]))
    (gx,) = t.differentiate((y * seed).sum(), [x])
    ref, dev = both(t, [w, y, gx])
    # windows [1,2,3], [3,4,5], [5,6,7]; element 8 is in none
    assert values(ref, w) == [1, 2, 3, 3, 4, 5, 5, 6, 7]
    assert values(ref, y) == [1, 2, 6, 4, 10, 6, 7, 0]
    # d/dx = unfold(seed) folded back onto x: the seed times each element's
    # window count
    assert values(ref, gx) == [0.0, 0.5, 2.0, 1.5, 4.0, 2.5, 3.0, 0.0]
    for v in (w, y, gx):
        assert dev[v.index].tobytes() == ref[v.index].tobytes()


def test_literals_mix_into_expressions(built):
    # graph/tests/value_tests.rs (payload_literals_mix_into_expressions): at
    # x = 3, y = 2x + 1 = 7 with dy/dx = 2, and z = 6 / x = 2 with
    # dz/dx = -6 / x^2 = -2/3; every literal is its own leaf
    t = Tape()
    x = t.parameter(tensor([], [3.0]))
    before = len(t)
    y = t.leaf(filled([], 2.0)) * x + t.leaf(filled([], 1.0))
    z = t.leaf(filled([], 6.0)) / x
    assert len(t) - before == 6  # 2, the product, 1, the sum, 6, the quotient
    gy, = t.differentiate(y, [x])
    gz, = t.differentiate(z, [x])
    ref, dev = both(t, [y, z, gy, gz])
    assert values(ref, y) == [7.0] and values(ref, z) == [2.0] and values(ref, gy) == [2.0]
    assert values(ref, gz) == [float(np.float32(-(np.float32(2.0) / np.float32(3.0))))]
    for v in (y, z, gy, gz):
        assert dev[v.index].tobytes() == ref[v.index].tobytes()
