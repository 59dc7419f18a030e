"""Pins the CPU oracle (and the host graph/plan mirror) against the known
answers of the reference's own tests.  The reference is Rust and cannot be
built here, so these assertions -- restated from its test files, cited per
test -- are what anchor the oracle's parity."""
import math
import struct

import numpy as np

import oracle
from poorgrad_b200 import neural
from poorgrad_b200.graph import Tape, filled, selection, tensor
from poorgrad_b200.plan import Request


def run(tape, roots, feeds=None):
    net = tape.into_network()
    cols = net.compile(Request(roots))
    return oracle.run(cols, net.parameters(), feeds)


def test_sigmoid_composition_value_and_gradient(built):
    # engine/tests/run_tests.rs:343-355: sigmoid(0) = 0.5, its derivative 0.25
    t = Tape()
    x = t.parameter(tensor([], [0.0]))
    one = t.leaf(filled([], 1.0))
    s = one / (one + (-x).exp())
    (g,) = t.differentiate(s, [x])
    out = run(t, [s, g])
    assert out[s.index] == 0.5 and out[g.index] == 0.25


def test_gather_and_scatter_known_rows(built):
    # payload/tests/tensor_tests.rs:995-1016
    t = Tape()
    table = t.leaf(tensor([3, 2], [1, 2, 3, 4, 5, 6]))
    sel = t.leaf(selection([0, 2, 0], 3))
    gathered = table.gather(sel)
    ones = t.leaf(filled([3, 2], 1.0))
    scattered = ones.scatter(sel, 3)
    out = run(t, [gathered, scattered])
    assert out[gathered.index].reshape(-1).tolist() == [1, 2, 5, 6, 1, 2]
    assert out[scattered.index].reshape(-1).tolist() == [2, 2, 0, 0, 1, 1]


def test_matmul_transpose_sum_broadcast(built):
    # payload/tests/tensor_tests.rs:232-250
    t = Tape()
    m = t.leaf(tensor([2, 2], [1, 2, 3, 4]))
    c = t.leaf(tensor([2, 1], [5, 6]))
    product = m.matmul(c)
    tr = m.transpose()
    total = m.sum()
    spread = total.broadcast_like(c)
    out = run(t, [product, tr, total, spread])
    assert out[product.index].reshape(-1).tolist() == [17, 39]
    assert out[tr.index].reshape(-1).tolist() == [1, 3, 2, 4]
    assert out[total.index] == 10
    assert out[spread.index].reshape(-1).tolist() == [10, 10]


def test_matmul_gradients_through_transposed_operands(built):
    # payload/tests/tensor_tests.rs:269-288
    t = Tape()
    a = t.parameter(tensor([2, 2], [1, 2, 3, 4]))
    b = t.parameter(tensor([2, 1], [5, 6]))
    loss = a.matmul(b).sum()
    ga, gb = t.differentiate(loss, [a, b])
    out = run(t, [loss, ga, gb])
    assert out[loss.index] == 56
    assert out[ga.index].reshape(-1).tolist() == [5, 6, 5, 6]
    assert out[gb.index].reshape(-1).tolist() == [4, 6]


def test_negative_zero_terms_keep_their_sign(built):
    # payload/tests/gemm_tests.rs:130-139
    t = Tape()
    left = t.leaf(tensor([1, 2], [-0.0, 0.0]))
    right = t.leaf(tensor([2, 1], [0.0, -0.0]))
    p = left.matmul(right)
    out = run(t, [p])
    assert math.copysign(1.0, float(out[p.index].reshape(-1)[0])) == -1.0


def test_product_matches_a_naive_in_order_loop_bitwise(built):
    # engine/tests/plan_tests.rs:542-591: 32x32x32 f32 product, serial k
    rng = np.random.default_rng(0)
    a = rng.standard_normal((32, 32)).astype(np.float32)
    b = rng.standard_normal((32, 32)).astype(np.float32)
    t = Tape()
    p = t.leaf(tensor(a.shape, a)).matmul(t.leaf(tensor(b.shape, b)))
    out = run(t, [p])[p.index]
    ref = a[:, 0:1] * b[0:1, :]
    for k in range(1, 32):
        ref = ref + a[:, k:k + 1] * b[k:k + 1, :]
    assert out.tobytes() == ref.astype(np.float32).tobytes()


def test_log_softmax_rows_and_gradient(built):
    # payload/tests/tensor_tests.rs:1119-1152 (f64 there; f32 tolerance here)
    t = Tape()
    logits = t.leaf(tensor([2, 2], [0, 0, 1, 3]))
    lp = logits.log_softmax(1)
    out = run(t, [lp])[lp.index]
    assert np.allclose(np.exp(out).sum(axis=1), 1.0, atol=1e-6)
    t = Tape()
    x = t.parameter(tensor([1, 2], [0.0, math.log(3.0)]))
    loss = x.log_softmax(1).sum()
    (g,) = t.differentiate(loss, [x])
    out = run(t, [g])[g.index].reshape(-1)
    assert np.allclose(out, [0.5, -0.5], atol=1e-6)


def test_relu_masks_gradients_by_sign(built):
    # payload/tests/tensor_tests.rs:1162-1178
    t = Tape()
    x = t.parameter(tensor([4], [-2.0, -0.5, 0.0, 3.0]))
    a = x.relu()
    loss = a.sum()
    (g,) = t.differentiate(loss, [x])
    out = run(t, [a, g])
    assert out[a.index].tolist() == [0, 0, 0, 3]
    assert out[g.index].tolist() == [0, 0, 1, 1]


def test_cross_entropy_gradient_is_probabilities_minus_targets(built):
    # neural/tests/loss_tests.rs:39-56
    t = Tape()
    logits = t.parameter(tensor([2, 2], [0.0, math.log(3.0), 0.0, 0.0]))
    targets = t.input(selection([0, 1], 2))
    loss = neural.cross_entropy(logits, targets)
    (g,) = t.differentiate(loss, [logits])
    out = run(t, [g])[g.index].reshape(-1)
    assert np.allclose(out, [-0.375, 0.375, 0.25, -0.25], atol=1e-6)


def test_cross_entropy_of_uniform_logits_is_log_classes(built):
    # neural/tests/loss_tests.rs:6-19
    t = Tape()
    logits = t.leaf(filled([2, 3], 0.0))
    targets = t.input(selection([0, 2], 3))
    loss = neural.cross_entropy(logits, targets)
    out = run(t, [loss])[loss.index]
    assert abs(float(out) - math.log(3.0)) < 1e-6


def test_extreme_finite_logits_keep_the_f32_loss_finite(built):
    # neural/tests/loss_tests.rs:124-133
    t = Tape()
    logits = t.leaf(tensor([1, 2], [-3.0e38, 3.0e38]))
    targets = t.input(selection([1], 2))
    loss = neural.cross_entropy(logits, targets)
    assert run(t, [loss])[loss.index] == 0.0


def _bits32(x):
    return [struct.unpack("<I", struct.pack("<f", float(v)))[0] for v in np.asarray(x).reshape(-1)]


def _f32_of(bits64):
    return [struct.unpack("<I", struct.pack("<f", struct.unpack("<d", struct.pack("<Q", b))[0]))[0]
            for b in bits64]


def test_seeded_streams_are_pinned(built):
    # neural/tests/init_tests.rs:81-134: the f32 path is the f64 stream
    # rounded once per element
    uni = [0xbfcc341e1ba6cdf8, 0xbfeeecf0ca02f0e8, 0x3fe9a610202eac4a, 0x3fc53aeb70673e28]
    nor = [0x3fffa194ec47d228, 0xc00dd3fde5949e97, 0x3f800ea29c8645d7, 0xbff0efc91ba890b4]
    assert _bits32(neural.uniform(7, 1.0)((4,))) == _f32_of(uni)
    assert _bits32(neural.normal(7, 2.0)((4,))) == _f32_of(nor)


def test_plan_columns_release_like_the_reference(built):
    # engine/tests/plan_tests.rs:133-150 (liveness diamond): a value with two
    # consumers is released by the later one; roots are never released
    t = Tape()
    x = t.parameter(tensor([2], [1.0, 2.0]))
    a = x.exp()
    b = a * a
    c = a + b
    net = t.into_network()
    cols = net.compile(Request([c]))
    assert a.index in cols.releases[c.index]
    assert all(c.index not in r for r in cols.releases)


def _norm_run(norm_cls, kw, rows, vals, grad_of_first=False):
    t = Tape()
    norm = norm_cls(t, 2, **kw)
    x = t.leaf(tensor((rows, 2), vals)) if not grad_of_first else t.parameter(tensor((rows, 2), vals))
    out = norm.express(x)
    if not grad_of_first:
        return run(t, [out])[out.index].reshape(-1).tolist()
    target = out.narrow(1, 0, 1).sum()
    grads = t.differentiate(target, [x] + norm.parameters())
    res = run(t, grads)
    return [res[g.index].reshape(-1).tolist() for g in grads]


def test_layer_norm_standardizes_and_applies_the_affine(built):
    # neural/tests/layer_norm_tests.rs:44-81
    assert _norm_run(neural.LayerNorm, dict(epsilon=0.0), 2, [1, 3, 2, 6]) == [-1, 1, -1, 1]
    assert _norm_run(neural.LayerNorm, dict(epsilon=0.0, scale=[2, 3], shift=[10, 20]), 2,
                     [1, 3, 2, 6]) == [8, 23, 8, 23]


def test_layer_norm_gradients_through_the_statistics(built):
    # neural/tests/layer_norm_tests.rs:143-177: x = [3, 1], eps 3 -> d n0/dx = [3/16, -3/16];
    # the scale sees the normalized value (0.5) and the shift the seed (1) on feature 0
    gx, gscale, gshift = _norm_run(neural.LayerNorm, dict(epsilon=3.0), 1, [3, 1], True)
    assert abs(gx[0] - 0.1875) < 1e-6 and abs(gx[1] + 0.1875) < 1e-6
    assert gscale == [0.5, 0.0] and gshift == [1.0, 0.0]


def test_rms_norm_normalizes_and_scales(built):
    # neural/tests/rms_norm_tests.rs:41-73
    assert _norm_run(neural.RmsNorm, dict(epsilon=0.0), 2, [2, 2, 3, -3]) == [1, 1, 1, -1]
    assert _norm_run(neural.RmsNorm, dict(epsilon=0.0, scale=[2, 5]), 2,
                     [2, 2, 3, -3]) == [2, 5, 2, -5]


def test_rms_norm_gradients_through_the_root_mean_square(built):
    # neural/tests/rms_norm_tests.rs:99-122: x = [2, 0], eps 2 -> [1/4, 0]; scale [1, 0]
    gx, gscale = _norm_run(neural.RmsNorm, dict(epsilon=2.0), 1, [2, 0], True)
    assert gx == [0.25, 0.0] and gscale == [1.0, 0.0]


def _conv(ishape, ivals, wshape, wvals, bvals, stride, padding):
    t = Tape()
    x = t.leaf(tensor(ishape, ivals))
    w = t.leaf(tensor(wshape, wvals))
    b = t.leaf(tensor((wshape[0],), bvals))
    out = neural.conv2d(x, w, b, stride, padding)
    return out.shape, run(t, [out])[out.index].reshape(-1).tolist()


def test_conv2d_known_answers(built):
    # neural/tests/convolution_tests.rs:6-81
    assert _conv((1, 1, 3, 3), list(range(1, 10)), (1, 1, 2, 2), [1, 0, 0, 1], [10], 1, 0) == \
        ((1, 1, 2, 2), [16, 18, 22, 24])
    assert _conv((1, 2, 2, 2), [1, 2, 3, 4, 10, 20, 30, 40], (2, 2, 1, 1), [1, 1, 2, 3], [0, 0],
                 1, 0) == ((1, 2, 2, 2), [11, 22, 33, 44, 32, 64, 96, 128])
    assert _conv((1, 1, 1, 5), [1, 2, 3, 4, 5], (1, 1, 1, 2), [1, 1], [0], 2, 0) == \
        ((1, 1, 1, 2), [3, 7])
    assert _conv((1, 1, 2, 2), [1, 2, 3, 4], (1, 1, 3, 3), [1] * 9, [0], 1, 1) == \
        ((1, 1, 2, 2), [10, 10, 10, 10])


def test_conv2d_gradients_known_answers(built):
    # neural/tests/convolution_tests.rs:84-114: window coverage counts, summed inputs, seeds
    t = Tape()
    x = t.parameter(tensor((1, 1, 3, 3), list(range(1, 10))))
    w = t.parameter(tensor((1, 1, 2, 2), [1, 1, 1, 1]))
    b = t.parameter(tensor((1,), [0]))
    loss = neural.conv2d(x, w, b, 1, 0).sum()
    gx, gw, gb = t.differentiate(loss, [x, w, b])
    out = run(t, [gx, gw, gb])
    assert out[gx.index].reshape(-1).tolist() == [1, 2, 1, 2, 4, 2, 1, 2, 1]
    assert out[gw.index].reshape(-1).tolist() == [12, 16, 24, 28]
    assert out[gb.index].reshape(-1).tolist() == [4]


def test_max_pool_takes_window_maxima_and_routes_ties_left(built):
    # neural/pooling.rs:49-61: a left fold of maximum over the window lanes
    t = Tape()
    x = t.parameter(tensor((1, 1, 2, 4), [1, 5, 2, 2, 3, 4, 2, 2]))
    pooled = neural.max_pool(x, 2, 2)
    (g,) = t.differentiate(pooled.sum(), [x])
    out = run(t, [pooled, g])
    assert out[pooled.index].reshape(-1).tolist() == [5, 2]
    # the second window's four 2s tie: the gradient goes to its first lane only
    assert out[g.index].reshape(-1).tolist() == [0, 1, 1, 0, 0, 0, 0, 0]


def test_linear_records_the_affine_alone(built):
    # neural/tests/linear_tests.rs:41-56: [1, 1] x [[1, 2], [3, 4]] + [10, 20]
    t = Tape()
    lin = neural.Linear(t, np.array([[1, 2], [3, 4]], np.float32), np.array([10, 20], np.float32))
    out = lin.express(t.leaf(tensor((1, 2), [1, 1])))
    assert run(t, [out])[out.index].reshape(-1).tolist() == [14, 26]


def test_confident_correct_logits_cost_nothing(built):
    # neural/tests/loss_tests.rs:21-36
    t = Tape()
    loss = neural.cross_entropy(t.leaf(tensor((1, 2), [1000.0, -1000.0])),
                                t.input(selection([0], 2)))
    assert run(t, [loss])[loss.index] == 0.0


def test_extreme_f32_logits_keep_loss_zero_and_gradients_finite(built):
    # neural/tests/loss_tests.rs:100-133 (the f32 range): either class order
    for row, cls in (([-3.0e38, 3.0e38], 1), ([3.0e38, -3.0e38], 0)):
        t = Tape()
        logits = t.parameter(tensor((1, 2), row))
        loss = neural.cross_entropy(logits, t.input(selection([cls], 2)))
        (g,) = t.differentiate(loss, [logits])
        out = run(t, [loss, g])
        assert out[loss.index] == 0.0
        assert np.all(np.isfinite(out[g.index]))


def test_zero_target_lanes_contribute_exact_zero(built):
    # neural/tests/loss_tests.rs:136-148: a dense soft target's zero lane
    # against an underflowing log-probability adds 0, never 0 * -inf
    t = Tape()
    loss = neural.cross_entropy(t.leaf(tensor((1, 2), [-3.0e38, 3.0e38])),
                                t.input(tensor((1, 2), [0.0, 1.0])))
    assert run(t, [loss])[loss.index] == 0.0


def test_log_sum_exp_known_answers(built):
    # function/tests/log_sum_exp_tests.rs:6-16, 31-40 (f32), 42-60, 62-75
    t = Tape()
    x = t.parameter(tensor([1, 3], [1.0, 2.0, 3.0]))
    lse = x.logsumexp(1)
    (g,) = t.differentiate((lse * t.leaf(filled([1], 2.0))).sum(), [x])
    out = run(t, [lse, g])
    z = math.exp(1) + math.exp(2) + math.exp(3)
    assert out[lse.index].shape == (1,)
    assert abs(float(out[lse.index][0]) - math.log(z)) < 1e-6
    assert np.allclose(out[g.index].reshape(-1), [2 * math.exp(v) / z for v in (1, 2, 3)],
                       atol=1e-6)
    for row in ([-3.0e38, 3.0e38], [3.0e38, -3.0e38]):
        t = Tape()
        x = t.parameter(tensor([2], row))
        lse = x.logsumexp(0)
        (g,) = t.differentiate(lse, [x])
        out = run(t, [lse, g])
        value = float(out[lse.index])
        assert math.isfinite(value) and abs(value - 3.0e38) < 3.0e31
        grad = out[g.index].tolist()
        winner = row.index(3.0e38)
        assert grad[1 - winner] == 0.0 and abs(grad[winner] - 1.0) < 1e-6


def test_log_softmax_known_answers(built):
    # function/tests/log_softmax_tests.rs:6-17, 19-30, 32-41, 43-68
    t = Tape()
    x = t.parameter(tensor([1, 3], [1.0, 2.0, 3.0]))
    lp = x.log_softmax(1)
    (g,) = t.differentiate((lp * t.leaf(tensor([1, 3], [1.0, 0.0, 0.0]))).sum(), [x])
    out = run(t, [lp, g])
    z = math.log(math.exp(1) + math.exp(2) + math.exp(3))
    assert np.allclose(out[lp.index].reshape(-1), [1 - z, 2 - z, 3 - z], atol=1e-6)
    soft = np.exp(out[lp.index].reshape(-1))
    assert np.allclose(out[g.index].reshape(-1), np.array([1.0, 0.0, 0.0]) - soft, atol=1e-6)
    t = Tape()
    lp = t.leaf(tensor([1, 2], [1000.0, 1000.0])).log_softmax(1)
    assert np.allclose(run(t, [lp])[lp.index], math.log(0.5), atol=1e-6)
    t = Tape()
    lp = t.leaf(tensor([2, 2], [0.0, 5.0, 0.0, -5.0])).log_softmax(0)
    p = np.exp(run(t, [lp])[lp.index].astype(np.float64))
    assert np.allclose(p.sum(axis=0), 1.0, atol=1e-6)
