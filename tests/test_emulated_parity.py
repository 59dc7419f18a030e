"""Device-parity cases run through the kernel emulator on the host: the same
kinds of graphs the GPU parity tests run (bit-exact elementwise groups and
views, serial-order scatter-add, reductions of odd shapes, LayerNorm and
RMSNorm with their gradients, a conv/pool network, extreme cross-entropy and
log-sum-exp rows), checked against the oracle without a GPU.  Elementwise and
index work is bit-exact here as on the device; the emulator's transcendentals
are the host's, so their agreement says nothing about CUDA's and is not
asserted bitwise."""
import math

import numpy as np
import pytest

import kernel_emulator
import oracle
from poorgrad_b200 import neural
from poorgrad_b200.graph import Tape, concat, selection, tensor
from poorgrad_b200.plan import Request


def both(t, roots, feeds=None):
    net = t.into_network()
    cols = net.compile(Request(roots))
    params = net.parameters()
    return oracle.run(cols, params, feeds), kernel_emulator.run_program(cols, params, feeds)


def rnd(shape, seed, lo=-1.0, hi=1.0):
    return np.random.default_rng(seed).uniform(lo, hi, size=shape)


@pytest.mark.parametrize("shape", [(7,), (33, 130), (2, 3, 8)])
def test_arithmetic_groups_are_bit_exact(built, shape):
    t = Tape()
    x = t.parameter(tensor(shape, rnd(shape, 1).reshape(-1)))
    y = t.parameter(tensor(shape, rnd(shape, 2, 0.5, 2.0).reshape(-1)))
    s = ((x * y - x / y) * (x + y)).sum()
    gx, gy = t.differentiate(s, [x, y])
    ref, emu = both(t, [s, gx, gy])
    for v in (gx, gy):
        assert emu[v.index].tobytes() == ref[v.index].tobytes()


def test_views_pad_and_concat_are_bit_exact(built):
    t = Tape()
    x = t.parameter(tensor((6, 10), rnd((6, 10), 3).reshape(-1)))
    parts = [x.narrow(1, 0, 4), x.narrow(1, 4, 6).permute([1, 0]).permute([1, 0])]
    joined = concat(parts, 1)
    e = joined.transpose().reshape((5, 12)).unfold(1, 3, 2, 1)
    loss = (e * e).sum()
    (g,) = t.differentiate(loss, [x])
    ref, emu = both(t, [e, g])
    assert emu[e.index].tobytes() == ref[e.index].tobytes()
    assert emu[g.index].tobytes() == ref[g.index].tobytes()


@pytest.mark.parametrize("count,vocab,width", [(1000, 27, 64), (300, 50, 5)])
def test_scatter_add_is_serial_order_exact(built, count, vocab, width):
    rng = np.random.default_rng(count)
    t = Tape()
    rows = t.parameter(tensor((count, width), rng.uniform(-1, 1, count * width)))
    sel = t.input(selection(rng.integers(0, vocab, count).tolist(), vocab))
    out = rows.scatter(sel, vocab)
    ref, emu = both(t, [out])
    assert emu[out.index].tobytes() == ref[out.index].tobytes()


@pytest.mark.parametrize("shape", [(5, 7), (300, 27), (2, 3, 129)])
def test_reductions(built, shape):
    t = Tape()
    x = t.parameter(tensor(shape, rnd(shape, 4).reshape(-1)))
    rows = x.sum_along(len(shape) - 1)
    cols = x.sum_along(0)
    total = x.sum()
    peak = x.logsumexp(len(shape) - 1)
    ref, emu = both(t, [rows, cols, total, peak])
    for v in (rows, cols, total, peak):
        # tree against serial order: the error scales with the output's size
        scale = max(1.0, float(np.abs(ref[v.index]).max()))
        np.testing.assert_allclose(emu[v.index], ref[v.index], rtol=1e-5, atol=1e-5 * scale)


def test_layer_norm_and_rms_norm_with_gradients(built):
    t = Tape()
    x = t.parameter(tensor((48, 64), rnd((48, 64), 5).reshape(-1)))
    ln = neural.LayerNorm(t, 64, scale=rnd(64, 6, 0.5, 1.5), shift=rnd(64, 7))
    rms = neural.RmsNorm(t, 64, scale=rnd(64, 8, 0.5, 1.5))
    y = ln.express(x).tanh() + rms.express(x)
    loss = (y * y).sum()
    grads = t.differentiate(loss, [x] + ln.parameters() + rms.parameters())
    ref, emu = both(t, [loss] + grads)
    for g in grads:
        scale = max(1.0, float(np.abs(ref[g.index]).max()))
        np.testing.assert_allclose(emu[g.index], ref[g.index], rtol=0, atol=1e-5 * scale)


def test_conv_pool_network_with_gradients(built):
    t = Tape()
    x = t.leaf(tensor((2, 2, 8, 8), rnd((2, 2, 8, 8), 9).reshape(-1)))
    w = t.parameter(tensor((4, 2, 3, 3), rnd((4, 2, 3, 3), 10, -0.4, 0.4).reshape(-1)))
    b = t.parameter(tensor((4,), rnd(4, 11, -0.1, 0.1)))
    head = t.parameter(tensor((64, 3), rnd((64, 3), 12, -0.2, 0.2).reshape(-1)))
    pooled = neural.max_pool(neural.conv2d(x, w, b, 1, 1).relu(), 2, 2)
    loss = neural.cross_entropy(pooled.reshape((2, 64)).matmul(head),
                                t.leaf(selection([1, 2], 3)))
    grads = t.differentiate(loss, [w, b, head])
    ref, emu = both(t, [loss] + grads)
    for v in [loss] + grads:
        scale = max(1.0, float(np.abs(ref[v.index]).max()))
        np.testing.assert_allclose(emu[v.index], ref[v.index], rtol=0, atol=3e-5 * scale)


@pytest.mark.parametrize("row,cls", [([1000.0, -1000.0], 0), ([-3.0e38, 3.0e38], 1),
                                     ([3.0e38, -3.0e38], 0)])
def test_cross_entropy_edge_rows(built, row, cls):
    t = Tape()
    logits = t.parameter(tensor((1, 2), row))
    loss = neural.cross_entropy(logits, t.input(selection([cls], 2)))
    (g,) = t.differentiate(loss, [logits])
    ref, emu = both(t, [loss, g])
    assert float(emu[loss.index]) == 0.0 == float(ref[loss.index])
    assert np.all(np.isfinite(emu[g.index]))
    np.testing.assert_allclose(emu[g.index], ref[g.index], rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("row", [[-3.0e38, 3.0e38], [1000.0, 1000.0], [1.0, 2.0, 3.0]])
def test_log_sum_exp_extreme_rows(built, row):
    t = Tape()
    x = t.parameter(tensor((1, len(row)), row))
    lse = x.logsumexp(1)
    (g,) = t.differentiate(lse.sum(), [x])
    ref, emu = both(t, [lse, g])
    assert np.all(np.isfinite(emu[lse.index]))
    np.testing.assert_allclose(emu[lse.index], ref[lse.index], rtol=1e-6)
    np.testing.assert_allclose(emu[g.index], ref[g.index], rtol=1e-6, atol=1e-7)
    assert math.isfinite(float(emu[g.index].sum()))


def test_long_flat_sums_split_into_virtual_rows(built):
    # a one-dimensional group with a full sum (the cross-entropy's batch sum)
    # runs as many 128-wide virtual rows instead of one team over the vector
    t = Tape()
    x = t.parameter(tensor((8192,), rnd((8192,), 21, 0.5, 2.0).reshape(-1)))
    y = t.parameter(tensor((8192,), rnd((8192,), 22).reshape(-1)))
    z = x.ln() + y
    loss = (z * y).sum()
    gx, gy = t.differentiate(loss, [x, y])
    ref, emu = both(t, [loss, z, gx, gy])
    np.testing.assert_allclose(emu[loss.index], ref[loss.index], rtol=1e-5)
    for v in (z, gx, gy):
        np.testing.assert_allclose(emu[v.index], ref[v.index], rtol=4e-6, atol=1e-7)
