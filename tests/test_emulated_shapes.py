"""Shape-dependent code paths of the emitted kernels, run by the kernel
emulator against the oracle: 256-thread teams with cross-warp reductions
(long rows), rows too long to keep phase values in registers, scalar
(`vec = 1`) rows of odd width, the four-stride unrolled flat loop (more than
4 · 1184 · 256 elements), and column sums of wide rows."""
import numpy as np

import kernel_emulator
import oracle
from poorgrad_b200 import neural
from poorgrad_b200.graph import Tape, selection, tensor
from poorgrad_b200.plan import Request


def check(t, roots, grads_of=None, tol=3e-5):
    loss = roots[0]
    grads = t.differentiate(loss, grads_of) if grads_of else []
    net = t.into_network()
    cols = net.compile(Request(list(roots) + grads))
    params = net.parameters()
    ref = oracle.run(cols, params)
    emu = kernel_emulator.run_program(cols, params)
    for v in list(roots) + grads:
        r = ref[v.index]
        scale = max(1.0, float(np.abs(r).max()))
        np.testing.assert_allclose(emu[v.index], r, rtol=0, atol=tol * scale, err_msg=str(v.index))
    return cols


def rnd(shape, seed, lo=-1.0, hi=1.0):
    return np.random.default_rng(seed).uniform(lo, hi, shape).reshape(-1)


def test_long_rows_layer_norm_forward_and_backward(built):
    # [16, 8192]: 256-thread teams, reductions across warps through shared memory
    t = Tape()
    x = t.parameter(tensor((16, 8192), rnd((16, 8192), 1)))
    ln = neural.LayerNorm(t, 8192)
    y = ln.express(x).tanh()
    check(t, [(y * y).sum()], [x] + ln.parameters())


def test_vocabulary_wide_cross_entropy(built):
    # [4, 50257]: scalar lanes, a row too long for register-held phase values
    rng = np.random.default_rng(2)
    t = Tape()
    logits = t.parameter(tensor((4, 50257), rng.normal(0, 2, 4 * 50257)))
    loss = neural.cross_entropy(logits, t.input(selection(rng.integers(0, 50257, 4).tolist(),
                                                          50257)))
    check(t, [loss], [logits])


def test_odd_width_softmax_rows(built):
    t = Tape()
    x = t.parameter(tensor((33, 1001), rnd((33, 1001), 3, -3, 3)))
    p = x.softmax(1)
    w = x.literal(tensor((33, 1001), rnd((33, 1001), 4)))
    check(t, [(p * w).sum()], [x])


def test_flat_groups_past_the_unrolled_threshold(built):
    # 1200 × 1024 elements: more than four grid strides of 1184 blocks
    t = Tape()
    x = t.parameter(tensor((1200, 1024), rnd((1200, 1024), 5)))
    y = t.parameter(tensor((1200, 1024), rnd((1200, 1024), 6, 0.5, 2.0)))
    s = (x * y - x / y).sum()
    check(t, [s], [x, y])


def test_column_sums_of_wide_rows(built):
    # [64, 4096] with column sums: the wide-row block cap
    t = Tape()
    x = t.parameter(tensor((64, 4096), rnd((64, 4096), 7)))
    b = t.parameter(tensor((4096,), rnd(4096, 8)))
    h = (x + b.broadcast_along(0, x)).tanh()
    # the loss sums 262,144 terms: serial against tree order differs by more
    # than the per-element bar
    check(t, [(h * h).sum(), h.sum_along(0)], [x, b], tol=2e-4)
