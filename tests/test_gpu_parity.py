"""Parity of the B200 device program with the CPU oracle, through the C ABI.

Bars (stated per assertion):
  * bit-exact for elementwise groups without transcendentals, views, gather,
    scatter-add and pad/concat;
  * transcendental groups (tanh/exp/ln/pow via CUDA's libm against glibc):
    relative error <= 4e-6 (a few ulp);
  * tree reductions: |dev - ref| <= 1e-6 * sum|terms| + tiny;
  * GEMM (3xTF32): |dev - ref| <= 8 eps sqrt(k) (1 + |ref|)
    (backend/cuda/tests/cuda_tests.rs:141-150).
"""
import math

import numpy as np
import pytest

import oracle
from oracle import optim
from poorgrad_b200 import backend, configs, neural
from poorgrad_b200.graph import Tape, concat, filled, selection, tensor
from poorgrad_b200.plan import Request

pytestmark = pytest.mark.gpu
EPS = np.finfo(np.float32).eps


def both(tape, roots, feeds=None, params=None):
    net = tape.into_network()
    cols = net.compile(Request(roots))
    p = net.parameters() if params is None else params
    ref = oracle.run(cols, p, feeds)
    plan = backend.DevicePlan(cols)
    dp = backend.DeviceParameters(plan, p)
    plan.forward(dp, feeds, sync=True)
    dev = {i: plan.of(i) for i in ref}
    return ref, dev, plan


def rnd(shape, seed, lo=-1.0, hi=1.0):
    rng = np.random.default_rng(seed)
    return rng.uniform(lo, hi, size=shape).astype(np.float32)


def assert_exact(a, b):
    assert a.shape == b.shape
    assert np.array_equal(a, b, equal_nan=True), f"max diff {np.nanmax(np.abs(a - b))}"


def assert_rel(dev, ref, rtol=4e-6, atol=1e-7):
    np.testing.assert_allclose(dev, ref, rtol=rtol, atol=atol)


def assert_gemm(dev, ref, k):
    tol = 8 * EPS * math.sqrt(k) * (1 + np.abs(ref))
    err = np.abs(dev - ref)
    assert np.all(err <= tol), f"worst ratio {np.max(err / tol)}"


# ------------------------------------------------------------ elementwise
@pytest.mark.parametrize("shape", [(7,), (3, 5), (64, 64), (33, 130), (2, 3, 8)])
def test_arithmetic_group_is_bit_exact(device, shape):
    t = Tape()
    x = t.parameter(tensor(shape, rnd(shape, 1)))
    y = t.parameter(tensor(shape, rnd(shape, 2, 0.5, 2.0)))
    z = ((x * y - x / y) + (-x)).maximum(y * x) + x.relu() * x.step(y)
    s = z.sqrt() if False else z
    loss = (s * s).sum()
    gx, gy = t.differentiate(loss, [x, y])
    ref, dev, plan = both(t, [s, gx, gy])
    assert_exact(dev[s.index], ref[s.index])
    assert_exact(dev[gx.index], ref[gx.index])
    assert_exact(dev[gy.index], ref[gy.index])


@pytest.mark.parametrize("op", ["tanh", "exp", "ln", "sqrt"])
def test_transcendental_maps(device, op):
    shape = (129, 67)
    t = Tape()
    lo = 0.1 if op in ("ln", "sqrt") else -4.0
    x = t.parameter(tensor(shape, rnd(shape, 3, lo, 4.0)))
    y = getattr(x, op)()
    loss = y.sum()
    (g,) = t.differentiate(loss, [x])
    ref, dev, _ = both(t, [y, g])
    if op == "sqrt":
        assert_exact(dev[y.index], ref[y.index])
    else:
        assert_rel(dev[y.index], ref[y.index])
    assert_rel(dev[g.index], ref[g.index], rtol=1e-5)


def test_powf_forward_and_gradients(device):
    shape = (31, 17)
    t = Tape()
    b = t.parameter(tensor(shape, rnd(shape, 4, 0.5, 2.0)))
    e = t.parameter(tensor(shape, rnd(shape, 5, -2.0, 2.0)))
    y = b.powf(e)
    gb, ge = t.differentiate(y.sum(), [b, e])
    ref, dev, _ = both(t, [y, gb, ge])
    for n in (y, gb, ge):
        assert_rel(dev[n.index], ref[n.index], rtol=2e-5)


# ------------------------------------------------------------ views and indexing
def test_views_pad_concat_are_bit_exact(device):
    t = Tape()
    x = t.parameter(tensor((4, 6), rnd((4, 6), 6)))
    y = t.parameter(tensor((6, 4), rnd((6, 4), 7)))
    a = x.transpose() * y
    b = x.narrow(1, 2, 3).pad(1, 1, 5)
    c = concat([x.narrow(1, 0, 2), y.transpose().narrow(1, 1, 3)], 1)
    d = x.reshape((2, 12)).permute((1, 0)).reshape((6, 4)) + y
    e = x.unfold(1, 3, 2, 1)
    loss = a.sum() + b.sum() + c.sum() + d.sum() + (e * e).sum()
    gx, gy = t.differentiate(loss, [x, y])
    ref, dev, _ = both(t, [a, b, c, d, e, gx, gy])
    for n in (a, b, c, d, e, gx, gy):
        if n in (gx, gy):
            assert_rel(dev[n.index], ref[n.index], rtol=1e-6, atol=1e-6)
        else:
            assert_exact(dev[n.index], ref[n.index])


def test_gather_and_scatter_known_rows(device):
    # payload/tests/tensor_tests.rs:995-1016 on the device
    t = Tape()
    table = t.parameter(tensor([3, 2], [1, 2, 3, 4, 5, 6]))
    sel = t.input(selection([0, 2, 0], 3))
    gathered = table.gather(sel)
    ones = t.leaf(filled([3, 2], 1.0))
    scattered = ones.scatter(sel, 3)
    ref, dev, _ = both(t, [gathered, scattered])
    assert dev[gathered.index].reshape(-1).tolist() == [1, 2, 5, 6, 1, 2]
    assert dev[scattered.index].reshape(-1).tolist() == [2, 2, 0, 0, 1, 1]


# the last three take the staged long-segment path (64+ sources per target row
# on average): skewed targets, an empty row, chunk and column-slice edges
@pytest.mark.parametrize("count,vocab,width", [(1000, 27, 64), (4097, 300, 5), (20000, 3, 7),
                                               (131072, 27, 64), (60001, 27, 100),
                                               (5000, 40, 33)])
def test_scatter_add_is_serial_order_exact(device, count, vocab, width):
    rng = np.random.default_rng(count)
    idx = rng.integers(0, vocab, count)
    if count > 20000:
        idx = np.minimum(idx, rng.integers(0, vocab, count))  # skewed towards row 0
        idx[idx == 1] = 0  # row 1 receives nothing
    g = rng.standard_normal((count, width)).astype(np.float32)
    t = Tape()
    gp = t.parameter(tensor(g.shape, g))
    sel = t.input(selection(idx, vocab))
    out = gp.scatter(sel, vocab)
    ref, dev, _ = both(t, [out])
    assert_exact(dev[out.index], ref[out.index])
    from poorgrad_b200.abi import load_library
    assert load_library().tbx_segment_error() == 0  # no bounded wait expired


# ------------------------------------------------------------ reductions and row ops
@pytest.mark.parametrize("shape", [(5, 7), (64, 8192), (300, 27), (2, 3, 129)])
def test_reductions(device, shape):
    t = Tape()
    x = t.parameter(tensor(shape, rnd(shape, 8)))
    r = len(shape)
    rows = x.sum_along(r - 1)
    cols = x.sum_along(0)
    total = x.sum()
    lse = x.logsumexp(r - 1)
    ls = x.log_softmax(r - 1)
    ref, dev, _ = both(t, [rows, cols, total, lse, ls])
    mag = np.abs(ref[ls.index]).max() + 1
    for n in (rows, cols, total):
        np.testing.assert_allclose(dev[n.index], ref[n.index], rtol=1e-5,
                                   atol=1e-6 * shape[-1] * 2)
    assert_rel(dev[lse.index], ref[lse.index], rtol=1e-5, atol=1e-6)
    assert_rel(dev[ls.index], ref[ls.index], rtol=1e-5, atol=1e-6 * mag)


def test_layer_norm_forward_and_gradients(device):
    t = Tape()
    x = t.parameter(tensor((40, 96), rnd((40, 96), 9, -3, 3)))
    ln = neural.LayerNorm(t, 96)
    y = ln.express(x)
    w = t.leaf(tensor((40, 96), rnd((40, 96), 10)))
    loss = (y * w).sum()
    grads = t.differentiate(loss, [x] + ln.parameters())
    ref, dev, _ = both(t, [y] + grads)
    for n in [y] + grads:
        np.testing.assert_allclose(dev[n.index], ref[n.index], rtol=2e-4, atol=2e-5)


def test_rms_norm_forward_and_gradients(device):
    # neural/rms_norm.rs:89-114 on a [48, 4100] input (a team of threads per row)
    t = Tape()
    x = t.parameter(tensor((48, 4100), rnd((48, 4100), 11, -3, 3)))
    rms = neural.RmsNorm(t, 4100, scale=rnd((4100,), 12, 0.5, 1.5))
    y = rms.express(x)
    w = t.leaf(tensor((48, 4100), rnd((48, 4100), 13)))
    loss = (y * w).sum()
    grads = t.differentiate(loss, [x] + rms.parameters())
    ref, dev, _ = both(t, [y] + grads)
    for n in [y] + grads:
        np.testing.assert_allclose(dev[n.index], ref[n.index], rtol=2e-4, atol=2e-5)


# ------------------------------------------------------------ GEMM
GRID = [(2, 3, 4), (5, 7, 3), (17, 33, 9), (64, 64, 64), (2, 64, 128), (129, 65, 257)]


@pytest.mark.parametrize("m,k,n", GRID)
@pytest.mark.parametrize("form", ["contiguous", "transposed", "narrowed"])
def test_gemm_shape_grid(device, m, k, n, form):
    # backend/cuda/tests/cuda_tests.rs:54-201: shape grid x stride forms
    t = Tape()
    if form == "contiguous":
        a = t.parameter(tensor((m, k), rnd((m, k), m)))
        b = t.parameter(tensor((k, n), rnd((k, n), n)))
        A, B = a, b
    elif form == "transposed":
        a = t.parameter(tensor((k, m), rnd((k, m), m)))
        b = t.parameter(tensor((n, k), rnd((n, k), n)))
        A, B = a.transpose(), b.transpose()
    else:
        a = t.parameter(tensor((m, k + 3), rnd((m, k + 3), m)))
        b = t.parameter(tensor((k, n + 2), rnd((k, n + 2), n)))
        A, B = a.narrow(1, 2, k), b.narrow(1, 1, n)
    c = A.matmul(B)
    ref, dev, _ = both(t, [c])
    assert_gemm(dev[c.index], ref[c.index], k)


def test_batched_gemm_and_gradients(device):
    t = Tape()
    a = t.parameter(tensor((3, 2, 20, 12), rnd((3, 2, 20, 12), 11)))
    b = t.parameter(tensor((3, 2, 12, 9), rnd((3, 2, 12, 9), 12)))
    c = a.matmul(b)
    ga, gb = t.differentiate((c * c).sum(), [a, b])
    ref, dev, _ = both(t, [c, ga, gb])
    assert_gemm(dev[c.index], ref[c.index], 12)
    np.testing.assert_allclose(dev[ga.index], ref[ga.index], rtol=1e-5, atol=1e-4)
    np.testing.assert_allclose(dev[gb.index], ref[gb.index], rtol=1e-5, atol=1e-4)


def test_repeated_runs_are_bitwise_identical(device):
    # backend/cuda/tests/cuda_tests.rs:241-257
    w = configs.fused(rows=96, cols=256)
    plan = backend.DevicePlan(w.columns)
    dp = backend.DeviceParameters(plan, w.network.parameters())
    outs = []
    for _ in range(3):
        plan.forward(dp, sync=True)
        outs.append([plan.of(g).copy() for g in w.grads])
    for o in outs[1:]:
        for x, y in zip(outs[0], o):
            assert x.tobytes() == y.tobytes()


# ------------------------------------------------------------ configs at test sizes
def _config_parity(w, feeds, rtol, atol):
    params = w.network.parameters()
    ref = oracle.run(w.columns, params, feeds)
    plan = backend.DevicePlan(w.columns)
    dp = backend.DeviceParameters(plan, params)
    plan.forward(dp, feeds, sync=True)
    for i, r in ref.items():
        d = plan.of(i)
        scale = np.abs(r).max() + 1e-30
        np.testing.assert_allclose(d, r, rtol=rtol, atol=atol * scale)
    return plan, dp


def test_c2_fused_microbench_small(device):
    w = configs.fused(rows=64, cols=520)
    _config_parity(w, {}, rtol=2e-5, atol=1e-5)


def test_c1_mlp_step_matches_oracle(device):
    w = configs.mlp(batch=128)
    feeds = w.feeds(0)
    _config_parity(w, feeds, rtol=1e-4, atol=2e-5)


def test_c4_char_mlp_small(device):
    w = configs.char_mlp(batch=256)
    _config_parity(w, w.feeds(0), rtol=1e-3, atol=1e-4)


def test_c5_gpt2_tiny(device):
    w = configs.gpt2(batch=2, seq=16, layers=2, d=32, heads=4, vocab=50, mlp=64)
    _config_parity(w, w.feeds(0), rtol=1e-3, atol=1e-4)


def test_c5_gpt2_with_raw_attention_operands(device):
    # 64-wide heads over 64 positions: every attention product reads its
    # operands as raw f32 values and splits them inside the GEMM
    w = configs.gpt2(batch=1, seq=64, layers=1, d=128, heads=2, vocab=50, mlp=256)
    assert ":raw" in backend.lower_describe(w.columns)
    _config_parity(w, w.feeds(0), rtol=1e-3, atol=1e-4)


def test_sgd_step_matches_the_reference_rule(device):
    w = configs.mlp(batch=128)
    feeds = w.feeds(0)
    params = w.network.parameters()
    ref = oracle.run(w.columns, params, feeds)
    plan = backend.DevicePlan(w.columns)
    dp = backend.DeviceParameters(plan, params)
    # first run without the optimizer to read this step's gradients
    plan.forward(dp, feeds, sync=True)
    grads = [plan.of(g) for g in w.grads]
    opt = backend.Optimizer(plan, dp, backend.SGD, zip(w.params, w.grads), 0.1)
    plan.forward(dp, feeds, sync=True)
    for p, g, sym in zip(params, grads, w.params):
        slot = w.columns.nodes[sym.index].slot
        expect = (p.reshape(g.shape) - g * np.float32(0.1)).astype(np.float32)
        assert_exact(dp.download(slot).reshape(g.shape), expect)


def test_adam_and_adamw_steps_match_the_reference_rule(device):
    w = configs.char_mlp(batch=128)
    feeds = w.feeds(0)
    params = w.network.parameters()
    for kind in (backend.ADAM, backend.ADAMW):
        plan = backend.DevicePlan(w.columns)
        dp = backend.DeviceParameters(plan, params)
        plan.forward(dp, feeds, sync=True)
        grads = [plan.of(g) for g in w.grads]
        opt = backend.Optimizer(plan, dp, kind, zip(w.params, w.grads), 1e-3, 0.9, 0.999, 1e-8,
                                decay=0.1)
        plan.forward(dp, feeds, sync=True)
        host = (optim.Adam(0.9, 0.999, 1e-8) if kind == backend.ADAM
                else optim.AdamW(0.9, 0.999, 1e-8, 0.1))
        expect = host.step([p.reshape(g.shape) for p, g in zip(params, grads)], grads, 1e-3)
        for e, sym in zip(expect, w.params):
            slot = w.columns.nodes[sym.index].slot
            assert_exact(dp.download(slot).reshape(e.shape), e)


@pytest.mark.parametrize("op,lo", [(9, -10.0), (10, 1e-3), (27, 0.0), (8, -5.0)])
def test_map_face_matches_libm(device, op, lo):
    # the `Elementary::map` face (payload/elementary.rs:89-95): exp, ln, sqrt, tanh
    import ctypes as C
    from poorgrad_b200.abi import fptr, load_library
    lib = load_library()
    x = np.random.default_rng(op).uniform(lo, 10.0, 1 << 18).astype(np.float32)
    out = np.empty_like(x)
    assert lib.tb_map_f32(op, fptr(x), x.size, fptr(out)) == 0
    ref = oracle.libm_map(op, x)
    if op == 27:
        assert_exact(out, ref)
    else:
        np.testing.assert_allclose(out, ref, rtol=4e-7, atol=1e-30)
    small = np.ones(16, np.float32)
    assert lib.tb_map_f32(op, fptr(small), 16, fptr(small)) == 5  # declined below 2^17


def test_standalone_optimizer_step_matches_the_reference_rule(device):
    # Parameters::step(&gradients, &mut optimizer) called by the caller
    # (graph/parameters.rs:90-146): once with the plan's own gradients, once
    # with caller-given device gradients (twice the plan's)
    import torch
    w = configs.mlp(batch=128)
    feeds = w.feeds(0)
    params = w.network.parameters()
    plan = backend.DevicePlan(w.columns)
    dp = backend.DeviceParameters(plan, params)
    opt = backend.Optimizer(plan, dp, backend.SGD, zip(w.params, w.grads), 0.1, attach=False)
    plan.forward(dp, feeds, sync=True)
    grads = [plan.of(g) for g in w.grads]
    opt.step()
    torch.cuda.synchronize()
    slots = [w.columns.nodes[p.index].slot for p in w.params]
    stepped = neural.sgd_reference([p.reshape(g.shape) for p, g in zip(params, grads)], grads, 0.1)
    for s, e in zip(slots, stepped):
        assert_exact(dp.download(s).reshape(e.shape), e)
    doubled = [torch.from_numpy(g * np.float32(2)).cuda() for g in grads]
    opt.step([d.data_ptr() for d in doubled])
    torch.cuda.synchronize()
    again = neural.sgd_reference(stepped, [g * np.float32(2) for g in grads], 0.1)
    for s, e in zip(slots, again):
        assert_exact(dp.download(s).reshape(e.shape), e)


def test_conv_pool_network_forward_and_gradients(device):
    # the mnist/cifar-style stack of the reference's examples: conv2d
    # (neural/convolution.rs:53-131: pad, unfolds, im2col GEMM), relu,
    # max_pool (neural/pooling.rs:49-61), linear head, cross-entropy
    t = Tape()
    rng = np.random.default_rng(21)
    x = t.input(tensor((8, 3, 16, 16), rng.uniform(-1, 1, (8, 3, 16, 16)).astype(np.float32)))
    y = t.input(selection(rng.integers(0, 10, 8), 10))
    w = t.parameter(tensor((8, 3, 3, 3), rng.uniform(-0.3, 0.3, (8, 3, 3, 3)).astype(np.float32)))
    b = t.parameter(tensor((8,), np.zeros(8, np.float32)))
    head = neural.Linear(t, rng.uniform(-0.1, 0.1, (8 * 8 * 8, 10)).astype(np.float32),
                         np.zeros(10, np.float32))
    h = neural.max_pool(neural.conv2d(x, w, b, 1, 1).relu(), 2, 2).reshape((8, 8 * 8 * 8))
    loss = neural.cross_entropy(head.express(h), y)
    grads = t.differentiate(loss, [w, b] + head.parameters())
    ref, dev, _ = both(t, [loss] + grads)
    for n in [loss] + grads:
        scale = np.abs(ref[n.index]).max() + 1e-30
        np.testing.assert_allclose(dev[n.index], ref[n.index], rtol=1e-3, atol=1e-4 * scale)


def test_batch_norm_face_is_bitwise_the_recorded_formula(device):
    # the `Elementary::batch_norm` face against the recorded formula
    # (payload/tensorial.rs:240-258) run by the oracle
    from poorgrad_b200.abi import fptr, load_library
    lib = load_library()
    batch, features = 512, 300
    rng = np.random.default_rng(31)
    x = rng.normal(0.5, 2.0, (batch, features)).astype(np.float32)
    scale = rng.uniform(0.5, 1.5, features).astype(np.float32)
    shift = rng.uniform(-1, 1, features).astype(np.float32)
    t = Tape()
    xv = t.leaf(tensor(x.shape, x))
    bn = neural.BatchNorm(t, features, 1e-5, scale, shift)
    out, mean, var = bn.express(xv)
    net = t.into_network()
    ref = oracle.run(net.compile(Request([out, mean, var])), net.parameters())
    o = np.empty_like(x)
    m = np.empty(features, np.float32)
    v = np.empty(features, np.float32)
    assert lib.tb_batch_norm_f32(fptr(x), fptr(scale), fptr(shift), np.float32(1e-5), batch,
                                 features, fptr(o), fptr(m), fptr(v)) == 0
    assert_exact(m, ref[mean.index].reshape(-1))
    assert_exact(v, ref[var.index].reshape(-1))
    assert_exact(o, ref[out.index].reshape(x.shape))
    small = np.zeros((4, 4), np.float32)  # below the size threshold: declined (TB_DECLINED)
    assert lib.tb_batch_norm_f32(fptr(small), fptr(scale), fptr(shift), np.float32(1e-5), 4, 4,
                                 fptr(small), fptr(m), fptr(v)) == 5


@pytest.mark.parametrize("row,cls", [([1000.0, -1000.0], 0), ([-3.0e38, 3.0e38], 1),
                                     ([3.0e38, -3.0e38], 0)])
def test_cross_entropy_edge_rows(device, row, cls):
    # neural/tests/loss_tests.rs:21-133 on the device, one row per plan as
    # there: a confidently correct or extreme finite row costs exactly 0 and
    # its gradient stays finite (in f32 two such rows in one batch would
    # overflow the loss's own sums, in the interpreter as well)
    t = Tape()
    logits = t.parameter(tensor((1, 2), row))
    loss = neural.cross_entropy(logits, t.input(selection([cls], 2)))
    (g,) = t.differentiate(loss, [logits])
    ref, dev, _ = both(t, [loss, g])
    assert dev[loss.index] == 0.0 and ref[loss.index] == 0.0
    assert np.all(np.isfinite(dev[g.index]))
    np.testing.assert_allclose(dev[g.index], ref[g.index], rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("row", [[-3.0e38, 3.0e38], [3.0e38, -3.0e38], [1000.0, 1000.0],
                                 [1.0, 2.0, 3.0]])
def test_log_sum_exp_and_log_softmax_extreme_rows(device, row):
    # function/tests/log_sum_exp_tests.rs:18-40, 62-75 and
    # log_softmax_tests.rs:19-30 on the device: a finite row whose
    # differences overflow keeps a finite normalizer, the losing lane's
    # gradient is exactly zero and the winner's is one
    t = Tape()
    x = t.parameter(tensor((1, len(row)), row))
    lse = x.logsumexp(1)
    lp = x.log_softmax(1)
    (g,) = t.differentiate(lse.sum(), [x])
    ref, dev, _ = both(t, [lse, lp, g])
    assert np.all(np.isfinite(dev[lse.index]))
    assert_rel(dev[lse.index], ref[lse.index])
    assert_rel(dev[lp.index], ref[lp.index])
    assert np.all(np.isfinite(dev[g.index]))
    assert_rel(dev[g.index], ref[g.index])
    if abs(row[0]) == 3.0e38:
        assert set(dev[g.index].reshape(-1).tolist()) == {0.0, 1.0}


def test_async_read_equals_the_waiting_read(device):
    # `Run::of` without waiting: the copy is enqueued behind the step, and a
    # later run does not change the copy already enqueued
    import torch
    w = configs.mlp(batch=128)
    plan = backend.DevicePlan(w.columns)
    dp = backend.DeviceParameters(plan, w.network.parameters())
    pinned = [torch.zeros((), dtype=torch.float32).pin_memory() for _ in range(2)]
    plan.forward(dp, w.feeds(0))
    plan.read_async(w.loss, pinned[0].data_ptr(), 1)
    plan.forward(dp, w.feeds(1))
    plan.read_async(w.loss, pinned[1].data_ptr(), 1)
    plan.synchronize()
    second = plan.of(w.loss)
    plan.forward(dp, w.feeds(0), sync=True)
    first = plan.of(w.loss)
    assert pinned[0].numpy().tobytes() == first.tobytes()
    assert pinned[1].numpy().tobytes() == second.tobytes()
