"""bf16 networks (payload/bf16.rs) in the oracle, pinned on the known answers
of payload/tests/bf16_tests.rs: rounding to nearest with ties to even, each
payload operation rounding its f32 result once, products, reductions and
scatters accumulating in f32 and rounding once, and networks differentiating
in bf16.  The device lowering of bf16 plans rounds every result and load in
the generated kernels; on the device a bf16 plan follows the bf16 oracle
within a few bf16 ulps (the reassociated f32 accumulations may round the
other way), and the emulated programs equal it bitwise
(`tests/test_emulated_programs.py`)."""
import struct

import numpy as np
import pytest

import oracle
from poorgrad_b200.graph import BF16, Tape, filled, selection, tensor
from poorgrad_b200.plan import Request


def bits(x):
    return struct.unpack("<I", struct.pack("<f", float(x)))[0]


def bf(x):
    return float(oracle.round_bf16(np.array([x], np.float32))[0])


def test_every_bit_pattern_round_trips_through_f32(built):
    # bf16_tests.rs:5-23
    patterns = np.arange(1 << 16, dtype=np.uint32) << 16
    values = patterns.view(np.float32)
    back = oracle.round_bf16(values).view(np.uint32)
    nan = np.isnan(values)
    assert np.array_equal(back[~nan], patterns[~nan])
    assert np.all(np.isnan(back[nan].view(np.float32)))


def test_rounding_is_nearest_with_ties_to_even(built):
    # bf16_tests.rs:25-37
    assert bf(1.00390625) == bf(1.0)
    assert bf(1.01171875) == bf(1.015625)
    assert bf(1.006) == bf(1.0078125)


def test_rounding_carries_into_the_extremes(built):
    # bf16_tests.rs:39-50
    f32max = float(np.finfo(np.float32).max)
    assert bf(f32max) == float("inf") and bf(-f32max) == float("-inf")
    assert bits(bf(-0.0)) == 0x80000000 and bits(bf(0.0)) == 0
    assert np.isnan(bf(float("nan")))


def test_counted_is_exact_up_to_256(built):
    # bf16_tests.rs:52-68
    for count in (0, 1, 100, 255, 256):
        assert bf(count) == count
    assert bf(257) == 256.0 and bf(259) == 260.0


def run(t, roots, feeds=None):
    net = t.into_network()
    cols = net.compile(Request(roots))
    return oracle.run(cols, net.parameters(), feeds)


def test_each_operation_rounds_the_f32_result_once(built):
    # bf16_tests.rs:70-78
    t = Tape(BF16)
    one, three, big = (t.leaf(filled((), v)) for v in (1.0, 3.0, 256.0))
    third = one / three
    swamped = big + one
    out = run(t, [third, swamped])
    assert float(out[third.index]) == bf(np.float32(1.0) / np.float32(3.0))
    assert float(out[swamped.index]) == 256.0


def test_matmul_accumulates_in_f32_and_rounds_once(built):
    # bf16_tests.rs:116-143, with a dense and a constant left operand
    t = Tape(BF16)
    right = t.leaf(tensor((3, 1), [256.0, 1.0, 1.0]))
    dense = t.leaf(tensor((1, 3), [1.0, 1.0, 1.0])).matmul(right)
    constant = t.leaf(filled((1, 3), 1.0)).matmul(right)
    left = t.leaf(tensor((1, 3), [256.0, 1.0, 1.0])).matmul(t.leaf(filled((3, 1), 1.0)))
    out = run(t, [dense, constant, left])
    for v in (dense, constant, left):
        assert out[v.index].reshape(-1).tolist() == [258.0]


def test_reductions_accumulate_in_f32(built):
    # bf16_tests.rs:145-155
    t = Tape(BF16)
    values = t.leaf(tensor((3,), [256.0, 1.0, 1.0]))
    rows = t.leaf(tensor((1, 3), [256.0, 1.0, 1.0]))
    total, along = values.sum(), rows.sum_along(1)
    out = run(t, [total, along])
    assert float(out[total.index]) == 258.0
    assert out[along.index].tolist() == [258.0]


def test_scatter_accumulates_duplicate_rows_in_f32(built):
    # bf16_tests.rs:157-167
    t = Tape(BF16)
    g = t.leaf(tensor((3, 1), [256.0, 1.0, 1.0]))
    folded = g.scatter(t.leaf(selection([0, 0, 0], 1)), 1)
    assert run(t, [folded])[folded.index].reshape(-1).tolist() == [258.0]


def test_scalar_networks_differentiate_bf16(built):
    # bf16_tests.rs:169-182
    t = Tape(BF16)
    x = t.parameter(filled((), 1.5))
    loss = x * x
    net = t.into_network()
    cols = net.compile(Request([loss]).backward())
    assert float(oracle.run(cols, net.parameters())[loss.index]) == 2.25
    (g,) = oracle.backward(cols, net.parameters(), loss, [x])
    assert float(g) == 3.0


def test_sources_enter_as_bf16(built):
    # bf16_tests.rs:184-203: narrowing rounds each element once, widening is
    # exact, so a second narrowing changes nothing
    t = Tape(BF16)
    x = t.leaf(tensor((2, 2), [1.0, 0.3, -2.5, 300.0]))
    y = x * x.literal(filled((2, 2), 1.0))
    out = run(t, [y])[y.index].reshape(-1)
    assert out.tolist() == [bf(v) for v in (1.0, 0.3, -2.5, 300.0)]
    assert oracle.round_bf16(out).tobytes() == out.tobytes()


def test_bf16_gradients_track_f32_within_epsilon(built):
    # bf16_tests.rs:205-245
    weights = [0.8, -1.3, 0.4, 2.1]
    xs = [0.5, -1.1, 1.9, 0.7]
    grads = []
    for element in (0, BF16):
        t = Tape(element)
        w = t.parameter(tensor((2, 2), weights))
        loss = t.leaf(tensor((2, 2), xs)).matmul(w).relu().sum()
        net = t.into_network()
        cols = net.compile(Request([loss]).backward())
        grads.append(oracle.backward(cols, net.parameters(), loss, [w])[0].reshape(-1))
    wide, narrow = grads
    eps = 7.8125e-3
    assert np.all(np.abs(narrow - wide) <= eps * (1 + np.abs(wide)))


def test_tensor_networks_differentiate_bf16(built):
    # bf16_tests.rs:247-261
    t = Tape(BF16)
    x = t.parameter(tensor((3,), [-2.0, 0.0, 3.0]))
    loss = x.abs().sum()
    net = t.into_network()
    cols = net.compile(Request([loss]).backward())
    assert float(oracle.run(cols, net.parameters())[loss.index]) == 5.0
    (g,) = oracle.backward(cols, net.parameters(), loss, [x])
    assert g.tolist() == [-1.0, 1.0, 1.0]


def test_recorded_gradients_close_in_bf16(built):
    # the closure contract (differentiate_tests.rs:11-28) holds per element
    # type: recorded bf16 gradients equal the bf16 reverse scan bitwise
    t = Tape(BF16)
    rng = np.random.default_rng(2)
    w = t.parameter(tensor((6, 5), rng.uniform(-1, 1, 30)))
    x = t.leaf(tensor((4, 6), rng.uniform(-1, 1, 24)))
    h = x.matmul(w).tanh()
    loss = (h.log_softmax(1) * h.literal(tensor((4, 5), rng.uniform(0, 1, 20)))).sum()
    (g,) = t.differentiate(loss, [w])
    net = t.into_network()
    cols = net.compile(Request([loss, g]))
    recorded = oracle.run(cols, net.parameters(), read=[g])[g.index]
    (scan,) = oracle.backward(cols, net.parameters(), loss, [w])
    assert recorded.tobytes() == scan.tobytes()
    assert oracle.round_bf16(recorded).tobytes() == recorded.tobytes()


@pytest.mark.gpu
def test_bf16_plans_on_the_device_follow_the_bf16_oracle(device):
    # values and gradients are bf16 numbers and agree with the oracle within
    # a few bf16 ulps of each output's scale
    from poorgrad_b200 import backend
    cols = _mixed_network(BF16)
    params = cols.network.parameters()
    ref = oracle.run(cols, params)
    plan = backend.DevicePlan(cols)
    dp = backend.DeviceParameters(plan, params)
    plan.forward(dp, sync=True)
    for node, r in ref.items():
        if not cols.readable[node]:
            continue
        got = plan.of(node)
        assert oracle.round_bf16(got).tobytes() == got.tobytes()
        scale = max(1.0, float(np.abs(r).max()))
        np.testing.assert_allclose(got, r, rtol=0, atol=2.0 ** -5 * scale)


@pytest.mark.gpu
def test_bf16_training_steps_on_the_device(device):
    # three Adam steps inside the plan's graph, in bf16 (optimizer_rule.h),
    # against the host bf16 restatement fed the oracle's gradients
    from oracle import optim
    from poorgrad_b200 import backend
    cols, wrt, grads = _mixed_network(BF16, detail=True)
    params0 = cols.network.parameters()  # slot order
    plan = backend.DevicePlan(cols)
    dp = backend.DeviceParameters(plan, params0)
    # hyperparameters exact in bf16 (0.999 would round to 1, and 1 - beta2^t to 0)
    b1, b2, eps = 0.875, 1.0 - 2.0 ** -7, 2.0 ** -20
    opt = backend.Optimizer(plan, dp, backend.ADAM, list(zip(wrt, grads)), 1e-2, b1, b2, eps)
    host = optim.Adam(b1, b2, eps, dtype=optim.BF16)
    slots = [cols.nodes[s.index].slot for s in wrt]
    params = [oracle.round_bf16(np.asarray(params0[k], np.float32).reshape(-1)).reshape(s.shape)
              for k, s in zip(slots, wrt)]
    for _ in range(3):
        in_slots = [None] * len(params0)
        for k, p in zip(slots, params):
            in_slots[k] = p
        ref = oracle.run(cols, in_slots, read=grads)
        plan.forward(dp, sync=True)
        params = host.step(params, [ref[g.index] for g in grads], 1e-2)
    for p, k in zip(params, slots):
        got = dp.download(k).reshape(p.shape)
        assert oracle.round_bf16(got.reshape(-1)).tobytes() == got.reshape(-1).tobytes()
        scale = max(1.0, float(np.abs(p).max()))
        np.testing.assert_allclose(got, p, rtol=0, atol=2.0 ** -4 * scale)
    del opt


def _mixed_network(element, detail=False):
    from poorgrad_b200 import neural
    rng = np.random.default_rng(6)
    t = Tape(element)
    x = t.input(tensor((64, 32), rng.uniform(-1, 1, 64 * 32)))
    w = t.parameter(tensor((32, 32), rng.uniform(-0.3, 0.3, 32 * 32)))
    ln = neural.LayerNorm(t, 32)
    h = ln.express(x.matmul(w)).tanh()
    table = t.parameter(tensor((10, 32), rng.uniform(-1, 1, 320)))
    sel = t.input(selection(rng.integers(0, 10, 64).tolist(), 10))
    g = h + table.gather(sel)
    loss = (g.log_softmax(1) * g).sum() + g.logsumexp(1).sum()
    wrt = [w, table] + ln.parameters()
    grads = t.differentiate(loss, wrt)
    cols = t.into_network().compile(Request([loss] + grads))
    return (cols, wrt, grads) if detail else cols


def test_bf16_plans_lower_with_rounding_and_compile(built):
    # the device lowering of a bf16 network: every generated kernel rounds
    # its results (`tb_rb`), log-sum-exp rows keep the two-pass form, and the
    # source compiles for sm_100a; f32 plans carry no rounding
    from poorgrad_b200 import backend
    bf = _mixed_network(BF16)
    text = backend.lower_describe(bf, with_source=True)
    bodies = text.split("extern \"C\" __global__")[1:]
    assert bodies and all("tb_rb(" in b for b in bodies)
    assert "tb_lse_push(" not in "".join(bodies)
    backend.nvrtc_check(bf)
    f32 = backend.lower_describe(_mixed_network(0), with_source=True)
    assert all("tb_rb(" not in b for b in f32.split("extern \"C\" __global__")[1:])
