"""Initializers (neural/init.rs) and the Mlp composition (neural/mlp.rs) of
the host mirror, pinned on the known answers of neural/tests/init_tests.rs
and neural/tests/mlp_tests.rs; the XOR run trains through the oracle."""
import math
import struct

import numpy as np
import pytest

import oracle
from poorgrad_b200 import neural
from poorgrad_b200.graph import Tape, tensor
from poorgrad_b200.plan import Request


def bits64(a):
    return [struct.unpack("<Q", struct.pack("<d", float(v)))[0] for v in np.asarray(a).reshape(-1)]


def bits32(a):
    return [struct.unpack("<I", struct.pack("<f", float(v)))[0] for v in np.asarray(a).reshape(-1)]


def f32_of(b64):
    return [bits32([np.float32(struct.unpack("<d", struct.pack("<Q", b))[0])])[0] for b in b64]


def test_fan_aware_streams_are_pinned(built):
    # init_tests.rs:80-135 (the xavier and kaiming goldens; uniform and
    # normal are pinned in test_oracle_pins)
    xavier = [0xbfd14566a85c9c0a, 0xbff2f01dbe7ab6a2, 0x3fef69c081567c5c, 0x3fca0063d7a5b7aa]
    kaiming = [0x3fefa194ec47d228, 0xbffdd3fde5949e97, 0x3f700ea29c8645d7, 0xbfe0efc91ba890b4]
    assert bits64(neural.xavier(7)((2, 2), f64=True)) == xavier
    assert bits64(neural.kaiming(7)((2, 2), f64=True)) == kaiming
    assert bits32(neural.xavier(7)((2, 2))) == f32_of(xavier)
    assert bits32(neural.kaiming(7)((2, 2))) == f32_of(kaiming)


def moments(values):
    v = np.asarray(values, np.float64).reshape(-1)
    return v.mean(), v.std()


def test_xavier_and_kaiming_bound_and_scale(built):
    # init_tests.rs:49-74
    w = neural.xavier(3)((30, 50), f64=True)
    assert np.all(np.abs(w) <= math.sqrt(6.0 / 80.0))
    assert np.all(neural.xavier(3)((50,)) == 0)
    _, dev = moments(neural.kaiming(3)((200, 100), f64=True))
    assert abs(dev - math.sqrt(2.0 / 200.0)) < 0.005
    assert np.all(neural.kaiming(3)((100,)) == 0)


def test_fan_aware_initializers_reject_other_ranks(built):
    # init_tests.rs:76-79, 162-166
    for init in (neural.xavier(1), neural.kaiming(1), neural.scaled(1, 1.0)):
        with pytest.raises(AssertionError, match="rank-2 weights or rank-1 biases"):
            init((2, 2, 2))


def test_scaled_matches_the_gain_over_the_fan(built):
    # init_tests.rs:136-160
    tanh = neural.Activation(neural.Activation.TANH)
    relu = neural.Activation(neural.Activation.RELU)
    mean, dev = moments(neural.scaled(7, tanh.gain())((400, 25), f64=True))
    assert abs(mean) < 0.01 and abs(dev - (5.0 / 3.0) / 20.0) < 0.005
    assert np.all(neural.scaled(7, tanh.gain())((25,)) == 0)
    _, a = moments(neural.scaled(7, relu.gain())((200, 50), f64=True))
    _, b = moments(neural.kaiming(7)((200, 50), f64=True))
    assert abs(a - b) < 0.005


def test_gains_state_the_standard_factors(built):
    # init_tests.rs:167-171
    assert neural.Activation(neural.Activation.TANH).gain() == 5.0 / 3.0
    assert neural.Activation(neural.Activation.RELU).gain() == math.sqrt(2.0)


def xorshift():
    # mlp_tests.rs:8-21
    state = [np.uint64(0x9E3779B97F4A7C15)]

    def draw(shape):
        out = []
        with np.errstate(over="ignore"):
            for _ in range(int(np.prod(shape))):
                s = state[0]
                s ^= s << np.uint64(13)
                s ^= s >> np.uint64(7)
                s ^= s << np.uint64(17)
                state[0] = s
                out.append(float(s >> np.uint64(11)) / float(1 << 53) - 0.5)
        return np.array(out).reshape(shape)
    return draw


def test_mlp_topology(built):
    # mlp_tests.rs:23-47
    t = Tape()
    mlp = neural.Mlp(t, [3, 4, 4, 1], xorshift())
    assert len(mlp.parameters()) == 6 and len(t) == 6
    with pytest.raises(AssertionError, match="input and an output width"):
        neural.Mlp(Tape(), [3], xorshift())
    t = Tape()
    out = neural.Mlp(t, [3, 4, 2], xorshift()).express(t.leaf(tensor((5, 3), [0.5] * 15)))
    assert out.shape == (5, 2)


def test_mlp_learns_xor(built):
    # mlp_tests.rs:49-83: 2000 SGD steps at rate 0.05 through the oracle
    t = Tape()
    mlp = neural.Mlp(t, [2, 4, 1], xorshift())
    x = t.leaf(tensor((4, 2), [0.0, 0.0, 0.0, 1.0, 1.0, 0.0, 1.0, 1.0]))
    y = t.leaf(tensor((4, 1), [-1.0, 1.0, 1.0, -1.0]))
    predicted = mlp.express(x)
    error = predicted - y
    loss = (error * error).sum()
    params = mlp.parameters()
    grads = t.differentiate(loss, params)
    net = t.into_network()
    cols = net.compile(Request([predicted] + grads))
    state = net.parameters()
    for _ in range(2000):
        out = oracle.run(cols, state, read=grads)
        state = [(p - out[g.index].reshape(-1) * np.float32(0.05)).astype(np.float32)
                 for p, g in zip(state, grads)]
    pred = oracle.run(cols, state, read=[predicted])[predicted.index].reshape(-1)
    assert np.all(np.abs(pred - np.array([-1.0, 1.0, 1.0, -1.0])) < 0.2), pred
