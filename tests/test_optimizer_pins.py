"""Pins the host optimizer restatement (``oracle/optim.py``), which the device
optimizer tests check against, on the known answers of the reference's own
optimizer tests.  Gradients come from recorded plans run by the f32 oracle,
the compiled-training route of neural/tests/adam_tests.rs:150-193."""
import numpy as np

import oracle
from oracle import optim
from poorgrad_b200.graph import Tape, tensor
from poorgrad_b200.plan import Request


class Model:
    """A recorded loss and its gradients, run by the oracle."""

    def __init__(self, build):
        t = Tape()
        self.loss, self.params = build(t)
        self.grads = t.differentiate(self.loss, self.params)
        net = t.into_network()
        self.columns = net.compile(Request([self.loss] + self.grads))
        self.initial = [np.asarray(p, np.float32).reshape(w.shape)
                        for p, w in zip(net.parameters(), self.params)]

    def __call__(self, parameters):
        out = oracle.run(self.columns, parameters, read=[self.loss] + self.grads)
        return float(out[self.loss.index]), [out[g.index] for g in self.grads]


def square(values):
    def build(t):
        w = t.parameter(tensor(np.shape(values), np.asarray(values, float).reshape(-1)))
        return (w * w).sum(), [w]
    return Model(build)


def affine_bowl(x_shape, x_values, w_values, b_values):
    # (x @ w + b)^2 summed: neural/tests/optimizer_tests.rs:3-13
    def build(t):
        w = t.parameter(tensor((2, 2), w_values))
        b = t.parameter(tensor((2,), b_values))
        x = t.leaf(tensor(x_shape, x_values))
        p = x.matmul(w)
        s = p + b.broadcast_along(0, p)
        return (s * s).sum(), [w, b]
    return Model(build)


def test_two_adam_steps_match_the_paper_trace():
    # neural/tests/adam_tests.rs:14-50: loss = w*w from w = 1, rate 0.1
    expected, m, v, p1, p2 = 1.0, 0.0, 0.0, 1.0, 1.0
    exact = optim.Adam(dtype=np.float64)
    params64 = [np.array(1.0)]
    model = square(1.0)
    adam32 = optim.Adam()
    params32 = [p.astype(np.float32) for p in model.initial]
    for _ in range(2):
        g = 2.0 * expected
        m = m * 0.9 + g * (1 - 0.9)
        v = v * 0.999 + g * g * (1 - 0.999)
        p1 *= 0.9
        p2 *= 0.999
        expected -= 0.1 * (m / (1 - p1)) / (np.sqrt(v / (1 - p2)) + 1e-8)
        params64 = exact.step(params64, [2.0 * params64[0]], 0.1)
        assert abs(float(params64[0]) - expected) < 1e-12
        _, grads = model(params32)
        params32 = adam32.step(params32, grads, 0.1)
        assert abs(float(params32[0].reshape(())) - expected) < 1e-6


def test_sgd_is_the_hand_written_rule_bitwise():
    # neural/tests/optimizer_tests.rs:15-39
    model = affine_bowl((3, 2), [1.0, 2.0, -1.0, 0.5, 0.25, -2.0],
                        [0.5, -0.25, 1.0, 0.75], [0.1, -0.2])
    params = model.initial
    _, grads = model(params)
    stepped = optim.Sgd().step(params, grads, 0.05)
    for p, g, s in zip(params, grads, stepped):
        hand = (p - g.reshape(p.shape) * np.float32(0.05)).astype(np.float32)
        assert hand.tobytes() == s.tobytes()


def test_adamw_decays_weights_and_spares_biases():
    # neural/tests/adam_tests.rs:77-114
    model = affine_bowl((1, 2), [1.0, -1.0], [1.0, -0.5, 0.25, 2.0], [0.5, -1.0])
    params = [p.astype(np.float64) for p in model.initial]
    _, grads = model(model.initial)
    grads = [g.astype(np.float64) for g in grads]
    by_adam = optim.Adam(dtype=np.float64).step(params, grads, 0.05)
    by_adamw = optim.AdamW(decay=0.1, dtype=np.float64).step(params, grads, 0.05)
    assert by_adam[1].tobytes() == by_adamw[1].tobytes()
    term = params[0] * 0.1 * 0.05
    assert np.all(np.abs(by_adam[0] - by_adamw[0] - term) < 1e-15)


def test_adamw_with_a_policy_that_decays_nothing_is_adam_bitwise():
    # neural/tests/adam_tests.rs:116-148
    model = square([[1.0, -0.5], [0.25, 2.0]])
    params = model.initial
    _, grads = model(params)
    by_adam = optim.Adam().step(params, grads, 0.05)
    spared = optim.AdamW(decay=0.1).step_where(params, grads, 0.05, lambda *_: False)
    assert by_adam[0].tobytes() == spared[0].tobytes()


def test_identical_adam_runs_are_bitwise_identical():
    # neural/tests/adam_tests.rs:52-75
    def trajectory():
        model = square([[1.0, -0.5], [0.25, 2.0]])
        adam, params = optim.Adam(), model.initial
        for _ in range(5):
            _, grads = model(params)
            params = adam.step(params, grads, 0.05)
        return params[0].tobytes()
    assert trajectory() == trajectory()


def test_every_strategy_descends():
    # neural/tests/optimizer_tests.rs:41-80: 25 steps at rate 0.01
    model = affine_bowl((3, 2), [1.0, 2.0, -1.0, 0.5, 0.25, -2.0],
                        [0.5, -0.25, 1.0, 0.75], [0.1, -0.2])
    for strategy in (optim.Sgd(), optim.Adam(), optim.AdamW(decay=0.01)):
        params, first = model.initial, None
        for _ in range(25):
            loss, grads = model(params)
            first = loss if first is None else first
            params = strategy.step(params, grads, 0.01)
        last, _ = model(params)
        assert np.isfinite(last) and last < first, (type(strategy).__name__, first, last)


def test_adam_beats_sgd_on_a_skewed_bowl():
    # neural/tests/adam_tests.rs:195-224: curvatures 100 and 0.01, 100 steps
    def build(t):
        w = t.parameter(tensor((2,), [5.0, 5.0]))
        c = t.leaf(tensor((2,), [100.0, 0.01]))
        return (w * w * c).sum(), [w]
    model = Model(build)

    def final(strategy):
        params = model.initial
        for _ in range(100):
            _, grads = model(params)
            params = strategy.step(params, grads, 0.01)
        return model(params)[0]

    sgd, adam = final(optim.Sgd()), final(optim.Adam())
    assert np.isfinite(sgd) and np.isfinite(adam)
    assert adam < sgd, (adam, sgd)
