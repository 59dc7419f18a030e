"""The derivative rules of the host mirror (`Tape::differentiate`,
graph/tape.rs:335-410, and each `Function::backward`) against central finite
differences, in the manner of engine/tests/run_tests.rs:49-160.  Each case is
written twice: on the tape (differentiated, then run by the f32 oracle) and in
numpy float64 (differenced numerically).  The bar is relative 2e-3: the
analytic side is f32."""
import numpy as np

import oracle
from poorgrad_b200 import neural
from poorgrad_b200.graph import Tape, selection, tensor
from poorgrad_b200.plan import Request

STEP = 1e-5


def check(values, graph_fn, numpy_fn, tol=2e-3):
    t = Tape()
    xs = [t.parameter(tensor(np.shape(v), np.asarray(v, np.float32).reshape(-1))) for v in values]
    y = graph_fn(*xs)
    if len(y.shape) > 0:
        y = y.sum()
    grads = t.differentiate(y, xs)
    net = t.into_network()
    out = oracle.run(net.compile(Request(grads)), net.parameters())
    base = [np.asarray(v, np.float64) for v in values]

    def f(vs):
        return float(np.sum(numpy_fn(*vs)))

    for i, g in enumerate(grads):
        analytic = out[g.index].reshape(-1).astype(np.float64)
        for pos in range(base[i].size):
            up = [b.copy() for b in base]
            down = [b.copy() for b in base]
            up[i].reshape(-1)[pos] += STEP
            down[i].reshape(-1)[pos] -= STEP
            numeric = (f(up) - f(down)) / (2 * STEP)
            assert abs(analytic[pos] - numeric) <= tol * (1 + abs(numeric)), \
                f"input {i} element {pos}: analytic {analytic[pos]}, numeric {numeric}"


def test_arithmetic():
    # run_tests.rs:48-56
    check([2.0, 3.0], lambda a, b: a + b, lambda a, b: a + b)
    check([2.0, 3.0], lambda a, b: a - b, lambda a, b: a - b)
    check([2.0, 3.0], lambda a, b: a * b, lambda a, b: a * b)
    check([2.0, 3.0], lambda a, b: a / b, lambda a, b: a / b)
    check([2.0], lambda a: -a, lambda a: -a)
    check([2.0, 3.0], lambda a, b: a * b + a - b / a, lambda a, b: a * b + a - b / a)


def test_transcendentals():
    # run_tests.rs:58-64
    check([0.5], lambda a: a.tanh(), np.tanh)
    check([0.8], lambda a: a.exp(), np.exp)
    check([1.7], lambda a: a.ln(), np.log)
    check([0.3, 1.2], lambda a, b: ((a * b).exp() + a.tanh()).ln(),
          lambda a, b: np.log(np.exp(a * b) + np.tanh(a)))
    check([2.5], lambda a: a.sqrt(), np.sqrt)
    check([1.3, 2.2], lambda a, b: a.powf(b), lambda a, b: a ** b)


def test_fan_out():
    # run_tests.rs:66-72: accumulation over several consumers
    def g(a):
        sq = a * a
        return sq * sq + sq + a
    check([1.5], g, g)


def test_dense_layer():
    # run_tests.rs:87-155: matmul, axis-wise bias broadcast, tanh, squared error
    x = np.array([[0.5, -1.0, 0.25], [1.5, 0.75, -0.5]])
    w = np.array([[1.0, 0.5], [-0.75, 0.25], [0.5, 1.25]])
    b = np.array([0.35, -0.15])
    y = np.array([[0.6, -0.5], [0.25, 0.75]])

    def graph(x, w, b, y):
        p = x.matmul(w)
        e = (p + b.broadcast_along(0, p)).tanh() - y
        return (e * e).sum()

    def ref(x, w, b, y):
        e = np.tanh(x @ w + b[None, :]) - y
        return np.sum(e * e)

    check([x, w, b, y], graph, ref)


def test_views_and_row_functions():
    x = np.array([[0.5, -1.0, 0.25, 2.0], [1.5, 0.75, -0.5, 0.1], [0.3, 0.2, -0.7, 1.1]])
    wts = np.linspace(-1, 1, 12).reshape(3, 4)

    def lsm(v):
        m = v.max(axis=1, keepdims=True)
        return v - m - np.log(np.exp(v - m).sum(axis=1, keepdims=True))

    check([x], lambda v: v.log_softmax(1) * v.literal(tensor((3, 4), wts.reshape(-1))),
          lambda v: lsm(v) * wts)
    check([x], lambda v: v.logsumexp(1), lambda v: np.log(np.exp(v).sum(axis=1)))
    check([x], lambda v: v.relu() * v, lambda v: np.maximum(v, 0) * v)
    check([x], lambda v: v.transpose().sum_along(0), lambda v: v.T.sum(axis=0))
    check([x], lambda v: v.narrow(1, 1, 2).exp(), lambda v: np.exp(v[:, 1:3]))
    check([x], lambda v: v.pad(1, 2, 7).tanh(), lambda v: np.tanh(v))
    check([x], lambda v: v.permute([1, 0]).reshape((2, 6)).tanh() * v.literal(
        tensor((2, 6), wts.reshape(-1))), lambda v: np.tanh(v.T.reshape(2, 6)) * wts.reshape(2, 6))
    check([x], lambda v: v.broadcast_along(0, v.literal(tensor((2, 3, 4), np.ones(24)))).tanh(),
          lambda v: np.tanh(np.broadcast_to(v, (2, 3, 4))))


def test_gather_and_scatter():
    table = np.array([[0.5, -1.0], [0.25, 2.0], [1.5, 0.75]])
    idx = [2, 0, 2, 1]
    check([table], lambda t_: (t_.gather(t_.literal(selection(idx, 3))).tanh()),
          lambda t_: np.tanh(t_[idx]))
    g = np.array([[0.5, -1.0], [0.25, 2.0], [1.5, 0.75], [0.1, 0.2]])

    def scattered(v):
        out = np.zeros((3, 2))
        for r, i in enumerate(idx):
            out[i] = out[i] + v[r]
        return np.tanh(out)

    check([g], lambda v: v.scatter(v.literal(selection(idx, 3)), 3).tanh(), scattered)


def test_convolution_and_pooling():
    rng = np.random.default_rng(5)
    x = rng.uniform(-1, 1, (1, 2, 5, 5))
    w = rng.uniform(-1, 1, (3, 2, 3, 3))
    b = rng.uniform(-1, 1, 3)

    def conv_ref(x, w, b):
        xp = np.pad(x, ((0, 0), (0, 0), (1, 1), (1, 1)))
        out = np.zeros((1, 3, 5, 5))
        for f in range(3):
            for i in range(5):
                for j in range(5):
                    out[0, f, i, j] = np.sum(xp[0, :, i:i + 3, j:j + 3] * w[f]) + b[f]
        return np.tanh(out)

    check([x, w, b], lambda x_, w_, b_: neural.conv2d(x_, w_, b_, 1, 1).tanh(), conv_ref)

    def pool_ref(x):  # 2x2 windows, stride 2
        return x.reshape(1, 2, 2, 2, 2, 2).max(axis=(3, 5))

    check([x[:, :, :4, :4]], lambda v: neural.max_pool(v, 2, 2), pool_ref)
