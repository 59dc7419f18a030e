"""Neural compositions recorded on a :class:`~poorgrad_b200.graph.Tape`: the
subset of topos `neural/` the training configs use.  Each records exactly the
formula of its reference, so the plan columns match what topos would compile.

- :class:`Linear` -- `neural/linear.rs:94-105`: ``x.matmul(W) + b.broadcast_along(0, .)``
- :class:`LayerNorm` -- `neural/layer_norm.rs:100-132`
- :func:`gelu` -- the tanh form of `examples/gpt2/model.rs:81-97`
- :func:`cross_entropy` -- `neural/loss.rs:44-63`
- initializers -- `neural/init.rs:50-216` (splitmix64 streams)
"""
from __future__ import annotations

import math
from typing import List

import numpy as np

from .graph import Dense, Tape, Value, counted, filled

GOLDEN = np.uint64(0x9E3779B97F4A7C15)
MIX1 = np.uint64(0xBF58476D1CE4E5B9)
MIX2 = np.uint64(0x94D049BB133111EB)


class Stream:
    """A splitmix64 state advanced once per draw (`init.rs:50-61`)."""

    def __init__(self, seed: int):
        self.state = np.uint64(seed)

    def raw(self, n: int) -> np.ndarray:
        with np.errstate(over="ignore"):
            steps = np.arange(1, n + 1, dtype=np.uint64)
            states = self.state + steps * GOLDEN
            self.state = self.state + np.uint64(n) * GOLDEN
            z = states
            z = (z ^ (z >> np.uint64(30))) * MIX1
            z = (z ^ (z >> np.uint64(27))) * MIX2
            return z ^ (z >> np.uint64(31))

    def unit(self, n: int) -> np.ndarray:
        """`unit`: the top 53 bits over 2^53, in f64."""
        return (self.raw(n) >> np.uint64(11)).astype(np.float64) / float(1 << 53)

    def standard_normal(self, n: int) -> np.ndarray:
        """Box-Muller with two draws per value (`init.rs:67-71`)."""
        u = self.unit(2 * n).reshape(n, 2)
        radius = np.sqrt(-2.0 * np.log(1.0 - u[:, 0]))
        angle = 2.0 * math.pi * u[:, 1]
        return radius * np.cos(angle)


def uniform(seed: int, scale: float):
    """`init::uniform`: ``(2u - 1) * scale``, cast to f32 once."""
    stream = Stream(seed)

    def draw(shape, override=None) -> np.ndarray:
        n = int(np.prod(shape)) if len(shape) else 1
        s = scale if override is None else override
        return ((stream.unit(n) * 2.0 - 1.0) * s).astype(np.float32).reshape(shape)
    return draw


def normal(seed: int, deviation: float):
    """`init::normal`: ``standard_normal * deviation``."""
    stream = Stream(seed)

    def draw(shape) -> np.ndarray:
        n = int(np.prod(shape)) if len(shape) else 1
        return (stream.standard_normal(n) * deviation).astype(np.float32).reshape(shape)
    return draw


def unit_uniform(seed: int):
    """``U[0, 1)`` from the same stream (`unit`)."""
    stream = Stream(seed)

    def draw(shape) -> np.ndarray:
        n = int(np.prod(shape)) if len(shape) else 1
        return stream.unit(n).astype(np.float32).reshape(shape)
    return draw


def dropout(seed: int, keep: float):
    """`init::dropout` (neural/init.rs:119-130): one stream across calls; per
    element ``1 / keep`` where the unit draw is below ``keep``, else 0."""
    assert 0.0 < keep <= 1.0, f"the keep probability must lie within (0, 1], got {keep}"
    stream = Stream(seed)

    def draw(shape) -> np.ndarray:
        n = int(np.prod(shape)) if len(shape) else 1
        return np.where(stream.unit(n) < keep, 1.0 / keep, 0.0).astype(np.float32).reshape(shape)
    return draw


def _fan_initializer(name: str, seed: int, weights):
    """Rank-2 ``[inputs, outputs]`` weights drawn by ``weights(stream, shape)``
    in f64, rank-1 biases zero (`neural/init.rs:145-216`); ``draw(shape,
    f64=True)`` returns the f64 values, the default rounds them once to f32."""
    stream = Stream(seed)

    def draw(shape, f64: bool = False) -> np.ndarray:
        shape = tuple(shape)
        if len(shape) == 1:
            out = np.zeros(shape)
        elif len(shape) == 2:
            out = weights(stream, shape).reshape(shape)
        else:
            raise AssertionError(f"{name} initialization expects rank-2 weights or rank-1 "
                                 f"biases, got {shape}")
        return out if f64 else out.astype(np.float32)
    return draw


def xavier(seed: int):
    """`init::xavier`: uniform within ``±sqrt(6 / (inputs + outputs))``."""
    return _fan_initializer("xavier", seed, lambda st, sh: (st.unit(sh[0] * sh[1]) * 2.0 - 1.0)
                            * math.sqrt(6.0 / float(sh[0] + sh[1])))


def kaiming(seed: int):
    """`init::kaiming`: normal with deviation ``sqrt(2 / inputs)``."""
    return _fan_initializer("kaiming", seed, lambda st, sh: st.standard_normal(sh[0] * sh[1])
                            * math.sqrt(2.0 / float(sh[0])))


def scaled(seed: int, gain: float):
    """`init::scaled`: normal with deviation ``gain / sqrt(inputs)``."""
    return _fan_initializer("scaled", seed, lambda st, sh: st.standard_normal(sh[0] * sh[1])
                            * (gain / math.sqrt(float(sh[0]))))


def integers(seed: int, high: int, n: int) -> np.ndarray:
    """Uniform integers ``0..high`` from one stream: ``floor(unit * high)``."""
    u = Stream(seed).unit(n)
    return np.minimum((u * high).astype(np.int64), high - 1)


class Linear:
    def __init__(self, tape: Tape, weights: np.ndarray, bias: np.ndarray):
        assert weights.ndim == 2 and bias.ndim == 1 and weights.shape[1] == bias.shape[0]
        self.weights = tape.parameter(Dense(weights.shape, weights))
        self.bias = tape.parameter(Dense(bias.shape, bias))

    def parameters(self) -> List[Value]:
        return [self.weights, self.bias]

    def express(self, x: Value) -> Value:
        product = x.matmul(self.weights)
        return product + self.bias.broadcast_along(0, product)

    def visit(self, visitor) -> None:
        # neural/linear.rs:107-110
        visitor.parameter("weights", self.weights)
        visitor.parameter("bias", self.bias)


class Dropout:
    """`neural/dropout.rs`: an input mask of the given shape, all ones until
    fed, multiplied into the expression; a training loop feeds a fresh
    `dropout` mask each step, an unfed run is the identity."""

    def __init__(self, tape: Tape, shape):
        self.mask = tape.input(counted(tuple(shape), 1))

    def express(self, x: Value) -> Value:
        return x * self.mask

    def visit(self, visitor) -> None:
        pass  # a mask input, no parameters


class Activation:
    """`neural/activation.rs:13-61`: a stateless stage, ``tanh`` or ``relu``."""
    TANH, RELU = "tanh", "relu"

    def __init__(self, kind: str):
        assert kind in (self.TANH, self.RELU), kind
        self.kind = kind

    def express(self, x: Value) -> Value:
        return x.tanh() if self.kind == self.TANH else x.relu()

    def gain(self) -> float:
        """`Activation::gain` (activation.rs:31-36)."""
        return 5.0 / 3.0 if self.kind == self.TANH else math.sqrt(2.0)

    def visit(self, visitor) -> None:
        pass


class Sequential:
    """`neural/sequential.rs`: stages applied in order; `visit` announces each
    stage's parameters under its index (`sequential.rs:57-63`)."""

    def __init__(self):
        self.stages = []

    def then(self, stage) -> "Sequential":
        self.stages.append(stage)
        return self

    def __len__(self):
        return len(self.stages)

    def express(self, x: Value) -> Value:
        for stage in self.stages:
            x = stage.express(x)
        return x

    def visit(self, visitor) -> None:
        for index, stage in enumerate(self.stages):
            visitor.enter(index)
            stage.visit(visitor)
            visitor.leave()


class Mlp:
    """`neural/mlp.rs`: Linear stages over consecutive widths, tanh between
    them and none after the last; ``initializer(shape)`` draws each weight,
    then its bias."""

    def __init__(self, tape: Tape, sizes, initializer):
        assert len(sizes) >= 2, "an MLP topology needs an input and an output width"
        self.stages = []
        for inputs, outputs in zip(sizes[:-1], sizes[1:]):
            weights = np.asarray(initializer((inputs, outputs)), np.float32)
            bias = np.asarray(initializer((outputs,)), np.float32)
            self.stages.append(Linear(tape, weights, bias))

    def parameters(self) -> List[Value]:
        return [p for stage in self.stages for p in stage.parameters()]

    def express(self, x: Value) -> Value:
        last = len(self.stages) - 1
        for index, stage in enumerate(self.stages):
            x = stage.express(x)
            if index != last:
                x = x.tanh()
        return x

    def visit(self, visitor) -> None:
        for index, stage in enumerate(self.stages):
            visitor.enter(index)
            stage.visit(visitor)
            visitor.leave()


class LayerNorm:
    """`neural/layer_norm.rs:100-132`: per-sample mean and biased variance
    along the features, ``(x - m) / sqrt(v + eps) * scale + shift``; scale
    and shift default to ones and zeros."""

    def __init__(self, tape: Tape, features: int, epsilon: float = 1e-5, scale=None, shift=None):
        scale = np.ones(features, np.float32) if scale is None else np.asarray(scale, np.float32)
        shift = np.zeros(features, np.float32) if shift is None else np.asarray(shift, np.float32)
        self.scale = tape.parameter(Dense((features,), scale))
        self.shift = tape.parameter(Dense((features,), shift))
        self.epsilon = tape.leaf(filled((), epsilon))

    def parameters(self) -> List[Value]:
        return [self.scale, self.shift]

    def express(self, x: Value) -> Value:
        assert len(x.shape) == 2
        mean = x.mean_along(1)
        centered = x - mean.broadcast_along(1, x)
        variance = (centered * centered).mean_along(1)
        deviation = (variance + self.epsilon.broadcast_like(variance)).sqrt()
        normalized = centered / deviation.broadcast_along(1, x)
        return normalized * self.scale.broadcast_along(0, x) + self.shift.broadcast_along(0, x)

    def visit(self, visitor) -> None:
        # neural/layer_norm.rs:148-151
        visitor.parameter("scale", self.scale)
        visitor.parameter("shift", self.shift)


class RmsNorm:
    """`neural/rms_norm.rs:89-114`: ``x / sqrt(mean(x^2) + eps) * scale`` per
    sample, no centering; scale defaults to ones."""

    def __init__(self, tape: Tape, features: int, epsilon: float = 1e-5, scale=None):
        scale = np.ones(features, np.float32) if scale is None else np.asarray(scale, np.float32)
        self.scale = tape.parameter(Dense((features,), scale))
        self.epsilon = tape.leaf(filled((), epsilon))

    def parameters(self) -> List[Value]:
        return [self.scale]

    def express(self, x: Value) -> Value:
        assert len(x.shape) == 2
        power = (x * x).mean_along(1)
        root = (power + self.epsilon.broadcast_like(power)).sqrt()
        return x / root.broadcast_along(1, x) * self.scale.broadcast_along(0, x)

    def visit(self, visitor) -> None:
        # neural/rms_norm.rs:130-132
        visitor.parameter("scale", self.scale)


def conv2d(x: Value, weights: Value, bias: Value, stride: int = 1, padding: int = 0) -> Value:
    """`neural/convolution.rs:53-131`: zero padding (`pad`), two single-axis
    unfolds into windows ``[batch, channels, out_h, kernel_h, out_w, kernel_w]``,
    the im2col matrix (window-major rows over ``[channels, kernel]``), one GEMM
    against the ``[columns, filters]`` weights, the bias along rows, back to
    ``[batch, filters, out_h, out_w]``."""
    batch, channels, height, width = x.shape
    filters, _, kh, kw = weights.shape
    padded = x
    if padding > 0:
        padded = padded.pad(2, padding, height + 2 * padding)
        padded = padded.pad(3, padding, width + 2 * padding)
    windows = padded.unfold(2, kh, stride, 1).unfold(4, kw, stride, 1)
    out_h, out_w = windows.shape[2], windows.shape[4]
    patches = windows.permute([0, 2, 4, 1, 3, 5]).reshape(
        (batch * out_h * out_w, channels * kh * kw))
    kernel = weights.permute([1, 2, 3, 0]).reshape((channels * kh * kw, filters))
    product = patches.matmul(kernel)
    shifted = product + bias.broadcast_along(0, product)
    return shifted.reshape((batch, out_h, out_w, filters)).permute([0, 3, 1, 2])


def max_pool(x: Value, size: int, stride: int) -> Value:
    """`neural/pooling.rs:16-61`: the window lanes (two unfolds, then
    ``[batch, channels, out_h, out_w, size*size]``) folded left with
    `maximum` in row-major window order (ties route to the earliest lane)."""
    windows = x.unfold(2, size, stride, 1).unfold(4, size, stride, 1)
    a = windows.shape
    lanes = windows.permute([0, 1, 2, 4, 3, 5]).reshape((a[0], a[1], a[2], a[4], size * size))
    largest = lanes.narrow(4, 0, 1)
    for lane in range(1, size * size):
        largest = largest.maximum(lanes.narrow(4, lane, 1))
    return largest.squeeze(4)


class BatchNorm:
    """`neural/batch_norm.rs:104-160` (training mode): per-feature mean and
    biased variance over the batch axis, ``(x - m) / sqrt(v + eps) * scale +
    shift``; `express` returns (output, mean, variance)."""

    def __init__(self, tape: Tape, features: int, epsilon: float = 1e-5, scale=None, shift=None):
        scale = np.ones(features, np.float32) if scale is None else np.asarray(scale, np.float32)
        shift = np.zeros(features, np.float32) if shift is None else np.asarray(shift, np.float32)
        self.scale = tape.parameter(Dense((features,), scale))
        self.shift = tape.parameter(Dense((features,), shift))
        self.epsilon = tape.leaf(filled((), epsilon))

    def parameters(self) -> List[Value]:
        return [self.scale, self.shift]

    def express(self, x: Value):
        mean = x.mean_along(0)
        centered = x - mean.broadcast_along(0, x)
        variance = (centered * centered).mean_along(0)
        return self._normalize(centered, variance), mean, variance

    def express_with(self, x: Value, mean: Value, variance: Value) -> Value:
        """Inference mode (`neural/batch_norm.rs:136-145`): normalization by
        supplied ``[features]`` statistics, typically per-run inputs fed with
        the running estimates."""
        return self._normalize(x - mean.broadcast_along(0, x), variance)

    def _normalize(self, centered: Value, variance: Value) -> Value:
        # the shared tail (`neural/batch_norm.rs:149-177`)
        assert len(centered.shape) == 2, \
            f"batch-norm input must be rank 2 [batch, features], got {centered.shape}"
        assert centered.shape[1] == self.scale.shape[0], \
            f"batch-norm input {centered.shape} and scale {self.scale.shape} disagree on features"
        deviation = (variance + self.epsilon.broadcast_like(variance)).sqrt()
        normalized = centered / deviation.broadcast_along(0, centered)
        return normalized * self.scale.broadcast_along(0, centered) + \
            self.shift.broadcast_along(0, centered)


class Gelu:
    """``0.5 x (1 + tanh(0.7978846 (x + 0.044715 x^3)))`` with scalar leaves."""

    def __init__(self, tape: Tape):
        self.half = tape.leaf(filled((), 0.5))
        self.one = tape.leaf(filled((), 1.0))
        self.root = tape.leaf(filled((), 0.7978846))
        self.coefficient = tape.leaf(filled((), 0.044715))

    def express(self, x: Value) -> Value:
        cubic = x * x * x * self.coefficient.broadcast_like(x)
        inner = ((x + cubic) * self.root.broadcast_like(x)).tanh()
        return x * (inner + self.one.broadcast_like(inner)) * self.half.broadcast_like(x)


def cross_entropy(logits: Value, targets: Value) -> Value:
    """`neural/loss.rs:44-63`: ``(Σ(Σ_1 t · lse(logits)) - Σ(t·logits)) / Σ t``."""
    assert len(logits.shape) == 2 and targets.shape == logits.shape
    normalizers = (targets.sum_along(1) * logits.logsumexp(1)).sum()
    alignment = (targets * logits).sum()
    return (normalizers - alignment) / targets.sum()


def sgd_reference(params, grads, lr):
    """Host f32 restatement of `Sgd::step` for checks: ``p - g·lr``."""
    lr = np.float32(lr)
    return [(p - g * lr).astype(np.float32) for p, g in zip(params, grads)]
