"""Host restatement of topos's optimizer rules -- TEST INFRASTRUCTURE.

The device applies SGD, Adam and AdamW inside each step's CUDA graph; the
tests check those updates against this restatement, which follows the
reference elementwise operation by operation so that f32 results agree to
the bit:

- ``Sgd``: ``parameter - gradient * rate`` (neural/optimizer.rs:40-51).
- ``Adam``: moments ``m = m * beta1 + g * (1 - beta1)`` and
  ``v = v * beta2 + (g * g) * (1 - beta2)``; beta powers by repeated
  products; direction ``(m / (1 - beta1^t)) / (sqrt(v / (1 - beta2^t)) + eps)``;
  update ``parameter - direction * rate`` (neural/adam.rs:40-104).
- ``AdamW``: the Adam update, then ``- (parameter * decay) * rate`` where the
  policy selects; the default policy is rank >= 2 (neural/adam.rs:106-170).

``dtype`` is float32 for the device checks, float64 for the reference's own
paper trace (neural/tests/adam_tests.rs:14-50), or ``BF16`` for a bf16
network: values are bf16 numbers held in float32 and every operation rounds
its result once (payload/bf16.rs:131-170), hyperparameters included.
"""
from __future__ import annotations

import numpy as np

BF16 = "bf16"


def _element(dtype):
    """(storage type, rounding of one result) of an element type."""
    if dtype == BF16:
        from . import round_bf16

        def r(x):
            a = round_bf16(np.asarray(x, np.float32).reshape(-1)).reshape(np.shape(x))
            return a if np.ndim(x) else np.float32(a)
        return np.float32, r
    return dtype, (lambda x: x)


class Sgd:
    def __init__(self, dtype=np.float32):
        self.dtype, self.r = _element(dtype)

    def step(self, parameters, gradients, rate):
        d, r = self.dtype, self.r
        rate = r(d(rate))
        return [r(p - r(np.asarray(g, d).reshape(p.shape) * rate)).astype(d)
                for p, g in zip(parameters, gradients)]


class Adam:
    def __init__(self, beta1=0.9, beta2=0.999, epsilon=1e-8, dtype=np.float32):
        d, r = self.dtype, self.r = _element(dtype)
        self.beta1, self.beta2, self.epsilon = r(d(beta1)), r(d(beta2)), r(d(epsilon))
        self.first_share = r(d(1) - self.beta1)
        self.second_share = r(d(1) - self.beta2)
        self.beta1_power = d(1)
        self.beta2_power = d(1)
        self.first = None
        self.second = None

    def direction(self, gradients):
        d, r = self.dtype, self.r
        gradients = [np.asarray(g, d) for g in gradients]
        first = self.first or [np.zeros_like(g) for g in gradients]
        second = self.second or [np.zeros_like(g) for g in gradients]
        first = [r(r(m * self.beta1) + r(g * self.first_share)) for m, g in zip(first, gradients)]
        second = [r(r(v * self.beta2) + r(r(g * g) * self.second_share))
                  for v, g in zip(second, gradients)]
        self.beta1_power = r(d(self.beta1_power * self.beta1))
        self.beta2_power = r(d(self.beta2_power * self.beta2))
        c1 = r(d(1) - self.beta1_power)
        c2 = r(d(1) - self.beta2_power)
        self.first, self.second = first, second
        return [r(r(m / c1) / r(r(np.sqrt(r(v / c2))) + self.epsilon))
                for m, v in zip(first, second)]

    def step(self, parameters, gradients, rate):
        d, r = self.dtype, self.r
        rate = r(d(rate))
        return [r(p - r(u.reshape(p.shape) * rate)).astype(d)
                for p, u in zip(parameters, self.direction(gradients))]


class AdamW:
    def __init__(self, beta1=0.9, beta2=0.999, epsilon=1e-8, decay=0.01, dtype=np.float32):
        self.adam = Adam(beta1, beta2, epsilon, dtype)
        self.dtype, self.r = _element(dtype)
        self.decay = self.r(self.dtype(decay))

    def step_where(self, parameters, gradients, rate, policy):
        d, r = self.dtype, self.r
        rate = r(d(rate))
        out = []
        for i, (p, u) in enumerate(zip(parameters, self.adam.direction(gradients))):
            stepped = r(p - r(u.reshape(p.shape) * rate))
            if policy(i, p):
                stepped = r(stepped - r(r(p * self.decay) * rate))
            out.append(stepped.astype(d))
        return out

    def step(self, parameters, gradients, rate):
        return self.step_where(parameters, gradients, rate, lambda _, p: np.ndim(p) >= 2)


def make(kind, hyper, dtype=np.float32):
    """The optimizer named by a workload's ``optimizer`` dict (``kind`` is
    "sgd", "adam" or "adamw")."""
    h = hyper
    if kind == "sgd":
        return Sgd(dtype)
    if kind == "adam":
        return Adam(h.get("beta1", 0.9), h.get("beta2", 0.999), h.get("eps", 1e-8), dtype)
    if kind == "adamw":
        return AdamW(h.get("beta1", 0.9), h.get("beta2", 0.999), h.get("eps", 1e-8),
                     h.get("decay", 0.0), dtype)
    raise ValueError(kind)
