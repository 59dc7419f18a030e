"""Dropout as the reference composes it (neural/dropout.rs: an input mask,
all ones until fed, multiplied in) with masks from the seeded stream of
neural/init.rs:119-130; the known answers of neural/tests/dropout_tests.rs
on the oracle, and a masked training loop on the device."""
import numpy as np
import pytest

import oracle
from poorgrad_b200 import backend, neural
from poorgrad_b200.graph import Tape, tensor
from poorgrad_b200.plan import Request


def test_masks_are_deterministic_in_seed_and_step():
    # dropout_tests.rs:6-17
    first, second = neural.dropout(11, 0.75), neural.dropout(11, 0.75)
    for _ in range(3):
        assert first((4, 8)).tobytes() == second((4, 8)).tobytes()
    assert neural.dropout(11, 0.75)((4, 8)).tobytes() != neural.dropout(12, 0.75)((4, 8)).tobytes()


def test_masks_hold_the_inverted_scale():
    # dropout_tests.rs:19-28
    mask = neural.dropout(7, 0.8)((64, 64))
    assert set(np.unique(mask).tolist()) <= {0.0, float(np.float32(1 / 0.8))}
    assert 2900 <= int(np.count_nonzero(mask)) < 3600


def test_a_zero_keep_probability_is_rejected():
    # dropout_tests.rs:30-34
    with pytest.raises(AssertionError, match="within \\(0, 1\\], got 0"):
        neural.dropout(1, 0.0)


def test_an_unfed_run_is_the_identity():
    # dropout_tests.rs:36-52
    t = Tape()
    x = t.parameter(tensor((2, 3), [0.5, -1.0, 2.0, 3.0, -0.25, 1.5]))
    masked = neural.Dropout(t, (2, 3)).express(x + x)
    plain = x + x
    net = t.into_network()
    out = oracle.run(net.compile(Request([masked, plain])), net.parameters())
    assert out[masked.index].tobytes() == out[plain.index].tobytes()


def test_gradients_route_through_the_mask():
    # dropout_tests.rs:54-65, 97-111
    t = Tape()
    x = t.parameter(tensor((1, 4), [1.0, 2.0, 3.0, 4.0]))
    drop = neural.Dropout(t, (1, 4))
    y = drop.express(x)
    (g,) = t.differentiate(y.sum(), [x])
    net = t.into_network()
    mask = np.array([[2.0, 0.0, 2.0, 0.0]], np.float32)
    out = oracle.run(net.compile(Request([y, g])), net.parameters(), {drop.mask: mask})
    assert out[g.index].reshape(-1).tolist() == [2.0, 0.0, 2.0, 0.0]
    assert out[y.index].reshape(-1).tolist() == [2.0, 0.0, 6.0, 0.0]


def masked_network(batch, features, hidden):
    rng = np.random.default_rng(3)
    t = Tape()
    w = t.parameter(tensor((features, hidden), rng.uniform(-0.5, 0.5, features * hidden)))
    x = t.input(tensor((batch, features), rng.uniform(-1, 1, batch * features)))
    drop = neural.Dropout(t, (batch, hidden))
    h = drop.express(x.matmul(w).tanh())
    loss = (h * h).sum()
    (g,) = t.differentiate(loss, [w])
    net = t.into_network()
    return net, net.compile(Request([loss, g])), w, x, drop, loss, g


def test_masked_training_replays_bitwise_under_matched_seeds():
    # dropout_tests.rs:67-95, on the oracle with the host SGD rule
    def final_loss():
        net, cols, w, x, drop, loss, g = masked_network(2, 2, 2)
        masks, params = neural.dropout(21, 0.5), net.parameters()
        for _ in range(8):
            out = oracle.run(cols, params, {drop.mask: masks((2, 2))})
            params = [(params[0].reshape(-1) - out[g.index].reshape(-1) * np.float32(0.05))
                      .astype(np.float32)]
        return out[loss.index].tobytes()
    assert final_loss() == final_loss()


@pytest.mark.gpu
def test_masked_training_on_the_device_tracks_the_oracle(device):
    # a fresh mask fed each step through the plan's input slot, the SGD step
    # inside the step's graph; gradients compared every step
    net, cols, w, x, drop, loss, g = masked_network(512, 64, 256)
    params = net.parameters()
    plan = backend.DevicePlan(cols)
    dp = backend.DeviceParameters(plan, params)
    opt = backend.Optimizer(plan, dp, backend.SGD, [(w, g)], 0.01)
    masks, host = neural.dropout(21, 0.9), [p.copy() for p in params]
    for _ in range(4):
        mask = masks((512, 256))
        ref = oracle.run(cols, host, {drop.mask: mask})
        plan.forward(dp, {drop.mask: mask}, sync=True)
        np.testing.assert_allclose(plan.of(loss), ref[loss.index], rtol=2e-5)
        # a 512-term sum on the tensor cores: absolute error relative to the
        # gradient's largest element
        scale = float(np.abs(ref[g.index]).max())
        np.testing.assert_allclose(plan.of(g), ref[g.index], rtol=1e-4, atol=2e-5 * scale)
        host = [(host[0].reshape(-1) - ref[g.index].reshape(-1) * np.float32(0.01))
                .astype(np.float32)]
    del opt


@pytest.mark.gpu
def test_an_unfed_mask_is_the_identity_on_the_device(device):
    # the mask's initial payload (`counted(shape, 1)`) fills its input buffer
    # until a feed replaces it
    t = Tape()
    x = t.parameter(tensor((64, 48), np.linspace(-2, 2, 64 * 48)))
    drop = neural.Dropout(t, (64, 48))
    masked = drop.express(x.tanh())
    plain = x.tanh()
    net = t.into_network()
    plan = backend.DevicePlan(net.compile(Request([masked, plain])))
    dp = backend.DeviceParameters(plan, net.parameters())
    plan.forward(dp, None, sync=True)
    assert plan.of(masked).tobytes() == plan.of(plain).tobytes()
    mask = neural.dropout(5, 0.5)((64, 48))
    plan.forward(dp, {drop.mask: mask}, sync=True)
    assert plan.of(masked).tobytes() == (plan.of(plain) * mask).astype(np.float32).tobytes()
