"""Loss trajectories over several training steps against the oracle at
identical seeds (C1 SGD, C4 Adam, C5 AdamW at test sizes).  The device runs
each step as one CUDA graph with the optimizer inside it; the oracle runs the
same recorded-gradient plan and a host f32 restatement of the update rule
(neural/optimizer.rs:40-51, neural/adam.rs:62-157) between steps.  The drift
of the loss (and of the parameters after the last step) must stay within the
tolerance each config states: the GEMMs and transcendentals differ from the
interpreter in the last bits, and training amplifies that slowly."""
import numpy as np
import pytest

import oracle
from poorgrad_b200 import backend, configs

pytestmark = pytest.mark.gpu
STEPS = 8


def host_step(kind, opt, params, grads, state, t):
    f = np.float32
    lr = f(opt["lr"])
    if kind == "sgd":
        return [(p - g.reshape(p.shape) * lr).astype(np.float32) for p, g in zip(params, grads)]
    b1, b2, eps = f(opt["beta1"]), f(opt["beta2"]), f(opt["eps"])
    decay = f(opt.get("decay", 0.0))
    state["p1"] = f(state.get("p1", f(1)) * b1)  # beta powers by repeated products
    state["p2"] = f(state.get("p2", f(1)) * b2)
    c1, c2 = f(1) - state["p1"], f(1) - state["p2"]
    out = []
    for i, (p, g) in enumerate(zip(params, grads)):
        g = g.reshape(p.shape).astype(np.float32)
        m = state.get(("m", i), np.zeros_like(g)) * b1 + g * (f(1) - b1)
        v = state.get(("v", i), np.zeros_like(g)) * b2 + (g * g) * (f(1) - b2)
        state[("m", i)], state[("v", i)] = m, v
        d = (m / c1) / (np.sqrt(v / c2) + eps)
        stepped = p - d * lr
        if kind == "adamw" and p.ndim >= 2:
            stepped = stepped - (p * decay) * lr
        out.append(stepped.astype(np.float32))
    return out


@pytest.mark.parametrize("name,kw,tol", [
    ("mlp", dict(batch=128), 1e-4),
    ("charmlp", dict(batch=256), 2e-3),
    ("gpt2", dict(batch=2, seq=16, layers=2, d=32, heads=4, vocab=50, mlp=64), 2e-3)])
def test_loss_trajectory_tracks_the_oracle(device, name, kw, tol):
    w = configs.BUILDERS[name](**kw)
    opt = w.optimizer
    kind = opt["kind"]
    params0 = w.network.parameters()
    plan = backend.DevicePlan(w.columns)
    dp = backend.DeviceParameters(plan, params0)
    code = {"sgd": backend.SGD, "adam": backend.ADAM, "adamw": backend.ADAMW}[kind]
    optimizer = backend.Optimizer(plan, dp, code, zip(w.params, w.grads), opt["lr"],
                                  opt.get("beta1", 0.9), opt.get("beta2", 0.999),
                                  opt.get("eps", 1e-8), opt.get("decay", 0.0))
    params, state = [p.copy() for p in params0], {}
    dev_loss, ref_loss = [], []
    for step in range(STEPS):
        feeds = w.feeds(step)
        plan.forward(dp, feeds, sync=True)
        dev_loss.append(float(plan.of(w.loss)))
        ref = oracle.run(w.columns, params, feeds, read=[w.loss.index] + [g.index for g in w.grads])
        ref_loss.append(float(ref[w.loss.index]))
        params = host_step(kind, opt, params, [ref[g.index] for g in w.grads], state, step + 1)
    drift = [abs(d - r) / max(abs(r), 1e-30) for d, r in zip(dev_loss, ref_loss)]
    assert max(drift) <= tol, f"loss drift per step {drift}"
    for p_ref, sym in zip(params, w.params):
        got = dp.download(w.columns.nodes[sym.index].slot).reshape(p_ref.shape)
        scale = np.abs(p_ref).max() + 1e-30
        np.testing.assert_allclose(got, p_ref, rtol=0, atol=50 * tol * scale)
    del optimizer
