"""Loss trajectories over several training steps against the oracle at
identical seeds (C1 SGD, C4 Adam, C5 AdamW at test sizes).  The device runs
each step as one CUDA graph with the optimizer inside it; the oracle runs the
same recorded-gradient plan and the host f32 restatement of the update rule
(``oracle/optim.py``, after neural/optimizer.rs:40-51 and neural/adam.rs:40-170)
between steps.  The drift
of the loss (and of the parameters after the last step) must stay within the
tolerance each config states: the GEMMs and transcendentals differ from the
interpreter in the last bits, and training amplifies that slowly."""
import numpy as np
import pytest

import oracle
from oracle import optim
from poorgrad_b200 import backend, configs

pytestmark = pytest.mark.gpu
STEPS = 8


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
    # shaped like their nodes: AdamW decays by rank (neural/adam.rs:159-169)
    params = [p.reshape(w.columns.nodes[s.index].shape).copy() for p, s in zip(params0, w.params)]
    host = optim.make(kind, opt)
    dev_loss, ref_loss = [], []
    for step in range(STEPS):
        feeds = w.feeds(step)
        plan.forward(dp, feeds, sync=True)
        dev_loss.append(float(plan.of(w.loss)))
        ref = oracle.run(w.columns, params, feeds, read=[w.loss.index] + [g.index for g in w.grads])
        ref_loss.append(float(ref[w.loss.index]))
        params = host.step(params, [ref[g.index] for g in w.grads], opt["lr"])
    drift = [abs(d - r) / max(abs(r), 1e-30) for d, r in zip(dev_loss, ref_loss)]
    assert max(drift) <= tol, f"loss drift per step {drift}"
    for p_ref, sym in zip(params, w.params):
        got = dp.download(w.columns.nodes[sym.index].slot).reshape(p_ref.shape)
        scale = np.abs(p_ref).max() + 1e-30
        np.testing.assert_allclose(got, p_ref, rtol=0, atol=50 * tol * scale)
    del optimizer
