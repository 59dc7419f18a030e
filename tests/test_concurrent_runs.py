"""Concurrent runs of one compiled plan (`Plan` and `Run` are Send + Sync and
run from many threads in the reference: engine/plan.rs:20, run.rs:14,
examples/makemore/mlp_parallel.rs:136-165).  Each `tb_run_begin` draws its own
instance (stream, arena, inputs) from the plan's pool, so threads running the
same plan on different feeds each get exactly the values a lone run of their
feeds produces (bitwise: same program, same kernels)."""
import threading

import numpy as np
import pytest

from poorgrad_b200 import backend, configs

pytestmark = pytest.mark.gpu


def test_threads_share_one_plan(device):
    w = configs.char_mlp(batch=512, hidden=64, embed=16)
    plan = backend.DevicePlan(w.columns)
    params = backend.DeviceParameters(plan, w.network.parameters())
    wanted = [w.loss] + list(w.grads)
    feeds = [w.feeds(i) for i in range(8)]
    alone = []
    for f in feeds:  # reference values, one run at a time on the main instance
        plan.forward(params, f, sync=True)
        alone.append([plan.of(v) for v in wanted])
    got = [None] * len(feeds)
    errors = []

    def worker(i):
        try:
            for rep in range(3):
                run = plan.begin(params, feeds[i])
                vals = [run.of(v) for v in wanted]
                run.release()
                if rep == 0:
                    got[i] = vals
                else:
                    for a, b in zip(vals, got[i]):
                        np.testing.assert_array_equal(a, b)
        except Exception as e:  # surfaced below
            errors.append((i, repr(e)))

    threads = [threading.Thread(target=worker, args=(i,)) for i in range(len(feeds))]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    assert not errors, errors
    for i in range(len(feeds)):
        for a, b in zip(got[i], alone[i]):
            np.testing.assert_array_equal(a, b)
    # a released run's instance is reused: a later run still agrees
    run = plan.begin(params, feeds[3])
    np.testing.assert_array_equal(run.of(w.loss), alone[3][0])
    run.release()
