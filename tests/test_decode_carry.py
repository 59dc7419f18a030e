"""Decode carry (engine/tests/plan_tests.rs:721-910): a full-context causal
attention stack and its one-token decode twin, recorded on one tape over the
same parameters.  The decode plan appends to capacity-shaped key/value caches
by `scatter` over a position selection and carries them from run to run as
fed inputs; at every step its row must equal the full plan's row of that
position, with the full window's future rows filled with garbage, so the
identity also proves the mask isolates the past."""
import numpy as np
import pytest

import oracle
from poorgrad_b200.graph import Tape, concat, filled, selection, tensor
from poorgrad_b200.plan import Request

CAPACITY, EMBED, HEADS, LAYERS = 4, 4, 2, 2
HEAD_DIM = EMBED // HEADS


def seeded(seed, count):
    return [(((at * 31 + seed * 17) % 23) - 11.0) / 16.0 for at in range(count)]


def record():
    t = Tape()
    layers = [(t.parameter(tensor((EMBED, 3 * EMBED), seeded(2 * l + 1, 3 * EMBED * EMBED))),
               t.parameter(tensor((EMBED, EMBED), seeded(2 * l + 2, EMBED * EMBED))))
              for l in range(LAYERS)]
    scale = t.leaf(filled((), float(np.float32(1.0) / np.sqrt(np.float32(HEAD_DIM)))))
    mask = t.leaf(tensor((CAPACITY, CAPACITY),
                         [0.0 if at % CAPACITY <= at // CAPACITY else -np.inf
                          for at in range(CAPACITY * CAPACITY)]))
    window = t.input(filled((CAPACITY, EMBED), 0.0))
    stream = window
    for fused_w, projection in layers:
        fused = stream.matmul(fused_w)
        heads = []
        for h in range(HEADS):
            q = fused.narrow(1, h * HEAD_DIM, HEAD_DIM)
            k = fused.narrow(1, EMBED + h * HEAD_DIM, HEAD_DIM)
            v = fused.narrow(1, 2 * EMBED + h * HEAD_DIM, HEAD_DIM)
            scores = q.matmul(k.transpose())
            heads.append((scores * scale.broadcast_like(scores) + mask).softmax(1).matmul(v))
        stream = stream + concat(heads, 1).matmul(projection)
    full_out = stream

    row_in = t.input(filled((1, EMBED), 0.0))
    position = t.input(selection([0], CAPACITY))
    mask_in = t.input(filled((1, CAPACITY), 0.0))
    caches = [(t.input(filled((CAPACITY, EMBED), 0.0)), t.input(filled((CAPACITY, EMBED), 0.0)))
              for _ in range(LAYERS)]
    row, updated = row_in, []
    for (fused_w, projection), (keys, values) in zip(layers, caches):
        fused = row.matmul(fused_w)
        keys = keys + fused.narrow(1, EMBED, EMBED).scatter(position, CAPACITY)
        values = values + fused.narrow(1, 2 * EMBED, EMBED).scatter(position, CAPACITY)
        heads = []
        for h in range(HEADS):
            q = fused.narrow(1, h * HEAD_DIM, HEAD_DIM)
            k = keys.narrow(1, h * HEAD_DIM, HEAD_DIM)
            v = values.narrow(1, h * HEAD_DIM, HEAD_DIM)
            scores = q.matmul(k.transpose())
            heads.append((scores * scale.broadcast_like(scores) + mask_in).softmax(1).matmul(v))
        row = row + concat(heads, 1).matmul(projection)
        updated.append((keys, values))
    net = t.into_network()
    full = net.compile(Request([full_out]))
    outputs = [c for pair in updated for c in pair]
    decode = net.compile(Request([row], observe=outputs))
    return net, full, decode, dict(window=window, full_out=full_out, row_in=row_in,
                                   position=position, mask_in=mask_in, caches=caches,
                                   updated=updated, row=row)


def steps():
    rows = [np.array(seeded(90 + at, EMBED), np.float32) for at in range(CAPACITY)]
    garbage = np.full(EMBED, 7.5, np.float32)
    for step in range(CAPACITY):
        window = np.stack([rows[at] if at <= step else garbage for at in range(CAPACITY)])
        mask_row = np.array([[0.0 if at <= step else -np.inf for at in range(CAPACITY)]],
                            np.float32)
        yield step, window, rows[step].reshape(1, EMBED), mask_row


def carry_loop(run_full, run_decode, n):
    """Runs both plans step by step; returns (full rows, decode rows)."""
    carry = {c: np.zeros((CAPACITY, EMBED), np.float32) for pair in n["caches"] for c in pair}
    full_rows, decode_rows = [], []
    for step, window, row, mask_row in steps():
        full_rows.append(run_full({n["window"]: window})[step])
        feeds = dict(carry)
        feeds.update({n["row_in"]: row, n["position"]: selection([step], CAPACITY),
                      n["mask_in"]: mask_row})
        out = run_decode(feeds)
        decode_rows.append(out[n["row"]].reshape(-1))
        carry = {}
        for (k_in, v_in), (k_out, v_out) in zip(n["caches"], n["updated"]):
            carry[k_in], carry[v_in] = out[k_out], out[v_out]
    return full_rows, decode_rows


def test_decode_carry_matches_the_full_context_plan_bitwise(built):
    net, full, decode, n = record()
    params = net.parameters()
    keys = [n["row"]] + [c for pair in n["updated"] for c in pair]

    def run_decode(feeds):
        out = oracle.run(decode, params, feeds, read=keys)
        return {k: out[k.index] for k in keys}

    full_rows, decode_rows = carry_loop(
        lambda feeds: oracle.run(full, params, feeds)[n["full_out"].index], run_decode, n)
    for step, (f, d) in enumerate(zip(full_rows, decode_rows)):
        assert f.tobytes() == d.tobytes(), f"the rows disagree at step {step}"


@pytest.mark.gpu
def test_decode_carry_on_the_device(device):
    # the device's full and decode plans each follow the oracle, and the
    # carried caches make the decode rows equal the full rows
    from poorgrad_b200 import backend
    net, full, decode, n = record()
    params = net.parameters()
    plans = {}
    for name, cols in (("full", full), ("decode", decode)):
        plan = backend.DevicePlan(cols)
        plans[name] = (plan, backend.DeviceParameters(plan, params))

    def run_full(feeds):
        plan, dp = plans["full"]
        plan.forward(dp, feeds, sync=True)
        got = plan.of(n["full_out"])
        ref = oracle.run(full, params, feeds)[n["full_out"].index]
        np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-6)
        return got

    def run_decode(feeds):
        plan, dp = plans["decode"]
        plan.forward(dp, feeds, sync=True)
        keys = [n["row"]] + [c for pair in n["updated"] for c in pair]
        out = {k: plan.of(k) for k in keys}
        ref = oracle.run(decode, params, feeds, read=keys)
        for k in keys:
            np.testing.assert_allclose(out[k], ref[k.index], rtol=1e-5, atol=1e-6)
        return out

    full_rows, decode_rows = carry_loop(run_full, run_decode, n)
    for step, (f, d) in enumerate(zip(full_rows, decode_rows)):
        np.testing.assert_allclose(d, f, rtol=1e-5, atol=1e-6, err_msg=f"step {step}")
