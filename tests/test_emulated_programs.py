"""Whole lowered device programs run on the host by the kernel emulator
(`tests/kernel_emulator.py`), against the oracle: the emitted kernels (fusion
groups and their phases, register-held values, column and full sums, preps,
gather and scatter) and the data flow between them, checked without a GPU.
The library kernels are restated in the emulator from their contracts, so
GEMM results agree within the product's tolerance, not bitwise.

bf16 networks are checked here end to end: their emulated programs equal the
bf16 oracle bitwise on these cases.  That bitwise agreement covers the
emulator's restatements only (a GEMM rounded once from an f64 hi/lo product,
column finals summed serially); the device accumulates 3xTF32 in chunks and
sums finals in strided groups, so device bf16 results are checked within
tolerance (tests/test_bf16.py), never bitwise.  Engine-backward plans (the reverse scan appended by
the lowering) follow the oracle's restatement of `Run::backward`."""
import numpy as np
import pytest

import kernel_emulator
import oracle
from poorgrad_b200 import configs
from poorgrad_b200.graph import BF16, Tape
from poorgrad_b200.plan import Request

from test_bf16 import _mixed_network
from test_closure import CASES
from test_random_graphs import random_graph


def compare(cols, params, feeds=None, tol=3e-5, bitwise=False):
    out = kernel_emulator.run_program(cols, params, feeds)
    ref = oracle.run(cols, params, feeds)
    assert out
    for node, v in out.items():
        r = ref[node]
        if bitwise:
            assert v.tobytes() == r.tobytes(), node
        else:
            scale = max(1.0, float(np.abs(r).max()))
            np.testing.assert_allclose(v, r, rtol=0, atol=tol * scale, err_msg=str(node))


@pytest.mark.parametrize("name,kw", [
    ("mlp", dict(batch=16)), ("charmlp", dict(batch=32)), ("fused", dict(rows=32, cols=64)),
    ("gpt2", dict(batch=1, seq=8, layers=1, d=16, heads=2, vocab=11, mlp=32)),
    ("gpt2", dict(batch=2, seq=16, layers=2, d=32, heads=4, vocab=50, mlp=64)),
    # 64-wide heads and sequence: every attention product reads raw f32 operands
    ("gpt2", dict(batch=1, seq=64, layers=1, d=128, heads=2, vocab=50, mlp=256))])
def test_config_programs_follow_the_oracle(built, name, kw):
    w = configs.BUILDERS[name](**kw)
    compare(w.columns, w.network.parameters(), w.feeds(0) if w.feeds else None)


@pytest.mark.parametrize("seed", [0, 3, 7, 11, 17, 22])
def test_random_programs_follow_the_oracle(built, seed):
    net, cols, _, _ = random_graph(seed)
    compare(cols, net.parameters())


@pytest.mark.parametrize("seed", [1, 4, 8, 12, 18, 23])
def test_random_bf16_programs_equal_the_bf16_oracle(built, seed):
    net, cols, _, _ = random_graph(seed, BF16)
    compare(cols, net.parameters(), bitwise=True)


def test_bf16_layer_norm_gather_and_softmax_program_equals_the_bf16_oracle(built):
    cols = _mixed_network(BF16)
    compare(cols, cols.network.parameters(), bitwise=True)


@pytest.mark.parametrize("name", sorted(CASES))
def test_engine_backward_programs_follow_the_engine_scan(built, name):
    # the reverse scan the lowering appends for `Request::backward`, run on
    # the host, against the oracle's restatement of `Run::backward`
    t = Tape()
    loss, wrt = CASES[name](t)
    net = t.into_network()
    cols = net.compile(Request([loss]).backward())
    params = net.parameters()
    out, grads = kernel_emulator.run_program(cols, params, gradients=True)
    scan = oracle.backward(cols, params, loss, wrt)
    for p, ref in zip(wrt, scan):
        got = out[grads[(loss.index, p.index)]]
        np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-6)


def test_decode_carry_programs_follow_the_oracle(built):
    # the full-context and one-token decode programs of the decode-carry test
    # (scatter-appended caches carried as feeds, a -inf mask), emulated
    from test_decode_carry import carry_loop, record
    net, full, decode, n = record()
    params = net.parameters()
    keys = [n["row"]] + [c for pair in n["updated"] for c in pair]

    def run_full(feeds):
        got = kernel_emulator.run_program(full, params, feeds)[n["full_out"].index]
        ref = oracle.run(full, params, feeds)[n["full_out"].index]
        np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-6)
        return got

    def run_decode(feeds):
        got = kernel_emulator.run_program(decode, params, feeds)
        ref = oracle.run(decode, params, feeds, read=keys)
        for k in keys:
            np.testing.assert_allclose(got[k.index], ref[k.index], rtol=1e-5, atol=1e-6)
        return {k: got[k.index] for k in keys}

    full_rows, decode_rows = carry_loop(run_full, run_decode, n)
    for f, d in zip(full_rows, decode_rows):
        np.testing.assert_allclose(d, f, rtol=1e-5, atol=1e-6)


def test_dropout_programs_follow_the_oracle(built):
    # a fed mask each run and an unfed run that is the identity
    from poorgrad_b200 import neural
    from test_dropout import masked_network
    net, cols, w, x, drop, loss, g = masked_network(64, 16, 32)
    params = net.parameters()
    for feeds in ({}, {drop.mask: neural.dropout(3, 0.75)((64, 32))}):
        out = kernel_emulator.run_program(cols, params, feeds)
        ref = oracle.run(cols, params, feeds)
        for v in (loss, g):
            scale = max(1.0, float(np.abs(ref[v.index]).max()))
            np.testing.assert_allclose(out[v.index], ref[v.index], rtol=0, atol=3e-5 * scale)


def test_composite_engine_backward_program_follows_the_oracle(built):
    # the compositions of the device composites test (broadcast_to, concat,
    # stack, masked softmax) in one engine-backward plan
    from poorgrad_b200.graph import concat, stack, tensor
    rng = np.random.default_rng(4)
    t = Tape()
    a = t.parameter(tensor((2, 1, 8), rng.uniform(-1, 1, 16)))
    b = t.parameter(tensor((8,), rng.uniform(-1, 1, 8)))
    s = t.parameter(tensor((4, 8), rng.uniform(-2, 2, 32)))
    mask = t.leaf(tensor((8,), [0.0] * 6 + [-np.inf] * 2))
    grid = a.broadcast_to((2, 4, 8)) + b.broadcast_to((2, 4, 8))
    probs = (s + mask.broadcast_to((4, 8))).softmax(1)
    joined = concat([grid.reshape((8, 8)), probs.abs()], 0)
    stacked = stack([probs, s.mean_along(0).broadcast_to((4, 8))], 0)
    loss = joined.tanh().sum() + stacked.logsumexp(2).sum()
    net = t.into_network()
    cols = net.compile(Request([loss, joined, stacked]).backward())
    params = net.parameters()
    out, grads = kernel_emulator.run_program(cols, params, gradients=True)
    ref = oracle.run(cols, params)
    for v in (joined, stacked, loss):
        np.testing.assert_allclose(out[v.index], ref[v.index], rtol=1e-5, atol=1e-6)
    for p, r in zip((a, b, s), oracle.backward(cols, params, loss, [a, b, s])):
        np.testing.assert_allclose(out[grads[(loss.index, p.index)]], r, rtol=1e-5, atol=1e-6)


def test_raw_operand_programs_follow_the_oracle(built):
    # a narrow MLP head whose activations reach both its products as raw f32
    # A operands (the logits, K-major, and the weight gradient, MN-major)
    import re
    from poorgrad_b200 import backend
    from poorgrad_b200.graph import Dense
    rng = np.random.default_rng(5)
    t = Tape()
    x = t.input(Dense((256, 96), rng.standard_normal((256, 96)).astype(np.float32)))
    w1 = t.parameter(Dense((96, 64), rng.standard_normal((96, 64)).astype(np.float32) * 0.1))
    w2 = t.parameter(Dense((64, 24), rng.standard_normal((64, 24)).astype(np.float32) * 0.1))
    h = x.matmul(w1).tanh()
    loss = (h.matmul(w2) * h.matmul(w2)).sum()
    grads = t.differentiate(loss, [w1, w2])
    net = t.into_network()
    cols = net.compile(Request([loss] + grads))
    text = backend.lower_describe(cols)
    assert re.search(r"a=k:raw", text) and re.search(r"a=mn:raw", text)
    compare(cols, net.parameters())


def test_power_of_two_divisors_divide_bitwise(built):
    # x / 2^k is emitted as x * 2^-k (an exact reciprocal: the same real
    # number rounded once), so exact kernels stay bit-identical to the
    # reference's division -- subnormal results, infinities, NaNs and signed
    # zeros included; a divisor that is not a power of two keeps the division
    import re
    from poorgrad_b200 import backend
    from poorgrad_b200.graph import Dense, filled
    vals = np.array([1.0, -3.0, 7e-39, -1e-45, 3.4e38, -0.0, 0.0, np.inf, -np.inf, np.nan,
                     1.17549435e-38, 0.1, 12345.678, -2.5e-40, 6.0, 1e30], np.float32)
    x_payload = Dense((4, 4), vals.reshape(4, 4))
    t = Tape()
    x = t.parameter(x_payload)
    outs = [x / x.literal(filled((4, 4), c)) for c in (4.0, 0.5, 2.0 ** -100, 2.0 ** 100, 3.0)]
    net = t.into_network()
    cols = net.compile(Request(outs))
    src = backend.lower_describe(cols, with_source=True)
    divisions = re.findall(r"__fdiv_rn\([^,]*, ([^)]*\))\)", src)
    assert divisions and set(divisions) == {"__int_as_float(0x40400000)"}  # only the one by 3
    compare(cols, net.parameters(), bitwise=True)
