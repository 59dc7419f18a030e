"""The five benchmark workloads of the reference's compiled-plan path, recorded
as topos graphs with the recorded-gradient training idiom
(`examples/makemore/mlp_compiled.rs:140-213`: ``differentiate`` once, one
forward-only plan computes loss and gradients).

Each builder returns a :class:`Workload` holding the network, the plan columns,
the parameter/gradient pairs, the input symbols and a seeded feed generator.
Inputs are synthetic, from the splitmix64 streams of `neural/init.rs`.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Callable, Dict, List

import numpy as np

from . import neural
from .graph import Dense, Selection, Tape, Value, counted, filled, selection
from .plan import Request


@dataclass
class Workload:
    name: str
    tape: Tape
    network: object
    columns: object
    loss: Value
    params: List[Value]
    grads: List[Value]
    inputs: Dict[str, Value]
    feeds: Callable[[int], dict]
    samples: int                 # samples per step (the metric's unit)
    optimizer: dict = field(default_factory=dict)
    flops: float = 0.0           # algorithmic FLOPs per step
    extra: dict = field(default_factory=dict)


def _compile(tape, loss, params, extra_roots=()):
    grads = tape.differentiate(loss, params)
    network = tape.into_network()
    columns = network.compile(Request([loss] + list(grads) + list(extra_roots)))
    return network, columns, grads


# ----------------------------------------------------------------- C1
def mlp(batch: int = 128, seed: int = 1) -> Workload:
    """C1: 784->256 (ReLU)->10, softmax cross-entropy, SGD lr 0.1."""
    tape = Tape()
    w1 = neural.uniform(seed, math.sqrt(6.0 / 784))
    l1 = neural.Linear(tape, w1((784, 256)), np.zeros(256, np.float32))
    l2 = neural.Linear(tape, w1((256, 10), math.sqrt(6.0 / 256)), np.zeros(10, np.float32))
    x = tape.input(Dense((batch, 784), np.zeros((batch, 784), np.float32)))
    y = tape.input(selection(np.zeros(batch, np.int64), 10))
    logits = l2.express(l1.express(x).relu())
    loss = neural.cross_entropy(logits, y)
    params = l1.parameters() + l2.parameters()
    network, columns, grads = _compile(tape, loss, params)

    def feeds(step: int):
        xs = neural.unit_uniform(seed * 1000 + step + 11)((batch, 784))
        ys = neural.integers(seed * 1000 + step + 12, 10, batch)
        return {x: Dense((batch, 784), xs), y: Selection(ys, 10)}

    flops = 2.0 * batch * (2 * 784 * 256 + 3 * 256 * 10)
    return Workload("mlp784", tape, network, columns, loss, params, grads, {"x": x, "y": y},
                    feeds, batch, {"kind": "sgd", "lr": 0.1}, flops=flops)


# ----------------------------------------------------------------- C2
def fused(rows: int = 8192, cols: int = 8192, seed: int = 2) -> Workload:
    """C2: y = tanh(a·X + b) · sigmoid(X), s = Σ_last y, loss = Σ s; grads
    w.r.t. X, b and a.  sigmoid is composed as 1/(1+exp(-x))."""
    tape = Tape()
    draw = neural.normal(seed, 1.0)
    X = tape.parameter(Dense((rows, cols), draw((rows, cols))))
    b = tape.parameter(Dense((cols,), draw((cols,))))
    a = tape.parameter(Dense((), np.array(0.5, np.float32)))
    one = tape.leaf(filled((), 1.0))
    z = a.broadcast_like(X) * X + b.broadcast_along(0, X)
    sig = one.broadcast_like(X) / (one.broadcast_like(X) + (-X).exp())
    y = z.tanh() * sig
    s = y.sum_along(1)
    loss = s.sum()
    params = [X, b, a]
    grads = tape.differentiate(loss, params)
    network = tape.into_network()
    columns = network.compile(Request([loss, s] + grads))
    return Workload("fused8192", tape, network, columns, loss, params, grads, {},
                    lambda step: {}, rows, {}, extra={"s": s})


# ----------------------------------------------------------------- C3
def gemm(m: int = 4096, k: int = 4096, n: int = 4096, seed: int = 3) -> Workload:
    """C3: C = A·B with upstream gradient dC: dA = dC·Bᵀ, dB = Aᵀ·dC, recorded
    as the loss Σ(C ⊙ dC) whose gradients are exactly those products."""
    tape = Tape()
    A = tape.parameter(Dense((m, k), neural.uniform(seed, 1.0)((m, k))))
    B = tape.parameter(Dense((k, n), neural.uniform(seed + 1, 1.0)((k, n))))
    dC = tape.input(Dense((m, n), neural.normal(seed + 2, 1.0)((m, n))))
    C = A.matmul(B)
    loss = (C * dC).sum()
    params = [A, B]
    grads = tape.differentiate(loss, params)
    network = tape.into_network()
    columns = network.compile(Request([loss, C] + grads))
    return Workload(f"gemm{m}x{k}x{n}", tape, network, columns, loss, params, grads, {"dC": dC},
                    lambda step: {}, 1, {}, flops=float(3 * 2 * m * n * k), extra={"C": C})


# ----------------------------------------------------------------- C4
def char_mlp(batch: int = 16384, context: int = 8, embed: int = 64, hidden: int = 512,
             vocab: int = 27, seed: int = 4) -> Workload:
    """C4: embedding gather, (Linear 512->512 -> LayerNorm -> tanh) x 2,
    Linear 512->27, cross-entropy, Adam."""
    tape = Tape()
    draw = neural.normal(seed, 1.0)
    table = tape.parameter(Dense((vocab, embed), draw((vocab, embed))))
    fan = context * embed
    layers = []
    width = fan
    for _ in range(2):
        w = neural.uniform(seed + 10 + len(layers), 1.0 / math.sqrt(width))((width, hidden))
        layers.append((neural.Linear(tape, w, np.zeros(hidden, np.float32)),
                       neural.LayerNorm(tape, hidden)))
        width = hidden
    head = neural.Linear(tape, neural.uniform(seed + 20, 1.0 / math.sqrt(hidden))((hidden, vocab)),
                         np.zeros(vocab, np.float32))
    ctx = tape.input(selection(np.zeros(batch * context, np.int64), vocab))
    tgt = tape.input(selection(np.zeros(batch, np.int64), vocab))
    h = table.gather(ctx).reshape((batch, fan))
    for lin, ln in layers:
        h = ln.express(lin.express(h)).tanh()
    logits = head.express(h)
    loss = neural.cross_entropy(logits, tgt)
    params = [table]
    for lin, ln in layers:
        params += lin.parameters() + ln.parameters()
    params += head.parameters()
    network, columns, grads = _compile(tape, loss, params)

    def feeds(step: int):
        c = neural.integers(seed * 7919 + step * 2 + 1, vocab, batch * context)
        t = neural.integers(seed * 7919 + step * 2 + 2, vocab, batch)
        return {ctx: Selection(c, vocab), tgt: Selection(t, vocab)}

    flops = 2.0 * batch * (fan * hidden + hidden * hidden + hidden * vocab) * 3
    return Workload("charmlp", tape, network, columns, loss, params, grads,
                    {"contexts": ctx, "targets": tgt}, feeds, batch,
                    {"kind": "adam", "lr": 1e-3, "beta1": 0.9, "beta2": 0.999, "eps": 1e-8},
                    flops=flops)


# ----------------------------------------------------------------- C5
def gpt2(batch: int = 8, seq: int = 1024, layers: int = 12, d: int = 768, heads: int = 12,
         vocab: int = 50257, mlp: int = 3072, seed: int = 5) -> Workload:
    """C5: GPT-2-small-shaped decoder (pre-LN, learned positions, GELU,
    tied head), batched attention over [B, H, T, Dh] with the causal -inf
    mask leaf, cross-entropy, AdamW (decay on rank >= 2)."""
    tape = Tape()
    draw = neural.normal(seed, 0.02)
    dh = d // heads
    tokens = batch * seq
    wte = tape.parameter(Dense((vocab, d), draw((vocab, d))))
    wpe = tape.parameter(Dense((seq, d), draw((seq, d))))
    mask = np.where(np.arange(seq)[None, :] <= np.arange(seq)[:, None], 0.0, -np.inf).astype(np.float32)
    mask_leaf = tape.leaf(Dense((seq, seq), mask))
    scale = tape.leaf(filled((), 1.0 / math.sqrt(dh)))
    gelu = neural.Gelu(tape)
    blocks = []
    for _ in range(layers):
        blocks.append({
            "ln1": neural.LayerNorm(tape, d),
            "qkv": neural.Linear(tape, draw((d, 3 * d)), np.zeros(3 * d, np.float32)),
            "proj": neural.Linear(tape, draw((d, d)), np.zeros(d, np.float32)),
            "ln2": neural.LayerNorm(tape, d),
            "fc": neural.Linear(tape, draw((d, mlp)), np.zeros(mlp, np.float32)),
            "out": neural.Linear(tape, draw((mlp, d)), np.zeros(d, np.float32)),
        })
    lnf = neural.LayerNorm(tape, d)
    ids = tape.input(selection(np.zeros(tokens, np.int64), vocab))
    tgt = tape.input(selection(np.zeros(tokens, np.int64), vocab))
    positions = tape.leaf(selection(np.tile(np.arange(seq), batch), seq))
    x = wte.gather(ids) + wpe.gather(positions)
    mask_b = mask_leaf
    for blk in blocks:
        h = blk["ln1"].express(x)
        qkv = blk["qkv"].express(h)                               # [B*T, 3D]
        qkv4 = qkv.reshape((batch, seq, 3 * heads, dh)).permute((0, 2, 1, 3))  # [B, 3H, T, Dh]
        q = qkv4.narrow(1, 0, heads)
        k = qkv4.narrow(1, heads, heads)
        v = qkv4.narrow(1, 2 * heads, heads)
        scores = q.matmul(k.permute((0, 1, 3, 2)))                # [B, H, T, T]
        ref4 = scores
        m = mask_b.broadcast_along(0, tape.leaf(counted((heads, seq, seq), 0)))
        m = m.broadcast_along(0, ref4)
        att = (scores * scale.broadcast_like(scores) + m).softmax(3)
        y = att.matmul(v)                                         # [B, H, T, Dh]
        y = y.permute((0, 2, 1, 3)).reshape((tokens, d))
        x = x + blk["proj"].express(y)
        h = blk["ln2"].express(x)
        x = x + blk["out"].express(gelu.express(blk["fc"].express(h)))
    h = lnf.express(x)
    logits = h.matmul(wte.transpose())
    loss = neural.cross_entropy(logits, tgt)
    params = [wte, wpe]
    for blk in blocks:
        for key in ("ln1", "qkv", "proj", "ln2", "fc", "out"):
            params += blk[key].parameters()
    params += lnf.parameters()
    network, columns, grads = _compile(tape, loss, params)

    def feeds(step: int):
        t = neural.integers(seed * 104729 + step * 2 + 1, vocab, tokens + 1)
        return {ids: Selection(t[:tokens], vocab), tgt: Selection(t[1:], vocab)}

    per_token = 6 * (layers * (d * 3 * d + d * d + 2 * d * mlp) + d * vocab) + 6 * layers * 2 * seq * d
    return Workload("gpt2small", tape, network, columns, loss, params, grads,
                    {"ids": ids, "targets": tgt}, feeds, batch,
                    {"kind": "adamw", "lr": 6e-4, "beta1": 0.9, "beta2": 0.95, "eps": 1e-8,
                     "decay": 0.1},
                    flops=float(per_token * tokens))


BUILDERS = {"mlp": mlp, "fused": fused, "gemm": gemm, "charmlp": char_mlp, "gpt2": gpt2}
