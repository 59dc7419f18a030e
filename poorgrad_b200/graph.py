"""Recorded graphs: the host-side mirror of topos's `graph/` layer.

A :class:`Tape` records a static graph one node at a time (topos
`graph/tape.rs:49`, `record` 191-220).  Each node carries the producing
operation (a ``Function`` variant, `function/function.rs:26-59`), its operand
links, its static shape and, for sources, the payload or slot.  The node
columns are exactly what topos's compiled ``Plan`` consumes
(`engine/plan.rs:309-346`), and they are what this package hands to the B200
backend through the C ABI (``include/topos_b200.h``).

:meth:`Tape.differentiate` is the tape-to-tape reverse-mode transform of
`graph/tape.rs:335-410`: the same reverse scan the engine runs, applied over
recording handles, so gradients become ordinary computed nodes (the
"recorded-gradient plan" every training config here compiles).

Payloads are the three storage representations of `payload/storage.rs:36-51`:
:class:`Dense` (row-major f32), :class:`Constant` (one value spread over a
shape) and :class:`Selection` (the one-hot ``[count, vocab]`` matrix stored as
its indices).  Values never depend on the representation
(`payload/tests/tensor_tests.rs:1209-1240`).
"""
from __future__ import annotations

import math
from typing import Iterable, List, Optional, Sequence

import numpy as np

# Function variant order, `function/function.rs:26-59`.  The index of a name
# is the opcode carried by `tb_node.op` in the C ABI.
OPS = [
    "Leaf", "Parameter", "Input", "Add", "Sub", "Mul", "Div", "Neg", "Tanh",
    "Exp", "Ln", "MatMul", "Transpose", "Sum", "SumAlong", "Broadcast",
    "BroadcastAlong", "Reshape", "Permute", "Narrow", "Pad", "Unfold", "Fold",
    "Gather", "Scatter", "LogSoftmax", "LogSumExp", "Sqrt", "Powf", "Maximum",
    "Relu", "Step",
]
OP = {name: index for index, name in enumerate(OPS)}

# Operand/output read contract of each derivative rule (`Function::reads`,
# `function/function.rs:295-328` and each rule file's `reads`): which payloads
# an engine-backward plan must retain.  (operand0, operand1, output)
READS = {
    "Mul": (True, True, False), "Div": (False, True, True),
    "Tanh": (False, False, True), "Exp": (False, False, True),
    "Ln": (True, False, False), "MatMul": (True, True, False),
    "Gather": (False, True, False), "Scatter": (False, True, False),
    "LogSoftmax": (False, False, True), "LogSumExp": (True, False, True),
    "Sqrt": (False, False, True), "Powf": (True, True, True),
    "Maximum": (True, True, False), "Relu": (True, False, False),
}
NOTHING = (False, False, False)

ARITY = {name: 2 for name in (
    "Add", "Sub", "Mul", "Div", "MatMul", "Broadcast", "BroadcastAlong",
    "Gather", "Scatter", "Powf", "Maximum", "Step")}
for _name in ("Leaf", "Parameter", "Input"):
    ARITY[_name] = 0
for _name in OPS:
    ARITY.setdefault(_name, 1)


def volume(shape: Sequence[int]) -> int:
    return int(math.prod(shape))


# ---------------------------------------------------------------- payloads
class Dense:
    """Row-major f32 elements of a shape (`Storage::Dense`, contiguous)."""

    kind = "dense"

    def __init__(self, shape, data):
        self.shape = tuple(int(e) for e in shape)
        array = np.ascontiguousarray(np.asarray(data, dtype=np.float32)).reshape(-1)
        assert array.size == volume(self.shape) and array.size > 0, \
            "tensors must hold at least one element"
        self.data = array

    def to_numpy(self) -> np.ndarray:
        return self.data.reshape(self.shape)


class Constant:
    """One value spread across a shape (`Storage::Constant`)."""

    kind = "constant"

    def __init__(self, shape, value):
        self.shape = tuple(int(e) for e in shape)
        assert volume(self.shape) > 0, "tensors must hold at least one element"
        self.value = np.float32(value)

    def to_numpy(self) -> np.ndarray:
        return np.full(self.shape, self.value, dtype=np.float32)


class Selection:
    """The one-hot ``[count, vocab]`` matrix stored as its row indices
    (`Tensor::selection`, `payload/tensor.rs:312-339`): row ``i`` holds
    ``one`` at column ``indices[i]`` and zero elsewhere."""

    kind = "selection"

    def __init__(self, indices, vocab: int, one: float = 1.0):
        indices = np.ascontiguousarray(np.asarray(indices, dtype=np.int64)).reshape(-1)
        assert vocab > 0, "a selection needs a non-empty vocabulary"
        assert indices.size > 0, "tensors must hold at least one element"
        assert indices.min() >= 0 and indices.max() < vocab, \
            "selection index is out of vocabulary"
        self.indices = indices.astype(np.int32)
        self.vocab = int(vocab)
        self.one = np.float32(one)
        self.shape = (int(indices.size), int(vocab))

    def to_numpy(self) -> np.ndarray:
        out = np.zeros(self.shape, dtype=np.float32)
        out[np.arange(self.shape[0]), self.indices] = self.one
        return out


def counted(shape, count: int) -> Constant:
    """`Differentiable::counted` for f32 tensors: ``count as f32`` spread over
    ``shape`` (`payload/tensor.rs:705-707`, `differentiable.rs:123-125`)."""
    return Constant(shape, np.float32(count))


def filled(shape, value) -> Constant:
    """`Tensor::filled` (`payload/tensor.rs:260`): one value over a shape."""
    return Constant(shape, value)


def tensor(shape, data) -> Dense:
    """`Tensor::new` (`payload/tensor.rs:250`)."""
    return Dense(shape, data)


def selection(indices, vocab: int, one: float = 1.0) -> Selection:
    return Selection(indices, vocab, one)


# ------------------------------------------------------------------- nodes
class Node:
    __slots__ = ("op", "operands", "attrs", "shape", "payload", "slot")

    def __init__(self, op, operands, attrs, shape, payload=None, slot=-1):
        self.op = op
        self.operands = tuple(operands)
        self.attrs = tuple(attrs)
        self.shape = tuple(int(e) for e in shape)
        self.payload = payload
        self.slot = slot

    @property
    def name(self) -> str:
        return OPS[self.op]


def _without(shape, axis):
    return tuple(e for i, e in enumerate(shape) if i != axis)


def infer_shape(name: str, attrs, shapes: List[tuple]) -> tuple:
    """Shape rule of each operation, with the reference's panics as
    assertions (each rule file's `infer_shape`)."""
    if name in ("Add", "Sub", "Mul", "Div", "Powf", "Maximum", "Step"):
        assert shapes[0] == shapes[1], f"{name} requires operands of equal shapes"
        return shapes[0]
    if name in ("Neg", "Tanh", "Exp", "Ln", "Sqrt", "Relu"):
        return shapes[0]
    if name == "MatMul":  # function/matmul.rs:24-55
        left, right = shapes
        assert len(left) >= 2, "matmul requires rank-2 or higher operands"
        assert len(left) == len(right), "matmul operands must agree in rank"
        split = len(left) - 2
        assert left[:split] == right[:split], "matmul batch axes must agree"
        assert left[split + 1] == right[split], "matmul cannot multiply"
        return left[:split + 1] + (right[split + 1],)
    if name == "Transpose":
        assert len(shapes[0]) <= 2, "transpose supports rank 2 at most"
        return tuple(reversed(shapes[0]))
    if name == "Sum":
        return ()
    if name == "SumAlong":
        return _without(shapes[0], attrs[0])
    if name == "Broadcast":
        assert volume(shapes[0]) == 1, "broadcast requires a single-element operand"
        return shapes[1]
    if name == "BroadcastAlong":
        assert shapes[0] == _without(shapes[1], attrs[0]), \
            "broadcast along an axis requires the remaining shape"
        return shapes[1]
    if name == "Reshape":
        assert volume(shapes[0]) == volume(attrs), "reshape changes the number of elements"
        return tuple(attrs)
    if name == "Permute":
        order = attrs
        assert sorted(order) == list(range(len(shapes[0]))), "permute order must cover every axis"
        return tuple(shapes[0][a] for a in order)
    if name == "Narrow":
        axis, start, length = attrs
        assert axis < len(shapes[0]) and length > 0 and start + length <= shapes[0][axis]
        return tuple(length if i == axis else e for i, e in enumerate(shapes[0]))
    if name == "Pad":
        axis, start, full = attrs
        assert axis < len(shapes[0]) and start + shapes[0][axis] <= full
        return tuple(full if i == axis else e for i, e in enumerate(shapes[0]))
    if name == "Unfold":  # function/unfold.rs:30-62
        axis, size, step, dilation = attrs
        extent = shapes[0][axis]
        span = dilation * (size - 1) + 1
        assert size > 0 and step > 0 and dilation > 0 and span <= extent
        count = (extent - span) // step + 1
        out = list(shapes[0])
        out[axis] = count
        out.insert(axis + 1, size)
        return tuple(out)
    if name == "Fold":  # function/fold.rs:31-79
        axis, size, step, dilation, extent = attrs
        operand = shapes[0]
        assert axis + 1 < len(operand)
        span = dilation * (size - 1) + 1
        assert span <= extent
        count = (extent - span) // step + 1
        assert operand[axis] == count and operand[axis + 1] == size
        out = list(operand)
        out[axis] = extent
        del out[axis + 1]
        return tuple(out)
    if name == "Gather":  # function/gather.rs:29-48
        table, sel = shapes
        assert len(sel) == 2 and len(table) >= 1 and sel[1] == table[0]
        return (sel[0],) + table[1:]
    if name == "Scatter":  # function/scatter.rs:30-58
        grad, sel = shapes
        (rows,) = attrs
        assert len(grad) >= 1 and len(sel) == 2 and sel[0] == grad[0] and sel[1] == rows
        return (rows,) + grad[1:]
    if name == "LogSoftmax":
        assert attrs[0] < len(shapes[0])
        return shapes[0]
    if name == "LogSumExp":
        assert attrs[0] < len(shapes[0])
        return _without(shapes[0], attrs[0])
    raise ValueError(name)


F32, BF16 = 0, 1  # payload element types (`Tensor<f32>`, `Tensor<Bf16>`: payload/bf16.rs)


class Tape:
    """Records a static graph (`graph/tape.rs:49`).  ``element`` is the
    payload element type of the whole tape, as `Tape<Tensor<E>>` fixes it
    in the reference: ``F32`` or ``BF16`` (payloads still travel as f32
    arrays; a bf16 network rounds them on entry)."""

    def __init__(self, element: int = F32):
        assert element in (F32, BF16), element
        self.element = element
        self.nodes: List[Node] = []
        self.parameter_payloads: List[Dense] = []
        self.input_payloads: list = []

    def __len__(self):
        return len(self.nodes)

    # -- sources (`tape.rs:107-160`)
    def leaf(self, payload) -> "Value":
        return self._push(Node(OP["Leaf"], (), (), payload.shape, payload=payload))

    def parameter(self, payload) -> "Value":
        if not isinstance(payload, Dense):
            payload = Dense(payload.shape, payload.to_numpy())
        slot = len(self.parameter_payloads)
        self.parameter_payloads.append(payload)
        return self._push(Node(OP["Parameter"], (), (), payload.shape, slot=slot))

    def input(self, initial) -> "Value":
        slot = len(self.input_payloads)
        self.input_payloads.append(initial)
        return self._push(Node(OP["Input"], (), (), initial.shape, slot=slot, payload=initial))

    def resolve(self, index: int) -> "Value":
        assert 0 <= index < len(self.nodes), "symbol is not allocated on this tape"
        return Value(self, index)

    def _push(self, node: Node) -> "Value":
        self.nodes.append(node)
        return Value(self, len(self.nodes) - 1)

    def record(self, name: str, operands: Sequence[int], attrs=()) -> "Value":
        assert len(operands) == ARITY[name], "operand count must match the operation's arity"
        shapes = [self.nodes[o].shape for o in operands]
        shape = infer_shape(name, attrs, shapes)
        return self._push(Node(OP[name], operands, attrs, shape))

    # -- reverse mode as a tape-to-tape transform (`tape.rs:335-410`)
    def differentiate(self, loss: "Value", wrt: Iterable["Value"]) -> List["Value"]:
        """Records the gradient of scalar ``loss`` w.r.t. each ``wrt`` value as
        ordinary nodes and returns them in ``wrt`` order.  The scan mirrors
        `Run::backward` exactly: a ``counted(shape, 1)`` seed, ancestor
        marking through present cotangents only, and each first contribution
        accumulated onto a recorded zero literal (`tape.rs:389-393`)."""
        wrt = list(wrt)
        assert self.nodes[loss.index].shape == (), \
            "differentiate requires a scalar loss; reduce it with `sum` first"
        out = loss.index
        frozen = len(self.nodes)
        cotangents: List[Optional[Value]] = [None] * (out + 1)
        cotangents[out] = self.leaf(counted((), 1))
        ancestors = [False] * (out + 1)
        ancestors[out] = True
        for index in range(out, -1, -1):
            if not ancestors[index]:
                continue
            node = self.nodes[index]
            if not node.operands:
                continue
            operands = [Value(self, o) for o in node.operands]
            recorded = backward_rule(node, operands, Value(self, index), cotangents[index])
            assert len(recorded) == len(node.operands)
            for link, contribution in zip(node.operands, recorded):
                if contribution is None:
                    continue
                ancestors[link] = True
                seeded = cotangents[link]
                if seeded is None:
                    seeded = Value(self, link).zero_like()
                cotangents[link] = seeded + contribution
        assert frozen <= len(self.nodes)
        result = []
        for target in wrt:
            grad = cotangents[target.index] if target.index <= out else None
            if grad is None:
                grad = self.leaf(counted(target.shape, 0))
            result.append(grad)
        return result

    def into_network(self) -> "Network":
        return Network(self)


class Network:
    """A sealed tape plus its initial parameter payloads
    (`graph/network.rs:37-60`)."""

    def __init__(self, tape: Tape):
        self.tape = tape
        self.nodes = tape.nodes

    def parameters(self) -> List[np.ndarray]:
        return [p.data.copy() for p in self.tape.parameter_payloads]

    def __len__(self):
        return len(self.nodes)

    def compile(self, request) -> "PlanColumns":
        from .plan import PlanColumns
        return PlanColumns(self, request)


class Value:
    """A recorded value: an index on its tape (`graph/value.rs`)."""

    __slots__ = ("tape", "index")

    def __init__(self, tape: Tape, index: int):
        self.tape = tape
        self.index = index

    @property
    def shape(self) -> tuple:
        return self.tape.nodes[self.index].shape

    def _same(self, other: "Value"):
        assert isinstance(other, Value) and other.tape is self.tape, \
            "values belong to different tapes"

    def _binary(self, name, other, attrs=()):
        self._same(other)
        return self.tape.record(name, (self.index, other.index), attrs)

    def _unary(self, name, attrs=()):
        return self.tape.record(name, (self.index,), attrs)

    def literal(self, payload) -> "Value":
        return self.tape.leaf(payload)

    # arithmetic (`value.rs:495-573`)
    def __add__(self, other):
        return self._binary("Add", other)

    def __sub__(self, other):
        return self._binary("Sub", other)

    def __mul__(self, other):
        return self._binary("Mul", other)

    def __truediv__(self, other):
        return self._binary("Div", other)

    def __neg__(self):
        return self._unary("Neg")

    def tanh(self):
        return self._unary("Tanh")

    def exp(self):
        return self._unary("Exp")

    def ln(self):
        return self._unary("Ln")

    def sqrt(self):
        return self._unary("Sqrt")

    def powf(self, exponent):
        return self._binary("Powf", exponent)

    def maximum(self, other):
        return self._binary("Maximum", other)

    def relu(self):
        return self._unary("Relu")

    def step(self, threshold):
        return self._binary("Step", threshold)

    def matmul(self, other):
        return self._binary("MatMul", other)

    def transpose(self):
        return self._unary("Transpose")

    def sum(self):
        return self._unary("Sum")

    def sum_along(self, axis):
        return self._unary("SumAlong", (axis,))

    def broadcast_like(self, reference):
        return self._binary("Broadcast", reference)

    def broadcast_along(self, axis, reference):
        return self._binary("BroadcastAlong", reference, (axis,))

    def reshape(self, shape):
        return self._unary("Reshape", tuple(int(e) for e in shape))

    def permute(self, order):
        return self._unary("Permute", tuple(int(a) for a in order))

    def unsqueeze(self, axis):
        axes = list(self.shape)
        axes.insert(axis, 1)
        return self.reshape(axes)

    def squeeze(self, axis):
        axes = list(self.shape)
        assert axes[axis] == 1, "squeeze requires an extent-1 axis"
        del axes[axis]
        return self.reshape(axes)

    def narrow(self, axis, start, length):
        return self._unary("Narrow", (axis, start, length))

    def pad(self, axis, start, full_extent):
        return self._unary("Pad", (axis, start, full_extent))

    def unfold(self, axis, size, step, dilation):
        return self._unary("Unfold", (axis, size, step, dilation))

    def fold(self, axis, size, step, dilation, extent):
        return self._unary("Fold", (axis, size, step, dilation, extent))

    def gather(self, sel):
        return self._binary("Gather", sel)

    def scatter(self, sel, rows):
        return self._binary("Scatter", sel, (rows,))

    def log_softmax(self, axis):
        return self._unary("LogSoftmax", (axis,))

    def logsumexp(self, axis):
        return self._unary("LogSumExp", (axis,))

    # the `Trace` twins of `zero_like`/`one_like` (`graph/trace.rs:42-45`)
    def zero_like(self):
        return self.literal(counted(self.shape, 0))

    def one_like(self):
        return self.literal(counted(self.shape, 1))

    # composites (`graph/composite.rs`)
    def abs(self):
        return self.maximum(-self)

    def softmax(self, axis):
        return self.log_softmax(axis).exp()

    def mean_along(self, axis):
        shape = self.shape
        assert axis < len(shape), f"axis {axis} is out of rank for {shape}"
        extent = shape[axis]
        return self.sum_along(axis) / self.literal(counted(_without(shape, axis), extent))

    def broadcast_to(self, shape):
        """`graph/composite.rs:77-131`: right-aligned broadcasting composed
        from `reshape` (prepended unit axes) and one `broadcast_along` per
        repeated axis, or a single `broadcast_like` for one element."""
        target, source = tuple(shape), self.shape
        if source == target:
            return self
        assert len(target) >= len(source), f"broadcast to {target} from {source} lowers the rank"
        offset = len(target) - len(source)
        for axis, extent in enumerate(source):
            aligned = target[offset + axis]
            assert extent in (aligned, 1), \
                (f"broadcast to {target} from {source} cannot align source axis {axis} "
                 f"of extent {extent} to extent {aligned}")
        if int(np.prod(source)) == 1:
            return self.broadcast_like(self.literal(counted(target, 0)))
        current = self if offset == 0 else self.reshape((1,) * offset + source)
        for axis in range(len(target)):
            if current.shape[axis] == target[axis]:
                continue
            widened = list(current.shape)
            widened[axis] = target[axis]
            current = current.squeeze(axis).broadcast_along(
                axis, self.literal(counted(tuple(widened), 0)))
        return current


def concat(values: Sequence[Value], axis: int) -> Value:
    """`graph/composite.rs:142-176`: the sum of zero-padded windows."""
    assert values, "concat needs at least one value"
    first = values[0]
    assert axis < len(first.shape), f"concat axis {axis} is out of rank for {first.shape}"
    for v in values:
        off = [e for i, e in enumerate(v.shape) if i != axis]
        assert len(v.shape) == len(first.shape) and off == [
            e for i, e in enumerate(first.shape) if i != axis], \
            "concat needs equal shapes off the axis"
    if len(values) == 1:
        return first
    combined = sum(v.shape[axis] for v in values)
    offset = 0
    total = None
    for v in values:
        padded = v.pad(axis, offset, combined)
        offset += v.shape[axis]
        total = padded if total is None else total + padded
    return total


def stack(values: Sequence[Value], axis: int) -> Value:
    return concat([v.unsqueeze(axis) for v in values], axis)


def _swapped(value: Value) -> Value:
    """`function/matmul.rs:87-96`."""
    rank = len(value.shape)
    if rank <= 2:
        return value.transpose()
    order = list(range(rank))
    order[rank - 2], order[rank - 1] = order[rank - 1], order[rank - 2]
    return value.permute(order)


def _inverse(order):
    inverse = [0] * len(order)
    for position, axis in enumerate(order):
        inverse[axis] = position
    return inverse


def backward_rule(node: Node, ops: List[Value], out: Value, g: Value):
    """Each operation's cotangents, recorded in the same evaluation order as
    the reference rules (files under `function/`, `backward`)."""
    name = node.name
    a = node.attrs
    if name == "Add":  # add.rs:40-42
        return [g, g]
    if name == "Sub":  # sub.rs:41-43
        return [g, -g]
    if name == "Mul":  # mul.rs:46-52
        return [g * ops[1], g * ops[0]]
    if name == "Div":  # div.rs:46-52
        return [g / ops[1], -((g * out) / ops[1])]
    if name == "Neg":
        return [-g]
    if name == "Tanh":  # tanh.rs:40-44
        one = out.one_like()
        derivative = one - out * out
        return [g * derivative]
    if name == "Exp":
        return [g * out]
    if name == "Ln":
        return [g / ops[0]]
    if name == "Sqrt":  # sqrt.rs:42-45
        return [g / (out + out)]
    if name == "Powf":  # powf.rs:47-54
        base, exponent = ops
        lowered = exponent - exponent.one_like()
        base_cot = (g * exponent) * base.powf(lowered)
        exp_cot = (g * out) * base.ln()
        return [base_cot, exp_cot]
    if name == "Maximum":  # maximum.rs:45-51
        winners = ops[0].step(ops[1])
        left = g * winners
        right = g * (winners.one_like() - winners)
        return [left, right]
    if name == "Relu":  # relu.rs:47-50
        zero = ops[0].zero_like()
        return [g * ops[0].step(zero)]
    if name == "Step":
        return [None, None]
    if name == "MatMul":  # matmul.rs:76-82
        left, right = ops
        return [g.matmul(_swapped(right)), _swapped(left).matmul(g)]
    if name == "Transpose":
        return [g.transpose()]
    if name == "Sum":
        return [g.broadcast_like(ops[0])]
    if name == "SumAlong":
        return [g.broadcast_along(a[0], ops[0])]
    if name == "Broadcast":
        return [g.sum().broadcast_like(ops[0]), None]
    if name == "BroadcastAlong":
        return [g.sum_along(a[0]), None]
    if name == "Reshape":
        return [g.reshape(ops[0].shape)]
    if name == "Permute":
        return [g.permute(_inverse(a))]
    if name == "Narrow":
        return [g.pad(a[0], a[1], ops[0].shape[a[0]])]
    if name == "Pad":
        return [g.narrow(a[0], a[1], ops[0].shape[a[0]])]
    if name == "Unfold":
        return [g.fold(a[0], a[1], a[2], a[3], ops[0].shape[a[0]])]
    if name == "Fold":
        return [g.unfold(a[0], a[1], a[2], a[3])]
    if name == "Gather":
        return [g.scatter(ops[1], ops[0].shape[0]), None]
    if name == "Scatter":
        return [g.gather(ops[1]), None]
    if name == "LogSoftmax":  # log_softmax.rs:66-72
        axis = a[0]
        total = g.sum_along(axis).broadcast_along(axis, g)
        return [g - out.exp() * total]
    if name == "LogSumExp":  # log_sum_exp.rs:66-74
        axis = a[0]
        probabilities = (ops[0] - out.broadcast_along(axis, ops[0])).exp()
        return [g.broadcast_along(axis, ops[0]) * probabilities]
    raise ValueError(f"no backward rule for {name}")
