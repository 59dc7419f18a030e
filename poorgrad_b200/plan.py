"""Plan requests and plan columns: the mirror of topos `engine/request.rs` and
the column half of `Plan::new` (`engine/plan.rs:143-283`).

`PlanColumns` computes exactly what topos's plan compiler computes from a
request: the ``wanted`` ancestor closure of roots and observes (154-172), the
``readable`` set, the read contract ``required`` of training plans from
`Function::reads` (201-225) and the last-consumer ``releases`` (226-268).
These columns, with the node columns of the network, are the input of the
B200 backend (`tb_plan_compile`) and of the CPU oracle.
"""
from __future__ import annotations

from typing import Iterable, List

from .graph import OPS, READS, NOTHING, Network, Value

FAST, EXACT = 0, 1


def _index(symbol) -> int:
    return symbol.index if isinstance(symbol, Value) else int(symbol)


class Request:
    """`engine/request.rs:36-88`."""

    def __init__(self, roots: Iterable, observe: Iterable = (), backward: bool = False,
                 numerics: int = FAST):
        self.roots = [_index(r) for r in roots]
        self.observe_ = [_index(o) for o in observe]
        self.backward_ = backward
        self.numerics_ = numerics

    @classmethod
    def of(cls, roots):
        return cls(roots)

    def observe(self, extra):
        self.observe_.extend(_index(o) for o in extra)
        return self

    def backward(self):
        self.backward_ = True
        return self

    def numerics(self, numerics: int):
        self.numerics_ = numerics
        return self


class PlanColumns:
    """The compiled columns of one request over one network."""

    def __init__(self, network: Network, request: Request):
        nodes = network.nodes
        length = len(nodes)
        self.network = network
        self.nodes = nodes
        self.roots = list(request.roots)
        self.observed = list(request.observe_)
        self.backward = bool(request.backward_)
        self.numerics = int(request.numerics_)
        self.element = int(getattr(network.tape, "element", 0))
        wanted = [False] * length
        readable = [False] * length
        for index in self.roots + self.observed:
            wanted[index] = True
            readable[index] = True
        for index in range(length - 1, -1, -1):
            if wanted[index]:
                for link in nodes[index].operands:
                    wanted[link] = True
        required = list(readable)
        if self.backward:
            for index in range(length):
                if not wanted[index]:
                    continue
                reads = READS.get(OPS[nodes[index].op], NOTHING)
                if reads[2]:
                    required[index] = True
                for position, link in enumerate(nodes[index].operands):
                    if reads[position]:
                        required[link] = True
        last_consumer: List[int] = [-1] * length
        for index in range(length):
            if wanted[index]:
                for link in nodes[index].operands:
                    last_consumer[link] = index
        releases: List[List[int]] = [[] for _ in range(length)]
        for slot in range(length):
            if not wanted[slot] or readable[slot] or required[slot]:
                continue
            if last_consumer[slot] >= 0:
                releases[last_consumer[slot]].append(slot)
        self.wanted = wanted
        self.readable = readable
        self.required = required
        self.releases = releases

    def __len__(self):
        return len(self.nodes)

    def describe(self) -> str:
        """A per-node listing in the spirit of `Plan::describe`
        (`engine/plan.rs:408-490`)."""
        lines = []
        for index, node in enumerate(self.nodes):
            if not self.wanted[index]:
                continue
            mark = "R" if self.readable[index] else " "
            lines.append(f"{index:6d} {mark} {node.name:<14} {list(node.operands)!s:<14} "
                         f"{node.shape} rel={self.releases[index]}")
        return "\n".join(lines)
