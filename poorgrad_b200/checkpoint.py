"""Checkpoints of a module's parameters (`neural/checkpoint.rs`,
`neural/module.rs:109-160`), for host or device-resident state.

A module announces its parameters through ``visit(visitor)``: the visitor sees
``parameter(name, symbol)`` per parameter and ``enter(segment)`` / ``leave()``
around each nested stage.  ``snapshot``/``restore`` identify parameters by
position in that order; ``named_snapshot``/``named_restore`` by dotted path
("0.weights").

``state`` is either host parameters (a list of arrays indexed by parameter
slot, as ``Network.parameters()`` returns) or ``backend.DeviceParameters``,
which are read and written on the device in place.  Optimizer state travels
separately (``backend.Optimizer.state_snapshot`` / ``state_restore``).
"""
from __future__ import annotations

from typing import Dict, Iterable, List, Sequence, Tuple

import numpy as np


class _Collector:
    def __init__(self):
        self.stack: List = []
        self.named: List[Tuple[str, object]] = []

    def parameter(self, name, symbol):
        self.named.append((".".join(str(s) for s in self.stack + [name]), symbol))

    def enter(self, segment):
        self.stack.append(segment)

    def leave(self):
        self.stack.pop()


def named_parameters(module) -> List[Tuple[str, object]]:
    """(path, symbol) per announced parameter, in visit order."""
    collector = _Collector()
    module.visit(collector)
    return collector.named


def parameters(module) -> List[object]:
    return [symbol for _, symbol in named_parameters(module)]


def _slot(symbol) -> int:
    return symbol.tape.nodes[symbol.index].slot


def _device(state) -> bool:
    return hasattr(state, "download") and hasattr(state, "upload")


def _read(state, symbol) -> np.ndarray:
    if _device(state):
        return state.download(_slot(symbol))
    return np.array(state[_slot(symbol)], dtype=np.float32, copy=True).reshape(symbol.shape)


def _with_payloads(state, replacements: Iterable[Tuple[object, np.ndarray]]):
    if _device(state):
        for symbol, payload in replacements:
            _upload(state, _slot(symbol), symbol, payload)
        return state
    out = [np.array(p, copy=True) for p in state]
    for symbol, payload in replacements:
        payload = np.asarray(payload, np.float32)
        assert payload.size == int(np.prod(symbol.shape)), "payload size disagrees with the parameter"
        out[_slot(symbol)] = payload.reshape(np.shape(out[_slot(symbol)])).copy()
    return out


def _upload(state, slot, symbol, payload):
    payload = np.ascontiguousarray(payload, np.float32)
    assert payload.size == int(np.prod(symbol.shape)), "payload size disagrees with the parameter"
    from . import abi
    from .backend import _check
    _check(state.lib.tb_params_upload(state.handle, slot, abi.fptr(payload.reshape(-1)),
                                      payload.size), "tb_params_upload")


def snapshot(state, module) -> List[np.ndarray]:
    """`checkpoint::snapshot` (checkpoint.rs): the payloads in visit order."""
    return [_read(state, symbol) for symbol in parameters(module)]


def restore(state, module, payloads: Sequence[np.ndarray]):
    """`checkpoint::restore`: the payloads, by position, into a state of the
    same topology; host state is returned as a new list, device state is
    written in place and returned."""
    symbols = parameters(module)
    assert len(payloads) == len(symbols), \
        (f"the checkpoint holds {len(payloads)} payloads but the module has "
         f"{len(symbols)} parameters")
    return _with_payloads(state, zip(symbols, payloads))


def named_snapshot(state, module) -> List[Tuple[str, np.ndarray]]:
    return [(path, _read(state, symbol)) for path, symbol in named_parameters(module)]


def named_restore(state, module, entries: Iterable[Tuple[str, np.ndarray]]):
    """`checkpoint::named_restore`: every parameter must find its path and
    every entry its parameter; a path announced twice (tied parameters)
    takes the later entry in visit order."""
    remaining: Dict[str, np.ndarray] = dict(entries)
    replacements, missing = [], []
    for path, symbol in named_parameters(module):
        if path in remaining:
            replacements.append((symbol, remaining.pop(path)))
        else:
            missing.append(path)
    assert not missing, f"the checkpoint is missing entries for: {', '.join(missing)}"
    assert not remaining, \
        f"the checkpoint holds entries no parameter matches: {', '.join(remaining)}"
    return _with_payloads(state, replacements)
