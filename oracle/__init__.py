"""CPU parity oracle for the topos B200 backend -- TEST INFRASTRUCTURE.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this package, and only as the checker (or the timed reference
CPU path).  The product never imports it.

``oracle.cpp`` restates the topos default-build interpreter (see its header
for the reference file:line each part follows); ``run`` executes a packed plan
descriptor on the host and returns the requested values, and ``backward`` runs
the engine's reverse scan over them.  ``optim.py`` restates the optimizers.  The reference is
Rust and cannot be built here (no cargo/rustc), so parity of this restatement
is pinned by the known-answer assertions of the reference's own test files
(``tests/test_oracle_pins.py``).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")


def build(force: bool = False) -> str:
    """Compiles ``oracle.cpp`` with the interpreter's arithmetic flags:
    no contraction, no fast-math."""
    src = os.path.join(HERE, "oracle.cpp")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.check_call([
            "g++", "-O2", "-std=c++17", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-pthread",
            "-shared", "-o", LIB_PATH, src])
    return LIB_PATH


_LIB = None


def lib():
    global _LIB
    if _LIB is None:
        build()
        _LIB = C.CDLL(LIB_PATH)
        _LIB.oracle_run.restype = C.c_int
        _LIB.oracle_backward.restype = C.c_int
        _LIB.oracle_last_error.restype = C.c_char_p
        _LIB.oracle_gemm.restype = None
        _LIB.oracle_map.restype = None
        _LIB.oracle_round_bf16.restype = None
        _LIB.oracle_set_threads.restype = None
    return _LIB


def set_threads(threads: int) -> None:
    """Host threads for the oracle's GEMMs (default 1, the interpreter's own
    single thread).  Each output row stays one serial chain, so the results
    are bit-identical for every thread count."""
    lib().oracle_set_threads(C.c_int(int(threads)))


def run(columns, parameters, feeds=None, read=None):
    """Runs ``columns`` (a ``PlanColumns``) on the CPU and returns
    ``{node_index: ndarray}`` for each node in ``read`` (default: the readable
    nodes)."""
    from poorgrad_b200.abi import PackedPlan, Feeds, fptr
    packed = PackedPlan(columns)
    feeds = Feeds(columns, feeds or {})
    params = [np.ascontiguousarray(p, dtype=np.float32).reshape(-1) for p in parameters]
    param_ptrs = (C.POINTER(C.c_float) * max(1, len(params)))(*[fptr(p) for p in params])
    if read is None:
        read = [i for i, r in enumerate(columns.readable) if r]
    read = [r.index if hasattr(r, "index") else int(r) for r in read]
    outs = [np.empty(columns.nodes[r].shape, dtype=np.float32) for r in read]
    out_ptrs = (C.POINTER(C.c_float) * max(1, len(outs)))(*[fptr(o) for o in outs])
    nodes = (C.c_int64 * max(1, len(read)))(*read)
    rc = lib().oracle_run(C.byref(packed.desc), param_ptrs, len(params), feeds.count,
                          feeds.array, len(read), nodes, out_ptrs)
    if rc != 0:
        raise RuntimeError("oracle: " + lib().oracle_last_error().decode())
    return dict(zip(read, outs))


def backward(columns, parameters, root, nodes, feeds=None):
    """The engine's reverse scan (`Run::backward`, engine/run.rs:229-318) from
    scalar ``root`` over the plan's forward values; returns the gradient of
    each of ``nodes`` in order (zeros for non-ancestors)."""
    from poorgrad_b200.abi import PackedPlan, Feeds, fptr
    packed = PackedPlan(columns)
    feeds = Feeds(columns, feeds or {})
    params = [np.ascontiguousarray(p, dtype=np.float32).reshape(-1) for p in parameters]
    param_ptrs = (C.POINTER(C.c_float) * max(1, len(params)))(*[fptr(p) for p in params])
    nodes = [n.index if hasattr(n, "index") else int(n) for n in nodes]
    outs = [np.empty(columns.nodes[n].shape, dtype=np.float32) for n in nodes]
    out_ptrs = (C.POINTER(C.c_float) * max(1, len(outs)))(*[fptr(o) for o in outs])
    index = (C.c_int64 * max(1, len(nodes)))(*nodes)
    root = root.index if hasattr(root, "index") else int(root)
    rc = lib().oracle_backward(C.byref(packed.desc), param_ptrs, len(params), feeds.count,
                               feeds.array, C.c_int64(root), len(nodes), index, out_ptrs)
    if rc != 0:
        raise RuntimeError("oracle: " + lib().oracle_last_error().decode())
    return outs


def gemm(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """The interpreter's serial-k GEMM (payload/gemm.rs:140-211)."""
    from poorgrad_b200.abi import fptr
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), dtype=np.float32)
    lib().oracle_gemm(fptr(a), fptr(b), fptr(c), C.c_int64(m), C.c_int64(k), C.c_int64(n))
    return c


def round_bf16(x: np.ndarray) -> np.ndarray:
    """`Bf16::from_f32(x).to_f32()` per element."""
    from poorgrad_b200.abi import fptr
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    lib().oracle_round_bf16(fptr(x), C.c_int64(x.size), fptr(out))
    return out


def libm_map(op: int, x: np.ndarray) -> np.ndarray:
    from poorgrad_b200.abi import fptr
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    lib().oracle_map(C.c_int32(op), fptr(x), C.c_int64(x.size), fptr(out))
    return out
