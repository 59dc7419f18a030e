"""Host-side emulation of a lowered device program -- TEST INFRASTRUCTURE.

Runs a plan's device program on the CPU so that the tests can check what the
lowering emits without a GPU: the generated kernels are compiled as host C++
against `kernel_emulator.h` (one OS thread per CUDA thread), and the library
kernels are restated here in numpy from their contracts:

- GEMM: the 3xTF32 product of the prepared hi/lo pairs (hi·hi + hi·lo +
  lo·hi), summed in f64 and rounded once to f32 -- within the tolerance the
  device parity tests give the tensor-core kernel;
- selection sort: a stable sort of the indices, with each row's segment;
- segment sums: each row summed from zero in sorted (source) order, in f32;
- column finals: the per-block partials summed in f32.

Buffers start as the runtime stages them (parameters, feeds or initial
payloads, leaves), and the arena's buffers sit at their planned offsets in one
array, as on the device: a buffer reused while still live clobbers a value and
shows as a wrong result.  The product never uses this module.
"""
from __future__ import annotations

import ctypes as C
import hashlib
import json
import os
import subprocess
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ARENA, PARAMETER, INPUT, LEAF, INPUT_INDICES, LEAF_INDICES = range(6)


def lowered(columns) -> dict:
    """The lowered program of `columns` (`tbx_lower_json`)."""
    from poorgrad_b200.abi import PackedPlan, load_library
    from poorgrad_b200.backend import last_error
    lib = load_library()
    fn = lib.tbx_lower_json
    fn.restype = C.c_int64
    packed = PackedPlan(columns)
    n = fn(C.byref(packed.desc), None, 0)
    if n < 0:
        raise RuntimeError("lowering failed: " + last_error())
    buf = C.create_string_buffer(int(n))
    fn(C.byref(packed.desc), buf, n)
    return json.loads(buf.value.decode())


def _host_source(source: str, names) -> str:
    out = []
    for line in source.splitlines():
        if 'asm volatile("griddepcontrol' in line:
            continue
        if 'asm("cvt.rna.tf32.f32' in line:
            line = "  r = emu_tf32_bits(x);"
        if 'asm volatile("bar.sync' in line:
            # a team's named barrier: every team of a block reaches its own
            # the same number of times, so a block barrier stands in for it
            line = "    __syncthreads();"
        if 'asm("rcp.approx.f32' in line:
            # the hardware reciprocal estimate, restated as the rounded reciprocal
            line = "  r = 1.0f / y;"
        out.append(line)
    for name in sorted(names):
        out.append(
            f'extern "C" void emu_run_{name}(void** p, int np, long grid, unsigned block) {{\n'
            f"  P_{name} prm;\n"
            f"  for (int i = 0; i < np; ++i) prm.p[i] = p[i];\n"
            f"  emu_launch(grid, block, [&]() {{ {name}(prm); }});\n"
            f"}}")
    return '#include "kernel_emulator.h"\n' + "\n".join(out) + "\n"


_CACHE = {}


def compiled(source: str, names) -> C.CDLL:
    """The generated kernels built as a host library (cached by source)."""
    text = _host_source(source, names)
    with open(os.path.join(HERE, "kernel_emulator.h")) as f:
        header = f.read()
    key = hashlib.sha1((header + text).encode()).hexdigest()[:16]
    if key in _CACHE:
        return _CACHE[key]
    work = os.path.join(tempfile.gettempdir(), "tb_kernel_emulator")
    os.makedirs(work, exist_ok=True)
    src = os.path.join(work, key + ".cpp")
    lib = os.path.join(work, key + ".so")
    if not os.path.exists(lib):
        with open(src, "w") as f:
            f.write(text)
        subprocess.check_call(
            ["g++", "-std=c++20", "-O1", "-ffp-contract=off", "-fno-fast-math", "-fPIC",
             "-shared", "-pthread", "-w", "-I", HERE, "-o", lib + ".tmp", src])
        os.replace(lib + ".tmp", lib)
    _CACHE[key] = C.CDLL(lib)
    return _CACHE[key]


def _round_bf16(x):
    import oracle
    return oracle.round_bf16(x)


def _tf32_pair(x):
    """hi = x rounded to tf32 (nearest, ties away from zero), lo = x - hi: the
    pair a GEMM splits a raw f32 operand into."""
    bits = x.view(np.uint32)
    hi = ((bits + np.uint32(0x1000)) & np.uint32(0xFFFFE000)).view(np.float32)
    hi = np.where(np.isfinite(x), hi, x).astype(np.float32)
    return hi, (x - hi).astype(np.float32)


def _operand(hi, lo, mn, ld, rows, batch, outer, inner):
    """The operand matrices [batch, outer, inner] from a prepared pair, or
    from raw f32 values (``lo`` None) split the way the GEMM splits them."""
    if lo is None:
        hi, lo = _tf32_pair(np.ascontiguousarray(hi[: batch * rows * ld]))
    h = hi[: batch * rows * ld].reshape(batch, rows, ld).astype(np.float64)
    l_ = lo[: batch * rows * ld].reshape(batch, rows, ld).astype(np.float64)
    if mn:  # stored [inner][outer]
        return h[:, :inner, :outer].transpose(0, 2, 1), l_[:, :inner, :outer].transpose(0, 2, 1)
    return h[:, :outer, :inner], l_[:, :outer, :inner]


def run_program(columns, parameters, feeds=None, gradients=False):
    """Runs the lowered program of `columns` on the host; returns
    ``{node_index: ndarray}`` for every readable value (the lowered program's
    node numbering: an engine-backward plan's gradients are appended nodes).
    With ``gradients``, also ``{(root, parameter): node}`` of such a plan."""
    from poorgrad_b200.graph import Constant, Dense, Selection
    prog = lowered(columns)
    kernels, buffers = prog["kernels"], prog["buffers"]
    names = {k["name"] for k in kernels if k["name"]}
    lib = compiled(prog["source"], names)
    nodes = columns.nodes
    fed = {}
    for sym, payload in (feeds or {}).items():
        fed[sym.index if hasattr(sym, "index") else int(sym)] = payload

    def payload_array(node, payload):
        if isinstance(payload, Selection):
            return np.ascontiguousarray(payload.indices, np.int32)
        if isinstance(payload, Constant):
            return np.full(int(np.prod(node.shape)) or 1, float(payload.value), np.float32)
        if isinstance(payload, Dense):
            return np.ascontiguousarray(payload.to_numpy(), np.float32).reshape(-1)
        a = np.asarray(payload)
        return np.ascontiguousarray(a, np.int32 if a.dtype == np.int32 else np.float32).reshape(-1)

    arena = np.zeros(max(prog["arena_bytes"], 16), np.uint8)
    mem = []
    for b in buffers:
        st, n = b["storage"], b["node"]
        if st == ARENA and b["placed"]:
            mem.append(arena[b["offset"]: b["offset"] + max(b["bytes"], 4)])
            continue
        raw = np.zeros(max(b["bytes"], 16), np.uint8)
        if st == PARAMETER:
            src = np.ascontiguousarray(parameters[b["slot"]], np.float32).reshape(-1)
        elif st in (INPUT, INPUT_INDICES):
            src = payload_array(nodes[n], fed[n] if n in fed else nodes[n].payload)
        elif st in (LEAF, LEAF_INDICES):
            src = payload_array(nodes[n], nodes[n].payload)
        else:
            src = None
        if src is not None:
            data = src.view(np.uint8)
            raw[: min(len(data), b["bytes"])] = data[: b["bytes"]]
        mem.append(raw)
    f32 = lambda i: mem[i].view(np.float32)
    i32 = lambda i: mem[i].view(np.int32)

    for K in kernels:
        t = K["type"]
        if K["name"]:
            ptrs = (C.c_void_p * max(1, len(K["params"])))(
                *[mem[b].ctypes.data for b in K["params"]])
            getattr(lib, "emu_run_" + K["name"])(ptrs, len(K["params"]), C.c_long(K["grid"]),
                                                 C.c_uint(K["block"]))
        elif t == "gemm":
            batch, m, n, k = K["batch"], K["m"], K["n"], K["k"]
            lo_of = lambda b: f32(b) if b >= 0 else None
            ah, al = _operand(f32(K["a_hi"]), lo_of(K["a_lo"]), K["a_mn"], K["a_ld"],
                              K["a_rows"], batch, m, k)
            # B is [k, n]: MN-major B stores it row-major, K-major B stores [n][k]
            bh, bl = _operand(f32(K["b_hi"]), lo_of(K["b_lo"]), not K["b_mn"], K["b_ld"],
                              K["b_rows"], batch, k, n)
            c = ah @ bh + ah @ bl + al @ bh
            f32(K["out"])[: batch * m * n] = c.astype(np.float32).reshape(-1)
        elif t == "sort":
            idx = i32(K["out"])[: K["count"]]
            order = np.argsort(idx, kind="stable").astype(np.int32)
            keys = idx[order]
            i32(K["keys"])[: K["count"]] = keys
            i32(K["vals"])[: K["count"]] = order
            rs, re_ = i32(K["rstart"]), i32(K["rend"])
            rs[: K["rows"]] = 0
            re_[: K["rows"]] = 0
            for r in np.unique(keys):
                where = np.nonzero(keys == r)[0]
                rs[r], re_[r] = where[0], where[-1] + 1
        elif t == "segsum":
            width, rows = K["final_width"], K["rows"]
            perm = f32(K["partial"])[: K["count"] * width].reshape(K["count"], width)
            out = np.zeros((rows, width), np.float32)
            rs, re_ = i32(K["rstart"]), i32(K["rend"])
            for r in range(rows):
                for q in range(rs[r], re_[r]):
                    out[r] = out[r] + perm[q]
            f32(K["final_out"])[: rows * width] = out.reshape(-1)
        elif t == "final":
            entries = (list(zip(K["final_parts"], K["final_outs"], K["final_widths"]))
                       or [(K["partial"], K["final_out"], K["final_width"])])
            for part, out, width in entries:
                p = f32(part)[: K["final_blocks"] * width].reshape(K["final_blocks"], width)
                total = np.zeros(width, np.float32)
                for row in p:
                    total = total + row
                f32(out)[:width] = total
        else:
            raise NotImplementedError(f"kernel type {t}")

    results = {}
    for node, (b, shape) in prog["readable"].items():
        shape = tuple(shape)
        v = f32(b)[: int(np.prod(shape)) if shape else 1].copy().reshape(shape)
        results[int(node)] = _round_bf16(v) if prog["bf16"] else v
    if gradients:
        return results, {(r, p): n for r, p, n in prog["gradients"]}
    return results
