"""Python face of the B200 backend: compiled plans, device parameters,
optimizer steps and the data-parallel gradient exchange, all through the C ABI
of ``libtopos_b200.so`` (``include/topos_b200.h``).

The names follow topos: ``Plan::forward`` -> :meth:`DevicePlan.forward`,
``Run::of`` -> :meth:`DevicePlan.of`, ``Parameters`` -> :class:`DeviceParameters`,
``Sgd``/``Adam``/``AdamW`` -> :class:`Optimizer`.  There is no CPU fallback:
every call goes to the CUDA library, and a missing library or device raises.
"""
from __future__ import annotations

import ctypes as C
from typing import Dict, Iterable, Optional, Sequence

import numpy as np

from .abi import (STATUS, Feeds, PackedPlan, TbOptimizerDesc, TbPlanStats, fptr, load_library)
from .plan import PlanColumns

SGD, ADAM, ADAMW = 0, 1, 2


class BackendError(RuntimeError):
    def __init__(self, code: int, what: str):
        self.code = code
        super().__init__(f"{what}: {STATUS.get(code, code)}: {last_error()}")


def last_error() -> str:
    return (load_library().tb_last_error() or b"").decode(errors="replace")


def _check(code: int, what: str):
    if code != 0:
        raise BackendError(code, what)


def status() -> tuple:
    """`Manifest::status` (backend/manifest.rs:16-37): (code, message)."""
    lib = load_library()
    buf = C.create_string_buffer(512)
    code = lib.tb_status(buf, 512)
    return code, buf.value.decode()


def lower_describe(columns: PlanColumns, with_source: bool = False) -> str:
    """Kernel list (and emitted source) of a plan, computed on the host only."""
    lib = load_library()
    fn = lib.tbx_lower_describe
    fn.restype = C.c_int64
    packed = PackedPlan(columns)
    n = fn(C.byref(packed.desc), None, 0, int(with_source))
    if n < 0:
        raise RuntimeError("lowering failed: " + last_error())
    buf = C.create_string_buffer(int(n))
    fn(C.byref(packed.desc), buf, n, int(with_source))
    return buf.value.decode()


def nvrtc_check(columns: PlanColumns) -> None:
    """Compiles a plan's emitted kernels for sm_100a with NVRTC (no device needed)."""
    lib = load_library()
    packed = PackedPlan(columns)
    rc = lib.tbx_nvrtc_check(C.byref(packed.desc))
    if rc != 0:
        raise RuntimeError("NVRTC rejected the emitted kernels:\n" + last_error())


class DeviceParameters:
    """Device-resident ``Parameters`` of a plan's network."""

    def __init__(self, plan: "DevicePlan", payloads: Optional[Sequence[np.ndarray]] = None):
        self.lib = load_library()
        self.handle = C.c_void_p()
        _check(self.lib.tb_params_create(plan.handle, C.byref(self.handle)), "tb_params_create")
        self.shapes = [plan.columns.network.tape.parameter_payloads[s].shape
                       for s in range(len(plan.columns.network.tape.parameter_payloads))]
        if payloads is not None:
            self.upload(payloads)

    def upload(self, payloads: Sequence[np.ndarray]):
        for slot, p in enumerate(payloads):
            a = np.ascontiguousarray(p, dtype=np.float32).reshape(-1)
            _check(self.lib.tb_params_upload(self.handle, slot, fptr(a), a.size), "tb_params_upload")

    def download(self, slot: int) -> np.ndarray:
        shape = self.shapes[slot]
        out = np.empty(shape, dtype=np.float32)
        _check(self.lib.tb_params_download(self.handle, slot, fptr(out), out.size),
               "tb_params_download")
        return out

    def __del__(self):
        if getattr(self, "handle", None):
            self.lib.tb_params_destroy(self.handle)
            self.handle = None


class DevicePlan:
    """A compiled plan lowered to a B200 device program."""

    def __init__(self, columns: PlanColumns):
        self.lib = load_library()
        self.columns = columns
        self.packed = PackedPlan(columns)
        self.handle = C.c_void_p()
        _check(self.lib.tb_plan_compile(C.byref(self.packed.desc), C.byref(self.handle)),
               "tb_plan_compile")
        self._feeds = None

    def forward(self, params: DeviceParameters, feeds: Optional[Dict] = None, sync: bool = False):
        """`Plan::forward`: enqueues one run (feeds copied in, then the CUDA graph)."""
        self._feeds = Feeds(self.columns, feeds or {})  # keep host arrays alive until the copy
        _check(self.lib.tb_plan_run(self.handle, params.handle, self._feeds.count,
                                    self._feeds.array), "tb_plan_run")
        if sync:
            self.synchronize()
        return self

    def synchronize(self):
        _check(self.lib.tb_plan_synchronize(self.handle), "tb_plan_synchronize")

    def begin(self, params: DeviceParameters, feeds: Optional[Dict] = None) -> "DeviceRun":
        """`Plan::forward` from any thread: a run on its own pooled instance
        (stream, arena, inputs), so runs of one plan proceed concurrently."""
        return DeviceRun(self, params, feeds)

    def of(self, symbol) -> np.ndarray:
        """`Run::of`: a readable value, copied to the host."""
        index = symbol.index if hasattr(symbol, "index") else int(symbol)
        out = np.empty(self.columns.nodes[index].shape, dtype=np.float32)
        _check(self.lib.tb_plan_read(self.handle, index, fptr(out), max(out.size, 1)),
               "tb_plan_read")
        return out

    def read_async(self, symbol, host_pointer: int, count: int):
        """`Run::of` without waiting: enqueues the copy of a readable value to
        page-locked host memory at ``host_pointer`` (``count`` floats) on the
        plan's stream; it is there once the stream passes the copy."""
        index = symbol.index if hasattr(symbol, "index") else int(symbol)
        _check(self.lib.tb_plan_read_async(self.handle, index, C.c_void_p(host_pointer), count),
               "tb_plan_read_async")

    def gradient(self, root, parameter) -> np.ndarray:
        """`Run::backward(root)` then `Gradients::of(parameter)` for a plan
        compiled with ``Request(...).backward()``."""
        r = root.index if hasattr(root, "index") else int(root)
        p = parameter.index if hasattr(parameter, "index") else int(parameter)
        node = C.c_int64()
        _check(self.lib.tb_plan_gradient_node(self.handle, r, p, C.byref(node)),
               "tb_plan_gradient_node")
        shape = self.columns.nodes[p].shape
        out = np.empty(shape, dtype=np.float32)
        _check(self.lib.tb_plan_read(self.handle, node.value, fptr(out), max(out.size, 1)),
               "tb_plan_read")
        return out

    def device_pointer(self, symbol) -> int:
        index = symbol.index if hasattr(symbol, "index") else int(symbol)
        ptr = C.c_void_p()
        _check(self.lib.tb_plan_device_pointer(self.handle, index, C.byref(ptr)),
               "tb_plan_device_pointer")
        return ptr.value

    def stream(self) -> int:
        return self.lib.tb_plan_stream(self.handle)

    def stats(self) -> dict:
        s = TbPlanStats()
        _check(self.lib.tb_plan_stats_get(self.handle, C.byref(s)), "tb_plan_stats_get")
        return {name: getattr(s, name) for name, _ in TbPlanStats._fields_}

    def describe(self) -> str:
        n = self.lib.tb_plan_describe(self.handle, None, 0)
        buf = C.create_string_buffer(int(n))
        self.lib.tb_plan_describe(self.handle, buf, n)
        return buf.value.decode()

    def __del__(self):
        if getattr(self, "handle", None):
            self.lib.tb_plan_destroy(self.handle)
            self.handle = None


class DeviceRun:
    """A run drawn from a plan's instance pool (the reference's `Run`): its
    readable values stay available until it is released (or collected)."""

    def __init__(self, plan: DevicePlan, params: DeviceParameters, feeds: Optional[Dict]):
        self.plan = plan
        self.lib = plan.lib
        self._feeds = Feeds(plan.columns, feeds or {})
        self.handle = C.c_void_p()
        _check(self.lib.tb_run_begin(plan.handle, params.handle, self._feeds.count,
                                     self._feeds.array, C.byref(self.handle)), "tb_run_begin")

    def synchronize(self):
        _check(self.lib.tb_run_synchronize(self.handle), "tb_run_synchronize")
        return self

    def of(self, symbol) -> np.ndarray:
        """`Run::of`: a readable value of this run, copied to the host."""
        index = symbol.index if hasattr(symbol, "index") else int(symbol)
        out = np.empty(self.plan.columns.nodes[index].shape, dtype=np.float32)
        _check(self.lib.tb_run_read(self.handle, index, fptr(out), max(out.size, 1)),
               "tb_run_read")
        return out

    def release(self):
        if getattr(self, "handle", None):
            self.lib.tb_run_release(self.handle)
            self.handle = None

    def __del__(self):
        self.release()


class Optimizer:
    """A device optimizer step bound to a plan's gradient outputs:
    SGD (`neural/optimizer.rs:40-51`), Adam and AdamW (`neural/adam.rs`)."""

    def __init__(self, plan: DevicePlan, params: DeviceParameters, kind: int,
                 pairs: Iterable, learning_rate: float, beta1: float = 0.9,
                 beta2: float = 0.999, epsilon: float = 1e-8, decay: float = 0.0,
                 gradient_scale: float = 1.0, attach: bool = True):
        self.lib = load_library()
        self.plan = plan
        pairs = list(pairs)
        slots = (C.c_int32 * max(1, len(pairs)))()
        nodes = (C.c_int64 * max(1, len(pairs)))()
        nodes_tape = plan.columns.nodes
        for i, (param, grad) in enumerate(pairs):
            pi = param.index if hasattr(param, "index") else int(param)
            gi = grad.index if hasattr(grad, "index") else int(grad)
            slots[i] = nodes_tape[pi].slot
            nodes[i] = gi
        self.slots = [slots[i] for i in range(len(pairs))]
        desc = TbOptimizerDesc(kind, learning_rate, beta1, beta2, epsilon, decay, gradient_scale)
        self.handle = C.c_void_p()
        _check(self.lib.tb_optimizer_create(plan.handle, params.handle, C.byref(desc), len(pairs),
                                            slots, nodes, C.byref(self.handle)),
               "tb_optimizer_create")
        if attach:
            _check(self.lib.tb_plan_attach_optimizer(plan.handle, self.handle),
                   "tb_plan_attach_optimizer")
        self.params = params

    def step(self, gradients=None, stream: int = 0):
        """`Parameters::step(&gradients, &mut optimizer)` now: with the plan's
        last gradients (``None``) or with one device pointer per bound slot."""
        arr = None
        if gradients is not None:
            ptrs = [int(g) for g in gradients]
            arr = (C.c_void_p * len(ptrs))(*ptrs)
        _check(self.lib.tb_optimizer_step(self.handle, arr, C.c_void_p(stream) if stream else None),
               "tb_optimizer_step")

    def set_learning_rate(self, lr: float):
        _check(self.lib.tb_optimizer_set_learning_rate(self.handle, lr), "set_learning_rate")

    def moments(self, slot: int):
        shape = self.params.shapes[slot]
        m = np.empty(shape, np.float32)
        v = np.empty(shape, np.float32)
        _check(self.lib.tb_optimizer_state(self.handle, slot, fptr(m), fptr(v), m.size),
               "tb_optimizer_state")
        return m, v

    def state_snapshot(self) -> dict:
        """The Adam/AdamW state a resumed run needs: per bound slot its
        moments, and the beta powers (``beta1^t``, ``beta2^t``)."""
        powers = (C.c_float * 2)()
        _check(self.lib.tb_optimizer_powers(self.handle, powers), "tb_optimizer_powers")
        return {"moments": {slot: self.moments(slot) for slot in self.slots},
                "powers": (powers[0], powers[1])}

    def state_restore(self, state: dict):
        """Writes a ``state_snapshot`` back: the next step continues the saved
        trajectory."""
        for slot, (m, v) in state["moments"].items():
            m = np.ascontiguousarray(m, np.float32).reshape(-1)
            v = np.ascontiguousarray(v, np.float32).reshape(-1)
            _check(self.lib.tb_optimizer_restore(self.handle, slot, fptr(m), fptr(v), m.size),
                   "tb_optimizer_restore")
        powers = (C.c_float * 2)(*state["powers"])
        _check(self.lib.tb_optimizer_restore_powers(self.handle, powers),
               "tb_optimizer_restore_powers")

    def __del__(self):
        if getattr(self, "handle", None):
            self.lib.tb_optimizer_destroy(self.handle)
            self.handle = None


class Comm:
    """An NCCL communicator over this process's GPU (one process per GPU)."""

    def __init__(self, rank: int, world: int, unique_id: bytes):
        self.lib = load_library()
        buf = (C.c_uint8 * 128).from_buffer_copy(unique_id)
        self.handle = C.c_void_p()
        _check(self.lib.tb_comm_init(rank, world, buf, C.byref(self.handle)), "tb_comm_init")
        self.rank, self.world = rank, world

    @staticmethod
    def unique_id() -> bytes:
        lib = load_library()
        buf = (C.c_uint8 * 128)()
        _check(lib.tb_comm_unique_id(buf), "tb_comm_unique_id")
        return bytes(buf)

    def attach(self, plan: DevicePlan, bucket_bytes: int = 32 << 20, reduction: str = "nccl"):
        """Sums the plan's optimizer-bound gradients across ranks before its
        optimizer step: ``reduction="nccl"`` (ncclAllReduce) or ``"tree"``
        (all-gather, then `tree_sum`'s pairwise order over ranks: bit-identical
        to the reference's host sum of the same shard gradients)."""
        _check(self.lib.tb_plan_attach_comm(plan.handle, self.handle, bucket_bytes),
               "tb_plan_attach_comm")
        code = {"nccl": 0, "tree": 1}[reduction]
        _check(self.lib.tb_plan_set_reduction(plan.handle, code), "tb_plan_set_reduction")

    def __del__(self):
        if getattr(self, "handle", None):
            self.lib.tb_comm_destroy(self.handle)
            self.handle = None


def gemm_f32(a: np.ndarray, b: np.ndarray) -> Optional[np.ndarray]:
    """The per-task GEMM face (`Elementary::gemm`); None when declined."""
    lib = load_library()
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    m, k = a.shape
    n = b.shape[1]
    sa = (C.c_int64 * 2)(a.strides[0] // 4, a.strides[1] // 4)
    sb = (C.c_int64 * 2)(b.strides[0] // 4, b.strides[1] // 4)
    base_a = np.lib.stride_tricks.as_strided(a, shape=(a.size,), strides=(4,)) if a.flags.c_contiguous else a
    out = np.empty((m, n), dtype=np.float32)
    ap = a.ctypes.data_as(C.POINTER(C.c_float))
    bp = b.ctypes.data_as(C.POINTER(C.c_float))
    span_a = (m - 1) * sa[0] + (k - 1) * sa[1] + 1
    span_b = (k - 1) * sb[0] + (n - 1) * sb[1] + 1
    del base_a
    rc = lib.tb_gemm_f32(ap, span_a, sa, bp, span_b, sb, m, k, n, fptr(out))
    if rc == 5:
        return None
    _check(rc, "tb_gemm_f32")
    return out
