"""ctypes mirror of ``include/topos_b200.h`` and the packing of plan columns
into its ``tb_plan_desc``.

The same descriptor feeds the B200 library (``libtopos_b200.so``) and the CPU
oracle, so both see byte-identical requests.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from .graph import OP, Constant, Dense, Selection

MAX_RANK = 8
PAYLOAD_NONE, PAYLOAD_DENSE, PAYLOAD_CONSTANT, PAYLOAD_SELECTION = 0, 1, 2, 3

STATUS = {0: "ok", 1: "NotCompiled", 2: "PlatformUnsupported", 3: "Initialization",
          4: "Poisoned", 5: "Declined", 6: "Invalid", 7: "Runtime"}


class TbNode(C.Structure):
    _fields_ = [
        ("op", C.c_int32), ("rank", C.c_int32), ("shape", C.c_int64 * MAX_RANK),
        ("operands", C.c_int32 * 2), ("attrs", C.c_int64 * MAX_RANK),
        ("slot", C.c_int32), ("payload", C.c_int32), ("constant", C.c_float),
        ("vocab", C.c_int32), ("dense", C.POINTER(C.c_float)),
        ("indices", C.POINTER(C.c_int32)), ("wanted", C.c_uint8), ("readable", C.c_uint8),
        ("required", C.c_uint8), ("reserved", C.c_uint8),
    ]


class TbPlanDesc(C.Structure):
    _fields_ = [("node_count", C.c_int64), ("nodes", C.POINTER(TbNode)),
                ("backward", C.c_int32), ("numerics", C.c_int32), ("element", C.c_int32)]


class TbFeed(C.Structure):
    _fields_ = [("slot", C.c_int32), ("on_device", C.c_int32),
                ("dense", C.POINTER(C.c_float)), ("indices", C.POINTER(C.c_int32))]


class TbPlanStats(C.Structure):
    _fields_ = [("kernels", C.c_int64), ("arena_bytes", C.c_int64),
                ("unplanned_bytes", C.c_int64), ("fused_nodes", C.c_int64),
                ("bit_identical", C.c_int32), ("gemms", C.c_int32)]


class TbOptimizerDesc(C.Structure):
    _fields_ = [("kind", C.c_int32), ("learning_rate", C.c_float), ("beta1", C.c_float),
                ("beta2", C.c_float), ("epsilon", C.c_float), ("decay", C.c_float),
                ("gradient_scale", C.c_float)]


def fptr(array: np.ndarray):
    return array.ctypes.data_as(C.POINTER(C.c_float))


def iptr(array: np.ndarray):
    return array.ctypes.data_as(C.POINTER(C.c_int32))


class PackedPlan:
    """A ``tb_plan_desc`` plus the host arrays it points into (kept alive)."""

    def __init__(self, columns):
        nodes = columns.nodes
        self.columns = columns
        self.array = (TbNode * len(nodes))()
        self._keep = []
        for index, node in enumerate(nodes):
            rec = self.array[index]
            rec.op = node.op
            rec.rank = len(node.shape)
            assert rec.rank <= MAX_RANK, "rank above the ABI maximum"
            for axis, extent in enumerate(node.shape):
                rec.shape[axis] = extent
            rec.operands[0] = node.operands[0] if len(node.operands) > 0 else -1
            rec.operands[1] = node.operands[1] if len(node.operands) > 1 else -1
            for position, value in enumerate(node.attrs):
                rec.attrs[position] = value
            rec.slot = node.slot
            rec.payload = PAYLOAD_NONE
            payload = node.payload
            if node.op in (OP["Leaf"], OP["Input"]) and payload is not None:
                self._payload(rec, payload)
            elif node.op == OP["Parameter"]:
                rec.payload = PAYLOAD_DENSE
            rec.wanted = columns.wanted[index]
            rec.readable = columns.readable[index]
            rec.required = columns.required[index]
        self.desc = TbPlanDesc(len(nodes), self.array, int(columns.backward),
                               int(columns.numerics), int(getattr(columns, "element", 0)))

    def _payload(self, rec, payload):
        if isinstance(payload, Constant):
            rec.payload = PAYLOAD_CONSTANT
            rec.constant = float(payload.value)
        elif isinstance(payload, Selection):
            rec.payload = PAYLOAD_SELECTION
            rec.constant = float(payload.one)
            rec.vocab = payload.vocab
            indices = np.ascontiguousarray(payload.indices, dtype=np.int32)
            self._keep.append(indices)
            rec.indices = iptr(indices)
        elif isinstance(payload, Dense):
            rec.payload = PAYLOAD_DENSE
            data = np.ascontiguousarray(payload.data, dtype=np.float32)
            self._keep.append(data)
            rec.dense = fptr(data)
        else:
            raise TypeError(type(payload))


class Feeds:
    """``tb_feed`` records for one run; values are numpy arrays (host) or
    ``(device_pointer, kind)`` pairs."""

    def __init__(self, columns, feeds: dict):
        nodes = columns.nodes
        self.array = (TbFeed * max(1, len(feeds)))()
        self.count = len(feeds)
        self._keep = []
        for position, (symbol, payload) in enumerate(feeds.items()):
            index = symbol.index if hasattr(symbol, "index") else int(symbol)
            node = nodes[index]
            assert node.op == OP["Input"], "only inputs can be fed"
            rec = self.array[position]
            rec.slot = node.slot
            if isinstance(payload, Selection):
                assert payload.shape == node.shape, "fed payload must match the input's shape"
                indices = np.ascontiguousarray(payload.indices, dtype=np.int32)
                self._keep.append(indices)
                rec.indices = iptr(indices)
            elif isinstance(payload, (Dense, Constant)):
                data = np.ascontiguousarray(payload.to_numpy(), dtype=np.float32).reshape(-1)
                assert payload.shape == node.shape, "fed payload must match the input's shape"
                self._keep.append(data)
                rec.dense = fptr(data)
            elif isinstance(payload, np.ndarray):
                if payload.dtype == np.int32:
                    indices = np.ascontiguousarray(payload)
                    self._keep.append(indices)
                    rec.indices = iptr(indices)
                else:
                    data = np.ascontiguousarray(payload, dtype=np.float32).reshape(-1)
                    self._keep.append(data)
                    rec.dense = fptr(data)
            elif isinstance(payload, tuple) and payload[0] in ("device", "host"):
                rec.on_device = 1 if payload[0] == "device" else 0
                if payload[2] == "indices":
                    rec.indices = C.cast(C.c_void_p(payload[1]), C.POINTER(C.c_int32))
                else:
                    rec.dense = C.cast(C.c_void_p(payload[1]), C.POINTER(C.c_float))
            else:
                raise TypeError(type(payload))


def library_path() -> str:
    return os.path.join(os.path.dirname(os.path.abspath(__file__)), "libtopos_b200.so")


_LIB = None


def load_library() -> C.CDLL:
    """Loads the in-tree ``libtopos_b200.so``; raises when it was not built
    (there is no CPU fallback)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = library_path()
    if not os.path.exists(path):
        raise RuntimeError(f"libtopos_b200.so is not built ({path}); run __graft_entry__.build()")
    lib = C.CDLL(path, mode=C.RTLD_GLOBAL)
    P = C.c_void_p
    sigs = {
        "tb_status": (C.c_int, [C.c_char_p, C.c_size_t]),
        "tb_last_error": (C.c_char_p, []),
        "tb_plan_compile": (C.c_int, [C.POINTER(TbPlanDesc), C.POINTER(P)]),
        "tb_plan_destroy": (None, [P]),
        "tb_plan_stats_get": (C.c_int, [P, C.POINTER(TbPlanStats)]),
        "tb_plan_describe": (C.c_int64, [P, C.c_char_p, C.c_size_t]),
        "tb_params_create": (C.c_int, [P, C.POINTER(P)]),
        "tb_params_destroy": (None, [P]),
        "tb_params_upload": (C.c_int, [P, C.c_int32, C.POINTER(C.c_float), C.c_int64]),
        "tb_params_download": (C.c_int, [P, C.c_int32, C.POINTER(C.c_float), C.c_int64]),
        "tb_plan_run": (C.c_int, [P, P, C.c_int32, C.POINTER(TbFeed)]),
        "tb_plan_synchronize": (C.c_int, [P]),
        "tb_plan_gradient_node": (C.c_int, [P, C.c_int64, C.c_int64, C.POINTER(C.c_int64)]),
        "tb_plan_read": (C.c_int, [P, C.c_int64, C.POINTER(C.c_float), C.c_int64]),
        "tb_plan_read_async": (C.c_int, [P, C.c_int64, C.c_void_p, C.c_int64]),
        "tb_plan_device_pointer": (C.c_int, [P, C.c_int64, C.POINTER(C.c_void_p)]),
        "tb_plan_stream": (P, [P]),
        "tb_run_begin": (C.c_int, [P, P, C.c_int32, C.POINTER(TbFeed), C.POINTER(P)]),
        "tb_run_synchronize": (C.c_int, [P]),
        "tb_run_read": (C.c_int, [P, C.c_int64, C.POINTER(C.c_float), C.c_int64]),
        "tb_run_device_pointer": (C.c_int, [P, C.c_int64, C.POINTER(C.c_void_p)]),
        "tb_run_stream": (P, [P]),
        "tb_run_release": (None, [P]),
        "tb_plan_set_reduction": (C.c_int, [P, C.c_int32]),
        "tb_optimizer_step": (C.c_int, [P, C.POINTER(C.c_void_p), P]),
        "tb_batch_norm_f32": (C.c_int, [C.POINTER(C.c_float)] * 3 + [C.c_float, C.c_int64, C.c_int64]
                              + [C.POINTER(C.c_float)] * 3),
        "tb_optimizer_create": (C.c_int, [P, P, C.POINTER(TbOptimizerDesc), C.c_int32,
                                          C.POINTER(C.c_int32), C.POINTER(C.c_int64),
                                          C.POINTER(P)]),
        "tb_optimizer_destroy": (None, [P]),
        "tb_optimizer_set_learning_rate": (C.c_int, [P, C.c_float]),
        "tb_plan_attach_optimizer": (C.c_int, [P, P]),
        "tb_optimizer_state": (C.c_int, [P, C.c_int32, C.POINTER(C.c_float),
                                         C.POINTER(C.c_float), C.c_int64]),
        "tb_optimizer_powers": (C.c_int, [P, C.POINTER(C.c_float)]),
        "tb_optimizer_restore": (C.c_int, [P, C.c_int32, C.POINTER(C.c_float),
                                           C.POINTER(C.c_float), C.c_int64]),
        "tb_optimizer_restore_powers": (C.c_int, [P, C.POINTER(C.c_float)]),
        "tb_comm_unique_id": (C.c_int, [C.POINTER(C.c_uint8)]),
        "tb_comm_init": (C.c_int, [C.c_int32, C.c_int32, C.POINTER(C.c_uint8), C.POINTER(P)]),
        "tb_comm_destroy": (None, [P]),
        "tb_plan_attach_comm": (C.c_int, [P, P, C.c_int64]),
        "tb_comm_allreduce": (C.c_int, [P, P, C.c_int64, P]),
        "tb_gemm_f32": (C.c_int, [C.POINTER(C.c_float), C.c_int64, C.POINTER(C.c_int64),
                                  C.POINTER(C.c_float), C.c_int64, C.POINTER(C.c_int64),
                                  C.c_int64, C.c_int64, C.c_int64, C.POINTER(C.c_float)]),
        "tb_map_f32": (C.c_int, [C.c_int32, C.POINTER(C.c_float), C.c_int64,
                                 C.POINTER(C.c_float)]),
        "tb_gemm_f32_noalloc": (C.c_int, [C.c_void_p, C.POINTER(C.c_int64), C.c_void_p,
                                          C.POINTER(C.c_int64), C.c_int64, C.c_int64, C.c_int64,
                                          C.c_void_p, C.c_void_p]),
    }
    for name, (restype, argtypes) in sigs.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _LIB = lib
    return lib


HEADER_SYMBOLS = None


def header_symbols() -> list:
    """Function names declared in ``include/topos_b200.h``."""
    import re
    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    text = open(os.path.join(here, "include", "topos_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tb_[a-z0-9_]+)\s*\(", text)))
