"""Failure handling made on the host: malformed requests answer TB_INVALID
(the reference panics) without poisoning the backend, and the product refuses
to run without its CUDA library (no CPU fallback)."""
import ctypes as C

import pytest

from poorgrad_b200 import abi, backend
from poorgrad_b200.graph import Tape, tensor
from poorgrad_b200.plan import Request


def _desc_with_forward_link():
    t = Tape()
    x = t.parameter(tensor([2], [1.0, 2.0]))
    y = x.exp()
    cols = t.into_network().compile(Request([y]))
    packed = abi.PackedPlan(cols)
    packed.array[1].operands[0] = 5  # points forward: malformed
    return packed


def test_malformed_descriptor_is_rejected_by_lowering(built):
    lib = abi.load_library()
    lib.tbx_lower_describe.restype = C.c_int64
    packed = _desc_with_forward_link()
    n = lib.tbx_lower_describe(C.byref(packed.desc), None, 0, 0)
    assert n == -1
    assert b"backwards" in lib.tb_last_error()


def test_unsupported_rank_is_rejected(built):
    lib = abi.load_library()
    lib.tbx_lower_describe.restype = C.c_int64
    t = Tape()
    x = t.parameter(tensor([2], [1.0, 2.0]))
    y = x.exp()
    packed = abi.PackedPlan(t.into_network().compile(Request([y])))
    packed.array[1].rank = 9
    assert lib.tbx_lower_describe(C.byref(packed.desc), None, 0, 0) == -1


def test_a_malformed_request_does_not_poison(built):
    lib = abi.load_library()
    packed = _desc_with_forward_link()
    h = C.c_void_p()
    rc = lib.tb_plan_compile(C.byref(packed.desc), C.byref(h))
    assert rc != 0
    code, _ = backend.status()
    assert code in (0, 2)  # ok on a GPU box, PlatformUnsupported without one; never Poisoned


def test_missing_library_fails_loudly(monkeypatch):
    monkeypatch.setattr(abi, "_LIB", None)
    monkeypatch.setattr(abi, "library_path", lambda: "/nonexistent/libtopos_b200.so")
    with pytest.raises(RuntimeError, match="not built"):
        abi.load_library()


@pytest.mark.parametrize("field,value,message", [
    ("shape", 0, b"empty extent"), ("op", 999, b"unknown opcode"), ("slot", -1, b"no slot")])
def test_invalid_descriptor_fields_are_rejected(built, field, value, message):
    # the reference has no empty values, no unknown functions and no unslotted
    # parameters: a descriptor with one answers TB_INVALID and poisons nothing
    lib = abi.load_library()
    lib.tbx_lower_describe.restype = C.c_int64
    t = Tape()
    x = t.parameter(tensor([2], [1.0, 2.0]))
    y = x.exp()
    packed = abi.PackedPlan(t.into_network().compile(Request([y])))
    node = packed.array[0]  # the parameter
    if field == "shape":
        node.shape[0] = value
    else:
        setattr(node, field, value)
    assert lib.tbx_lower_describe(C.byref(packed.desc), None, 0, 0) == -1
    assert message in lib.tb_last_error()
    code, _ = backend.status()
    assert code in (0, 2)
