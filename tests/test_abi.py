"""The C ABI on a machine without a GPU: the library loads, exports every
symbol include/topos_b200.h declares, reports PlatformUnsupported, and the
host half of the backend (lowering, NVRTC compilation of the emitted kernels
for sm_100a) runs."""

import pytest

from poorgrad_b200 import abi, backend, configs


def _no_gpu():
    import torch
    return not torch.cuda.is_available()


def test_library_exports_every_declared_symbol(built):
    lib = abi.load_library()
    declared = abi.header_symbols()
    assert len(declared) >= 28
    missing = [name for name in declared if not hasattr(lib, name)]
    assert not missing, missing


@pytest.mark.skipif(not _no_gpu(), reason="checks the device-less answers")
def test_status_without_a_device_is_platform_unsupported(built):
    code, _ = backend.status()
    assert code == 2  # BackendUnavailable::PlatformUnsupported
    w = configs.mlp(batch=8)
    with pytest.raises(backend.BackendError) as err:
        backend.DevicePlan(w.columns)
    assert err.value.code == 2


@pytest.mark.parametrize("name,kw", [
    ("mlp", dict(batch=16)), ("fused", dict(rows=32, cols=64)), ("gemm", dict(m=64, k=32, n=48)),
    ("charmlp", dict(batch=32)),
    ("gpt2", dict(batch=1, seq=8, layers=1, d=16, heads=2, vocab=11, mlp=32))])
def test_configs_lower_and_their_kernels_compile_for_sm100a(built, name, kw):
    w = configs.BUILDERS[name](**kw)
    text = backend.lower_describe(w.columns)
    assert "arena" in text
    backend.nvrtc_check(w.columns)


def test_c2_is_one_fused_pass_over_x(built):
    # forward row sum, db column sum, da full sum and dX share one kernel
    # (more than 256 rows: shorter column sums fold serially on their own)
    w = configs.fused(rows=512, cols=64)
    text = backend.lower_describe(w.columns)
    first = text.splitlines()[0]
    assert first.startswith("0: row") and len(first.split("members=")[1].split()) >= 4


def test_noalloc_gemm_refuses_oversized_requests_before_any_cuda_call():
    # the size check comes first and cannot overflow: an absurd extent is an
    # invalid request, answered without touching a device
    import ctypes as C
    lib = abi.load_library()
    s = (C.c_int64 * 2)(1, 1)
    big = (1 << 58) - 1
    for m, k, n in [(big, 1, 1), (1, big, 1), (1, 1, big), (4096, 1024, 4096)]:
        rc = lib.tb_gemm_f32_noalloc(C.c_void_p(256), s, C.c_void_p(256), s, m, k, n,
                                     C.c_void_p(256), None)
        assert rc == 6, (m, k, n)
        assert b"fixed scratch holds" in lib.tb_last_error()
