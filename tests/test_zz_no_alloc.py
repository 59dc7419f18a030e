"""The allocation-free GEMM entry point, through the C ABI.

`tb_gemm_f32_noalloc` exists for callers that cannot let this library call
cudaMalloc: a host framework whose own memory pool owns and accounts for every
device allocation, or code that must not allocate after start-up.  They pass
device inputs and output; the library's only scratch is a fixed 16 MiB device
array.  This file checks it against the allocating entry point `tb_gemm_f32`
on the same inputs, twice in a row (the shared scratch keeps the previous
call's contents), within the GEMM bar of the other tests
(8 eps sqrt(k) (1 + |ref|), backend/cuda/tests/cuda_tests.rs:141-150), and
that a request beyond the fixed scratch is rejected with a clear error.
It is collected last so that a run stopping at the first failure has already
run every other test."""
import ctypes as C
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
EPS = float(np.finfo(np.float32).eps)


def _gemm_host(lib, a, b):
    m, k = a.shape
    n = b.shape[1]
    out = np.empty((m, n), np.float32)
    sa = (C.c_int64 * 2)(k, 1)
    sb = (C.c_int64 * 2)(n, 1)
    f = lambda x: x.ctypes.data_as(C.POINTER(C.c_float))
    rc = lib.tb_gemm_f32(f(a), a.size, sa, f(b), b.size, sb, m, k, n, f(out))
    assert rc == 0, lib.tb_last_error()
    return out


def test_noalloc_gemm_matches_the_allocating_entry_point(device):
    import torch
    from poorgrad_b200.abi import load_library
    lib = load_library()
    m, k, n = 384, 320, 256
    rng = np.random.default_rng(7)
    for call in range(2):
        a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        expected = _gemm_host(lib, a, b)
        da = torch.from_numpy(a).cuda()
        db = torch.from_numpy(b).cuda()
        out = torch.full((m, n), float("nan"), device="cuda")
        sa = (C.c_int64 * 2)(k, 1)
        sb = (C.c_int64 * 2)(n, 1)
        stream = torch.cuda.current_stream().cuda_stream
        rc = lib.tb_gemm_f32_noalloc(da.data_ptr(), sa, db.data_ptr(), sb, m, k, n,
                                     out.data_ptr(), stream)
        assert rc == 0, lib.tb_last_error()
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        tol = 8 * EPS * math.sqrt(k) * (1 + np.abs(expected))
        assert np.all(np.abs(got - expected) <= tol), f"call {call}"


def test_noalloc_gemm_rejects_requests_beyond_its_scratch(device):
    import torch
    from poorgrad_b200.abi import load_library
    lib = load_library()
    m, k, n = 4096, 1024, 4096          # needs 2*(m+n)*k = 16.8M floats > 4.19M
    x = torch.zeros(1, device="cuda")
    sa = (C.c_int64 * 2)(k, 1)
    sb = (C.c_int64 * 2)(n, 1)
    rc = lib.tb_gemm_f32_noalloc(x.data_ptr(), sa, x.data_ptr(), sb, m, k, n, x.data_ptr(), 0)
    assert rc == 6  # TB_INVALID
    assert b"fixed scratch holds" in lib.tb_last_error()
