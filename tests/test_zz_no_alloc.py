"""The allocation-free GEMM entry point, through the C ABI.

`tb_gemm_f32_noalloc` exists for callers that cannot let this library call
cudaMalloc: a host framework whose own memory pool owns and accounts for every
device allocation, or code that must not allocate after start-up.  They pass
device inputs and output; the library's only scratch is a fixed 16 MiB device
array that every call shares.

This file checks the entry point against the CPU oracle's serial-k product
(`oracle.gemm`, the interpreter's `gemm.rs:140-211` loop) within the GEMM bar
of the other tests, 8 eps sqrt(k) (1 + |ref|)
(backend/cuda/tests/cuda_tests.rs:141-150):
  * the reference's shape grid under every pair of stride forms (contiguous,
    transposed, narrowed; cuda_tests.rs:54-201), on a non-default stream;
  * two calls in a row, and a smaller call after a larger one, since the shared
    scratch keeps the previous call's contents (a k that is not a multiple of
    32 exercises the zero padding each call rewrites);
  * the existing entry point `tb_gemm_f32` on the same inputs agrees too.
It also checks that a request beyond the fixed scratch is rejected with a clear
error.  It is collected last so that a run stopping at the first failure has
already run every other test."""
import ctypes as C
import math

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
EPS = float(np.finfo(np.float32).eps)

SHAPES = [(2, 3, 4), (5, 8, 13), (16, 16, 16), (63, 64, 65), (100, 127, 3), (128, 100, 64),
          (2, 64, 128)]


def varied(rows, cols, seed):
    # cuda_tests.rs `varied`: distinct, sign-varied values
    i = np.arange(rows * cols, dtype=np.int64)
    return (((i * 7 + seed * 13) % 23 - 11) / 4.0).astype(np.float32).reshape(rows, cols)


def stored(logical, form):
    """(flat buffer, strides) holding `logical` under one stride form."""
    rows, cols = logical.shape
    if form == "contiguous":
        return logical.reshape(-1).copy(), (cols, 1)
    if form == "transposed":
        return logical.T.copy().reshape(-1), (1, rows)
    padded = np.zeros((rows, cols + 3), np.float32)
    padded[:, :cols] = logical
    return padded.reshape(-1), (cols + 3, 1)


def assert_gemm(got, expected, k, what):
    tol = 8 * EPS * math.sqrt(k) * (1 + np.abs(expected))
    err = np.abs(got - expected)
    assert np.all(err <= tol), f"{what}: worst ratio {np.max(err / tol)}"


def noalloc(lib, torch, a, b, form_a="contiguous", form_b="contiguous", stream=None):
    m, k = a.shape
    n = b.shape[1]
    buf_a, sa = stored(a, form_a)
    buf_b, sb = stored(b, form_b)
    da = torch.from_numpy(buf_a).cuda()
    db = torch.from_numpy(buf_b).cuda()
    out = torch.full((m, n), float("nan"), device="cuda")
    s = stream if stream is not None else torch.cuda.current_stream()
    with torch.cuda.stream(s):
        rc = lib.tb_gemm_f32_noalloc(da.data_ptr(), (C.c_int64 * 2)(*sa), db.data_ptr(),
                                     (C.c_int64 * 2)(*sb), m, k, n, out.data_ptr(),
                                     C.c_void_p(s.cuda_stream))
    assert rc == 0, lib.tb_last_error()
    s.synchronize()
    assert lib.tbx_gemm_error() == 0
    return out.cpu().numpy()


def test_noalloc_gemm_follows_the_oracle_on_the_shape_grid(device):
    import torch
    from poorgrad_b200.abi import load_library
    lib = load_library()
    side = torch.cuda.Stream()
    forms = ["contiguous", "transposed", "narrowed"]
    for m, k, n in SHAPES:
        a = varied(m, k, 3)
        b = varied(k, n, 4)
        expected = oracle.gemm(a, b)
        for fa in forms:
            for fb in forms:
                got = noalloc(lib, torch, a, b, fa, fb, stream=side)
                assert_gemm(got, expected, k, f"{(m, k, n)} {fa}/{fb}")


def test_noalloc_gemm_twice_in_a_row_and_smaller_after_larger(device):
    import torch
    from poorgrad_b200 import backend
    from poorgrad_b200.abi import load_library
    lib = load_library()
    rng = np.random.default_rng(7)
    # a larger product, then the same twice, then a smaller ragged one whose
    # k (300) is not a multiple of 32
    for m, k, n in [(384, 320, 256), (384, 320, 256), (130, 300, 70), (130, 300, 70)]:
        a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        expected = oracle.gemm(a, b)
        got = noalloc(lib, torch, a, b, "transposed", "narrowed", stream=torch.cuda.Stream())
        assert_gemm(got, expected, k, f"{(m, k, n)}")
        # the existing, allocating entry point agrees on the same inputs
        if 2 * m * n * k >= 1 << 24:
            assert_gemm(backend.gemm_f32(a, b), expected, k, f"tb_gemm_f32 {(m, k, n)}")


def test_noalloc_gemm_rejects_requests_beyond_its_scratch(device):
    import torch
    from poorgrad_b200.abi import load_library
    lib = load_library()
    m, k, n = 4096, 1024, 4096          # needs 2*(m+n)*k = 16.8M floats > 4.19M
    x = torch.zeros(1, device="cuda")
    sa = (C.c_int64 * 2)(k, 1)
    sb = (C.c_int64 * 2)(n, 1)
    rc = lib.tb_gemm_f32_noalloc(x.data_ptr(), sa, x.data_ptr(), sb, m, k, n, x.data_ptr(), None)
    assert rc == 6  # TB_INVALID
    assert b"fixed scratch holds" in lib.tb_last_error()
