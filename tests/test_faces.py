"""The per-task faces (`Elementary::gemm`, payload/elementary.rs:74-80) against
the CPU oracle, through the C ABI.

`tb_gemm_f32` replaces the cuda backend's `executed_f32`
(backend/cuda/kernels/gemm.rs:54-163): host slices in, an owned row-major
result out.  Its results are compared with the interpreter's serial-k product
(`oracle.gemm`, payload/gemm.rs:140-211) under the reference's bar
8 eps sqrt(k) (1 + |ref|) (backend/cuda/tests/cuda_tests.rs:141-150), on a
shape grid (squares, rectangles, primes) under every pair of the reference's
stride forms (contiguous, transposed, narrowed; cuda_tests.rs:54-201).  The
grid is the reference's scaled up past the face's size threshold (tasks
below 2mnk = 2^24 decline, backend/cuda/kernels/mod.rs:34); the unscaled grid
runs through the allocation-free entry point, which has no threshold.

A runtime failure of a face poisons the library for good
(backend/cuda/kernels/mod.rs:94-105); that is checked in a child process, with
an allocation the device cannot satisfy as the failure."""
import math
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle
from poorgrad_b200 import backend

pytestmark = pytest.mark.gpu
EPS = float(np.finfo(np.float32).eps)
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SHAPES = [(256, 300, 128), (252, 256, 260), (1000, 127, 300), (128, 1000, 66),
          (513, 257, 129), (2048, 64, 128), (4, 4096, 1024)]


def varied(rows, cols, seed):
    i = np.arange(rows * cols, dtype=np.int64)
    return (((i * 7 + seed * 13) % 23 - 11) / 4.0).astype(np.float32).reshape(rows, cols)


def view(logical, form):
    """A numpy view holding `logical` under one stride form."""
    if form == "contiguous":
        return np.ascontiguousarray(logical)
    if form == "transposed":
        return np.ascontiguousarray(logical.T).T
    rows, cols = logical.shape
    padded = np.zeros((rows, cols + 3), np.float32)
    padded[:, :cols] = logical
    return padded[:, :cols]


@pytest.mark.parametrize("m,k,n", SHAPES)
def test_gemm_face_follows_the_oracle_in_every_stride_form(device, m, k, n):
    a = varied(m, k, 1)
    b = varied(k, n, 2)
    expected = oracle.gemm(a, b)
    tol = 8 * EPS * math.sqrt(k) * (1 + np.abs(expected))
    for fa in ("contiguous", "transposed", "narrowed"):
        for fb in ("contiguous", "transposed", "narrowed"):
            got = backend.gemm_f32(view(a, fa), view(b, fb))
            assert got is not None, "declined"
            err = np.abs(got - expected)
            assert np.all(err <= tol), f"{fa}/{fb}: worst ratio {np.max(err / tol)}"


def test_gemm_face_uniform_operands_and_negative_zero(device):
    rng = np.random.default_rng(5)
    a = rng.uniform(-1, 1, (700, 513)).astype(np.float32)
    b = rng.uniform(-1, 1, (513, 333)).astype(np.float32)
    expected = oracle.gemm(a, b)
    got = backend.gemm_f32(a, b)
    assert np.all(np.abs(got - expected) <= 8 * EPS * math.sqrt(513) * (1 + np.abs(expected)))
    # gemm_tests.rs:130-139: a product of -0.0 terms keeps its sign
    z = np.full((256, 256), -0.0, np.float32)
    one = np.ones((256, 256), np.float32)
    out = backend.gemm_f32(z, one)
    assert np.all(out == 0)


def test_gemm_face_declines_small_tasks(device):
    assert backend.gemm_f32(varied(5, 8, 1), varied(8, 13, 2)) is None


CHILD = r"""
import ctypes as C, sys
sys.path.insert(0, %r)
from poorgrad_b200.abi import load_library
lib = load_library()
buf = C.create_string_buffer(256)
assert lib.tb_status(buf, 256) == 0
x = (C.c_float * 4)()
# 2**40 elements: the face's device workspace cannot be allocated
rc = lib.tb_map_f32(9, x, C.c_int64(1 << 40), x)
status = lib.tb_status(buf, 256)
print(rc, status, buf.value.decode())
"""


def test_a_face_failure_poisons_the_library(device):
    out = subprocess.run([sys.executable, "-c", CHILD % ROOT], capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr
    rc, status = out.stdout.split()[:2]
    assert rc == "7"       # TB_RUNTIME
    assert status == "4"   # TB_POISONED from then on
