"""The tcgen05 3xTF32 GEMM against an f64 reference and against the SIMT
engine, on prepared K-major tf32 hi/lo operands, including ragged tiles,
batches and split-K.  Bar: |dev - ref| <= 8 eps sqrt(k) (1 + |ref|)
(backend/cuda/tests/cuda_tests.rs:141-150) up to k = 1024; beyond that a
serial f32 sum itself (the interpreter order, and the SIMT engine) drifts
past 8x, so the bar there is 16 eps sqrt(k) (1 + |ref|)."""
import ctypes as C
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
EPS = float(np.finfo(np.float32).eps)


def _prep(torch, x, kp):
    # hi = rna_tf32(x) via the 13-bit rounding of the f32 pattern, lo = x - hi
    b, r, k = x.shape
    pad = torch.zeros((b, r, kp), dtype=torch.float32, device=x.device)
    pad[:, :, :k] = x
    bits = pad.view(torch.int32)
    hi = ((bits + 0x1000) & ~0x1FFF).view(torch.float32)
    hi = torch.where(torch.isfinite(pad), hi, pad)
    return hi.contiguous(), (pad - hi).contiguous()


@pytest.mark.parametrize("batch,m,n,k,splits", [
    (1, 128, 128, 32, 1), (1, 256, 384, 96, 1), (2, 130, 70, 40, 1), (1, 1, 5, 7, 1),
    (3, 200, 136, 300, 1), (1, 512, 512, 4096, 4), (1, 128, 256, 1024, 3)])
@pytest.mark.parametrize("tile", [32, 64, 128, 256])
def test_tcgen05_matches_f64(device, batch, m, n, k, splits, tile):
    import torch
    from poorgrad_b200.abi import load_library
    lib = load_library()
    lib.tbx_gemm_prepared.restype = C.c_int
    lib.tbx_gemm_prepared.argtypes = [C.c_void_p] * 6 + [C.c_int] + [C.c_int64] * 4 + [C.c_int]
    g = torch.Generator(device="cuda").manual_seed(batch * m + n + k)
    a = torch.rand((batch, m, k), device="cuda", generator=g) * 2 - 1
    bt = torch.rand((batch, n, k), device="cuda", generator=g) * 2 - 1
    kp = (k + 31) // 32 * 32
    ahi, alo = _prep(torch, a, kp)
    bhi, blo = _prep(torch, bt, kp)
    ref = torch.bmm(a.double(), bt.double().transpose(1, 2))
    factor = 8 if k <= 1024 else 16
    tol = factor * EPS * math.sqrt(k) * (1 + ref.abs())
    lib.tbx_set_gemm_tile_n(tile)
    for engine in (2, 1):
        c = torch.full((batch, m, n), float("nan"), device="cuda")
        part = torch.empty((max(splits, 1), batch, m, n), device="cuda")
        rc = lib.tbx_gemm_prepared(ahi.data_ptr(), alo.data_ptr(), bhi.data_ptr(), blo.data_ptr(),
                                   c.data_ptr(), part.data_ptr(), splits, batch, m, n, kp, engine)
        assert rc == 0, f"engine {engine} rc {rc}"
        assert lib.tbx_gemm_error() == 0
        err = (c.double() - ref).abs()
        assert torch.all(err <= tol), f"engine {engine}: worst {(err / tol).max().item()}"
    lib.tbx_set_gemm_tile_n(0)


@pytest.mark.parametrize("batch,m,n,k,splits", [
    (1, 128, 128, 32, 1), (2, 130, 70, 40, 1), (1, 64, 96, 17, 1), (1, 300, 200, 1000, 3),
    (1, 512, 27, 2048, 4)])
@pytest.mark.parametrize("a_mn,b_mn", [(0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("tile", [32, 64, 128, 256])
def test_mn_major_operands_match_f64(device, batch, m, n, k, splits, a_mn, b_mn, tile):
    # an MN-major operand is the value [batch, k, mn] in its own row-major
    # layout, the mn axis padded to a multiple of 32 (how the plan prepares an
    # activation once for a product and for the transposed weight gradient)
    import torch
    from poorgrad_b200.abi import load_library
    lib = load_library()
    f = lib.tbx_gemm_prepared_layout
    f.restype = C.c_int
    f.argtypes = ([C.c_void_p, C.c_void_p, C.c_int, C.c_int64] * 2 + [C.c_void_p, C.c_void_p, C.c_int]
                  + [C.c_int64] * 5 + [C.c_int])
    g = torch.Generator(device="cuda").manual_seed(7 * batch + m + n + k)
    a = torch.rand((batch, m, k), device="cuda", generator=g) * 2 - 1
    bt = torch.rand((batch, n, k), device="cuda", generator=g) * 2 - 1
    kp = (k + 31) // 32 * 32

    def operand(x, mn):
        rows = x.shape[1]
        if not mn:
            return _prep(torch, x, kp), kp
        ld = (rows + 31) // 32 * 32
        return _prep(torch, x.transpose(1, 2).contiguous(), ld), ld

    (ahi, alo), a_ld = operand(a, a_mn)
    (bhi, blo), b_ld = operand(bt, b_mn)
    ref = torch.bmm(a.double(), bt.double().transpose(1, 2))
    tol = 16 * EPS * math.sqrt(k) * (1 + ref.abs())
    lib.tbx_set_gemm_tile_n(tile)
    try:
        for engine in (2, 1):
            c = torch.full((batch, m, n), float("nan"), device="cuda")
            part = torch.empty((splits, batch, m, n), device="cuda")
            rc = f(ahi.data_ptr(), alo.data_ptr(), a_mn, a_ld, bhi.data_ptr(), blo.data_ptr(), b_mn,
                   b_ld, c.data_ptr(), part.data_ptr(), splits, batch, m, n, k, kp, engine)
            assert rc == 0, f"engine {engine} rc {rc}"
            assert lib.tbx_gemm_error() == 0
            err = (c.double() - ref).abs()
            assert torch.all(err <= tol), f"engine {engine}: worst {(err / tol).max().item()}"
    finally:
        lib.tbx_set_gemm_tile_n(0)


@pytest.mark.parametrize("m,n,k,a_mn,tile", [
    (16384, 512, 512, 0, 256), (4096, 4096, 512, 0, 256), (20000, 64, 256, 0, 128),
    (2000, 3000, 100, 1, 256), (1500, 900, 700, 1, 128)])
def test_stream_k_matches_f64_and_whole_tiles(device, m, n, k, a_mn, tile):
    # Shapes whose tiles leave the last wave of 148 SMs partly idle: with the
    # (opt-in) stream-K schedule their last tiles are cut into pieces whose
    # partial sums the owning CTA adds in k order.  Checked against f64,
    # against whole tiles (the default schedule), and bitwise against itself
    # on a second launch (the hand-over flags reset).
    import torch
    from poorgrad_b200.abi import load_library
    lib = load_library()
    f = lib.tbx_gemm_prepared_layout
    f.restype = C.c_int
    f.argtypes = ([C.c_void_p, C.c_void_p, C.c_int, C.c_int64] * 2 + [C.c_void_p, C.c_void_p, C.c_int]
                  + [C.c_int64] * 5 + [C.c_int])
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = torch.rand((1, m, k), device="cuda", generator=g) * 2 - 1
    bt = torch.rand((1, n, k), device="cuda", generator=g) * 2 - 1
    kp = (k + 31) // 32 * 32
    if a_mn:
        a_ld = (m + 31) // 32 * 32
        ahi, alo = _prep(torch, a.transpose(1, 2).contiguous(), a_ld)
    else:
        a_ld = kp
        ahi, alo = _prep(torch, a, kp)
    bhi, blo = _prep(torch, bt, kp)
    ref = torch.bmm(a.double(), bt.double().transpose(1, 2))
    tol = 8 * EPS * math.sqrt(k) * (1 + ref.abs())
    lib.tbx_set_gemm_tile_n(tile)
    outs = {}
    try:
        for label, sk in (("stream-k", 1), ("stream-k again", 1), ("whole tiles", 0)):
            lib.tbx_set_gemm_stream_k(sk)
            c = torch.full((1, m, n), float("nan"), device="cuda")
            rc = f(ahi.data_ptr(), alo.data_ptr(), a_mn, a_ld, bhi.data_ptr(), blo.data_ptr(), 0,
                   kp, c.data_ptr(), 0, 1, 1, m, n, k, kp, 2)
            assert rc == 0, f"{label} rc {rc}"
            assert lib.tbx_gemm_error() == 0, label
            err = (c.double() - ref).abs()
            assert torch.all(err <= tol), f"{label}: worst {(err / tol).max().item()}"
            outs[label] = c
    finally:
        lib.tbx_set_gemm_stream_k(0)
        lib.tbx_set_gemm_tile_n(0)
    assert torch.equal(outs["stream-k"], outs["stream-k again"])


@pytest.mark.parametrize("batch,m,n,k,splits", [
    (1, 128, 27, 64, 1), (2, 130, 70, 40, 1), (1, 300, 64, 1000, 3), (1, 512, 27, 2048, 4),
    (3, 64, 200, 96, 1)])
@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("raw", [1, 2, 3])
@pytest.mark.parametrize("tile", [32, 64, 128, 256])
def test_raw_operands_equal_prepared_pairs(device, batch, m, n, k, splits, a_mn, b_mn, raw, tile):
    # A raw operand is the f32 values in the prepared layout (no lo buffer).
    # The tcgen05 GEMM splits a raw A, each row by one epilogue lane, into its
    # tf32 pair in tensor memory, the pair the plan's prep writes: the product
    # is bitwise the product over prepared pairs, for either layout, any tile
    # (the 256-wide request runs on the 128-wide tile) and split-K.  It
    # declines a raw B; the SIMT engine takes either.
    import torch
    from poorgrad_b200.abi import load_library
    lib = load_library()
    f = lib.tbx_gemm_prepared_layout
    f.restype = C.c_int
    f.argtypes = ([C.c_void_p, C.c_void_p, C.c_int, C.c_int64] * 2 + [C.c_void_p, C.c_void_p, C.c_int]
                  + [C.c_int64] * 5 + [C.c_int])
    g = torch.Generator(device="cuda").manual_seed(11 * batch + m + n + k + raw)
    a = torch.randn((batch, m, k), device="cuda", generator=g)
    bt = torch.randn((batch, n, k), device="cuda", generator=g)
    kp = (k + 31) // 32 * 32

    def operand(x, mn):
        rows = x.shape[1]
        src = x.transpose(1, 2).contiguous() if mn else x
        ld = (rows + 31) // 32 * 32 if mn else kp
        hi, lo = _prep(torch, src, ld)
        padded = torch.zeros_like(hi)
        padded[:, :, :src.shape[2]] = src
        return hi, lo, padded.contiguous(), ld

    ahi, alo, araw, a_ld = operand(a, a_mn)
    bhi, blo, braw, b_ld = operand(bt, b_mn)
    ref = torch.bmm(a.double(), bt.double().transpose(1, 2))
    tol = 16 * EPS * math.sqrt(k) * (1 + ref.abs())
    lib.tbx_set_gemm_tile_n(tile)
    try:
        for engine in (2, 1):
            outs = []
            for use_raw in (0, raw):
                pa = (araw.data_ptr(), None) if use_raw & 1 else (ahi.data_ptr(), alo.data_ptr())
                pb = (braw.data_ptr(), None) if use_raw & 2 else (bhi.data_ptr(), blo.data_ptr())
                c = torch.full((batch, m, n), float("nan"), device="cuda")
                part = torch.empty((splits, batch, m, n), device="cuda")
                rc = f(pa[0], pa[1], a_mn, a_ld, pb[0], pb[1], b_mn, b_ld, c.data_ptr(),
                       part.data_ptr(), splits, batch, m, n, k, kp, engine)
                if engine == 2 and use_raw & 2:
                    assert rc == 5, "the tensor-core path declines a raw B"  # TB_DECLINED
                    outs.append(None)
                    continue
                assert rc == 0, f"engine {engine} raw {use_raw} rc {rc}"
                assert lib.tbx_gemm_error() == 0
                outs.append(c)
            if outs[1] is None:
                continue
            err = (outs[1].double() - ref).abs()
            assert torch.all(err <= tol), f"engine {engine}: worst {(err / tol).max().item()}"
            assert torch.equal(outs[0], outs[1]), "raw operands changed the product's bits"
    finally:
        lib.tbx_set_gemm_tile_n(0)
