"""Lowering decisions, checked on the host (no GPU): how the charmlp (C4)
training plan is split into kernels, which GEMM operands are read K-major or
MN-major, which operand preps ride inside the fusion group that computes the
value, and how column finals share launches.  These are the structure the
bench numbers depend on; the GPU tests check the values."""
import ctypes as C
import re

import pytest

from poorgrad_b200 import backend, configs


@pytest.fixture(scope="module")
def charmlp_lines(built):
    w = configs.char_mlp()
    return [l for l in backend.lower_describe(w.columns).splitlines() if re.match(r"\d+: ", l)]


def test_weight_gradients_read_the_forward_preps_transposed(charmlp_lines):
    gemms = [l for l in charmlp_lines if "gemm3xtf32" in l]
    assert len(gemms) == 9
    # dW = h^T . dY (m=n=512, k=batch): both operands are the activations'
    # own row-major preps, read MN-major -- no transposing prep exists
    dw = [l for l in gemms if "m=512 n=512 k=16384" in l]
    assert len(dw) == 2 and all("a=mn b=mn" in l for l in dw)
    # every prepared value is prepared once (9 GEMMs, fewer than 18 preps)
    preps = [l for l in charmlp_lines if ": prep " in l]
    fused = [l for l in charmlp_lines if "prep" in l and (": row " in l or ": ew " in l)]
    assert len(preps) + len(fused) < 18


def test_activation_preps_ride_in_their_producing_row_kernels(charmlp_lines):
    # the LayerNorm forward (tanh output) and backward (dX) row kernels write
    # the tf32 pair of the GEMM operand they compute -- all but the second
    # hidden layer's output, which only the 27-wide head products read
    rows = [l for l in charmlp_lines if ": row " in l and "space=[16384,512]" in l]
    assert sum("prep" in l for l in rows) == 3
    standalone = [l for l in charmlp_lines if ": prep " in l and "[1,16384,512]" in l]
    assert not standalone


def test_operands_of_memory_bound_products_stay_f32(charmlp_lines):
    # the head's logits (n=27) and its weight gradient (m=512, n=27) read the
    # second hidden layer's output as raw f32 values, split into the tf32
    # pair inside the GEMM: no pair of it is written
    gemms = [l for l in charmlp_lines if "gemm3xtf32" in l]
    raw = [l for l in gemms if ":raw" in l]
    assert len(raw) == 2
    assert any("m=16384 n=27 k=512" in l and "a=k:raw" in l for l in raw)
    assert any("m=512 n=27 k=16384" in l and "a=mn:raw" in l for l in raw)
    # products wide enough for the tensor cores keep prepared pairs
    assert not any(":raw" in l for l in gemms if " n=512 " in l)


def test_raw_operands_can_be_turned_off(built, monkeypatch):
    monkeypatch.setenv("TB_RAW_OPERANDS", "0")
    w = configs.char_mlp()
    assert ":raw" not in backend.lower_describe(w.columns)


def test_narrow_column_finals_share_a_launch(charmlp_lines):
    finals = [l for l in charmlp_lines if ": final " in l]
    assert any(l.count(",") >= 2 for l in finals)  # three 512-wide finals in one launch
    assert len(finals) <= 6


def test_the_selection_sort_leads_the_program(charmlp_lines):
    assert " sort selection" in charmlp_lines[0]


def test_gemm_tile_and_split_rules(built):
    from poorgrad_b200.abi import load_library
    lib = load_library()
    lib.tbx_gemm_splits.restype = C.c_int
    lib.tbx_gemm_splits.argtypes = [C.c_int64] * 4
    # split-K fills one wave of 148 SMs at most: 512x512 outputs in 256-wide
    # tiles are 8 tiles -> 18 splits (144 work items)
    assert lib.tbx_gemm_splits(1, 512, 512, 16384) == 18
    # long-M products need no split
    assert lib.tbx_gemm_splits(1, 16384, 512, 512) == 1
    # outputs at most 32 wide take the 32-wide tile: 4 tiles -> 37 splits
    assert lib.tbx_gemm_splits(1, 512, 27, 16384) == 37


@pytest.mark.parametrize("name", ["mlp", "fused", "gemm", "charmlp", "gpt2"])
def test_no_config_stores_a_large_value_nobody_reads(built, name):
    # a full-size value that no other kernel reads (not a result) is a store
    # nobody needs or a round trip through memory inside its own kernel: the
    # waste of materializing broadcast row statistics and phase-crossing
    # values.  What remains are per-row statistics the kernel also keeps in
    # registers.
    from poorgrad_b200 import backend, configs
    w = configs.BUILDERS[name]()
    dead = [l for l in backend.lower_describe(w.columns).splitlines() if l.startswith("dead")]
    assert all(int(l.split()[-1]) < (1 << 20) for l in dead), dead


def test_values_past_two_to_the_31_elements_index_in_64_bits(built):
    # a [65536, 40000] input (2.6e9 elements; a constant payload, so nothing
    # is allocated): its kernels take 64-bit indices and still compile
    from poorgrad_b200.graph import Tape, filled
    from poorgrad_b200.plan import Request
    t = Tape()
    x = t.input(filled((65536, 40000), 1.0))
    rows = (x * x.literal(filled((65536, 40000), 0.5))).tanh().sum_along(1)
    cols = t.into_network().compile(Request([rows]))
    text = backend.lower_describe(cols, with_source=True)
    assert "typedef long long I;" in text
    backend.nvrtc_check(cols)


def test_gradient_seeds_over_products_and_sums_need_no_copy_kernels(charmlp_lines):
    # Tape::differentiate's `0 + c` seeds (graph/tape.rs:389-393) over a
    # product, a scatter-add or a fused sum are that value's own buffer: the
    # step ends with the optimizer inputs written by their producers, not by
    # copy kernels (the only flat kernels left are the gather, the loss scale
    # and the tail of the cross-entropy gradient)
    flat = [l for l in charmlp_lines if re.match(r"\d+: ew ", l)]
    assert len(flat) <= 3, flat


def test_window_patterns_lower_without_materialized_windows(built):
    # conv -> max-pool: the im2col view chain is read by the operand prep
    # (the tf32 pair the tensor-core product needs) and the pool's window max
    # runs inside the kernel that adds the bias and restores NCHW: no window
    # lanes are stored (engine/pattern/window.rs, reduce_window.rs)
    import numpy as np
    from poorgrad_b200 import neural
    from poorgrad_b200.graph import Dense, Tape
    from poorgrad_b200.plan import Request
    t = Tape()
    rng = np.random.default_rng(0)
    x = t.input(Dense((8, 4, 16, 16), rng.standard_normal((8, 4, 16, 16)).astype(np.float32)))
    w = t.parameter(Dense((8, 4, 3, 3), rng.standard_normal((8, 4, 3, 3)).astype(np.float32)))
    b = t.parameter(Dense((8,), np.zeros(8, np.float32)))
    p = neural.max_pool(neural.conv2d(x, w, b, stride=1, padding=1), 2, 2)
    net = t.into_network()
    lines = [l for l in backend.lower_describe(net.compile(Request([p]))).splitlines()
             if re.match(r"\d+: ", l)]
    kinds = [l.split()[1] for l in lines]
    assert kinds.count("gemm3xtf32") == 1
    assert kinds.count("prep") == 2 and kinds.count("ew") == 1 and len(lines) == 4, lines


def test_attention_probabilities_stay_f32_for_their_narrow_products(built):
    # the probabilities [heads, T, T] feed P.V and dV = P^T.dO, both 64 wide
    # (the head width): raw f32 operands.  The score gradient dS also feeds
    # dK^T = Q^T.dS as B, a 1024-wide product on the 256-wide tile, so it
    # keeps its prepared pair.
    w = configs.gpt2(batch=1, seq=1024, layers=1, vocab=64)
    lines = [l for l in backend.lower_describe(w.columns).splitlines() if "batch=12 " in l]
    assert any("m=1024 n=64 k=1024" in l and "a=k:raw" in l for l in lines)
    assert any("m=1024 n=64 k=1024" in l and "a=mn:raw" in l for l in lines)
    assert any("m=1024 n=64 k=1024" in l and "a=k b=mn" in l for l in lines)  # dQ = dS.K
    assert not any(":raw" in l for l in lines if "m=64 n=1024" in l or "n=1024 k=64" in l)
    # a raw operand is always A: the tensor-core path splits A only
    every = backend.lower_describe(w.columns)
    assert not re.search(r"b=(k|mn):raw", every)


def _product_lines(build):
    from poorgrad_b200.graph import Tape
    from poorgrad_b200.plan import Request
    t = Tape()
    roots = build(t)
    cols = t.into_network().compile(Request(roots))
    return [l for l in backend.lower_describe(cols).splitlines() if "gemm3xtf32" in l]


def test_which_operands_stay_raw(built):
    # raw: the A operand of products at most 64 wide, stored densely with
    # rows of a multiple of 32 floats -- an input as it is, a computed value
    # once in f32; everything else keeps its prepared pair
    import numpy as np
    from poorgrad_b200.graph import Dense, filled
    rng = np.random.default_rng(1)

    def dense(shape):
        return Dense(shape, rng.standard_normal(shape).astype(np.float32))

    # an input feeding a 48-wide product: raw, no prep for it
    lines = _product_lines(lambda t: [t.input(dense((256, 64))).matmul(t.parameter(dense((64, 48))))])
    assert len(lines) == 1 and "a=k:raw" in lines[0]
    # the same input also feeding a 256-wide product: pairs for both
    def two(t):
        x = t.input(dense((256, 64)))
        return [x.matmul(t.parameter(dense((64, 48)))), x.matmul(t.parameter(dense((64, 256))))]
    assert not any(":raw" in l for l in _product_lines(two))
    # rows that are not a multiple of 32 floats: a pair (it would need padding)
    lines = _product_lines(lambda t: [t.input(dense((256, 40))).matmul(t.parameter(dense((40, 48))))])
    assert not any(":raw" in l for l in lines)
    # a computed value read by a narrow product: raw, stored by its fusion group
    lines = _product_lines(
        lambda t: [(t.input(dense((256, 64))).tanh()).matmul(t.parameter(dense((64, 16))))])
    assert len(lines) == 1 and "a=k:raw" in lines[0]
    # a value read transposed as A (a weight gradient's shape): raw, MN-major
    lines = _product_lines(
        lambda t: [t.input(dense((512, 64))).transpose().matmul(t.input(dense((512, 32))))])
    assert len(lines) == 1 and "a=mn:raw" in lines[0] and "b=mn" in lines[0]
    # the B side of a narrow product (its own M is large) is never raw
    assert "b=mn:raw" not in lines[0] and "b=k:raw" not in lines[0]


def test_bf16_networks_keep_prepared_pairs(built):
    import numpy as np
    from poorgrad_b200.graph import BF16, Dense, Tape
    from poorgrad_b200.plan import Request
    rng = np.random.default_rng(2)
    t = Tape(BF16)
    x = t.input(Dense((256, 64), rng.standard_normal((256, 64)).astype(np.float32)))
    y = x.matmul(t.parameter(Dense((64, 16), rng.standard_normal((64, 16)).astype(np.float32))))
    cols = t.into_network().compile(Request([y]))
    assert ":raw" not in backend.lower_describe(cols)
