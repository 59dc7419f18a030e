"""The deterministic gradient reduction: `tree_sum` of
examples/makemore/mlp_parallel.rs:59-71 sums shard gradients pairwise
(left + right, an odd last shard carried up) until one remains.  The device
kernel that runs after the all-gather must give exactly the host tree's f32
result for every shard count."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def host_tree_sum(shards):
    layer = [s.astype(np.float32) for s in shards]
    while len(layer) > 1:
        nxt = []
        for j in range(0, len(layer), 2):
            nxt.append(layer[j] + layer[j + 1] if j + 1 < len(layer) else layer[j])
        layer = nxt
    return layer[0]


@pytest.mark.parametrize("n", [1, 2, 3, 5, 7, 8, 13])
def test_device_tree_matches_the_host_tree(device, n):
    import torch
    from poorgrad_b200.abi import load_library
    lib = load_library()
    lib.tbx_tree_sum.restype = C.c_int
    lib.tbx_tree_sum.argtypes = [C.c_void_p, C.c_int, C.c_int64, C.c_void_p]
    rng = np.random.default_rng(n)
    count = 4099
    # magnitudes spread over many binades so that the order of additions shows
    g = (rng.standard_normal((n, count)) * np.exp2(rng.integers(-20, 20, (n, count)))).astype(np.float32)
    dg = torch.from_numpy(g).cuda()
    out = torch.empty(count, device="cuda")
    assert lib.tbx_tree_sum(dg.data_ptr(), n, count, out.data_ptr()) == 0
    expect = host_tree_sum(list(g))
    assert out.cpu().numpy().tobytes() == expect.tobytes()
