"""Data parallel on 2 GPUs through the C ABI: each rank runs the training
plan on its shard, the gradients are summed by the in-graph NCCL all-reduce,
and the SGD step (with gradient_scale = 1/N) leaves identical parameters on
every rank that match the full-batch update computed by the oracle (a
tolerance: NCCL's reduction order is not the reference's tree_sum)."""
import os
import socket
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port, out, reduction="nccl"):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    from poorgrad_b200 import backend, configs
    from poorgrad_b200.graph import Selection
    full = configs.char_mlp(batch=128, hidden=64, embed=16)
    feeds = full.feeds(0)
    c = feeds[full.inputs["contexts"]].indices.reshape(128, 8)
    t = feeds[full.inputs["targets"]].indices
    w = configs.char_mlp(batch=128 // world, hidden=64, embed=16)
    sl = slice(rank * 128 // world, (rank + 1) * 128 // world)
    sfeeds = {w.inputs["contexts"]: Selection(c[sl].reshape(-1), 27),
              w.inputs["targets"]: Selection(t[sl], 27)}
    plan = backend.DevicePlan(w.columns)
    dp = backend.DeviceParameters(plan, w.network.parameters())
    opt = backend.Optimizer(plan, dp, backend.SGD, zip(w.params, w.grads), 0.1,
                            gradient_scale=1.0 / world)  # kept alive: it detaches when freed
    uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
    if rank == 0:
        uid.copy_(torch.tensor(list(backend.Comm.unique_id()), dtype=torch.uint8))
    dist.broadcast(uid, 0)
    comm = backend.Comm(rank, world, bytes(uid.cpu().tolist()))
    comm.attach(plan, reduction=reduction)
    plan.forward(dp, sfeeds, sync=True)
    slots = [w.columns.nodes[p.index].slot for p in w.params]
    out[rank] = [dp.download(s) for s in slots]
    dist.barrier()
    # leave without destructors: communicators bound into a captured graph are
    # not torn down at interpreter exit
    sys.stdout.flush()
    os._exit(0)


@pytest.mark.timeout(300)
def test_two_rank_sgd_step_matches_the_full_batch_update(device):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import oracle
    from poorgrad_b200 import configs
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_rank, args=(2, _port(), out), nprocs=2, join=True)
    full = configs.char_mlp(batch=128, hidden=64, embed=16)
    params = full.network.parameters()
    ref = oracle.run(full.columns, params, full.feeds(0), read=[g.index for g in full.grads])
    for i, g in enumerate(full.grads):
        expect = params[i].reshape(ref[g.index].shape) - ref[g.index] * np.float32(0.1)
        np.testing.assert_array_equal(out[0][i], out[1][i])
        np.testing.assert_allclose(out[0][i].reshape(expect.shape), expect, rtol=1e-4, atol=1e-5)


def _shard_gradients(world):
    """Each shard's device gradients, computed one shard at a time without a
    communicator (what every rank contributes to the exchange)."""
    sys.path.insert(0, ROOT)
    from poorgrad_b200 import backend, configs
    from poorgrad_b200.graph import Selection
    full = configs.char_mlp(batch=128, hidden=64, embed=16)
    feeds = full.feeds(0)
    c = feeds[full.inputs["contexts"]].indices.reshape(128, 8)
    t = feeds[full.inputs["targets"]].indices
    w = configs.char_mlp(batch=128 // world, hidden=64, embed=16)
    plan = backend.DevicePlan(w.columns)
    dp = backend.DeviceParameters(plan, w.network.parameters())
    out = []
    for rank in range(world):
        sl = slice(rank * 128 // world, (rank + 1) * 128 // world)
        sfeeds = {w.inputs["contexts"]: Selection(c[sl].reshape(-1), 27),
                  w.inputs["targets"]: Selection(t[sl], 27)}
        plan.forward(dp, sfeeds, sync=True)
        out.append([plan.of(g) for g in w.grads])
    return w, out


@pytest.mark.timeout(300)
def test_tree_reduction_is_bitwise_the_reference_tree_sum(device):
    # TB_REDUCTION_TREE: all-gather, then tree_sum's pairwise order; the SGD step
    # p - (sum * (1/N)) * lr must equal the host restatement bit for bit
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_rank, args=(world, _port(), out, "tree"), nprocs=world, join=True)
    w, shards = _shard_gradients(world)
    params = w.network.parameters()
    scale = np.float32(1.0 / world)
    for i, g in enumerate(w.grads):
        layer = [s[i] for s in shards]
        while len(layer) > 1:
            layer = [layer[j] + layer[j + 1] if j + 1 < len(layer) else layer[j]
                     for j in range(0, len(layer), 2)]
        expect = params[i].reshape(layer[0].shape) - (layer[0] * scale) * np.float32(0.1)
        np.testing.assert_array_equal(out[0][i], out[1][i])
        assert out[0][i].reshape(expect.shape).astype(np.float32).tobytes() == \
            expect.astype(np.float32).tobytes()
