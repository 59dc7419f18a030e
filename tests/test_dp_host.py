"""Host-side logic of data-parallel training, as gloo ranks on CPU.

The reference's data-parallel idiom (examples/makemore/mlp_parallel.rs:59-71,
136-171) sums shard gradients and scales by 1/shards; each shard's
cross-entropy normalizes by its own target mass, so with equal shards the mean
of shard gradients is the full-batch gradient.  The device path does the sum
with NCCL inside the step and folds 1/N into the optimizer; here the same
arithmetic runs on the oracle per rank with a gloo all-reduce, and the
bootstrap failure modes (a rank that never joins) end in an error, not a hang."""
import os
import socket
import sys

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _dp_worker(rank, world, port, out):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import oracle
    from poorgrad_b200 import configs
    from poorgrad_b200.graph import Selection
    full = configs.char_mlp(batch=64, hidden=32, embed=8)
    feeds = full.feeds(0)
    ctx, tgt = full.inputs["contexts"], full.inputs["targets"]
    c = feeds[ctx].indices.reshape(64, 8)
    t = feeds[tgt].indices
    shard = configs.char_mlp(batch=64 // world, hidden=32, embed=8)
    sl = slice(rank * 64 // world, (rank + 1) * 64 // world)
    sfeeds = {shard.inputs["contexts"]: Selection(c[sl].reshape(-1), 27),
              shard.inputs["targets"]: Selection(t[sl], 27)}
    ref = oracle.run(shard.columns, shard.network.parameters(), sfeeds,
                     read=[g.index for g in shard.grads])
    scale = np.float32(1.0 / world)
    for i, g in enumerate(shard.grads):
        buf = torch.from_numpy(ref[g.index].copy())
        dist.all_reduce(buf)
        mean = buf.numpy() * scale
        if rank == 0:
            out[i] = mean
    dist.barrier()
    dist.destroy_process_group()


def test_mean_of_shard_gradients_is_the_full_batch_gradient(built):
    import oracle
    from poorgrad_b200 import configs
    world = 2
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_dp_worker, args=(world, _port(), out), nprocs=world, join=True)
    full = configs.char_mlp(batch=64, hidden=32, embed=8)
    ref = oracle.run(full.columns, full.network.parameters(), full.feeds(0),
                     read=[g.index for g in full.grads])
    for i, g in enumerate(full.grads):
        np.testing.assert_allclose(out[i], ref[g.index], rtol=2e-4, atol=1e-6)


def _lonely(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=3))
    except Exception:
        sys.exit(17)
    sys.exit(0)


def test_a_rank_that_never_joins_ends_in_an_error(built):
    ctx = mp.get_context("spawn")
    p = ctx.Process(target=_lonely, args=(0, 2, _port()))
    p.start()
    p.join(60)
    assert not p.is_alive()
    assert p.exitcode == 17
