"""Multi-rank host logic on CPU: world-size-2 gloo ranks shard a batch the way
bench.py does, each rank evaluates its slice (the oracle stands in for the
device), and the rank outputs placed in batch order equal the full-batch result;
the timing reduction takes the max over ranks."""
import importlib
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out_dir):
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ob = importlib.import_module("onnx-rs_b200")
    from oracle import oracle as orc
    nodes, inits, ins, outs = ob.workloads.stem_conv(0, batch=4)
    x = ob.synth.uniform(0, "X", (4, 3, 32, 32), -1, 1)
    lo, hi = ob.sharding.shard_range(4, world, rank)
    y = orc.conv2d(x[lo:hi], inits["W"], inits["B"], (2, 2), (3, 3, 3, 3))
    t = torch.from_numpy(np.ascontiguousarray(y))
    gathered = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(gathered, t)
    ms = torch.tensor([10.0 + rank], dtype=torch.float64)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    if rank == 0:
        np.save(os.path.join(out_dir, "gathered.npy"), torch.cat(gathered).numpy())
        np.save(os.path.join(out_dir, "max_ms.npy"), ms.numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_shard_ranges(ob):
    assert ob.sharding.all_ranges(256, 8) == [(32 * r, 32 * (r + 1)) for r in range(8)]
    assert ob.sharding.shard_range(256, 1, 0) == (0, 256)
    with pytest.raises(ValueError):
        ob.sharding.shard_range(256, 3, 0)
    with pytest.raises(ValueError):
        ob.sharding.shard_range(256, 2, 2)


def test_two_rank_shard_and_concat(tmp_path, ob, oracle):
    port = _free_port()
    mp.start_processes(_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    gathered = np.load(tmp_path / "gathered.npy")
    nodes, inits, ins, outs = ob.workloads.stem_conv(0, batch=4)
    x = ob.synth.uniform(0, "X", (4, 3, 32, 32), -1, 1)
    full = oracle.conv2d(x, inits["W"], inits["B"], (2, 2), (3, 3, 3, 3))
    np.testing.assert_array_equal(gathered, full)
    assert float(np.load(tmp_path / "max_ms.npy")[0]) == 11.0
