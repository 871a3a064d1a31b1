"""Batch sharding: slice arithmetic and a 2-rank gloo gather on CPU."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from turbompc_b200.sharding import gather_batch, shard_params, shard_range


@pytest.mark.parametrize("nb,world", [(65536, 8), (10, 3), (3, 4), (0, 2)])
def test_shard_range_covers_batch_exactly(nb, world):
    got = [shard_range(nb, world, r) for r in range(world)]
    assert got[0][0] == 0 and got[-1][1] == nb
    assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
    assert max(h - l for l, h in got) - min(h - l for l, h in got) <= 1


def test_shard_params_slices_batched_only():
    p = {"initial_state": torch.arange(10.0)[:, None].repeat(1, 3), "w": torch.ones(3), "horizon": 5,
         "dyn": {"A": torch.zeros(10, 2, 2), "c": torch.zeros(2, 2)}}
    s = shard_params(p, 10, 3, 7, batched={"initial_state", "dyn.A"})
    assert s["initial_state"].shape == (4, 3) and s["initial_state"][0, 0] == 3
    assert s["w"].shape == (3,) and s["dyn"]["A"].shape == (4, 2, 2) and s["dyn"]["c"].shape == (2, 2)


def test_shard_params_leaves_shared_tensors_whose_size_matches_the_batch():
    # a weight matrix with nb rows is shared, not a batch axis
    p = {"initial_state": torch.zeros(6, 6), "mlp_W1": torch.ones(6, 9),
         "dynamics_state_dot_params": {"A": torch.eye(6)}}
    s = shard_params(p, 6, 2, 4)
    assert s["initial_state"].shape == (2, 6)
    assert s["mlp_W1"].shape == (6, 9) and s["dynamics_state_dot_params"]["A"].shape == (6, 6)


def _worker(rank, world, port, nb, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    lo, hi = shard_range(nb, world, rank)
    local = torch.arange(lo, hi, dtype=torch.float64)[:, None].repeat(1, 2)
    full = gather_batch(local, nb)
    q.put((rank, full.tolist()))
    dist.destroy_process_group()


def test_gloo_two_rank_gather():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, 7, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    want = [[float(i)] * 2 for i in range(7)]
    assert res[0] == want and res[1] == want
