"""Data-parallel sharding on CPU ranks (gloo, world size 2).

Rank 0 builds the seeded weights and broadcasts them; each rank generates its
shard of the global batch and runs the forward on it (the CPU oracle stands in
for a GPU here). Gathered shards must equal the unsharded run bit for bit, and
every rank must hold the identical weight blob.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import orbit_wars_b200 as ow
from orbit_wars_b200.shard import broadcast_weights, shard_inputs, shard_range

PER_RANK = 4
WORLD = 2


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, out_dir):
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(repo), str(repo / "orbit-wars-2d-transformer_b200")]
    import torch.distributed as dist
    from oracle import bind
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg = ow.preset(1)
    w = broadcast_weights(cfg, seed=17, rank=rank)
    # the communicator id of the library's NCCL weight broadcast travels over the same group
    from orbit_wars_b200.shard import share_comm_id
    uid = share_comm_id(rank, bytes(range(128)) if rank == 0 else None)
    feats, counts = shard_inputs(cfg, 17, rank, PER_RANK)
    lg, v, a = bind.policy_forward(cfg, w, feats, counts, f64=False, threads=1)
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), w=w, lg=lg, v=v, a=a, counts=counts,
             uid=np.frombuffer(uid, np.uint8))
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_forward_equals_unsharded(tmp_path, oracle):
    port = _free_port()
    mp.start_processes(_rank_main, args=(WORLD, port, str(tmp_path)), nprocs=WORLD, join=True, start_method="spawn")
    cfg = ow.preset(1)
    ranks = [np.load(tmp_path / f"rank{r}.npz") for r in range(WORLD)]
    assert np.array_equal(ranks[0]["w"], ranks[1]["w"])
    assert all(np.array_equal(r["uid"], np.arange(128, dtype=np.uint8)) for r in ranks)
    assert np.array_equal(ranks[0]["w"], ow.make_weights(cfg, seed=17))
    feats, counts = ow.make_inputs(cfg, batch=WORLD * PER_RANK, seed=17)
    lg, v, a = oracle.policy_forward(cfg, ranks[0]["w"], feats, counts, f64=False, threads=1)
    for r in range(WORLD):
        lo, hi = shard_range(r, PER_RANK)
        assert np.array_equal(ranks[r]["counts"], counts[lo:hi])
        assert np.array_equal(ranks[r]["lg"], lg[lo:hi])
        assert np.array_equal(ranks[r]["v"], v[lo:hi])
        assert np.array_equal(ranks[r]["a"], a[lo:hi])
