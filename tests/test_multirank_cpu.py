"""Multi-rank sharding on CPU with the gloo backend (world size 2): each rank
projects its slice of the batch with the oracle, the slices are gathered, and
the result equals the single-rank projection of the whole batch.  Also a rank
that raises before the gather makes the others fail fast instead of hanging."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG_DIR, ROOT


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n, out_path, fail_rank):
    import sys
    sys.path[:0] = [ROOT, PKG_DIR]
    import datetime

    import oracle
    from mhc_proj.sharding import shard_range

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        rng = np.random.default_rng(0)
        R = rng.standard_normal((n, 4, 4)).astype(np.float32)
        a, b = shard_range(n, rank, world)
        if rank == fail_rank:
            raise RuntimeError("injected failure on the host")
        T = torch.from_numpy(oracle.birkhoff_proj_n4(R[a:b], 1e-6, threads=1))
        sizes = [b2 - a2 for a2, b2 in (shard_range(n, r, world) for r in range(world))]
        parts = [torch.empty(s, 4, 4) for s in sizes]
        dist.all_gather(parts, T) if len(set(sizes)) == 1 else _gather_ragged(parts, T)
        if rank == 0:
            np.save(out_path, torch.cat(parts).numpy())
    finally:
        dist.destroy_process_group()


def _gather_ragged(parts, T):
    rank = dist.get_rank()
    for r, p in enumerate(parts):
        buf = T.clone() if r == rank else p
        dist.broadcast(buf, src=r)
        if r != rank:
            p.copy_(buf)
        else:
            parts[r] = T


@pytest.mark.parametrize("n", [4096, 1001])
def test_two_rank_shards_reassemble(tmp_path, n):
    import oracle

    out = str(tmp_path / "T.npy")
    mp.start_processes(_worker, args=(2, _free_port(), n, out, -1), nprocs=2, join=True, start_method="spawn")
    rng = np.random.default_rng(0)
    R = rng.standard_normal((n, 4, 4)).astype(np.float32)
    assert np.array_equal(np.load(out), oracle.birkhoff_proj_n4(R, 1e-6, threads=1))


def test_failing_rank_is_reported(tmp_path):
    out = str(tmp_path / "T.npy")
    with pytest.raises(Exception):
        mp.start_processes(_worker, args=(2, _free_port(), 512, out, 1), nprocs=2, join=True, start_method="spawn")
    assert not os.path.exists(out)
