"""The batch sharded over two GPUs, one process per GPU with NCCL (runs only
where two GPUs are visible): each rank projects and differentiates its slice
of the batch on its own device -- no collective on the data path -- and the
gathered slices equal the single-GPU results bit for bit.  NCCL only gathers
the results for the check, after the work."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG_DIR, ROOT

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n, out_path):
    import sys
    sys.path[:0] = [ROOT, PKG_DIR]
    import mhc_proj
    from mhc_proj.sharding import shard_range, shard_sizes
    from mhc_proj.workloads import make_logits

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        R = make_logits("sigma_mix", n, seed=5, device=dev)  # the same batch on every rank
        G = make_logits("normal", n, seed=6, device=dev)
        a, b = shard_range(n, rank, world)
        T = mhc_proj.torch.birkhoff_proj_n4(R[a:b].contiguous(), 1e-6)["T"]
        D = mhc_proj.torch.birkhoff_proj_n4_backward(G[a:b].contiguous(), T)["D"]
        torch.cuda.synchronize(dev)
        sizes = shard_sizes(n, world)
        width = max(sizes)
        pad = lambda x: torch.cat([x, x.new_zeros(width - x.shape[0], 4, 4)])  # noqa: E731
        gT = [torch.empty(width, 4, 4, device=dev) for _ in range(world)]
        gD = [torch.empty(width, 4, 4, device=dev) for _ in range(world)]
        dist.all_gather(gT, pad(T))
        dist.all_gather(gD, pad(D))
        if rank == 0:
            Tall = torch.cat([g[:m] for g, m in zip(gT, sizes)])
            Dall = torch.cat([g[:m] for g, m in zip(gD, sizes)])
            T1 = mhc_proj.torch.birkhoff_proj_n4(R, 1e-6)["T"]
            D1 = mhc_proj.torch.birkhoff_proj_n4_backward(G, T1)["D"]
            ok = (torch.equal(Tall.view(torch.int32), T1.view(torch.int32))
                  and torch.equal(Dall.view(torch.int32), D1.view(torch.int32)))
            with open(out_path, "w") as f:
                f.write("ok" if ok else "mismatch")
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_shards_equal_one_gpu(tmp_path):
    out = str(tmp_path / "result")
    n = (1 << 20) + 3  # uneven shards
    mp.start_processes(_worker, args=(2, _free_port(), n, out), nprocs=2, join=True, start_method="spawn")
    assert open(out).read() == "ok"
