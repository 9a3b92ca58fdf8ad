"""Column-sharded layer on real GPUs: NCCL ranks, the library's kernels as each rank's product, the gathered
output bit-identical to the unsharded product.  Needs two or more GPUs (skipped otherwise)."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, M, N, K, out_dir):
    import datetime
    import torch.distributed as dist
    from apsi_b200 import sharded, kernels
    from apsi_b200._lib import FMT_INT4_G128
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        gen = torch.Generator(device=dev)
        gen.manual_seed(17)                             # the same W and x on every rank
        W = torch.randn((N, K), generator=gen, device=dev) * 0.02
        x = torch.randn((M, K), generator=gen, device=dev).to(torch.bfloat16)
        layer = sharded.ColumnShardedLinear.from_weight(W, FMT_INT4_G128)
        y = layer(x)
        torch.cuda.synchronize(dev)
        if rank == 0:
            packed, s16, _ = kernels.quant_int4_g128(W, want_scale32=False)
            full = kernels.linear(FMT_INT4_G128, x, packed, s16, N)
            torch.cuda.synchronize(dev)
            np.save(os.path.join(out_dir, "y.npy"), y.view(torch.int16).cpu().numpy())
            np.save(os.path.join(out_dir, "full.npy"), full.view(torch.int16).cpu().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("M,N,K", [(1, 11008, 4096), (4, 4096, 11008), (64, 2048, 4096)])
def test_nccl_column_shards_match_unsharded_bits(tmp_path, M, N, K):
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), M, N, K, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    y = np.load(tmp_path / "y.npy")
    full = np.load(tmp_path / "full.npy")
    assert y.shape == full.shape == (M, N)
    assert np.array_equal(y, full)
