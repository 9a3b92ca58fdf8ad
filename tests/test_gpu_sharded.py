"""Column-sharded layer on real GPUs: NCCL ranks, the library's kernels as each rank's product, the assembled
output bit-identical to the unsharded product -- through the NCCL all-gather, and with the gather fused into
the product (peer stores over NVLink + the flag barrier).  The multi-rank tests need two or more GPUs (skipped
otherwise); the barrier's timeout is tested on one GPU."""
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


def _worker(rank, world, port, M, N, K, out_dir, mode="nccl"):
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
        peers = sharded.PeerOutputs(N, M, dev) if mode == "p2p" else None
        layer = sharded.ColumnShardedLinear.from_weight(W, FMT_INT4_G128, peers=peers)
        outs = []
        for call in range(3):                           # p2p: both output buffers, then the first again
            xc = x if call == 0 else torch.randn((M, K), generator=gen, device=dev).to(torch.bfloat16)
            y = layer(xc)
            torch.cuda.synchronize(dev)
            outs.append((xc, y.clone()))
        if mode == "p2p":
            assert kernels.device_errors(dev) == 0
        packed, s16, _ = kernels.quant_int4_g128(W, want_scale32=False)
        for call, (xc, y) in enumerate(outs):
            full = kernels.linear(FMT_INT4_G128, xc, packed, s16, N)
            torch.cuda.synchronize(dev)
            np.save(os.path.join(out_dir, f"y{rank}_{call}.npy"), y.view(torch.int16).cpu().numpy())
            np.save(os.path.join(out_dir, f"full{rank}_{call}.npy"), full.view(torch.int16).cpu().numpy())
        if peers is not None:
            peers.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("mode", ["nccl", "p2p"])
@pytest.mark.parametrize("M,N,K", [(1, 11008, 4096), (4, 4096, 11008), (64, 2048, 4096), (1, 8192, 28672),
                                   (64, 28672, 8192), (64, 8192, 28672)])
def test_column_shards_match_unsharded_bits(tmp_path, M, N, K, mode, world):
    """Every rank's assembled [M, N] output equals the unsharded product bit for bit, at 2, 4 and 8 ranks (as
    many as the machine has GPUs), over three calls (both p2p output buffers)."""
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.start_processes(_worker, args=(world, _free_port(), M, N, K, str(tmp_path), mode), nprocs=world, join=True,
                       start_method="spawn")
    for rank in range(world):
        for call in range(3):
            y = np.load(tmp_path / f"y{rank}_{call}.npy")
            full = np.load(tmp_path / f"full{rank}_{call}.npy")
            assert y.shape == full.shape == (M, N)
            assert np.array_equal(y, full), (rank, call)


def test_rank_barrier_reports_a_rank_that_never_arrives(cuda):
    """One GPU: a barrier of two ranks where the second never arrives (its flag is never written) gives up
    after its time limit, reports LB_DEVERR_PEER_TIMEOUT, and the context stays usable."""
    from apsi_b200 import kernels
    from apsi_b200._lib import DEVERR_PEER_TIMEOUT, FMT_INT4_G128
    kernels.device_errors(cuda)                          # start clean
    mine = torch.zeros(2, dtype=torch.int32, device=cuda)
    other = torch.zeros(2, dtype=torch.int32, device=cuda)
    kernels.rank_barrier([mine.data_ptr(), other.data_ptr()], 0, 1, cuda, timeout_ms=50)
    torch.cuda.synchronize(cuda)
    assert kernels.device_errors(cuda) == DEVERR_PEER_TIMEOUT
    assert mine.tolist() == [1, 0] and other.tolist() == [1, 0]   # rank 0 arrived in both arrays
    # both ranks arrived: no timeout
    other_side = torch.tensor([1, 1], dtype=torch.int32, device=cuda)
    kernels.rank_barrier([other_side.data_ptr(), other.data_ptr()], 0, 1, cuda, timeout_ms=50)
    torch.cuda.synchronize(cuda)
    assert kernels.device_errors(cuda) == 0
    W = torch.randn((256, 1024), device=cuda) * 0.02
    p, s16, _ = kernels.quant_int4_g128(W, want_scale32=False)
    x = torch.randn((1, 1024), device=cuda).to(torch.bfloat16)
    y = kernels.linear(FMT_INT4_G128, x, p, s16, 256)
    torch.cuda.synchronize(cuda)
    assert torch.isfinite(y.float()).all() and kernels.device_errors(cuda) == 0
