"""Host logic of the column-sharded layer on CPU: two gloo ranks, the oracle as each rank's local product.

What runs here is the part that is not a kernel: the row split, the quantisation of a shard (equal to the same
rows of the whole layer's), the all-gather and the reassembly of [G][M][N/G] into [M, N].  The product on a
GPU is the library's kernel (tests/test_gpu_linear.py checks that shards are bit-identical there)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from apsi_b200 import sharded
from apsi_b200._lib import FMT_INT4_G128, FMT_INT8_ROW, LowbitError
from oracle import lowbit_oracle as ora


def _free_port():
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_quantize(fmt):
    def q(rows):
        W = rows.numpy()
        if fmt == FMT_INT4_G128:
            packed, _, s16 = ora.quant_int4_g128(W)
            return torch.from_numpy(packed), torch.from_numpy(s16)
        codes, _, s16 = ora.quant_int8_rows(W)
        return torch.from_numpy(codes), torch.from_numpy(s16)
    return q


def _oracle_product(fmt):
    def op(x, codes, scales, n_local, bias):
        if fmt == FMT_INT4_G128:
            Wd = ora.dequant_int4_g128(codes.numpy(), scales.numpy())
        else:
            Wd = ora.dequant_int8_rows(codes.numpy(), scales.numpy())
        y = ora.linear_ref(x.numpy(), Wd, None if bias is None else bias.numpy())
        return torch.from_numpy(y.astype(np.float32))
    return op


def _worker(rank, world, port, fmt, M, N, K, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, W = ora.make_config_inputs(M, N, K, seed=3)
        bias = np.random.default_rng(5).standard_normal(N).astype(np.float32)
        layer = sharded.ColumnShardedLinear.from_weight(
            torch.from_numpy(W), fmt, bias=torch.from_numpy(bias), quantize=_oracle_quantize(fmt),
            local_op=_oracle_product(fmt))
        y = layer(torch.from_numpy(x))
        np.save(os.path.join(out_dir, f"y{rank}.npy"), y.numpy())
        np.save(os.path.join(out_dir, f"codes{rank}.npy"), layer.codes.numpy())
        np.save(os.path.join(out_dir, f"rows{rank}.npy"), np.array([layer.row0, layer.row1]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fmt", [FMT_INT4_G128, FMT_INT8_ROW])
def test_two_rank_column_shards_reassemble_the_full_layer(tmp_path, fmt):
    M, N, K, world = 3, 96, 256, 2
    mp.start_processes(_worker, args=(world, _free_port(), fmt, M, N, K, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    x, W = ora.make_config_inputs(M, N, K, seed=3)
    bias = np.random.default_rng(5).standard_normal(N).astype(np.float32)
    if fmt == FMT_INT4_G128:
        codes_full, _, s16 = ora.quant_int4_g128(W)
        Wd = ora.dequant_int4_g128(codes_full, s16)
    else:
        codes_full, _, s16 = ora.quant_int8_rows(W)
        Wd = ora.dequant_int8_rows(codes_full, s16)
    ref = ora.linear_ref(x, Wd, bias).astype(np.float32)
    for r in range(world):
        y = np.load(tmp_path / f"y{r}.npy")
        assert y.shape == (M, N)
        assert np.array_equal(y, ref), f"rank {r}: gathered output differs from the unsharded product"
        r0, r1 = np.load(tmp_path / f"rows{r}.npy")
        assert (r0, r1) == (r * N // world, (r + 1) * N // world)
        assert np.array_equal(np.load(tmp_path / f"codes{r}.npy"), codes_full[r0:r1]), "shard codes != full rows"


def test_shard_rows_split_and_rejects_uneven():
    assert sharded.shard_rows(11008, 8, 3) == (4128, 5504)
    assert sharded.shard_rows(28672, 4, 0) == (0, 7168)
    with pytest.raises(LowbitError):
        sharded.shard_rows(100, 8, 0)
    with pytest.raises(LowbitError):
        sharded.shard_rows(96, 2, 2)
