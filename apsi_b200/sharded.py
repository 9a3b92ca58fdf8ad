"""Column-sharded low-bit linear layer over the ranks of a process group (one process per GPU).

Rank r of G holds output rows [r * N / G, (r + 1) * N / G) of the packed weights: codes and scales.  The int4
groups of 128 run along K, so a shard never splits a group, and the quantisation of a shard equals the
corresponding rows of the whole layer's quantisation.  x is replicated.  Every rank multiplies its shard with
the library's kernels.  One all-gather (NCCL over NVLink on GPUs) collects the [M, N / G] outputs rank-major,
and the interleave kernel turns [G][M][N / G] into the row-major [M, N].  The kernels' summation structure
depends only on K, so the gathered result is bit-identical to the unsharded layer's.

The reference has no multi-GPU inference path; this module is the scale-out of apsi/precision.py:294-299
(``qmatmul``) for layers too large for one GPU or for more weight bandwidth.
"""
import torch
import torch.distributed as dist

from . import kernels
from ._lib import LowbitError, LB_E_ARG, FMT_INT4_G128, FMT_INT8_ROW

__all__ = ["shard_rows", "ColumnShardedLinear", "gather_columns"]


def shard_rows(N, world, rank):
    """[start, stop) of the output rows that rank `rank` of `world` holds.  N must divide evenly."""
    if world < 1 or not 0 <= rank < world:
        raise LowbitError(LB_E_ARG, f"rank {rank} is not in a world of {world}")
    if N % world:
        raise LowbitError(LB_E_ARG, f"N ({N}) must be a multiple of the number of shards ({world})")
    per = N // world
    return rank * per, (rank + 1) * per


def _all_gather(y_local, group):
    """[M, Nl] on every rank -> [G, M, Nl] (rank-major) on every rank."""
    world = dist.get_world_size(group)
    out = torch.empty((world,) + tuple(y_local.shape), dtype=y_local.dtype, device=y_local.device)
    if y_local.is_cuda and dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out.view(-1), y_local.contiguous().view(-1), group=group)
    else:
        dist.all_gather(list(out.unbind(0)), y_local.contiguous(), group=group)
    return out


def gather_columns(y_local, group=None):
    """The [M, N] output from every rank's [M, N / G] column shard (all ranks receive it)."""
    if dist.get_world_size(group) == 1:
        return y_local
    g = _all_gather(y_local, group)
    G, M, Nl = g.shape
    if g.is_cuda:
        return kernels.interleave_cols(g, G, M, Nl)
    # host tensors (gloo process groups): the same reassembly as a copy, no arithmetic
    return g.permute(1, 0, 2).reshape(M, G * Nl).contiguous()


class ColumnShardedLinear:
    """y[M, N] = x[M, K] . deq(W)[N, K]^T (+ bias) with W's rows split over the ranks of `group`.

    ``local_op(x, codes, scales, n_local, bias_local) -> y_local`` computes one rank's product.  By default
    it is the library's kernel, ``kernels.linear``, which takes CUDA tensors only.
    """

    def __init__(self, fmt, codes, scales, N, K, bias=None, group=None, local_op=None):
        if fmt not in (FMT_INT4_G128, FMT_INT8_ROW):
            raise LowbitError(LB_E_ARG, f"format {fmt} has no product kernel")
        self.fmt, self.N, self.K, self.group = fmt, int(N), int(K), group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.row0, self.row1 = shard_rows(self.N, self.world, self.rank)
        self.n_local = self.row1 - self.row0
        if codes.shape[0] != self.n_local or scales.shape[0] != self.n_local:
            raise LowbitError(LB_E_ARG, f"rank {self.rank} holds {codes.shape[0]} rows, expected {self.n_local}")
        self.codes, self.scales = codes, scales
        self.bias = bias[self.row0:self.row1].contiguous() if bias is not None and bias.shape[0] == self.N else bias
        self.local_op = local_op or self._kernel_product

    @classmethod
    def from_weight(cls, W, fmt=FMT_INT4_G128, bias=None, group=None, local_op=None, quantize=None):
        """Quantise this rank's rows of a full [N, K] weight (every rank passes the same W).

        ``quantize(W_rows) -> (codes, scales)`` defaults to the library's kernels (CUDA tensors)."""
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        N, K = W.shape
        r0, r1 = shard_rows(N, world, rank)
        rows = W[r0:r1].contiguous()
        if quantize is None:
            if fmt == FMT_INT4_G128:
                codes, scales, _ = kernels.quant_int4_g128(rows, want_scale32=False)
            else:
                codes, scales, _ = kernels.quant_int8_rows(rows, want_scale32=False)
        else:
            codes, scales = quantize(rows)
        return cls(fmt, codes, scales, N, K, bias=bias, group=group, local_op=local_op)

    def _kernel_product(self, x, codes, scales, n_local, bias):
        return kernels.linear(self.fmt, x, codes, scales, n_local, bias=bias)

    def local(self, x):
        """This rank's [M, N / G] columns."""
        return self.local_op(x, self.codes, self.scales, self.n_local, self.bias)

    def __call__(self, x):
        return gather_columns(self.local(x), self.group)
