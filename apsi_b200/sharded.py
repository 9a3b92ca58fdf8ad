"""Column-sharded low-bit linear layer over the ranks of a process group (one process per GPU).

Rank r of G holds output rows [r * N / G, (r + 1) * N / G) of the packed weights: codes and scales.  The int4
groups of 128 run along K, so a shard never splits a group, and the quantisation of a shard equals the
corresponding rows of the whole layer's quantisation.  x is replicated.  Every rank multiplies its shard with
the library's kernels.  The kernels' summation structure depends only on K, so the assembled result is
bit-identical to the unsharded layer's.

Two ways to assemble the [M, N] output on every rank:

* without ``peers``: each rank writes its [M, N / G] block locally, one all-gather (NCCL over NVLink on GPUs,
  gloo on CPU) collects the blocks rank-major and the interleave kernel turns [G][M][N / G] into [M, N];
* with ``peers`` (a ``PeerOutputs``, GPUs): the gather is fused into the product.  Every rank's GEMV / GEMM
  epilogue stores its columns straight into every rank's [M, N] output over NVLink (the other ranks' output
  buffers are mapped through CUDA IPC), then one flag barrier with a bounded wait says all columns have
  arrived.  No collective launch and no interleave pass remain on the path.

The reference has no multi-GPU inference path; this module is the scale-out of apsi/precision.py:294-299
(``qmatmul``) for layers too large for one GPU or for more weight bandwidth.
"""
import torch
import torch.distributed as dist

from . import kernels
from ._lib import LowbitError, LB_E_ARG, FMT_INT4_G128, FMT_INT8_ROW

__all__ = ["shard_rows", "ColumnShardedLinear", "gather_columns", "PeerOutputs"]


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


class PeerOutputs:
    """Output buffers that every rank of `group` can write: per rank, two [max_rows, N] bfloat16 buffers (used
    alternately, so a rank writing call n + 1 never overwrites what another rank still reads from call n) and
    one flag array for the barrier, allocated with ``kernels.peer_alloc`` and mapped on the other ranks.

    ``out(M)`` gives this call's buffer pointers (all ranks) and a [M, N] view of the local one; ``finish()``
    runs the barrier on the current stream.  ``close()`` unmaps and frees (every rank, collectively)."""

    def __init__(self, N, max_rows, device, group=None, timeout_ms=0):
        self.N, self.max_rows, self.device = int(N), int(max_rows), torch.device(device)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.timeout_ms = timeout_ms
        nbytes = self.max_rows * self.N * 2
        self._views, self._own, handles = [], [], []
        for _ in range(2):
            t, p, h = kernels.peer_alloc(nbytes, self.device)
            self._views.append(t.view(torch.bfloat16).view(self.max_rows, self.N))
            self._own.append(p)
            handles.append(h)
        tf, pf, hf = kernels.peer_alloc(4 * (self.world + 1), self.device)   # G flags + the epoch counter
        self._own.append(pf)
        handles.append(hf)
        everyone = [None] * self.world
        dist.all_gather_object(everyone, handles, group=group)
        self._opened = []
        self.ptrs = []                            # [buffer 0, buffer 1, flags] -> one pointer per rank
        for j in range(3):
            row = []
            for g in range(self.world):
                if g == self.rank:
                    row.append(self._own[j])
                else:
                    p = kernels.peer_open(everyone[g][j], self.device)
                    self._opened.append(p)
                    row.append(p)
            self.ptrs.append(row)
        self.epoch = 0

    def out(self, M):
        """(pointers of every rank's output buffer for the next call, the local [M, N] view of it)."""
        if M > self.max_rows:
            raise LowbitError(LB_E_ARG, f"{M} rows exceed the {self.max_rows} the buffers hold")
        b = (self.epoch + 1) & 1
        return self.ptrs[b], self._views[b][:M]

    def view0(self, M):
        """The local [M, N] view of output buffer 0 (the one a caller that passes ``ptrs[0]`` itself writes)."""
        return self._views[0][:M]

    def finish(self):
        """Barrier: every rank's stores of this call are visible on every rank (on the current stream).  The
        barrier's epoch comes from the device-side counter, so its flags stay in step when a CUDA graph replays
        it.  The choice between the two output buffers is made on the host (``out``), so a captured graph
        replays into the buffers it was captured with: capture two consecutive calls (one per buffer) in one
        graph, or a faster rank's next replay may overwrite columns a slower rank is still reading."""
        self.epoch += 1
        kernels.rank_barrier(self.ptrs[2], self.rank, 0, self.device, self.timeout_ms)

    def close(self):
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)            # nobody writes into a buffer that is being unmapped
        for p in self._opened:
            kernels.peer_close(p, self.device)
        dist.barrier(group=self.group)
        for p in self._own:
            kernels.peer_free(p, self.device)
        self._opened, self._own, self.ptrs = [], [], []


class ColumnShardedLinear:
    """y[M, N] = x[M, K] . deq(W)[N, K]^T (+ bias) with W's rows split over the ranks of `group`.

    ``local_op(x, codes, scales, n_local, bias_local) -> y_local`` computes one rank's product.  By default
    it is the library's kernel, ``kernels.linear``, which takes CUDA tensors only.
    """

    def __init__(self, fmt, codes, scales, N, K, bias=None, group=None, local_op=None, peers=None):
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
        self.peers = peers                        # PeerOutputs: gather fused into the product (p2p)

    @classmethod
    def from_weight(cls, W, fmt=FMT_INT4_G128, bias=None, group=None, local_op=None, quantize=None, peers=None):
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
        return cls(fmt, codes, scales, N, K, bias=bias, group=group, local_op=local_op, peers=peers)

    def _kernel_product(self, x, codes, scales, n_local, bias):
        return kernels.linear(self.fmt, x, codes, scales, n_local, bias=bias)

    def local(self, x):
        """This rank's [M, N / G] columns."""
        return self.local_op(x, self.codes, self.scales, self.n_local, self.bias)

    def __call__(self, x, static_weights=False):
        """The full [M, N] output on every rank.  With ``peers`` (p2p), it is a view of the shared output
        buffer, valid until the call after next; copy it to keep it longer."""
        if self.peers is None or self.world == 1:
            return gather_columns(self.local(x), self.group)
        K = x.shape[-1]
        M = x.numel() // K
        ptrs, view = self.peers.out(M)
        kernels.linear_sharded(self.fmt, x, self.codes, self.scales, self.n_local, ptrs, self.rank, self.peers.N,
                               bias=self.bias, static_weights=static_weights)
        self.peers.finish()
        return view
