"""N-sharded quantized linear layers across the GPUs of one node.

A layer's output columns are split evenly over the ranks of a process group: rank r owns
columns [r*N/P, (r+1)*N/P). For AWQ that is a slice of the packed words of `qweight` and `qzeros`
and of the columns of `scales`; for W8A8 it is a block of rows of the [N, K] weight and of its
per-channel scales. Weights are sliced once, at construction. A forward call runs the local
kernel on the rank's slice (no communication inside the kernel) and, when the consumer needs
the whole output, gathers the slices with one all-gather over NCCL (NVLink / NVSwitch), then
lays them out as [M, N].

The compute step is a constructor argument so the bookkeeping runs unchanged on CPU ranks of a
gloo group in tests; the default is the sm_100a kernel of this package.
"""

from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist


def _world(group) -> tuple[int, int]:
    if group is None and not dist.is_initialized():
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def shard_bounds(n: int, rank: int, world: int, multiple: int = 1) -> tuple[int, int]:
    """Column range [lo, hi) of `rank`; N must split into equal parts that are multiples of
    `multiple` (8 for AWQ's packed words)."""
    if n % world != 0 or (n // world) % multiple != 0:
        raise ValueError(f"N={n} does not split into {world} shards of a multiple of {multiple}")
    per = n // world
    return rank * per, (rank + 1) * per


def shard_awq(qweight: torch.Tensor, scales: torch.Tensor, qzeros: torch.Tensor, rank: int,
              world: int):
    """This rank's column slice of AWQ weights (contiguous copies)."""
    n = qweight.shape[1] * 8
    lo, hi = shard_bounds(n, rank, world, 8)
    return (qweight[:, lo // 8:hi // 8].contiguous(), scales[:, lo:hi].contiguous(),
            qzeros[:, lo // 8:hi // 8].contiguous())


def shard_w8a8(weight: torch.Tensor, weight_scale: torch.Tensor, block_n: int, rank: int,
               world: int):
    """This rank's rows of a W8A8 weight [N, K] and the matching rows of its block scales
    (a per-tensor scale, one block over all N, is replicated)."""
    n = weight.shape[0]
    lo, hi = shard_bounds(n, rank, world, 1)
    if block_n >= n:
        return weight[lo:hi].contiguous(), weight_scale.contiguous(), hi - lo
    if lo % block_n != 0 or hi % block_n != 0:
        raise ValueError(f"shard rows [{lo}, {hi}) do not align with block_n={block_n}")
    return (weight[lo:hi].contiguous(), weight_scale[lo // block_n:hi // block_n].contiguous(),
            block_n)


def gather_columns(local: torch.Tensor, group=None, layout: str = "mn") -> torch.Tensor:
    """All-gathers the [M, N/P] slices of every rank. layout "mn" returns [M, N]; "pmn" returns
    the gathered [P, M, N/P] without the final reshuffle (for consumers that accept it)."""
    rank, world = _world(group)
    if world == 1:
        return local if layout == "mn" else local.unsqueeze(0)
    m, npr = local.shape
    local = local.contiguous()
    out = torch.empty(world, m, npr, dtype=local.dtype, device=local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, local, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), local, group=group)
    if layout == "pmn":
        return out
    return out.permute(1, 0, 2).reshape(m, world * npr)


class ShardedAWQLinear:
    """y = x @ dequant(W) with W's columns split across the group (tileops/quant_awq.py:112)."""

    def __init__(self, qweight, scales, qzeros, group=None,
                 compute: Optional[Callable] = None):
        self.group = group
        self.rank, self.world = _world(group)
        self.n = qweight.shape[1] * 8
        self.qweight, self.scales, self.qzeros = shard_awq(qweight, scales, qzeros, self.rank,
                                                           self.world)
        if compute is None:
            from .quant_awq import awq_gemm

            compute = lambda x, qw, s, qz: awq_gemm(x, qw, s, qz, 1)  # noqa: E731
        self.compute = compute

    def local(self, x: torch.Tensor) -> torch.Tensor:
        return self.compute(x, self.qweight, self.scales, self.qzeros)

    def __call__(self, x: torch.Tensor, gather: bool = True, layout: str = "mn") -> torch.Tensor:
        y = self.local(x)
        return gather_columns(y, self.group, layout) if gather else y


class ShardedW8A8Linear:
    """C = dequant(A) @ dequant(B).T with B's rows (output columns) split across the group
    (tileops/quant_int8.py:180, tileops/quant_fp8.py:188)."""

    def __init__(self, weight, weight_scale, block_size, group=None,
                 output_dtype: torch.dtype = torch.bfloat16,
                 compute: Optional[Callable] = None):
        self.group = group
        self.rank, self.world = _world(group)
        self.weight, self.weight_scale, block_n = shard_w8a8(weight, weight_scale, block_size[0],
                                                             self.rank, self.world)
        self.block_size = [block_n, block_size[1]]
        self.output_dtype = output_dtype
        if compute is None:
            if weight.dtype == torch.int8:
                from .quant_int8 import w8a8_block_int8_matmul as mm
            else:
                from .quant_fp8 import w8a8_block_fp8_matmul as mm
            compute = lambda a, b, a_s, b_s, bs, od: mm(a, b, a_s, b_s, bs, od)  # noqa: E731
        self.compute = compute

    def local(self, a: torch.Tensor, a_s: torch.Tensor) -> torch.Tensor:
        return self.compute(a, self.weight, a_s, self.weight_scale, self.block_size,
                            self.output_dtype)

    def __call__(self, a: torch.Tensor, a_s: torch.Tensor, gather: bool = True,
                 layout: str = "mn") -> torch.Tensor:
        y = self.local(a, a_s)
        return gather_columns(y, self.group, layout) if gather else y
