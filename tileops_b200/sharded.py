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

AWQ layers on CUDA can also run the gather inside the GEMM (`ShardedAWQLinear.gathered`,
`gathered_gemm`): every rank maps every peer's output buffer (`PeerBuffers`, CUDA IPC over
NVLink), the kernel (the decode kernel for 1-32 tokens, the tensor-core GEMM above) stores each
finished output tile of its slice into all of them, and a rank barrier on the GPU
(`PeerBarrier`: flags raised in every rank's mapped memory, no collective) orders the peers'
reads after every rank's stores. The exchange overlaps the GEMM and needs no reshuffle: each
buffer is the [M, N] output.
"""

from __future__ import annotations

import ctypes
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


class _DeviceArray:
    """Exposes a raw device allocation to torch.as_tensor (no copy, no ownership)."""

    def __init__(self, ptr_value: int, shape: tuple[int, ...], typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr,
                                         "data": (ptr_value, False), "version": 3,
                                         "strides": None}


class PeerBuffers:
    """`count` output buffers of [m, n] 16-bit elements on every rank of `group`, each mapped
    into every rank's process: ptrs[b][r] is rank r's buffer b as seen from this process and
    tensors[b] this rank's own buffer b. Collective: every rank constructs it with the same
    shape. close() is collective too."""

    def __init__(self, m: int, n: int, dtype: torch.dtype, group=None, count: int = 2):
        from . import _lib

        if dtype not in (torch.float16, torch.bfloat16):
            raise TypeError(f"PeerBuffers: 16-bit outputs only (got {dtype})")
        self.group = group
        self.rank, self.world = _world(group)
        self.shape = (m, n)
        dev = torch.device("cuda", torch.cuda.current_device())
        nbytes = m * n * 2
        own, handles = [], []
        for _ in range(count):
            p, h = _lib.ipc_alloc(nbytes)
            own.append(p)
            handles.append(h)
        self._opened: list[int] = []
        self.ptrs: list[list[int]] = []
        try:
            table: list = [None] * self.world
            dist.all_gather_object(table, (handles, (m, n, str(dtype))), group=group)
            for r, (_, meta) in enumerate(table):
                if tuple(meta) != (m, n, str(dtype)):
                    raise ValueError(f"PeerBuffers: rank {r} has {meta}, rank {self.rank} has "
                                     f"{(m, n, str(dtype))}")
            for b in range(count):
                row = []
                for r in range(self.world):
                    if r == self.rank:
                        row.append(own[b])
                    else:
                        q = _lib.ipc_open(table[r][0][b])
                        self._opened.append(q)
                        row.append(q)
                self.ptrs.append(row)
        except Exception:
            for q in self._opened:
                _lib.ipc_close(q)
            for p in own:
                _lib.ipc_free(p)
            raise
        self._own = own
        self.tensors = [torch.as_tensor(_DeviceArray(p, (m, n), "<i2"), device=dev).view(dtype)
                        for p in own]
        self._next = 0

    def next_index(self) -> int:
        """Buffers are used in turn; a buffer is reused every `count` calls."""
        b = self._next
        self._next = (self._next + 1) % len(self._own)
        return b

    def close(self) -> None:
        from . import _lib

        if not self._own:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)  # no peer writes into our buffers any more
        self.tensors = []
        for q in self._opened:
            _lib.ipc_close(q)
        dist.barrier(group=self.group)  # every peer has unmapped ours
        for p in self._own:
            _lib.ipc_free(p)
        self._opened, self._own, self.ptrs = [], [], []


class PeerBarrier:
    """The GPU-side rank barrier of a group (to_peer_barrier): every rank's flag array mapped
    into every rank's process plus this rank's barrier count. wait() queues the barrier on the
    current stream: work queued after it sees every rank's stores queued before theirs.
    Collective: every rank constructs it, calls wait() the same number of times, and closes it."""

    def __init__(self, group=None):
        from . import _lib

        self.group = group
        self.rank, self.world = _world(group)
        dev = torch.device("cuda", torch.cuda.current_device())
        nbytes = int(_lib.load().to_peer_flags_bytes())
        own, handle = _lib.ipc_alloc(nbytes)
        torch.as_tensor(_DeviceArray(own, (nbytes,), "|u1"), device=dev).zero_()
        self.counter = torch.zeros(1, dtype=torch.int64, device=dev)
        torch.cuda.synchronize()  # zeroed before any peer can raise a slot
        self._own, self._opened = own, []
        try:
            table: list = [None] * self.world
            dist.all_gather_object(table, handle, group=group)
            ptrs = []
            for r in range(self.world):
                if r == self.rank:
                    ptrs.append(own)
                else:
                    q = _lib.ipc_open(table[r])
                    self._opened.append(q)
                    ptrs.append(q)
        except Exception:
            for q in self._opened:
                _lib.ipc_close(q)
            _lib.ipc_free(own)
            raise
        self._table = (ctypes.c_void_p * self.world)(*ptrs)
        dist.barrier(group=group)  # every rank's flags are zero and mapped

    def wait(self) -> None:
        from . import _lib

        _lib.check(_lib.load().to_peer_barrier(self._table, self.world, self.rank,
                                               self.counter.data_ptr(), _lib.stream_ptr()),
                   "peer_barrier")

    def close(self) -> None:
        from . import _lib

        if self._own is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for q in self._opened:
            _lib.ipc_close(q)
        dist.barrier(group=self.group)
        _lib.ipc_free(self._own)
        self._own, self._opened = None, []


_BARRIERS: dict = {}


def peer_barrier(group=None) -> PeerBarrier:
    """The group's rank barrier, created on first use (collectively) and shared by its layers."""
    key = id(group) if group is not None else None
    b = _BARRIERS.get(key)
    if b is None:
        b = PeerBarrier(group)
        _BARRIERS[key] = b
    return b


def close_peer_barriers() -> None:
    """Releases every group's rank barrier (collective over each group)."""
    for b in list(_BARRIERS.values()):
        b.close()
    _BARRIERS.clear()


def gathered_gemm(x: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor,
                  qzeros: torch.Tensor, bufs: "PeerBuffers", group=None) -> Optional[torch.Tensor]:
    """y = x @ dequant(W) for this rank's column slice, all-gathered inside the kernel: each
    rank stores its [M, N/P] slice into every rank's [M, N] buffer of `bufs` (the next one in
    turn), then the group's GPU rank barrier orders the reads. Returns this rank's full [M, N]
    buffer, or None (nothing launched) for shapes the gathering kernels do not take."""
    from . import _lib
    from .quant_awq import _as_words

    rank, world = _world(group)
    _lib.ensure_device(x, "awq_gemm_gather")
    m, k = x.shape
    dtype = scales.dtype
    b = bufs.next_index()
    xx = x.to(dtype).contiguous()
    qw, qz = _as_words(qweight), _as_words(qzeros)
    n_local = qweight.shape[1] * 8
    group_size = k // qzeros.shape[0]
    lib = _lib.load()
    ws_bytes = _lib.workspace_bytes("to_awq_gemm_workspace_size", m, k, n_local, group_size)
    ws = _lib.workspace(ws_bytes, x.get_device())
    table = (ctypes.c_void_p * world)(*bufs.ptrs[b])
    rc = lib.to_awq_gemm_gather(xx.data_ptr(), qw.data_ptr(), scales.data_ptr(),
                                _lib.DTYPE_CODES[dtype], qz.data_ptr(), table, world, rank, m, k,
                                n_local, group_size, _lib.ptr(ws), ws_bytes, _lib.stream_ptr())
    if rc == _lib.TO_EUNSUPPORTED:
        return None
    _lib.check(rc, "awq_gemm_gather")
    peer_barrier(group).wait()
    return bufs.tensors[b]


def gathered_gemm_act(x: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor,
                      qzeros: torch.Tensor, bufs: "PeerBuffers", act: int = 0,
                      group=None) -> Optional[torch.Tensor]:
    """act(gate) * up of this rank's slice of a gate_up linear (interleaved by
    awq_interleave_gate_up; N/P columns, N/(2P) outputs), all-gathered inside the decode kernel
    into every rank's [M, N/2] buffer of `bufs`, then the GPU rank barrier. Returns this rank's
    full [M, N/2] buffer, or None (nothing launched) where the decode kernel does not take the
    shapes (more than 32 tokens): run awq_gemm_silu_and_mul and gather_columns instead."""
    from . import _lib
    from .quant_awq import _as_words

    rank, world = _world(group)
    _lib.ensure_device(x, "awq_gemm_act_gather")
    m, k = x.shape
    dtype = scales.dtype
    b = bufs.next_index()
    xx = x.to(dtype).contiguous()
    qw, qz = _as_words(qweight), _as_words(qzeros)
    n_local = qweight.shape[1] * 8
    group_size = k // qzeros.shape[0]
    lib = _lib.load()
    ws_bytes = _lib.workspace_bytes("to_awq_gemm_workspace_size", m, k, n_local, group_size)
    ws = _lib.workspace(ws_bytes, x.get_device())
    table = (ctypes.c_void_p * world)(*bufs.ptrs[b])
    rc = lib.to_awq_gemm_act_gather(xx.data_ptr(), qw.data_ptr(), scales.data_ptr(),
                                    _lib.DTYPE_CODES[dtype], qz.data_ptr(), table, world, rank,
                                    m, k, n_local, group_size, act, _lib.ptr(ws), ws_bytes,
                                    _lib.stream_ptr())
    if rc == _lib.TO_EUNSUPPORTED:
        return None
    _lib.check(rc, "awq_gemm_act_gather")
    peer_barrier(group).wait()
    return bufs.tensors[b]


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
        self._peer_buffers: dict[int, PeerBuffers] = {}

    @classmethod
    def from_shard(cls, qweight, scales, qzeros, group=None,
                   compute: Optional[Callable] = None) -> "ShardedAWQLinear":
        """A layer from this rank's column slice, already cut (N = world x the slice's)."""
        self = cls.__new__(cls)
        self.group = group
        self.rank, self.world = _world(group)
        self.n = qweight.shape[1] * 8 * self.world
        self.qweight, self.scales, self.qzeros = qweight, scales, qzeros
        if compute is None:
            from .quant_awq import awq_gemm

            compute = lambda x, qw, s, qz: awq_gemm(x, qw, s, qz, 1)  # noqa: E731
        self.compute = compute
        self._peer_buffers = {}
        return self

    def local(self, x: torch.Tensor) -> torch.Tensor:
        return self.compute(x, self.qweight, self.scales, self.qzeros)

    def __call__(self, x: torch.Tensor, gather: bool = True, layout: str = "mn") -> torch.Tensor:
        y = self.local(x)
        return gather_columns(y, self.group, layout) if gather else y

    def gathered(self, x: torch.Tensor) -> torch.Tensor:
        """The whole [M, N] output with the all-gather done inside the GEMM (CUDA ranks of an
        NCCL group) and a GPU rank barrier after it. The result is one of two buffers per M that
        the layer reuses in turn: it stays valid until the layer's second-next call with the
        same M. Shapes the fused kernels do not take run the local GEMM and an all-gather."""
        if self.world == 1:
            return self.local(x)
        m = x.shape[0]
        bufs = self._peer_buffers.get(m)
        if bufs is None:
            bufs = PeerBuffers(m, self.n, self.scales.dtype, self.group)
            self._peer_buffers[m] = bufs
        y = gathered_gemm(x, self.qweight, self.scales, self.qzeros, bufs, self.group)
        return y if y is not None else gather_columns(self.local(x), self.group)

    def close(self) -> None:
        """Releases the peer-mapped output buffers (collective)."""
        for bufs in self._peer_buffers.values():
            bufs.close()
        self._peer_buffers = {}


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
