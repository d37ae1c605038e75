"""Row-sharded INT4 / INT8 GEMV over the GPUs of one node (one process per GPU).

The weight matrix is split into contiguous row shards, one per rank of a
torch.distributed group; x is replicated (every rank holds the same x); after
a step every rank holds all N rows of y.  This is the multi-GPU form of the
reference's GEMV path for its 70B-class MLP shapes (N=28672,K=8192 and
N=8192,K=28672): the reference itself runs on one GPU and names "rows
sharded, x broadcast, y all-gathered by NCCL" as the scaling scheme.

Two ways to finish a step:
  * mode="fused" (default): cl_int4gemv_sharded / cl_qgemv_sharded -- each
    CTA stores its rows straight into every rank's y buffer over NVLink peer
    mappings and the ranks complete the step through a flag block, so the
    all-gather overlaps the GEMV (one kernel, no collective launch);
  * mode="nccl": the single-GPU GEMV into a local shard, then
    torch.distributed.all_gather_into_tensor (the unfused baseline).

The peer buffers are plain cudaMalloc memory shared by CUDA IPC handles
(cl_peer_alloc / cl_peer_open); no multicast objects are created.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _native as nat

_ALIGN = 256


def shard_rows(N: int, world: int, rank: int) -> tuple[int, int]:
    """Balanced contiguous split of N rows: (first row, row count) of `rank`.
    The first N % world ranks get one extra row."""
    if N <= 0 or world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad shard request N={N} world={world} rank={rank}")
    base, rem = divmod(N, world)
    row0 = rank * base + min(rank, rem)
    return row0, base + (1 if rank < rem else 0)


def gather_shards(y_shard: torch.Tensor, y_gather: torch.Tensor, N: int, group=None) -> torch.Tensor:
    """All-gather of equally padded shards into y.  `y_shard` is [n_max] or
    [M, n_max] (n_max = ceil(N/world), the first shard_rows(...)[1] columns
    valid); `y_gather` holds world * M * n_max values.  Returns y [N] (a view
    of `y_gather` when N divides evenly) or [M, N]."""
    world = dist.get_world_size(group)
    n_max = y_shard.shape[-1]
    dist.all_gather_into_tensor(y_gather, y_shard.reshape(-1), group=group)
    if y_shard.dim() == 1:
        if N == world * n_max:
            return y_gather
        parts = [y_gather[p * n_max: p * n_max + shard_rows(N, world, p)[1]]
                 for p in range(world)]
        return torch.cat(parts)
    M = y_shard.shape[0]
    g = y_gather.view(world, M, n_max)
    parts = [g[p, :, : shard_rows(N, world, p)[1]] for p in range(world)]
    return torch.cat(parts, dim=1)


def _round_up(v: int, a: int = _ALIGN) -> int:
    return (v + a - 1) // a * a


@dataclass
class _Layout:
    """One rank's peer allocation: [y parity 0 | y parity 1 | flag block]; a y
    buffer holds up to max_batch rows of N halves."""
    N: int
    max_batch: int = 1

    @property
    def y_bytes(self) -> int:
        return _round_up(2 * self.N * self.max_batch)

    def y_off(self, parity: int) -> int:
        return parity * self.y_bytes

    @property
    def flag_off(self) -> int:
        return 2 * self.y_bytes

    @property
    def total(self) -> int:
        return self.flag_off + _round_up(nat.CL_PEER_FLAG_BYTES)


class _CudaBackend:
    """Device memory through the C ABI (cl_peer_alloc / open / close / free)."""

    def __init__(self):
        self.lib = nat.load()

    def alloc(self, nbytes: int) -> tuple[int, bytes]:
        ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(nat.CL_IPC_HANDLE_BYTES)
        rc = self.lib.cl_peer_alloc(nbytes, ctypes.byref(ptr), handle)
        if rc != nat.CL_OK:
            raise RuntimeError(f"cl_peer_alloc failed ({rc}): {nat.last_error(self.lib)}")
        return ptr.value, handle.raw

    def open(self, handle: bytes) -> int:
        ptr = ctypes.c_void_p()
        rc = self.lib.cl_peer_open(handle, ctypes.byref(ptr))
        if rc != nat.CL_OK:
            raise RuntimeError(f"cl_peer_open failed ({rc}): {nat.last_error(self.lib)}")
        return ptr.value

    def close(self, ptr: int) -> None:
        self.lib.cl_peer_close(ctypes.c_void_p(ptr))

    def free(self, ptr: int) -> None:
        self.lib.cl_peer_free(ctypes.c_void_p(ptr))


class _DeviceView:
    """Zero-copy torch view of raw device memory (CUDA array interface)."""

    def __init__(self, ptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr,
                                         "data": (ptr, False), "version": 2}


class PeerBuffers:
    """y buffers (two step parities) and a flag block on every rank, each
    mapped into every rank's address space.  Handles are exchanged with
    all_gather_object over `group`; `backend` supplies alloc/open/close/free
    (the C ABI by default)."""

    def __init__(self, N_total: int, group=None, backend=None, max_batch: int = 1):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > nat.CL_MAX_PEERS:
            raise ValueError(f"at most {nat.CL_MAX_PEERS} ranks, got {self.world}")
        if not 1 <= max_batch <= 16:
            raise ValueError(f"max_batch must be in [1, 16], got {max_batch}")
        self.layout = _Layout(N_total, max_batch)
        self.backend = backend or _CudaBackend()
        self.local_ptr, handle = self.backend.alloc(self.layout.total)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        self.base = []
        self._opened = []
        for p, h in enumerate(handles):
            if p == self.rank:
                self.base.append(self.local_ptr)
            else:
                ptr = self.backend.open(h)
                self._opened.append(ptr)
                self.base.append(ptr)
        lay = self.layout
        self.y_ptrs = [[b + lay.y_off(par) for b in self.base] for par in (0, 1)]
        self.flag_ptrs = [b + lay.flag_off for b in self.base]
        self._y_array = (ctypes.c_void_p * (2 * self.world))(*(self.y_ptrs[0] + self.y_ptrs[1]))
        self._flag_array = (ctypes.c_void_p * self.world)(*self.flag_ptrs)

    def y_array(self):
        """Parity-0 buffers of all ranks, then parity-1 buffers."""
        return self._y_array

    def flag_array(self):
        return self._flag_array

    def local_y(self, parity: int) -> torch.Tensor:
        """This rank's y buffer of one parity as a flat [max_batch * N] view."""
        ptr = self.local_ptr + self.layout.y_off(parity)
        n = self.layout.N * self.layout.max_batch
        return torch.as_tensor(_DeviceView(ptr, n, "<f2"), device="cuda")

    def close(self) -> None:
        for ptr in self._opened:
            self.backend.close(ptr)
        self._opened = []
        if self.local_ptr:
            self.backend.free(self.local_ptr)
            self.local_ptr = 0


class ShardedGemv:
    """One rank's part of a row-sharded GEMV.

    kind: "int4gemv" (W_shard uint8 [n, K/2], scale fp16 [n, K/128]) or
    "qgemv" (W_shard int8 [n, K], scale fp32 [n]); the shard holds rows
    shard_rows(N_total, world, rank).  forward(x) takes x [K] or X [M, K]
    (M <= max_batch <= 16) and returns y [N_total] or Y [M, N_total] fp16 on
    every rank.  In fused mode the returned tensor is this step's parity
    buffer: it stays valid until the step after next (two steps later the
    same buffer is rewritten).  Every rank must call forward the same number
    of times, in the same order.  The step count lives on the device, so a
    captured graph of fused steps replays correctly; `self.epoch` counts the
    eager calls only (it picks the returned buffer).
    """

    def __init__(self, kind: str, W_shard: torch.Tensor, scale_shard: torch.Tensor,
                 N_total: int, K: int, group=None, variant: str | None = None,
                 mode: str = "fused", backend=None, peers: "PeerBuffers | None" = None,
                 max_batch: int = 1):
        if kind not in ("int4gemv", "qgemv"):
            raise ValueError(f"unknown kind {kind}")
        if mode not in ("fused", "nccl"):
            raise ValueError(f"unknown mode {mode}")
        self.kind, self.mode, self.group = kind, mode, group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.N, self.K = N_total, K
        self.row0, self.n = shard_rows(N_total, self.world, self.rank)
        if W_shard.shape[0] != self.n:
            raise ValueError(f"rank {self.rank}: shard has {W_shard.shape[0]} rows, "
                             f"expected {self.n} (rows {self.row0}..{self.row0 + self.n})")
        self.W, self.scale = W_shard.contiguous(), scale_shard.contiguous()
        self.variant = variant or ("int4gemv_mma" if kind == "int4gemv" else "qgemv_mma")
        self.max_batch = max_batch
        self.epoch = 0
        if mode == "fused":
            self.lib = nat.load()
            # several weight sets of one shape may share the buffers (and the step count)
            self._own_peers = peers is None
            self.peers = (peers if peers is not None
                          else PeerBuffers(N_total, group, backend, max_batch))
            if self.peers.layout.N != N_total or self.peers.layout.max_batch < max_batch:
                raise ValueError("shared peer buffers were made for another N or batch")
            self._fn = (self.lib.cl_int4gemv_sharded if kind == "int4gemv"
                        else self.lib.cl_qgemv_sharded)
            self._y = [self.peers.local_y(0), self.peers.local_y(1)]
        else:
            from .build import build
            self.ext = build(kind)
            self.n_max = -(-N_total // self.world)
            dev = self.W.device
            self.y_shard = torch.zeros(max_batch, self.n_max, dtype=torch.float16, device=dev)
            self.y_gather = torch.empty(self.world * max_batch * self.n_max, dtype=torch.float16,
                                        device=dev)

    def forward(self, x: torch.Tensor, flags: int = 0) -> torch.Tensor:
        if x.dtype != torch.float16 or x.dim() not in (1, 2) or x.shape[-1] != self.K:
            raise RuntimeError(f"x must be fp16 [{self.K}] or [M, {self.K}]")
        M = 1 if x.dim() == 1 else x.shape[0]
        if not 1 <= M <= self.max_batch:
            raise RuntimeError(f"batch of {M} rows exceeds max_batch={self.max_batch}")
        x = x.contiguous()
        self.epoch += 1
        if self.mode == "nccl":
            # the local shard buffer is read by the previous step's all-gather,
            # so its GEMV must wait before storing
            flags &= ~nat.CL_LAUNCH_OUTPUTS_FREE
            if x.dim() == 1:
                self.ext.forward_into(self.variant, self.W, self.scale, x,
                                      self.y_shard[0, : self.n], flags=flags)
                g = self.y_gather[: self.world * self.n_max]
                return gather_shards(self.y_shard[0], g, self.N, self.group)
            ys = self.y_shard[:M]
            out = torch.empty(M, self.n, dtype=torch.float16, device=x.device)
            self.ext.forward_batched_into(self.variant, self.W, self.scale, x, out, flags=flags)
            ys[:, : self.n].copy_(out)
            g = self.y_gather[: self.world * M * self.n_max]
            return gather_shards(ys, g, self.N, self.group)
        stream = torch.cuda.current_stream(self.W.device).cuda_stream
        rc = self._fn(self.variant.encode(), self.W.data_ptr(), self.scale.data_ptr(),
                      x.data_ptr(), M, self.peers.y_array(), self.peers.flag_array(),
                      self.rank, self.world, self.row0, self.n, self.N, self.K, stream, flags)
        if rc != nat.CL_OK:
            raise RuntimeError(f"{self.kind} sharded step failed ({rc}): {nat.last_error()}")
        y = self._y[self.epoch & 1]
        return y[: self.N] if x.dim() == 1 else y[: M * self.N].view(M, self.N)

    def close(self) -> None:
        if self.mode == "fused" and self._own_peers:
            torch.cuda.synchronize(self.W.device)
            self.peers.close()
