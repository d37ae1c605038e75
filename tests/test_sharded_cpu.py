"""Host logic of the row-sharded GEMV on CPU: shard arithmetic, the padded
all-gather + assembly (gloo, world size 2, shards computed by the oracle) and
the peer-buffer handle exchange (gloo, fake device memory)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cudalab_b200.sharded import PeerBuffers, gather_shards, shard_rows
from oracle import int4gemv_oracle as o4


@pytest.mark.parametrize("N", [1, 7, 16, 1000, 4096, 8192, 28672])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_rows_partition(N, world):
    if N < world:
        pytest.skip("fewer rows than ranks")
    spans = [shard_rows(N, world, r) for r in range(world)]
    assert spans[0][0] == 0
    for (a0, an), (b0, _) in zip(spans, spans[1:]):
        assert a0 + an == b0
    assert spans[-1][0] + spans[-1][1] == N
    sizes = [n for _, n in spans]
    assert max(sizes) - min(sizes) <= 1 and min(sizes) >= 1


def test_shard_rows_rejects():
    for args in [(0, 1, 0), (8, 0, 0), (8, 2, 2), (8, 2, -1)]:
        with pytest.raises(ValueError):
            shard_rows(*args)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)


def _gather_worker(rank, world, port, N, K, q):
    try:
        _init(rank, world, port)
        rng = np.random.default_rng(5)
        W = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
        x = rng.standard_normal(K).astype(np.float16)
        Wp, s16 = o4.quantize_w(W)
        row0, n = shard_rows(N, world, rank)
        y_local = o4.gemv_ref(Wp[row0:row0 + n], s16[row0:row0 + n], x)
        n_max = -(-N // world)
        y_shard = torch.zeros(n_max, dtype=torch.float16)
        y_shard[:n] = torch.from_numpy(y_local.view(np.float16).copy())
        y_gather = torch.empty(world * n_max, dtype=torch.float16)
        y = gather_shards(y_shard, y_gather, N, None)
        ref = o4.gemv_ref(Wp, s16, x).view(np.float16)
        q.put((rank, bool(np.array_equal(y.numpy().view(np.uint16), ref.view(np.uint16)))))
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001
        q.put((rank, repr(exc)))


@pytest.mark.parametrize("N", [256, 1000])
def test_gather_shards_gloo(N):
    world, K = 2, 256
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, N, K, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}, res


class _FakeBackend:
    """Host memory standing in for cl_peer_alloc / open: a handle carries the
    owner's rank, and open() maps it to a distinct fake address."""

    def __init__(self, rank):
        self.rank = rank
        self.freed = []
        self.closed = []

    def alloc(self, nbytes):
        return 0x10000000 * (self.rank + 1), f"rank{self.rank}:{nbytes}".encode().ljust(64, b"\0")

    def open(self, handle):
        owner = int(handle.split(b":")[0][4:])
        return 0x100000000 * (owner + 1) + self.rank

    def close(self, ptr):
        self.closed.append(ptr)

    def free(self, ptr):
        self.freed.append(ptr)


def _peer_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        be = _FakeBackend(rank)
        pb = PeerBuffers(1000, None, backend=be)
        lay = pb.layout
        ok = pb.base[rank] == 0x10000000 * (rank + 1)
        for p in range(world):
            if p != rank:
                ok &= pb.base[p] == 0x100000000 * (p + 1) + rank
            ok &= pb.y_ptrs[0][p] == pb.base[p] and pb.y_ptrs[1][p] == pb.base[p] + lay.y_bytes
            ok &= pb.flag_ptrs[p] == pb.base[p] + 2 * lay.y_bytes
        ok &= list(pb.y_array()) == pb.y_ptrs[0] + pb.y_ptrs[1]
        ok &= list(pb.flag_array()) == pb.flag_ptrs
        ok &= lay.y_bytes % 256 == 0 and lay.y_bytes >= 2000 and lay.total >= lay.flag_off + 64
        pb.close()
        ok &= be.freed == [0x10000000 * (rank + 1)] and len(be.closed) == world - 1
        q.put((rank, bool(ok)))
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001
        q.put((rank, repr(exc)))


def test_peer_buffer_exchange_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}, res
