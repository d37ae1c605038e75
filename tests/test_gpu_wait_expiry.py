"""A bounded device-side wait that runs out, on one GPU, without a fault.

The fused sharded step of rank 0 in a group of two is launched alone: both
ranks' buffers and flag blocks are local allocations, and nothing ever writes
rank 1's slot of rank 0's flag block.  With the wait bound lowered to 10^6 SM
cycles (about half a millisecond) the last CTA's wait for rank 1 runs out,
records status 5 (peer timeout) in the device status word and returns: the
call completes, the context stays usable, and the rows this rank computed
(stored before the wait) equal the single-GPU GEMV.  This exercises the
missing-rank path of the sharded protocol the way a failed peer would,
without withholding a real rank while others wait."""
import ctypes

import pytest
import torch

from cudalab_b200 import _native as nat
from cudalab_b200.build import build
from cudalab_b200.operators.int4gemv import make_w4, make_x4

pytestmark = pytest.mark.gpu

SHORT_BUDGET = 1_000_000  # SM cycles


@pytest.fixture()
def short_waits():
    prev = nat.set_wait_budget(SHORT_BUDGET)
    try:
        yield
    finally:
        nat.set_wait_budget(prev)


def test_peer_wait_expires_and_reports(short_waits):
    lib = nat.load()
    ext = build("int4gemv")
    assert nat.device_status(clear=True) == 0
    N, K, world, rank = 1024, 2048, 2, 0
    row0, n = 0, N // 2  # rank 0's shard of a 2-way split
    Wp, s, _ = make_w4(N, K, seed=61)
    x = make_x4(K, seed=62)
    Ws, ss = Wp[row0:row0 + n].contiguous(), s[row0:row0 + n].contiguous()
    ys = [torch.full((N,), float("nan"), dtype=torch.float16, device="cuda")
          for _ in range(2 * world)]
    flags = [torch.zeros(nat.CL_PEER_FLAG_BYTES // 4, dtype=torch.int32, device="cuda")
             for _ in range(world)]
    y_arr = (ctypes.c_void_p * (2 * world))(*[t.data_ptr() for t in ys])
    f_arr = (ctypes.c_void_p * world)(*[t.data_ptr() for t in flags])
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.cl_int4gemv_sharded(b"int4gemv_mma", Ws.data_ptr(), ss.data_ptr(), x.data_ptr(), 1,
                                 y_arr, f_arr, rank, world, row0, n, N, K, stream, 0)
    assert rc == nat.CL_OK, nat.last_error(lib)
    torch.cuda.synchronize()  # returns: the wait was bounded
    assert nat.device_status(clear=True) == 5
    # step 1 writes the parity-1 buffers of both ranks before waiting
    ref = ext.forward("int4gemv_mma", Ws, ss, x)
    torch.cuda.synchronize()
    for p in range(world):
        assert torch.equal(ys[world + p][row0:row0 + n], ref), p
    # this rank published its own arrival, rank 1's slot stays empty
    f0 = flags[0].cpu()
    assert int(f0[0]) == 1 and int(f0[1]) == 0
    # the context is still healthy and later launches use the default bound
    nat.set_wait_budget(0)
    y = ext.forward("int4gemv_mma", Ws, ss, x)
    torch.cuda.synchronize()
    assert torch.equal(y, ref) and nat.device_status(clear=True) == 0

