"""Quantisation-contract CPU tests (the checks of the reference's
tests/test_int4gemv_cpu.py, applied to the product quantiser and to the
independent numpy oracle):

  1. all 256 bytes unpack to sign-extended (lo, hi) and repack bijectively;
  2. every value -8..7 round-trips through the low and the high nibble;
  3. scale == fp16(amax/7), q == clamp(round(W/s32), -7, 7), zero groups;
  4. rejection paths (ValueError);
  5. fidelity metrics sanity;
  6. dequantize_w reads the stored fp16 scale.
"""
import math

import numpy as np
import pytest
import torch

from cudalab_b200.int4gemv_quantize import (GROUP_SIZE, INT4_MAX, dequantize_w,
                                            fidelity_metrics, pack_q, quantize_w, unpack_w)
from oracle import int4gemv_oracle as orc


def _py_sign_extend(b: int):
    lo = (b & 0x0F) - 16 if (b & 0x08) else (b & 0x0F)
    hi = ((b >> 4) & 0x0F) - 16 if (b & 0x80) else ((b >> 4) & 0x0F)
    return lo, hi


def test_exhaustive_byte_bijection():
    Wp = torch.arange(256, dtype=torch.uint8).view(1, 256)
    Wq = unpack_w(Wp)
    assert tuple(Wq.shape) == (1, 512)
    assert int(Wq.min()) >= -8 and int(Wq.max()) <= 7
    for b in range(256):
        assert (int(Wq[0, 2 * b]), int(Wq[0, 2 * b + 1])) == _py_sign_extend(b)
    assert torch.equal(pack_q(Wq), Wp)
    # the oracle agrees element for element
    assert np.array_equal(orc.unpack_w(Wp.numpy()), Wq.numpy())
    assert np.array_equal(orc.pack_q(Wq.numpy()), Wp.numpy())


def test_value_roundtrip_all_positions():
    v = torch.arange(-8, 8, dtype=torch.int32)
    even = torch.zeros(32, dtype=torch.int32)
    even[0::2] = v
    odd = torch.zeros(32, dtype=torch.int32)
    odd[1::2] = v
    assert torch.equal(unpack_w(pack_q(even.view(1, -1)))[0][0::2], v)
    assert torch.equal(unpack_w(pack_q(odd.view(1, -1)))[0][1::2], v)
    b = torch.tensor([-7, 0, 7], dtype=torch.int32)
    e = torch.zeros(6, dtype=torch.int32)
    e[0::2] = b
    o = torch.zeros(6, dtype=torch.int32)
    o[1::2] = b
    assert torch.equal(unpack_w(pack_q(e.view(1, -1)))[0][0::2], b)
    assert torch.equal(unpack_w(pack_q(o.view(1, -1)))[0][1::2], b)


def test_quantizer_contract():
    torch.manual_seed(0)
    N, G, K = 4, 3, 384
    W = (torch.randn(N, K) * 0.5).to(torch.float16)
    W.view(N, G, GROUP_SIZE)[:, 1, :].fill_(0)
    Wp, s16 = quantize_w(W)
    assert tuple(Wp.shape) == (N, K // 2) and Wp.dtype == torch.uint8
    assert tuple(s16.shape) == (N, G) and s16.dtype == torch.float16
    Wq = unpack_w(Wp)
    assert int(Wq.abs().max()) <= INT4_MAX
    assert bool((s16[:, 1] == 0).all())
    assert bool((Wq[:, 128:256] == 0).all())
    Wg = W.float().view(N, G, GROUP_SIZE)
    s32 = Wg.abs().amax(dim=2) / 7
    assert torch.equal(s16, s32.to(torch.float16))
    q_ref = torch.round(Wg / torch.where(s32 == 0, torch.ones_like(s32), s32).unsqueeze(2))
    q_ref = q_ref.clamp(-7, 7)
    q_ref = torch.where(s32.unsqueeze(2) == 0, torch.zeros_like(q_ref), q_ref)
    assert torch.equal(Wq.view(N, G, GROUP_SIZE), q_ref.to(torch.int32))
    s32c = torch.where(s32 == 0, torch.ones_like(s32), s32)
    err = (Wg - q_ref * s32c.unsqueeze(2)).abs()
    assert bool((err <= (0.5 * s32c + 1e-6).unsqueeze(2)).all())
    Wpz, sz = quantize_w(torch.zeros(2, K, dtype=torch.float16))
    assert bool((sz == 0).all()) and bool((Wpz == 0).all()) and bool(torch.isfinite(sz).all())
    # oracle quantiser: byte-identical on the same W
    owp, os16 = orc.quantize_w(W.numpy())
    assert np.array_equal(owp, Wp.numpy())
    assert np.array_equal(os16.view(np.uint16), s16.numpy().view(np.uint16))


@pytest.mark.parametrize("bad", [
    lambda: quantize_w(torch.randn(2, 256, dtype=torch.float16).view(-1)),
    lambda: quantize_w(torch.randn(2, 256, dtype=torch.float16).view(2, 2, 128)),
    lambda: quantize_w(torch.randn(2, 256)),
    lambda: quantize_w(torch.randn(256, 2, dtype=torch.float16).t()),
    lambda: quantize_w(torch.randn(2, 200, dtype=torch.float16)),
    lambda: quantize_w(torch.tensor([[float("nan")] + [0.0] * 127], dtype=torch.float16)),
    lambda: quantize_w(torch.tensor([[float("inf")] + [0.0] * 127], dtype=torch.float16)),
    lambda: pack_q(torch.zeros(1, 3, dtype=torch.int32)),
    lambda: pack_q(torch.tensor([[8, 0]], dtype=torch.int32)),
    lambda: pack_q(torch.tensor([[-9, 0]], dtype=torch.int32)),
])
def test_quantizer_rejections(bad):
    with pytest.raises(ValueError):
        bad()


def test_fidelity_small():
    torch.manual_seed(1)
    N, K = 4, 256
    W = torch.randn(N, K, dtype=torch.float16)
    x = torch.randn(K, dtype=torch.float16)
    Wp, s16 = quantize_w(W)
    fid = fidelity_metrics(W, x, Wp, s16)
    for k in ("max_abs", "rmse", "max_dequant_abs_err", "max_dequant_step_err"):
        assert math.isfinite(fid[k])
    assert fid["cosine"] is not None and 0.9 < fid["cosine"] <= 1.0 + 1e-9
    assert fid["max_dequant_step_err"] < 0.52
    assert fidelity_metrics(W, torch.zeros(K, dtype=torch.float16), Wp, s16)["cosine"] is None
    Wz = torch.zeros(N, K, dtype=torch.float16)
    Wpz, sz = quantize_w(Wz)
    fz = fidelity_metrics(Wz, x, Wpz, sz)
    assert fz["cosine"] is None and fz["max_abs"] == 0.0


def test_dequantize_uses_stored_fp16_scale():
    N, G, K = 2, 2, 256
    Wq = torch.randint(-7, 8, (N, K), dtype=torch.int32)
    Wp = pack_q(Wq)
    s16 = (torch.rand(N, G) * 0.1 + 0.01).to(torch.float16)
    Wd = dequantize_w(Wp, s16)
    assert torch.equal(Wd, Wq.float() * s16.float().repeat_interleave(GROUP_SIZE, dim=1))
    assert np.array_equal(orc.dequantize_w(Wp.numpy(), s16.numpy()), Wd.numpy())
