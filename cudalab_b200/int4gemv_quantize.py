"""W4A16 symmetric group-wise INT4 quantisation and nibble packing.

Data contract (identical to the reference, cudalab/int4gemv_quantize.py:1-36,
because W_packed / scale produced by either side must be interchangeable):

  * group size G = 128 along K, K % 128 == 0, zero point 0;
  * scale32[n, g] = max|W[n, g*128:(g+1)*128]| / 7 computed in fp32, stored as
    fp16 (the kernels and every reference read the stored fp16 value);
  * q = clamp(round_half_even(W / scale32), -7, 7); an all-zero group has
    scale 0 and q == 0 (no division by zero);
  * W_packed[n, b] = (q[n, 2b+1] & 0xF) << 4 | (q[n, 2b] & 0xF): low nibble is
    element 2b, high nibble element 2b+1, 4-bit two's complement.

Quantisation happens offline (outside every timed region).  Inputs must be
finite fp16, 2-D, contiguous; violations raise ValueError, as in the
reference (cudalab/int4gemv_quantize.py:44-58).
"""
from __future__ import annotations

import torch

INT4_MAX = 7
GROUP_SIZE = 128


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _check_w(W: torch.Tensor) -> None:
    _require(W.dim() == 2, f"expected a 2-D W (N, K), got {W.dim()}-D")
    _require(W.dtype == torch.float16, f"quantize_w accepts fp16 weights only, got {W.dtype}")
    _require(W.is_contiguous(), "quantize_w requires a contiguous W")
    _require(W.size(1) % GROUP_SIZE == 0,
             f"K must be divisible by {GROUP_SIZE} (group size), got K={W.size(1)}")
    _require(bool(torch.isfinite(W).all()), "quantize_w requires finite W (no NaN/Inf)")


def quantize_w(W: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """fp16 W [N, K] -> (W_packed uint8 [N, K/2], scale fp16 [N, K/128]).

    Works on any device; the arithmetic is elementwise fp32 (division,
    round-half-even, clamp) so CPU and CUDA give identical bytes.
    Follows cudalab/int4gemv_quantize.py:61-89.
    """
    _check_w(W)
    N, K = W.shape
    groups = W.float().reshape(N, K // GROUP_SIZE, GROUP_SIZE)
    s32 = groups.abs().amax(dim=2) / INT4_MAX
    is_zero = s32 == 0
    denom = torch.where(is_zero, torch.ones_like(s32), s32).unsqueeze(2)
    q = torch.clamp(torch.round(groups / denom), -INT4_MAX, INT4_MAX)
    q = torch.where(is_zero.unsqueeze(2), torch.zeros_like(q), q)
    W_packed = pack_q(q.reshape(N, K).to(torch.int32))
    return W_packed, s32.to(torch.float16).contiguous()


def quantize_w_device(W: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """quantize_w on the GPU through the C ABI (cl_int4gemv_quantize): the same
    checks and the same bytes, one pass over W on the current stream."""
    _check_w(W)
    _require(W.is_cuda, "quantize_w_device requires a CUDA tensor")
    from . import _native as nat
    lib = nat.load()
    N, K = W.shape
    Wp = torch.empty(N, K // 2, dtype=torch.uint8, device=W.device)
    s = torch.empty(N, K // GROUP_SIZE, dtype=torch.float16, device=W.device)
    with torch.cuda.device(W.device):
        rc = lib.cl_int4gemv_quantize(W.data_ptr(), N, K, Wp.data_ptr(), s.data_ptr(),
                                      torch.cuda.current_stream(W.device).cuda_stream)
    if rc != nat.CL_OK:
        raise RuntimeError(f"cl_int4gemv_quantize failed ({rc}): {nat.last_error(lib)}")
    return Wp, s


def pack_q(q: torch.Tensor) -> torch.Tensor:
    """int [N, K] with values in [-8, 7] -> uint8 [N, K/2] (low nibble = even k).
    Follows cudalab/int4gemv_quantize.py:92-114."""
    _require(q.dim() == 2, f"pack_q expects a 2-D (N, K) tensor, got {q.dim()}-D")
    N, K = q.shape
    _require(K % 2 == 0, f"pack_q requires an even K, got K={K}")
    if q.numel():
        _require(int(q.min()) >= -8 and int(q.max()) <= 7,
                 "pack_q value out of the INT4 two's-complement range [-8, 7]")
    pairs = q.to(torch.int32).reshape(N, K // 2, 2) & 0xF
    return (pairs[..., 0] | (pairs[..., 1] << 4)).to(torch.uint8).contiguous()


def unpack_w(W_packed: torch.Tensor) -> torch.Tensor:
    """uint8 [N, K/2] -> int32 [N, K] in [-8, 7], the exact inverse of pack_q.
    Follows cudalab/int4gemv_quantize.py:117-134."""
    _require(W_packed.dim() == 2, f"unpack_w expects a 2-D (N, K/2) tensor, got "
                                  f"{W_packed.dim()}-D")
    _require(W_packed.dtype == torch.uint8, f"unpack_w accepts uint8 only, got {W_packed.dtype}")
    N, H = W_packed.shape
    b = W_packed.to(torch.int32)
    nib = torch.stack((b & 0xF, b >> 4), dim=-1)          # (N, H, 2), 0..15
    return (nib - ((nib & 0x8) << 1)).reshape(N, 2 * H).contiguous()  # sign-extend


def dequantize_w(W_packed: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """fp32 [N, K] = unpack(W_packed) * stored fp16 scale (promoted to fp32).
    Follows cudalab/int4gemv_quantize.py:137-149."""
    q = unpack_w(W_packed)
    N, K = q.shape
    _require(tuple(scale.shape) == (N, K // GROUP_SIZE),
             f"scale shape {tuple(scale.shape)} does not match ({N}, {K // GROUP_SIZE})")
    return q.float() * scale.float().repeat_interleave(GROUP_SIZE, dim=1)


def fidelity_metrics(W: torch.Tensor, x: torch.Tensor, W_packed: torch.Tensor,
                     scale: torch.Tensor) -> dict:
    """Quantisation fidelity, report-only (cudalab/int4gemv_quantize.py:152-198):
    y_orig = W @ x vs y_quant = dequant(W) @ x (both fp32 accumulation)."""
    xf = x.float()
    y_orig = torch.mv(W.float(), xf)
    Wd = dequantize_w(W_packed, scale)
    y_quant = torch.mv(Wd, xf)
    diff = y_quant - y_orig
    no, nq = float(y_orig.norm()), float(y_quant.norm())
    cosine = (float(torch.dot(y_orig, y_quant)) / (no * nq)) if (no > 0 and nq > 0) else None
    step = scale.float().clamp_min(1e-30).repeat_interleave(GROUP_SIZE, dim=1)
    deq = (W.float() - Wd).abs()
    return {
        "max_abs": float(diff.abs().max()) if diff.numel() else 0.0,
        "rmse": float(diff.pow(2).mean().sqrt()) if diff.numel() else 0.0,
        "cosine": cosine,
        "y_orig_norm": no,
        "y_quant_norm": nq,
        "max_dequant_abs_err": float(deq.max()) if deq.numel() else 0.0,
        "max_dequant_step_err": float((deq / step).max()) if deq.numel() else 0.0,
        "n_zero_scale_groups": int((scale == 0).sum()),
        "max_abs_q": int(unpack_w(W_packed).abs().max()) if W_packed.numel() else 0,
        "note": "quantisation fidelity: quantisation error, not a kernel defect (report only)",
    }
