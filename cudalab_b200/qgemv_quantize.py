"""INT8 weight-only symmetric per-row quantisation.

Data contract (identical to the reference, cudalab/qgemv_quantize.py:1-24):
scale[n] = max_k |W[n,k]| / 127 in fp32 (stored fp32, 1-D [N]);
q = clamp(round_half_even(W / scale), -127, 127) as int8; an all-zero row has
scale 0 and q == 0.  Inputs must be finite fp16, 2-D, contiguous (ValueError
otherwise).  Quantisation happens offline.
"""
from __future__ import annotations

import torch

INT8_MAX = 127


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def quantize_w(W: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """fp16 W [N, K] -> (W_q int8 [N, K], scale fp32 [N]).
    Follows cudalab/qgemv_quantize.py:33-64."""
    _require(W.dim() == 2, f"expected a 2-D W (N, K), got {W.dim()}-D")
    _require(W.dtype == torch.float16, f"quantize_w accepts fp16 weights only, got {W.dtype}")
    _require(W.is_contiguous(), "quantize_w requires a contiguous W")
    _require(bool(torch.isfinite(W).all()), "quantize_w requires finite W (no NaN/Inf)")
    Wf = W.float()
    scale = Wf.abs().amax(dim=1) / INT8_MAX
    is_zero = scale == 0
    denom = torch.where(is_zero, torch.ones_like(scale), scale).unsqueeze(1)
    q = torch.clamp(torch.round(Wf / denom), -INT8_MAX, INT8_MAX)
    q = torch.where(is_zero.unsqueeze(1), torch.zeros_like(q), q)
    return q.to(torch.int8), scale


def quantize_w_device(W: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """quantize_w on the GPU through the C ABI (cl_qgemv_quantize): the same
    checks and the same bytes."""
    _require(W.dim() == 2, f"expected a 2-D W (N, K), got {W.dim()}-D")
    _require(W.dtype == torch.float16, f"quantize_w accepts fp16 weights only, got {W.dtype}")
    _require(W.is_contiguous(), "quantize_w requires a contiguous W")
    _require(bool(torch.isfinite(W).all()), "quantize_w requires finite W (no NaN/Inf)")
    _require(W.is_cuda, "quantize_w_device requires a CUDA tensor")
    from . import _native as nat
    lib = nat.load()
    N, K = W.shape
    Wq = torch.empty(N, K, dtype=torch.int8, device=W.device)
    s = torch.empty(N, dtype=torch.float32, device=W.device)
    with torch.cuda.device(W.device):
        rc = lib.cl_qgemv_quantize(W.data_ptr(), N, K, Wq.data_ptr(), s.data_ptr(),
                                   torch.cuda.current_stream(W.device).cuda_stream)
    if rc != nat.CL_OK:
        raise RuntimeError(f"cl_qgemv_quantize failed ({rc}): {nat.last_error(lib)}")
    return Wq, s


def dequantize_w(W_q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """fp32 [N, K] = W_q * scale[:, None] (cudalab/qgemv_quantize.py:67-70)."""
    return W_q.float() * scale.unsqueeze(1)


def fidelity_metrics(W: torch.Tensor, x: torch.Tensor, W_q: torch.Tensor,
                     scale: torch.Tensor) -> dict:
    """Quantisation fidelity, report-only (cudalab/qgemv_quantize.py:73-119)."""
    xf = x.float()
    y_orig = torch.mv(W.float(), xf)
    Wd = dequantize_w(W_q, scale)
    y_quant = torch.mv(Wd, xf)
    diff = y_quant - y_orig
    no, nq = float(y_orig.norm()), float(y_quant.norm())
    cosine = (float(torch.dot(y_orig, y_quant)) / (no * nq)) if (no > 0 and nq > 0) else None
    deq = (W.float() - Wd).abs()
    return {
        "max_abs": float(diff.abs().max()) if diff.numel() else 0.0,
        "max_rel": float((diff.abs() / y_orig.abs().clamp_min(1e-3)).max()) if diff.numel() else 0.0,
        "rmse": float(diff.pow(2).mean().sqrt()) if diff.numel() else 0.0,
        "cosine": cosine,
        "y_orig_norm": no,
        "y_quant_norm": nq,
        "max_dequant_abs_err": float(deq.max()) if deq.numel() else 0.0,
        "max_dequant_step_err": float((deq / scale.clamp_min(1e-30).unsqueeze(1)).max())
        if deq.numel() else 0.0,
        "n_zero_scale_rows": int((scale == 0).sum()),
        "max_abs_q": int(W_q.abs().max()) if W_q.numel() else 0,
        "note": "quantisation fidelity: quantisation error, not a kernel defect (report only)",
    }
