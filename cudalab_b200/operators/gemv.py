"""Deterministic fp16 weight / activation generators shared by the INT4 and
INT8 operators (the roles of cudalab/operators/gemv.py:106-189).

Modes: "normal" N(0, scale), "zeros", "tiny" N(0, 1e-4), "large" N(0, large),
"mixed_sign" (|N(0,1)| with a checkerboard sign on W and an independent
Bernoulli sign on x, so row sums really cancel).

The random stream is always drawn from a CPU torch.Generator and then moved
to the requested device, so a (seed, mode, shape) triple names the same tensor
on every device.  (The reference draws from a generator on the target device,
so its CUDA tensors differ from its CPU tensors for the same seed; the CPU
streams of both are identical because the same torch calls are made in the
same order.)
"""
from __future__ import annotations

import torch

MODES = ("normal", "zeros", "tiny", "large", "mixed_sign")


def _gen(seed: int) -> torch.Generator:
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    return g


def make_w(N: int, K: int, dtype: torch.dtype = torch.float16, device: str = "cpu",
           seed: int = 0, mode: str = "normal", scale: float = 1.0,
           large: float = 10.0) -> torch.Tensor:
    g = _gen(seed)
    if mode == "normal":
        w = torch.randn(N, K, generator=g, dtype=torch.float32) * scale
    elif mode == "zeros":
        w = torch.zeros(N, K, dtype=torch.float32)
    elif mode == "tiny":
        w = torch.randn(N, K, generator=g, dtype=torch.float32) * 1e-4
    elif mode == "large":
        w = torch.randn(N, K, generator=g, dtype=torch.float32) * large
    elif mode == "mixed_sign":
        a = torch.randn(N, K, generator=g, dtype=torch.float32).abs()
        i = torch.arange(N).unsqueeze(1)
        j = torch.arange(K).unsqueeze(0)
        w = a * torch.where(((i + j) % 2) == 0, 1.0, -1.0)
    else:
        raise ValueError(f"unknown input mode: {mode}")
    return w.to(dtype).contiguous().to(device)


def make_x(K: int, dtype: torch.dtype = torch.float16, device: str = "cpu", seed: int = 0,
           mode: str = "normal", scale: float = 1.0, large: float = 10.0) -> torch.Tensor:
    g = _gen(seed)
    if mode == "normal":
        x = torch.randn(K, generator=g, dtype=torch.float32) * scale
    elif mode == "zeros":
        x = torch.zeros(K, dtype=torch.float32)
    elif mode == "tiny":
        x = torch.randn(K, generator=g, dtype=torch.float32) * 1e-4
    elif mode == "large":
        x = torch.randn(K, generator=g, dtype=torch.float32) * large
    elif mode == "mixed_sign":
        a = torch.randn(K, generator=g, dtype=torch.float32).abs()
        s = torch.randint(0, 2, (K,), generator=g, dtype=torch.int32)
        x = a * torch.where(s == 0, 1.0, -1.0)
    else:
        raise ValueError(f"unknown input mode: {mode}")
    return x.to(dtype).contiguous().to(device)


# ---- the dense GEMV operator itself (cudalab/operators/gemv.py:192-201,
#      :283-289 of the reference) ----

# LLM hidden / MLP projection shapes (N, K) of the reference's bench matrix.
BENCH_MATRIX_GEMV = ((1024, 4096), (4096, 1024), (4096, 4096), (11008, 4096), (4096, 11008))
PRIMARY_TARGET = (4096, 4096)


def gemv_ref(W: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """Reference result: fp16 -> fp16(mv(W.float(), x.float())); fp32 -> mv(W, x)."""
    if W.dim() != 2:
        raise ValueError(f"expected a 2-D W (N, K), got {W.dim()}-D")
    if x.dim() != 1:
        raise ValueError(f"expected a 1-D x (K,), got {x.dim()}-D")
    if W.dtype == torch.float16:
        return torch.mv(W.float(), x.float()).to(torch.float16)
    return torch.mv(W, x)


def algorithmic_bytes_gemv(N: int, K: int, element_size: int = 2) -> int:
    """W read + x read + y write: (N*K + K + N) * element_size."""
    return (N * K + K + N) * element_size
