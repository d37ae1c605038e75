"""INT8 weight-only operator adapter (mirror of cudalab/operators/qgemv.py:
make_w_q/make_x_q :104-125, pool :142-212, algorithmic_bytes :214-227).

    W_q int8 [N, K], scale fp32 [N], x fp16 [K], y fp16 [N]
    y[n] = sum_k (scale[n] * W_q[n, k]) * x[k]

Pools as for int4gemv ("hot", "streaming", "l2cold").
"""
from __future__ import annotations

from pathlib import Path

import torch

from ..evaluator.bench import SEED, BenchPool
from ..qgemv_quantize import quantize_w
from .base import Operator
from .gemv import make_w as _make_w_fp16
from .gemv import make_x as _make_x_fp16

ROOT = Path(__file__).resolve().parents[2]

BENCH_MATRIX_QGEMV = [
    (1024, 4096),
    (4096, 1024),
    (4096, 4096),
    (11008, 4096),
    (4096, 11008),
]
PRIMARY_TARGET = (4096, 4096)


def make_w_q(N: int, K: int, seed: int = 0, mode: str = "normal", scale: float = 1.0,
             large: float = 10.0, device: str = "cuda"):
    """Seeded fp16 W -> (W_q int8, scale fp32, W_fp16), quantised offline."""
    W = _make_w_fp16(N, K, torch.float16, device="cpu", seed=seed, mode=mode, scale=scale,
                     large=large)
    W = W.to(device)
    W_q, s = quantize_w(W)  # elementwise IEEE fp32: same bytes on every device
    return W_q, s, W


def make_x_q(K: int, seed: int = 0, mode: str = "normal", large: float = 10.0,
             device: str = "cuda") -> torch.Tensor:
    return _make_x_fp16(K, torch.float16, device=device, seed=seed, mode=mode, large=large)


def algorithmic_bytes_int8(N: int, K: int, M: int = 1) -> int:
    """W_q + scale + x + y: N*K + 4*N + 2*M*K + 2*M*N."""
    return N * K + 4 * N + 2 * M * K + 2 * M * N


class QgemvOperator(Operator):
    name = "qgemv"
    dtypes = ("float16",)
    bench_shapes = BENCH_MATRIX_QGEMV
    primary_target = PRIMARY_TARGET
    ncu_kernel_regex = "qgemv|gemv_vec_kernel"
    profiles_dir = ROOT / "profiles"

    def build(self):
        from ..build import build
        return build("qgemv")

    def make_bench_pool(self, M: int, K: int, dtype: torch.dtype = torch.float16,
                        mode: str = "streaming", seed: int = SEED, pool_size: int = 16,
                        weight_dist: float = 1.0) -> BenchPool:
        N = M
        if dtype != torch.float16:
            raise NotImplementedError(f"qgemv takes fp16 activations only, got {dtype}")
        dev = "cuda"
        n = 1 if mode == "hot" else pool_size
        xs = [make_x_q(K, seed=seed + i, device=dev) for i in range(n)]
        outs = [torch.empty(N, dtype=torch.float16, device=dev) for _ in xs]
        n_w = pool_size if mode == "l2cold" else 1
        weights = []
        for i in range(n_w):
            Wq, s, _ = make_w_q(N, K, seed=seed + 100000 + i, scale=weight_dist, device=dev)
            weights.append((Wq, s))
        wset_bytes = N * K + 4 * N

        def launch(ext, variant: str, i: int, flags: int = 0):
            Wq, s = weights[i % len(weights)]
            ext.forward_into(variant, Wq, s, xs[i % len(xs)], outs[i % len(outs)], flags=flags)

        return BenchPool(
            xs=xs, outs=outs, pool_size=n, working_set_bytes=n * (2 * K + 2 * N),
            element_size=2, mode=mode, launch=launch,
            shared={"weights": weights}, shared_bytes=n_w * wset_bytes,
            pool_extra={"weight_sets": n_w, "weight_set_bytes": wset_bytes,
                        "weights_total_bytes": n_w * wset_bytes,
                        "quantization_offline": True})

    def algorithmic_bytes(self, M: int, K: int, element_size: int = 2) -> int:
        return algorithmic_bytes_int8(M, K)

    def experiment_prefix(self) -> str:
        return "QGEMV"

    def run_correctness(self, ext, variant: str) -> dict:
        from ..qgemv_correctness import run_suite, summarize
        results = run_suite(variant, ext)
        s = summarize(results)
        return {"all_pass": bool(s["all_pass"]), "summary": s}

    def run_negative(self, ext, variant: str | None = None) -> dict:
        from ..qgemv_negative import run_negative_suite
        return run_negative_suite(ext, variant=variant or "qgemv_baseline")


qgemv = QgemvOperator()
