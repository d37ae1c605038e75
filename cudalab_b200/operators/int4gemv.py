"""INT4 (W4A16) operator adapter: generators, benchmark pools, logical bytes.

Mirror of cudalab/operators/int4gemv.py (make_w4/make_x4 :119-142, bench pool
:159-236, algorithmic_bytes :238-249).  Operator:

    W_packed uint8 [N, K/2], scale fp16 [N, K/128], x fp16 [K], y fp16 [N]
    y[n] = sum_k (scale[n, k/128] * unpack(W_packed)[n, k]) * x[k]

Pools:
  * "hot"       one x / out, resident weights (the reference's hot mode);
  * "streaming" x / out rotate over `pool_size` buffers, one resident weight
                set (the reference's streaming mode, :186-197).  On a B200 the
                126 MB L2 holds a 4096x4096 weight set, so this regime is
                L2-warm;
  * "l2cold"    x / out AND (W_packed, scale) rotate over `pool_size` (>= 64)
                independently seeded weight sets whose total is far above the
                L2 size, so every launch streams its weights from HBM.
"""
from __future__ import annotations

from pathlib import Path

import torch

from ..evaluator.bench import SEED, BenchPool
from ..int4gemv_quantize import GROUP_SIZE, quantize_w
from .base import Operator
from .gemv import make_w as _make_w_fp16
from .gemv import make_x as _make_x_fp16

ROOT = Path(__file__).resolve().parents[2]

BENCH_MATRIX_INT4GEMV = [
    (1024, 4096),
    (4096, 1024),
    (4096, 4096),
    (11008, 4096),
    (4096, 11008),
]
PRIMARY_TARGET = (4096, 4096)
L2_COLD_POOL = 64


def make_w4(N: int, K: int, seed: int = 0, mode: str = "normal", scale: float = 1.0,
            large: float = 10.0, device: str = "cuda"):
    """Seeded fp16 W -> (W_packed, scale, W_fp16), quantised outside any timed
    region.  K % 128 == 0 is required (the quantiser rejects otherwise)."""
    W = _make_w_fp16(N, K, torch.float16, device="cpu", seed=seed, mode=mode, scale=scale,
                     large=large)
    W = W.to(device)
    W_packed, s = quantize_w(W)  # elementwise IEEE fp32: same bytes on every device
    return W_packed, s, W


def make_x4(K: int, seed: int = 0, mode: str = "normal", large: float = 10.0,
            device: str = "cuda") -> torch.Tensor:
    return _make_x_fp16(K, torch.float16, device=device, seed=seed, mode=mode, large=large)


def algorithmic_bytes_int4(N: int, K: int, M: int = 1) -> int:
    """W_packed + scale + x + y: N*K/2 + N*(K/128)*2 + 2*M*K + 2*M*N."""
    return N * K // 2 + N * (K // GROUP_SIZE) * 2 + 2 * M * K + 2 * M * N


class Int4gemvOperator(Operator):
    name = "int4gemv"
    dtypes = ("float16",)
    bench_shapes = BENCH_MATRIX_INT4GEMV
    primary_target = PRIMARY_TARGET
    ncu_kernel_regex = "int4gemv|gemv_vec_kernel"
    profiles_dir = ROOT / "profiles"

    def build(self):
        from ..build import build
        return build("int4gemv")

    def make_bench_pool(self, M: int, K: int, dtype: torch.dtype = torch.float16,
                        mode: str = "streaming", seed: int = SEED, pool_size: int = 16,
                        weight_dist: float = 1.0) -> BenchPool:
        """Pre-allocate every tensor a timed launch touches (protocol (M, H) ->
        (N, K)).  `weight_dist` scales the fp16 weights before quantisation
        (N(0, weight_dist^2)); the roofline is indifferent to it."""
        N = M
        if dtype != torch.float16:
            raise NotImplementedError(f"int4gemv takes fp16 activations only, got {dtype}")
        if K % GROUP_SIZE != 0:
            raise NotImplementedError(f"int4gemv requires K % 128 == 0, got K={K}")
        dev = "cuda"
        n = 1 if mode == "hot" else pool_size
        xs = [make_x4(K, seed=seed + i, device=dev) for i in range(n)]
        outs = [torch.empty(N, dtype=torch.float16, device=dev) for _ in xs]
        n_w = pool_size if mode == "l2cold" else 1
        weights = []
        for i in range(n_w):
            Wp, s, _ = make_w4(N, K, seed=seed + 100000 + i, scale=weight_dist, device=dev)
            weights.append((Wp, s))
        wset_bytes = N * K // 2 + N * (K // GROUP_SIZE) * 2

        def launch(ext, variant: str, i: int, flags: int = 0):
            Wp, s = weights[i % len(weights)]
            ext.forward_into(variant, Wp, s, xs[i % len(xs)], outs[i % len(outs)], flags=flags)

        return BenchPool(
            xs=xs, outs=outs, pool_size=n, working_set_bytes=n * (2 * K + 2 * N),
            element_size=2, mode=mode, launch=launch,
            shared={"weights": weights}, shared_bytes=n_w * wset_bytes,
            pool_extra={"weight_sets": n_w, "weight_set_bytes": wset_bytes,
                        "weights_total_bytes": n_w * wset_bytes,
                        "quantization_offline": True})

    def algorithmic_bytes(self, M: int, K: int, element_size: int = 2) -> int:
        return algorithmic_bytes_int4(M, K)

    def experiment_prefix(self) -> str:
        return "INT4GEMV"

    def run_correctness(self, ext, variant: str) -> dict:
        from ..int4gemv_correctness import run_suite, summarize
        results = run_suite(variant, ext)
        s = summarize(results)
        return {"all_pass": bool(s["all_pass"]), "summary": s}

    def run_negative(self, ext, variant: str | None = None) -> dict:
        from ..int4gemv_negative import run_negative_suite
        return run_negative_suite(ext, variant=variant or "int4gemv_baseline")


int4gemv = Int4gemvOperator()
