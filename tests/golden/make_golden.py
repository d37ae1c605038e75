"""Generate the golden vectors that pin the oracle and the product quantisers.

Runs ONLY in the build container, where the reference tree is mounted
beside the repository (directory `reference` next to the repository root;
override with CUDALAB_REFERENCE).  It imports the
reference's own CPU code -- its generators (cudalab/operators/gemv.py:
make_w/make_x), quantisers (cudalab/int4gemv_quantize.py,
cudalab/qgemv_quantize.py), layer-A references and fp64 exact values -- and
stores inputs and outputs as small .npz fixtures next to this script (the
dense GEMV fixture: the reference's gemv_ref and gate,
cudalab/operators/gemv.py:192-201, cudalab/gemv_correctness.py:163-191).  The
fixtures travel; the reference does not.

    python tests/golden/make_golden.py               # all fixtures
    python tests/golden/make_golden.py --only-gemv   # the dense GEMV fixture
    python tests/golden/make_golden.py --only-rmsnorm  # RMSNorm and fused fixtures
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REF = Path(os.environ.get("CUDALAB_REFERENCE", HERE.parents[2] / "reference"))

INT4_CASES = [  # (N, K, mode, seed_w, seed_x)
    (8, 128, "normal", 0, 1),
    (3, 256, "mixed_sign", 0, 1),
    (16, 512, "large", 2, 3),
    (4, 1024, "tiny", 4, 5),
    (2, 128, "zeros", 0, 1),
    (32, 2048, "normal", 6, 7),
    (5, 384, "normal", 8, 9),
]
GEMV_CASES = [  # (dtype, N, K, mode, seed_w, seed_x)
    ("float16", 8, 64, "normal", 0, 1),
    ("float16", 16, 13, "mixed_sign", 0, 1),
    ("float16", 4, 4096, "large", 2, 3),
    ("float16", 5, 7, "tiny", 4, 5),
    ("float16", 2, 16, "zeros", 0, 1),
    ("float16", 32, 1024, "normal", 6, 7),
    ("float32", 8, 64, "normal", 0, 1),
    ("float32", 16, 13, "mixed_sign", 0, 1),
    ("float32", 3, 4096, "large", 2, 3),
    ("float32", 64, 1, "normal", 4, 5),
    ("float32", 32, 1024, "tiny", 6, 7),
]
INT8_CASES = [
    (8, 64, "normal", 0, 1),
    (16, 13, "mixed_sign", 0, 1),
    (1, 4096, "large", 2, 3),
    (64, 1, "normal", 4, 5),
    (5, 7, "tiny", 6, 7),
    (2, 16, "zeros", 0, 1),
    (32, 1024, "normal", 8, 9),
]


def _bits16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def _raw(t: torch.Tensor) -> np.ndarray:
    """Element bits of an fp16 / fp32 tensor."""
    if t.dtype == torch.float16:
        return _bits16(t)
    return t.contiguous().view(torch.int32).numpy().view(np.uint32).copy()


def make_gemv() -> None:
    """Dense GEMV fixtures: the reference's generators, gemv_ref and gate."""
    from cudalab.operators.gemv import make_w, make_x, gemv_ref  # reference code
    from cudalab.gemv_correctness import arith_ratio

    out = {}
    for i, (dt, N, K, mode, sw, sx) in enumerate(GEMV_CASES):
        dtype = getattr(torch, dt)
        W = make_w(N, K, dtype, device="cpu", seed=sw, mode=mode, large=10.0)
        x = make_x(K, dtype, device="cpu", seed=sx, mode=mode, large=10.0)
        y_ref = gemv_ref(W, x)
        exact = torch.mv(W.double(), x.double())
        S = (W.double().abs() * x.double().abs().unsqueeze(0)).sum(dim=1)
        ratio, _, _ = arith_ratio(y_ref, W, x, dt)
        p = f"c{i}_"
        out[p + "meta"] = np.array([N, K, sw, sx], np.int64)
        out[p + "dtype"] = np.array(dt)
        out[p + "mode"] = np.array(mode)
        out[p + "W"] = _raw(W)
        out[p + "x"] = _raw(x)
        out[p + "y_ref"] = _raw(y_ref)
        out[p + "exact"] = exact.numpy()
        out[p + "S"] = S.numpy()
        out[p + "ref_ratio"] = np.array(ratio)
    out["n_cases"] = np.array(len(GEMV_CASES))
    np.savez_compressed(HERE / "gemv_golden.npz", **out)
    print("wrote", HERE / "gemv_golden.npz")


RMSNORM_CASES = [  # (M, H, mode, seed): the reference's RMSNorm on its own generator
    (1, 4096, "normal", 0),
    (3, 1024, "tiny", 1),
    (2, 2048, "biased", 2),
    (1, 512, "zeros", 3),
    (4, 8192, "normal", 4),
]
FUSED_CASES = [  # (N, K, M, mode, seed_w, seed_x): RMSNorm of x, then the INT4 layer-A
    (64, 1024, 1, "normal", 0, 1),
    (16, 4096, 3, "biased", 2, 3),
    (40, 2048, 2, "tiny", 4, 5),
]


def make_rmsnorm() -> None:
    """RMSNorm fixtures (cudalab/reference.py:rmsnorm_ref and make_inputs) and
    fused RMSNorm -> INT4 GEMV fixtures: the reference's RMSNorm output fed
    to its INT4 layer-A reference and fp64 exact values."""
    from cudalab.reference import make_inputs, rmsnorm_ref  # reference code
    from cudalab.operators.gemv import make_w
    from cudalab import int4gemv_quantize as q4

    out = {}
    for i, (M, H, mode, seed) in enumerate(RMSNORM_CASES):
        x, w = make_inputs(M, H, torch.float16, device="cpu", seed=seed, mode=mode)
        y = rmsnorm_ref(x, w)
        p = f"c{i}_"
        out[p + "meta"] = np.array([M, H, seed], np.int64)
        out[p + "mode"] = np.array(mode)
        out[p + "x"] = _bits16(x)
        out[p + "w"] = _bits16(w)
        out[p + "y_ref"] = _bits16(y)
    out["n_cases"] = np.array(len(RMSNORM_CASES))
    out["eps"] = np.array(1e-5)
    for i, (N, K, M, mode, sw, sx) in enumerate(FUSED_CASES):
        W = make_w(N, K, torch.float16, device="cpu", seed=sw, mode="normal")
        Wp, s16 = q4.quantize_w(W)
        x, g = make_inputs(M, K, torch.float16, device="cpu", seed=sx, mode=mode)
        xn = rmsnorm_ref(x, g)
        Wd = q4.dequantize_w(Wp, s16)
        y_ref = torch.stack([torch.mv(Wd, xn[m].float()) for m in range(M)]).to(torch.float16)
        a = q4.unpack_w(Wp).double() * s16.double().repeat_interleave(128, dim=1)
        exact = xn.double() @ a.t()
        S = xn.double().abs() @ a.abs().t()
        p = f"f{i}_"
        out[p + "meta"] = np.array([N, K, M, sw, sx], np.int64)
        out[p + "W_packed"] = Wp.numpy()
        out[p + "scale"] = _bits16(s16)
        out[p + "x"] = _bits16(x)
        out[p + "g"] = _bits16(g)
        out[p + "xn_ref"] = _bits16(xn)
        out[p + "y_ref"] = _bits16(y_ref)
        out[p + "exact"] = exact.numpy()
        out[p + "S"] = S.numpy()
    out["n_fused"] = np.array(len(FUSED_CASES))
    np.savez_compressed(HERE / "rmsnorm_golden.npz", **out)
    print("wrote", HERE / "rmsnorm_golden.npz")


def main() -> None:
    if not REF.exists():
        raise SystemExit(f"reference tree not found at {REF}; fixtures are committed already")
    sys.path.insert(0, str(REF))
    if "--only-rmsnorm" in sys.argv:
        make_rmsnorm()
        return
    if "--only-gemv" not in sys.argv:
        make_quantized()
    make_gemv()
    make_rmsnorm()


def make_quantized() -> None:
    from cudalab.operators.gemv import make_w, make_x  # reference generators
    from cudalab import int4gemv_quantize as q4
    from cudalab import qgemv_quantize as q8
    from cudalab.int4gemv_correctness import arith_ratio as ar4
    from cudalab.qgemv_correctness import arith_ratio as ar8

    out4 = {}
    for i, (N, K, mode, sw, sx) in enumerate(INT4_CASES):
        W = make_w(N, K, torch.float16, device="cpu", seed=sw, mode=mode, large=10.0)
        if i == 6:  # one all-zero group inside an otherwise normal row
            W.view(N, K // 128, 128)[1, 1, :] = 0
        x = make_x(K, torch.float16, device="cpu", seed=sx, mode=mode, large=10.0)
        Wp, s16 = q4.quantize_w(W)
        y_ref = torch.mv(q4.dequantize_w(Wp, s16), x.float()).to(torch.float16)
        Wq = q4.unpack_w(Wp).double()
        a = Wq * s16.double().repeat_interleave(128, dim=1)
        exact = torch.mv(a, x.double())
        S = (a.abs() * x.double().abs().unsqueeze(0)).sum(dim=1)
        ratio, _, _ = ar4(y_ref, Wp, s16, x, "float16")
        p = f"c{i}_"
        out4[p + "meta"] = np.array([N, K, sw, sx], np.int64)
        out4[p + "mode"] = np.array(mode)
        out4[p + "W_fp16"] = _bits16(W)
        out4[p + "x"] = _bits16(x)
        out4[p + "W_packed"] = Wp.numpy()
        out4[p + "scale"] = _bits16(s16)
        out4[p + "y_ref"] = _bits16(y_ref)
        out4[p + "exact"] = exact.numpy()
        out4[p + "S"] = S.numpy()
        out4[p + "ref_ratio"] = np.array(ratio)
    table = torch.arange(256, dtype=torch.uint8).view(1, 256)
    out4["byte_table_unpacked"] = q4.unpack_w(table).numpy().astype(np.int8)
    out4["n_cases"] = np.array(len(INT4_CASES))
    np.savez_compressed(HERE / "int4gemv_golden.npz", **out4)

    out8 = {}
    for i, (N, K, mode, sw, sx) in enumerate(INT8_CASES):
        W = make_w(N, K, torch.float16, device="cpu", seed=sw, mode=mode, large=10.0)
        x = make_x(K, torch.float16, device="cpu", seed=sx, mode=mode, large=10.0)
        Wq, s = q8.quantize_w(W)
        y_ref = torch.mv(q8.dequantize_w(Wq, s), x.float()).to(torch.float16)
        a = Wq.double() * s.double().unsqueeze(1)
        exact = torch.mv(a, x.double())
        S = (a.abs() * x.double().abs().unsqueeze(0)).sum(dim=1)
        ratio, _, _ = ar8(y_ref, Wq, s, x, "float16")
        p = f"c{i}_"
        out8[p + "meta"] = np.array([N, K, sw, sx], np.int64)
        out8[p + "mode"] = np.array(mode)
        out8[p + "W_fp16"] = _bits16(W)
        out8[p + "x"] = _bits16(x)
        out8[p + "W_q"] = Wq.numpy()
        out8[p + "scale"] = s.numpy()
        out8[p + "y_ref"] = _bits16(y_ref)
        out8[p + "exact"] = exact.numpy()
        out8[p + "S"] = S.numpy()
        out8[p + "ref_ratio"] = np.array(ratio)
    out8["n_cases"] = np.array(len(INT8_CASES))
    np.savez_compressed(HERE / "qgemv_golden.npz", **out8)
    print("wrote", HERE / "int4gemv_golden.npz", HERE / "qgemv_golden.npz")


if __name__ == "__main__":
    main()
