"""Host-side operator extensions: the drop-in replacement of the reference's
per-operator pybind modules.

`Int4gemvExt` mirrors kernels/int4gemv/bindings.cpp (forward :145-159,
forward_into :163-176, native_timing :180-253, variant lists :258-285) and
`QgemvExt` mirrors kernels/qgemv/bindings.cpp (:66-115, :281-306), `GemvExt`
kernels/gemv/bindings.cpp (dense fp16 / fp32 GEMV).  The
tensor-metadata checks run here, before any device work, in the reference's
order (variant lookup, then W: dim -> N>0 -> K>0 -> dtype -> [K%128] ->
contiguous -> is_cuda, then scale, x, out), and raise RuntimeError whose first
line carries the same message substring as the reference (its negative suite
matches those substrings), followed by an English rendering.  The computation
itself always goes through the C ABI of libcudalab_gemv.so.
"""
from __future__ import annotations

import ctypes
import statistics

import torch

from . import _native as nat

NATIVE_NOTE = ("native kernel-loop timing: back-to-back launches issued from C++, "
               "CUDA events around each window / launches per window; excludes the "
               "Python boundary (distinct from the API-path and ncu durations)")


def timing_result(variant: str, warmup: int, n_windows: int, launches_per_window: int,
                  per_window_us) -> dict:
    """The dict native_timing returns (kernels/*/bindings.cpp native_timing of
    the reference): per-window single-launch times and their statistics."""
    per = [float(v) for v in per_window_us]
    s = sorted(per)
    return {
        "variant": variant,
        "warmup": warmup,
        "n_windows": n_windows,
        "launches_per_window": launches_per_window,
        "window_median_us": per,
        "median_us": statistics.median(s),
        "min_us": s[0],
        "max_us": s[-1],
        "mean_us": sum(s) / len(s),
        "note": NATIVE_NOTE,
    }


def _chk(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


_U8, _I8, _F16, _F32 = torch.uint8, torch.int8, torch.float16, torch.float32
# Raw handle of the current stream / index of the current device without
# building Python objects (about 0.1 us each instead of several us).
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)
_cur_device = getattr(torch._C, "_cuda_getDevice", None)


def _stream_ptr(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _stream_of(idx: int) -> int:
    if _raw_stream is not None:
        return _raw_stream(idx)
    return torch.cuda.current_stream(idx).cuda_stream


def _device_is_current(idx: int) -> bool:
    return (_cur_device() if _cur_device is not None else torch.cuda.current_device()) == idx


def _same_device(idx: int, *ts) -> bool:
    for t in ts:
        if not t.is_cuda or t.get_device() != idx:
            return False
    return True


_BINDING = []  # [module or None], loaded once


def _binding():
    """The torch binding of the success path (csrc/torch_fast.cpp), built in
    the library folder by build.build_binding; None when it is absent, in
    which case every call takes the ctypes path (the same C ABI and kernels)."""
    if not _BINDING:
        mod = None
        from .build import binding_path
        p = binding_path()
        if p.exists():
            import importlib.util
            spec = importlib.util.spec_from_file_location("cudalab_b200._cl_torch", p)
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
        _BINDING.append(mod)
    return _BINDING[0]


class _ExtBase:
    kind = ""          # "int4gemv" | "qgemv"
    w_name = ""        # "W_packed" | "W_q"
    _kind_code = -1    # operator code of the torch binding

    def __init__(self) -> None:
        self._lib = nat.load()
        self._tb = _binding()
        self._cache = {}
        # every registered name (normal and quarantined) -> its bytes for the C call
        self._encoded = {v: v.encode() for v in self.all_variants()}

    # ---- variant registry ----
    def variants(self) -> list[str]:
        return nat.list_variants(self.kind, nat.CL_VARIANTS_NORMAL)

    def all_variants(self) -> list[str]:
        return nat.list_variants(self.kind, nat.CL_VARIANTS_ALL)

    def quarantined_variants(self) -> list[str]:
        return nat.list_variants(self.kind, nat.CL_VARIANTS_QUARANTINED)

    def _check_variant(self, name: str) -> None:
        allv = self._cache.get("all")
        if allv is None:
            allv = self._cache["all"] = set(self.all_variants())
        if name not in allv:
            normal = " ".join(self.variants())
            raise RuntimeError(f"未知 {self.kind} 变体 '{name}'。正常可用: {normal} "
                               f"(unknown {self.kind} variant)")

    # ---- shared checks on x / out (reference order: dim, size, dtype,
    #      contiguous, is_cuda, same device) ----
    def _validate_x(self, W: torch.Tensor, x: torch.Tensor, K: int) -> None:
        _chk(x.dim() == 1, f"x 必须是 1 维 (K,)，实际 {x.dim()} 维 (x must be 1-D)")
        _chk(x.size(0) == K, f"x 长度必须等于 K: x={x.size(0)} K={K} (len(x) must equal K)")
        _chk(x.dtype == torch.float16,
             f"x 必须是 float16（FP16 activation）, 实际 {x.dtype} (x must be float16)")
        _chk(x.is_contiguous(), "x 必须是连续内存 (x must be contiguous)")
        _chk(x.is_cuda, "x 必须是 CUDA 张量 (x must be a CUDA tensor)")
        _chk(x.device == W.device,
             f"x 必须与 {self.w_name} 在同一 CUDA 设备上 (x must be on the device of "
             f"{self.w_name})")

    def _validate_out(self, W: torch.Tensor, out: torch.Tensor) -> None:
        N = W.size(0)
        _chk(out.dim() == 1, f"out 必须是 1 维 (N,)，实际 {out.dim()} 维 (out must be 1-D)")
        _chk(out.size(0) == N,
             f"out 长度必须等于 N: out={out.size(0)} N={N} (len(out) must equal N)")
        _chk(out.dtype == torch.float16,
             f"out 必须是 float16，实际 {out.dtype} (out must be float16)")
        _chk(out.is_contiguous(), "out 必须是连续内存 (out must be contiguous)")
        _chk(out.is_cuda, "out 必须是 CUDA 张量 (out must be a CUDA tensor)")
        _chk(out.device == W.device,
             f"out 必须与 {self.w_name} 在同一 CUDA 设备上 (out must be on the device of "
             f"{self.w_name})")

    # subclasses: _validate_w, _validate_scale, _k_of, _call
    def _validate_inputs(self, W, scale, x) -> int:
        self._validate_w(W)
        self._validate_scale(W, scale)
        K = self._k_of(W)
        self._validate_x(W, x, K)
        return K

    def _launch(self, name: str, W, scale, x, out, flags: int = 0) -> None:
        idx = W.get_device()
        args = (self._encoded.get(name) or name.encode(), W.data_ptr(), scale.data_ptr(),
                x.data_ptr(), out.data_ptr(), W.size(0), self._k_of(W))
        if _device_is_current(idx):
            rc = self._call(*args, _stream_of(idx), flags)
        else:
            with torch.cuda.device(idx):
                rc = self._call(*args, _stream_of(idx), flags)
        if rc != nat.CL_OK:
            raise RuntimeError(f"{self.kind} launch failed ({rc}): {nat.last_error(self._lib)}")

    # Success-path predicate: true only when every ordered check of
    # _check_variant / _validate_inputs / _validate_out would pass (it may be
    # stricter, never looser), so the common call skips building messages; on
    # False the ordered checks run and raise the reference's message.
    def _fast_ok(self, variant, W, scale, x, out) -> bool:
        if variant not in self._encoded or not self._fast_inputs(W, scale, x):
            return False
        return (out is None or (out.dtype is _F16 and out.shape == (W.shape[0],)
                                and out.is_contiguous() and _same_device(W.get_device(), out)))

    # ---- public API (names and keyword names of the reference module) ----
    # The torch binding takes the common call whole (checks in C++, then the C
    # ABI); whenever it declines, the ordered checks below run and raise.
    def forward(self, variant: str, W, scale, x, flags: int = 0) -> torch.Tensor:
        if self._tb is not None:
            out = self._tb.forward(self._kind_code, variant, W, scale, x, flags)
            if out is not None:
                return out
        if not self._fast_ok(variant, W, scale, x, None):
            self._check_variant(variant)
            self._validate_inputs(W, scale, x)
        out = torch.empty(W.size(0), dtype=torch.float16, device=W.device)
        self._launch(variant, W, scale, x, out, flags)
        return out

    def forward_into(self, variant: str, W, scale, x, out, flags: int = 0) -> None:
        if self._tb is not None and \
                self._tb.forward_into(self._kind_code, variant, W, scale, x, out, flags) == 0:
            return
        if not self._fast_ok(variant, W, scale, x, out):
            self._check_variant(variant)
            self._validate_inputs(W, scale, x)
            self._validate_out(W, out)
        self._launch(variant, W, scale, x, out, flags)

    # ---- batched activations (no reference counterpart; English messages) ----
    def _validate_batch(self, W, X: torch.Tensor, K: int) -> int:
        _chk(X.dim() == 2, f"X must be 2-D (M, K), got {X.dim()}-D")
        _chk(X.size(0) > 0, "X must have at least one row")
        _chk(X.size(1) == K, f"X must have K={K} columns, got {X.size(1)}")
        _chk(X.dtype == torch.float16, f"X must be float16, got {X.dtype}")
        _chk(X.is_contiguous(), "X must be contiguous")
        _chk(X.is_cuda and X.device == W.device, f"X must be on the device of {self.w_name}")
        return X.size(0)

    def _launch_batched(self, name: str, W, scale, X, out, flags: int) -> None:
        N, K, M = W.size(0), self._k_of(W), X.size(0)
        dev = W.device
        with torch.cuda.device(dev):
            rc = self._batched(name.encode(), W.data_ptr(), scale.data_ptr(), X.data_ptr(),
                               out.data_ptr(), M, N, K, _stream_ptr(dev), flags)
        if rc != nat.CL_OK:
            raise RuntimeError(f"{self.kind} batched launch failed ({rc}): "
                               f"{nat.last_error(self._lib)}")

    def forward_batched(self, variant: str, W, scale, X, flags: int = 0) -> torch.Tensor:
        """Y [M, N] = rows of X [M, K] through the quantised W."""
        self._check_variant(variant)
        self._validate_w(W)
        self._validate_scale(W, scale)
        M = self._validate_batch(W, X, self._k_of(W))
        out = torch.empty(M, W.size(0), dtype=torch.float16, device=W.device)
        self._launch_batched(variant, W, scale, X, out, flags)
        return out

    def forward_batched_into(self, variant: str, W, scale, X, out, flags: int = 0) -> None:
        self._check_variant(variant)
        self._validate_w(W)
        self._validate_scale(W, scale)
        M = self._validate_batch(W, X, self._k_of(W))
        _chk(out.dim() == 2 and out.size(0) == M and out.size(1) == W.size(0),
             f"out must be [M={M}, N={W.size(0)}]")
        _chk(out.dtype == torch.float16 and out.is_contiguous(), "out must be contiguous float16")
        _chk(out.is_cuda and out.device == W.device, f"out must be on the device of {self.w_name}")
        self._launch_batched(variant, W, scale, X, out, flags)

    def native_timing(self, variant: str, W, scale, x, out, warmup: int = 200,
                      n_windows: int = 10, launches_per_window: int = 64,
                      flags: int = 0) -> dict:
        self._check_variant(variant)
        _chk(warmup >= 0, f"warmup 必须 >= 0，实际 {warmup} (warmup must be >= 0)")
        _chk(n_windows >= 1, f"n_windows 必须 >= 1，实际 {n_windows} (n_windows must be >= 1)")
        _chk(launches_per_window >= 1,
             f"launches_per_window 必须 >= 1，实际 {launches_per_window} "
             "(launches_per_window must be >= 1)")
        self._validate_inputs(W, scale, x)
        self._validate_out(W, out)
        N, K = W.size(0), self._k_of(W)
        buf = (ctypes.c_double * n_windows)()
        dev = W.device
        with torch.cuda.device(dev):
            rc = self._timing(variant.encode(), W.data_ptr(), scale.data_ptr(), x.data_ptr(),
                              out.data_ptr(), N, K, warmup, n_windows, launches_per_window,
                              _stream_ptr(dev), flags, buf)
        if rc != nat.CL_OK:
            raise RuntimeError(f"native_timing failed ({rc}): {nat.last_error(self._lib)}")
        return timing_result(variant, warmup, n_windows, launches_per_window, buf)


class Int4gemvExt(_ExtBase):
    """W4A16: W_packed uint8 [N, K/2], scale fp16 [N, K/128], x fp16 [K]."""
    kind = "int4gemv"
    w_name = "W_packed"
    _kind_code = 0

    def __init__(self) -> None:
        super().__init__()
        self._call = self._lib.cl_int4gemv_ex
        self._batched = self._lib.cl_int4gemv_batched
        self._timing = self._lib.cl_int4gemv_native_timing

    def _k_of(self, W) -> int:
        return 2 * W.size(1)

    # ---- fused RMSNorm -> INT4 GEMV (no reference counterpart; English messages) ----
    def rmsnorm_variants(self) -> list[str]:
        return ["int4gemv_rmsnorm", "int4gemv_rmsnorm_w2", "int4gemv_rmsnorm_w4",
                "int4gemv_rmsnorm_w8", "int4gemv_rmsnorm_w8c2", "int4gemv_rmsnorm_w16"]

    def forward_rmsnorm(self, variant: str, W_packed, scale, X, norm_weight, eps: float = 1e-5,
                        out=None, flags: int = 0) -> torch.Tensor:
        """Y = W * RMSNorm(X, norm_weight) per row of X ([M, K] -> [M, N], or
        [K] -> [N]) in one launch per 16 rows; equal bit for bit to rmsnorm()
        followed by forward_batched(variant 'int4gemv_mma_w8c2')."""
        _chk(variant in self.rmsnorm_variants(),
             f"unknown int4gemv_rmsnorm variant '{variant}'; available: "
             f"{' '.join(self.rmsnorm_variants())}")
        self._validate_w(W_packed)
        self._validate_scale(W_packed, scale)
        K, N = self._k_of(W_packed), W_packed.size(0)
        X2 = X.unsqueeze(0) if X.dim() == 1 else X
        M = self._validate_batch(W_packed, X2, K)
        _chk(norm_weight.dim() == 1 and norm_weight.size(0) == K,
             f"norm_weight must be 1-D of length K={K}")
        _chk(norm_weight.dtype == torch.float16 and norm_weight.is_contiguous(),
             "norm_weight must be contiguous float16")
        _chk(norm_weight.is_cuda and norm_weight.device == W_packed.device,
             "norm_weight must be on the device of W_packed")
        _chk(eps >= 0.0 and eps == eps and eps != float("inf"), "eps must be finite and >= 0")
        shape = (N,) if X.dim() == 1 else (M, N)
        if out is None:
            out = torch.empty(shape, dtype=torch.float16, device=W_packed.device)
        else:
            _chk(tuple(out.shape) == shape and out.dtype == torch.float16 and out.is_contiguous()
                 and out.is_cuda and out.device == W_packed.device,
                 f"out must be contiguous float16 {list(shape)} on the device of W_packed")
        dev = W_packed.device
        with torch.cuda.device(dev):
            rc = self._lib.cl_int4gemv_rmsnorm(
                variant.encode(), W_packed.data_ptr(), scale.data_ptr(), X2.data_ptr(),
                norm_weight.data_ptr(), float(eps), out.data_ptr(), M, N, K, _stream_ptr(dev),
                flags)
        if rc != nat.CL_OK:
            raise RuntimeError(f"int4gemv_rmsnorm launch failed ({rc}): "
                               f"{nat.last_error(self._lib)}")
        return out

    @staticmethod
    def _fast_inputs(Wp, scale, x) -> bool:
        if Wp.dtype is not _U8 or Wp.dim() != 2 or not Wp.is_contiguous():
            return False
        n, kh = Wp.shape
        if n <= 0 or kh <= 0 or kh % 64:  # K = 2 kh, K % 128 == 0
            return False
        return (scale.dtype is _F16 and scale.shape == (n, kh // 64) and scale.is_contiguous()
                and x.dtype is _F16 and x.shape == (2 * kh,) and x.is_contiguous()
                and Wp.is_cuda and _same_device(Wp.get_device(), scale, x))

    def _validate_w(self, Wp: torch.Tensor) -> None:
        _chk(Wp.dim() == 2, f"W_packed 必须是 2 维 (N, K/2)，实际 {Wp.dim()} 维 "
                            "(W_packed must be 2-D)")
        _chk(Wp.size(0) > 0, f"N 必须 > 0，实际 {Wp.size(0)} (N must be > 0)")
        _chk(Wp.size(1) > 0, f"K/2 必须 > 0，实际 {Wp.size(1)} (K/2 must be > 0)")
        _chk(Wp.dtype == torch.uint8,
             f"W_packed 必须是 uint8（torch uint8 为 kByte），实际 {Wp.dtype} "
             "(W_packed must be uint8)")
        K = 2 * Wp.size(1)
        _chk(K % 128 == 0, f"K 必须可被 128 整除（group_size=128 合同）, 实际 K={K} "
                           "(K must be divisible by 128)")
        _chk(Wp.is_contiguous(), "W_packed 必须是连续内存 (W_packed must be contiguous)")
        _chk(Wp.is_cuda, "W_packed 必须是 CUDA 张量 (W_packed must be a CUDA tensor)")

    def _validate_scale(self, Wp: torch.Tensor, scale: torch.Tensor) -> None:
        N, K = Wp.size(0), 2 * Wp.size(1)
        _chk(scale.dim() == 2, f"scale 必须是 2 维 (N, K/128)，实际 {scale.dim()} 维 "
                               "(scale must be 2-D)")
        _chk(scale.size(0) == N, f"scale 行数必须等于 N: scale={scale.size(0)} N={N} "
                                 "(scale rows must equal N)")
        _chk(scale.size(1) == K // 128,
             f"scale 组数必须等于 K/128（invalid group count）: scale={scale.size(1)} "
             f"K/128={K // 128} (scale groups must equal K/128)")
        _chk(scale.dtype == torch.float16,
             f"scale 必须是 float16（group-wise 合同）, 实际 {scale.dtype} "
             "(scale must be float16)")
        _chk(scale.is_contiguous(), "scale 必须是连续内存 (scale must be contiguous)")
        _chk(scale.is_cuda, "scale 必须是 CUDA 张量 (scale must be a CUDA tensor)")
        _chk(scale.device == Wp.device,
             "scale 必须与 W_packed 在同一 CUDA 设备上 (scale must be on the device of W_packed)")


class QgemvExt(_ExtBase):
    """INT8: W_q int8 [N, K], scale fp32 [N], x fp16 [K]."""
    kind = "qgemv"
    w_name = "W_q"
    _kind_code = 1

    def __init__(self) -> None:
        super().__init__()
        self._call = self._lib.cl_qgemv_ex
        self._batched = self._lib.cl_qgemv_batched
        self._timing = self._lib.cl_qgemv_native_timing

    def _k_of(self, W) -> int:
        return W.size(1)

    @staticmethod
    def _fast_inputs(Wq, scale, x) -> bool:
        if Wq.dtype is not _I8 or Wq.dim() != 2 or not Wq.is_contiguous():
            return False
        n, k = Wq.shape
        if n <= 0 or k <= 0:
            return False
        return (scale.dtype is _F32 and scale.shape == (n,) and scale.is_contiguous()
                and x.dtype is _F16 and x.shape == (k,) and x.is_contiguous()
                and Wq.is_cuda and _same_device(Wq.get_device(), scale, x))

    def _validate_w(self, Wq: torch.Tensor) -> None:
        _chk(Wq.dim() == 2, f"W_q 必须是 2 维 (N, K)，实际 {Wq.dim()} 维 (W_q must be 2-D)")
        _chk(Wq.size(0) > 0, f"N 必须 > 0，实际 {Wq.size(0)} (N must be > 0)")
        _chk(Wq.size(1) > 0, f"K 必须 > 0，实际 {Wq.size(1)} (K must be > 0)")
        _chk(Wq.dtype == torch.int8,
             f"W_q 必须是 int8（torch int8 为 kChar），实际 {Wq.dtype} (W_q must be int8)")
        _chk(Wq.is_contiguous(), "W_q 必须是连续内存 (W_q must be contiguous)")
        _chk(Wq.is_cuda, "W_q 必须是 CUDA 张量 (W_q must be a CUDA tensor)")

    def _validate_scale(self, Wq: torch.Tensor, scale: torch.Tensor) -> None:
        _chk(scale.dim() == 1, f"scale 必须是 1 维 (N,)，实际 {scale.dim()} 维 "
                               "(scale must be 1-D)")
        _chk(scale.size(0) == Wq.size(0),
             f"scale 长度必须等于 N: scale={scale.size(0)} N={Wq.size(0)} "
             "(len(scale) must equal N)")
        _chk(scale.dtype == torch.float32,
             f"scale 必须是 float32，实际 {scale.dtype} (scale must be float32)")
        _chk(scale.is_contiguous(), "scale 必须是连续内存 (scale must be contiguous)")
        _chk(scale.is_cuda, "scale 必须是 CUDA 张量 (scale must be a CUDA tensor)")
        _chk(scale.device == Wq.device,
             "scale 必须与 W_q 在同一 CUDA 设备上 (scale must be on the device of W_q)")


_EXTS: dict = {}


class GemvExt:
    """Dense GEMV, y = W @ x with W fp16 / fp32 [N, K], x [K], y [N] of the
    same dtype, fp32 accumulation: mirrors kernels/gemv/bindings.cpp (checks
    :86-125 in that order, forward :136-162, forward_into :166-191,
    native_timing :195-266, variant lists :271-306), each message's first
    part the reference's text, then an English rendering."""
    kind = "gemv"

    def __init__(self) -> None:
        self._lib = nat.load()
        self._cache = {}

    def variants(self) -> list[str]:
        return nat.list_variants("gemv", nat.CL_VARIANTS_NORMAL)

    def all_variants(self) -> list[str]:
        return nat.list_variants("gemv", nat.CL_VARIANTS_ALL)

    def quarantined_variants(self) -> list[str]:
        return nat.list_variants("gemv", nat.CL_VARIANTS_QUARANTINED)

    def _check_variant(self, name: str) -> None:
        allv = self._cache.get("all")
        if allv is None:
            allv = self._cache["all"] = set(self.all_variants())
        if name not in allv:
            normal = " ".join(self.variants())
            quarantined = " ".join(self.quarantined_variants())
            raise RuntimeError(f"未知 gemv 变体 '{name}'。正常可用: {normal} "
                               f"；被隔离（NOT_FOR_NORMAL_DISPATCH）: {quarantined} "
                               "（显式命名仍可调用，属受控历史审计入口） (unknown gemv variant)")

    @staticmethod
    def _validate_w(W: torch.Tensor) -> None:
        _chk(W.dim() == 2, f"W 必须是 2 维 (N, K)，实际 {W.dim()} 维 (W must be 2-D)")
        _chk(W.size(0) > 0, f"N 必须 > 0，实际 {W.size(0)} (N must be > 0)")
        _chk(W.size(1) > 0, f"K 必须 > 0，实际 {W.size(1)} (K must be > 0)")
        _chk(W.dtype in (torch.float16, torch.float32),
             f"仅支持 float16 / float32，实际 {W.dtype} (only float16 / float32)")
        _chk(W.is_contiguous(), "W 必须是连续内存 (W must be contiguous)")
        _chk(W.is_cuda, "W 必须是 CUDA 张量 (W must be a CUDA tensor)")

    @staticmethod
    def _validate_x(W: torch.Tensor, x: torch.Tensor) -> None:
        _chk(x.dim() == 1, f"x 必须是 1 维 (K,)，实际 {x.dim()} 维 (x must be 1-D)")
        _chk(x.size(0) == W.size(1),
             f"x 长度必须等于 K: x={x.size(0)} K={W.size(1)} (len(x) must equal K)")
        _chk(x.dtype == W.dtype,
             f"x 的 dtype 必须与 W 一致: x={x.dtype} W={W.dtype} (x dtype must equal W dtype)")
        _chk(x.is_contiguous(), "x 必须是连续内存 (x must be contiguous)")
        _chk(x.is_cuda, "x 必须是 CUDA 张量 (x must be a CUDA tensor)")
        _chk(x.device == W.device, "x 必须与 W 在同一 CUDA 设备上 (x must be on the device of W)")

    @staticmethod
    def _validate_out(W: torch.Tensor, out: torch.Tensor) -> None:
        _chk(out.dim() == 1, f"out 必须是 1 维 (N,)，实际 {out.dim()} 维 (out must be 1-D)")
        _chk(out.size(0) == W.size(0),
             f"out 长度必须等于 N: out={out.size(0)} N={W.size(0)} (len(out) must equal N)")
        _chk(out.dtype == W.dtype,
             f"out 的 dtype 必须与 W 一致: out={out.dtype} W={W.dtype} "
             "(out dtype must equal W dtype)")
        _chk(out.is_contiguous(), "out 必须是连续内存 (out must be contiguous)")
        _chk(out.is_cuda, "out 必须是 CUDA 张量 (out must be a CUDA tensor)")
        _chk(out.device == W.device,
             "out 必须与 W 在同一 CUDA 设备上 (out must be on the device of W)")

    @staticmethod
    def _dtype_code(W: torch.Tensor) -> int:
        return nat.CL_DTYPE_F16 if W.dtype == torch.float16 else nat.CL_DTYPE_F32

    def _launch(self, name: str, W, x, out, flags: int = 0) -> None:
        dev = W.device
        with torch.cuda.device(dev):
            rc = self._lib.cl_gemv_ex(name.encode(), W.data_ptr(), x.data_ptr(), out.data_ptr(),
                                      W.size(0), W.size(1), self._dtype_code(W), _stream_ptr(dev),
                                      flags)
        if rc != nat.CL_OK:
            raise RuntimeError(f"gemv launch failed ({rc}): {nat.last_error(self._lib)}")

    def forward(self, variant: str, W, x, flags: int = 0) -> torch.Tensor:
        self._check_variant(variant)
        self._validate_w(W)
        self._validate_x(W, x)
        out = torch.empty(W.size(0), dtype=W.dtype, device=W.device)
        self._launch(variant, W, x, out, flags)
        return out

    def forward_into(self, variant: str, W, x, out, flags: int = 0) -> None:
        self._check_variant(variant)
        self._validate_w(W)
        self._validate_x(W, x)
        self._validate_out(W, out)
        self._launch(variant, W, x, out, flags)

    def native_timing(self, variant: str, W, x, out, warmup: int = 200, n_windows: int = 10,
                      launches_per_window: int = 64, flags: int = 0) -> dict:
        self._check_variant(variant)
        _chk(warmup >= 0, f"warmup 必须 >= 0，实际 {warmup} (warmup must be >= 0)")
        _chk(n_windows >= 1, f"n_windows 必须 >= 1，实际 {n_windows} (n_windows must be >= 1)")
        _chk(launches_per_window >= 1,
             f"launches_per_window 必须 >= 1，实际 {launches_per_window} "
             "(launches_per_window must be >= 1)")
        self._validate_w(W)
        self._validate_x(W, x)
        self._validate_out(W, out)
        buf = (ctypes.c_double * n_windows)()
        dev = W.device
        with torch.cuda.device(dev):
            rc = self._lib.cl_gemv_native_timing(
                variant.encode(), W.data_ptr(), x.data_ptr(), out.data_ptr(), W.size(0),
                W.size(1), self._dtype_code(W), warmup, n_windows, launches_per_window,
                _stream_ptr(dev), flags, buf)
        if rc != nat.CL_OK:
            raise RuntimeError(f"native_timing failed ({rc}): {nat.last_error(self._lib)}")
        return timing_result(variant, warmup, n_windows, launches_per_window, buf)


class RmsnormExt:
    """fp16 RMSNorm: mirrors `forward` / `forward_into` / `variants` of
    kernels/rmsnorm/bindings.cpp:91-115 (argument names and the checks of
    validate_common, :24-41) for the one kernel here, registered as
    'rmsnorm_f16'.  fp32 rows are not supported (RuntimeError); H must be a
    multiple of 8."""
    kind = "rmsnorm"

    def __init__(self) -> None:
        self._lib = nat.load()

    def variants(self) -> list[str]:
        return ["rmsnorm_f16"]

    def _validate(self, variant: str, x, w, eps: float) -> None:
        _chk(variant in self.variants(),
             f"未知 rmsnorm 变体 '{variant}'。可用: rmsnorm_f16 (unknown rmsnorm variant)")
        _chk(x.dim() == 2, f"x 必须是 2 维 (M, H)，实际 {x.dim()} 维 (x must be 2-D)")
        _chk(w.dim() == 1, f"w 必须是 1 维 (H,)，实际 {w.dim()} 维 (w must be 1-D)")
        _chk(x.size(0) > 0, f"M 必须 > 0，实际 {x.size(0)} (M must be > 0)")
        _chk(x.size(1) > 0, f"H 必须 > 0，实际 {x.size(1)} (H must be > 0)")
        _chk(x.size(1) == w.size(0), f"维度不匹配: H={x.size(1)} vs w={w.size(0)} "
                                     "(H must equal len(w))")
        _chk(x.dtype == w.dtype, "x 与 w 必须同 dtype (x and w must have the same dtype)")
        _chk(x.dtype == torch.float16, f"only float16 rows are supported, got {x.dtype}")
        _chk(x.is_contiguous(), "x 必须是连续内存 (x must be contiguous)")
        _chk(w.is_contiguous(), "w 必须是连续内存 (w must be contiguous)")
        _chk(x.is_cuda, "x 必须是 CUDA 张量 (x must be a CUDA tensor)")
        _chk(w.is_cuda, "w 必须是 CUDA 张量 (w must be a CUDA tensor)")
        _chk(x.device == w.device, "w 必须与 x 在同一 CUDA 设备上 (w must be on the device of x)")
        _chk(eps >= 0.0 and eps == eps and eps != float("inf"),
             f"eps 必须是有限且 >= 0，实际 {eps} (eps must be finite and >= 0)")
        _chk(x.size(1) % 8 == 0, f"H must be a multiple of 8, got {x.size(1)}")

    def _launch(self, x, w, out, eps: float, flags: int) -> None:
        dev = x.device
        with torch.cuda.device(dev):
            rc = self._lib.cl_rmsnorm_f16(x.data_ptr(), w.data_ptr(), float(eps), out.data_ptr(),
                                          x.size(0), x.size(1), _stream_ptr(dev), flags)
        if rc != nat.CL_OK:
            raise RuntimeError(f"rmsnorm launch failed ({rc}): {nat.last_error(self._lib)}")

    def forward(self, variant: str, x, w, eps: float = 1e-5, flags: int = 0) -> torch.Tensor:
        self._validate(variant, x, w, eps)
        out = torch.empty_like(x)
        self._launch(x, w, out, eps, flags)
        return out

    def forward_into(self, variant: str, x, w, out, eps: float = 1e-5, flags: int = 0) -> None:
        self._validate(variant, x, w, eps)
        _chk(out.dim() == 2, f"out 必须是 2 维 (M, H)，实际 {out.dim()} 维 (out must be 2-D)")
        _chk(out.shape == x.shape, "out 形状必须与 x 一致 (out must have the shape of x)")
        _chk(out.dtype == x.dtype, "out 必须与 x 同 dtype (out must have the dtype of x)")
        _chk(out.is_contiguous(), "out 必须是连续内存 (out must be contiguous)")
        _chk(out.is_cuda, "out 必须是 CUDA 张量 (out must be a CUDA tensor)")
        _chk(out.device == x.device, "out 必须与 x 在同一 CUDA 设备上 (out must be on the "
                                     "device of x)")
        self._launch(x, w, out, eps, flags)


_EXT_TYPES = {"int4gemv": Int4gemvExt, "qgemv": QgemvExt, "gemv": GemvExt, "rmsnorm": RmsnormExt}


def get_ext(op: str):
    """Singleton extension object for `op`."""
    if op not in _EXT_TYPES:
        raise RuntimeError(f"unknown operator {op!r}; available: {', '.join(_EXT_TYPES)}")
    if op not in _EXTS:
        _EXTS[op] = _EXT_TYPES[op]()
    return _EXTS[op]
