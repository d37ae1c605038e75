"""The bit trick of the tensor-core kernels' INT4 dequantisation, checked
exhaustively on the CPU.

The kernels turn two packed nibbles into two fp16 operands with one lop3 that
places each nibble under a binary16 exponent, followed by one fp16 add of an
immediate that removes the bias.  The constants are read from
the kernel sources, so an edit that breaks exactness fails here before any
GPU run.  numpy's float16 arithmetic rounds like the GPU's fp16 add / fma for
these operands (every result is a small integer, exactly representable).
"""
import re
from pathlib import Path

import numpy as np

CSRC = Path(__file__).resolve().parents[1] / "cudalab_b200" / "csrc"


def _nib_pair_consts():
    """(mask, pattern, bias bits) of nib_pair_lo and nib_pair_hi."""
    src = (CSRC / "gemv_mma.cuh").read_text()
    consts = dict(re.findall(r"constexpr unsigned short (kH_\w+) = (0x[0-9A-Fa-f]+);",
                             (CSRC / "gemv_common.cuh").read_text()))
    out = {}
    for name in ("nib_pair_lo", "nib_pair_hi"):
        body = src[src.index(f"uint32_t {name}(uint32_t w)"):]
        body = body[:body.index("}")]
        m = re.search(r"__hadd2\(u32_as_h2\(lop3_sel_xor_i<(0x[0-9A-Fa-f]+)u, (0x[0-9A-Fa-f]+)u>"
                      r"\(w\)\),\s*h2_const\((kH_\w+)\)\)", body)
        assert m, f"{name}: unexpected form"
        out[name] = (int(m.group(1), 16), int(m.group(2), 16), int(consts[m.group(3)], 16))
    return out


def _h16(bits):
    return np.asarray(bits, dtype=np.uint16).view(np.float16)


def _signed_nibbles(w, shift):
    n = (w >> shift) & 0xF
    return np.where(n >= 8, n.astype(np.int64) - 16, n.astype(np.int64))


def test_nibble_pairs_exact_for_every_word_half():
    """Every 16-bit half of a weight word (all 65536): the low pair yields
    nibble 0 of the half, the high pair nibble 1, as exact fp16 integers, and
    a zero nibble gives +0 (the same bits as the earlier fma form)."""
    c = _nib_pair_consts()
    half = np.arange(1 << 16, dtype=np.uint32)
    w = half | (half << 16)  # both halves of the word
    for name, shift in (("nib_pair_lo", 0), ("nib_pair_hi", 4)):
        mask, pat, bias = c[name]
        v = ((w & mask) ^ pat) & 0xFFFFFFFF  # lop3 LUT 0x6A: mask ? w ^ pat : pat
        lo16 = _h16((v & 0xFFFF).astype(np.uint16))
        got = (lo16 + _h16(np.full(v.shape, bias, dtype=np.uint16))).astype(np.float16)
        want = _signed_nibbles(half, shift)
        assert np.array_equal(got.astype(np.float64), want.astype(np.float64)), name
        assert not np.any(np.signbit(got[want == 0])), name
        hi16 = _h16(((v >> 16) & 0xFFFF).astype(np.uint16))
        assert np.array_equal(hi16, lo16)


def test_nibble_pairs_match_earlier_fma_form():
    """The add-immediate forms give the values of the fma forms the CUDA-core
    kernels keep (exponent of 1024 for both pairs, the high one rescaled by
    1/16), bit for bit."""
    half = np.arange(1 << 16, dtype=np.uint32)
    one, sixteenth = np.float16(1.0), np.float16(0.0625)
    lo_old = (_h16(((half & 0x000F) ^ 0x6408).astype(np.uint16)) * one
              + np.float16(-1032)).astype(np.float16)
    hi_old = (_h16(((half & 0x00F0) ^ 0x6480).astype(np.uint16)) * sixteenth
              + np.float16(-72)).astype(np.float16)
    c = _nib_pair_consts()
    outs = []
    for name in ("nib_pair_lo", "nib_pair_hi"):
        mask, pat, bias = c[name]
        v = _h16((((half & mask) ^ pat) & 0xFFFF).astype(np.uint16))
        outs.append((v + _h16(np.full(half.shape, bias, dtype=np.uint16))).astype(np.float16))
    assert np.array_equal(outs[0].view(np.uint16), lo_old.view(np.uint16))
    assert np.array_equal(outs[1].view(np.uint16), hi_old.view(np.uint16))
