"""The trace kernel's exit quotient (navi_b200/csrc/exit_quotient.cuh) against the IEEE
division __fdiv_rn on the device, bit for bit.

The grid kernel computes each quotient of a void cell's exit distance by one fused
residual correction of RN(a * RN(1 / d)) instead of a division.  These tests check that
identity over slices of the binary32 significand pairs (exhaustively over all 2^46 pairs
with NAVI_QUOTIENT_EXHAUSTIVE=1, about a minute on one B200) and over sampled exponents
and signs, through navi_b200/csrc/quotient_check.cu in libnavi_probe.so.
"""

from __future__ import annotations

import ctypes
import os
import struct

import pytest
import torch

from tests.gpu_util import dev

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu


def _lib():
    path = os.path.join(ROOT, "navi_b200", "_lib", "libnavi_probe.so")
    assert os.path.exists(path), "libnavi_probe.so not built (navi_b200/build.py)"
    lib = ctypes.CDLL(path)
    lib.navi_check_exit_quotient.restype = ctypes.c_int
    lib.navi_check_exit_quotient.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p]
    lib.navi_check_exit_quotient_scaled.restype = ctypes.c_int
    lib.navi_check_exit_quotient_scaled.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_int,
                                                    ctypes.c_void_p]
    return lib


def _floats(word: int) -> tuple[float, float]:
    a = struct.unpack("<f", struct.pack("<I", (word >> 32) & 0xFFFFFFFF))[0]
    d = struct.unpack("<f", struct.pack("<I", word & 0xFFFFFFFF))[0]
    return a, d


def _exhaustive(lib, slices) -> list[int]:
    d = dev()
    out = torch.zeros(2, dtype=torch.int64, device=d)
    stream = torch.cuda.current_stream(d)
    for first, count in slices:
        rc = lib.navi_check_exit_quotient(first, count, ctypes.c_void_p(out.data_ptr()),
                                          ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0, f"launch failed: cudaError {rc}"
    torch.cuda.synchronize(d)
    return out.cpu().tolist()


def test_exit_quotient_on_significand_slices():
    """All 2^23 dividends against divisors next to 1 and 2 (the reciprocal at the top and
    bottom of its binade), powers of two and 1024 random divisor significands."""
    lib = _lib()
    g = torch.Generator().manual_seed(5)
    rand = torch.randint(0, 1 << 23, (1024,), generator=g).tolist()
    slices = [(0, 2048), ((1 << 23) - 2048, 2048)] + [(int(r), 1) for r in rand]
    bad, first = _exhaustive(lib, slices)
    assert bad == 0, f"{bad} mismatches; first a, d = {_floats(first)}"


@pytest.mark.skipif(os.environ.get("NAVI_QUOTIENT_EXHAUSTIVE") != "1",
                    reason="full sweep of 2^46 pairs: set NAVI_QUOTIENT_EXHAUSTIVE=1")
def test_exit_quotient_all_significand_pairs():
    lib = _lib()
    step = 1 << 15
    bad, first = _exhaustive(lib, [(f, step) for f in range(0, 1 << 23, step)])
    assert bad == 0, f"{bad} mismatches; first a, d = {_floats(first)}"


def test_exit_quotient_scaled_and_clamped():
    """2^30 pairs over the exponent range: the quotient where exact by construction, and the
    clamped exit distance (with the kernel's fallback division for |d| >= 2^126) everywhere."""
    lib = _lib()
    d = dev()
    out = torch.zeros(4, dtype=torch.int64, device=d)
    stream = torch.cuda.current_stream(d)
    sms = torch.cuda.get_device_properties(d).multi_processor_count
    for seed in (1, 2, 3, 4):
        rc = lib.navi_check_exit_quotient_scaled(seed, 1 << 28, ctypes.c_void_p(out.data_ptr()), sms * 8,
                                                 ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0, f"launch failed: cudaError {rc}"
    torch.cuda.synchronize(d)
    bad_q, first_q, bad_c, first_c = out.cpu().tolist()
    assert bad_q == 0, f"quotient: {bad_q} mismatches; first a, d = {_floats(first_q)}"
    assert bad_c == 0, f"clamped exit: {bad_c} mismatches; first a, d = {_floats(first_c)}"
