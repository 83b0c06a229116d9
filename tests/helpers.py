"""Shared test helpers: tolerance metric, tensor conversion, op-input builders."""
from __future__ import annotations

import ctypes
import os

import numpy as np

import w4a8_oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "w4a8_b200.h")
LIB = os.path.join(ROOT, "rdna4-vllm_b200", "w4a8_fp8_wmma", "libw4a8_b200.so")

# North-star tolerance for GEMM outputs: max |ours - ref| / max |ref| <= 1e-2.
MAX_ABS_REL = 1e-2


def max_abs_rel(ours, ref) -> float:
    ours = np.asarray(ours, np.float64)
    ref = np.asarray(ref, np.float64)
    den = max(np.abs(ref).max(), 1e-30) if ref.size else 1.0
    return float(np.abs(ours - ref).max() / den) if ref.size else 0.0


def reference_tolerance_ok(ours, ref, atol=0.15, rtol=0.03, mean_tol=2e-3, mean_rtol=0.01):
    """The reference's own pass rule (w4a8_fp8_wmma/test_correctness.py:146-158)."""
    ours = np.asarray(ours, np.float64)
    ref = np.asarray(ref, np.float64)
    diff = np.abs(ours - ref)
    eff = max(mean_tol, mean_rtol * np.abs(ref).mean())
    return diff.mean() <= eff and int((diff > atol + rtol * np.abs(ref)).sum()) == 0


def header_symbols() -> list[str]:
    import re
    src = open(HEADER).read()
    return sorted(set(re.findall(r"\b(w4a8_[a-z0-9_]+)\s*\(", src)))


def load_lib():
    return ctypes.CDLL(LIB)


def packed_dense(codes, scales, zeros):
    """numpy (N,K) codes, (N,G) scales, (N,G) zeros|None -> packed numpy arrays."""
    return O.pack_int4(codes), scales, (O.pack_zeros(zeros) if zeros is not None else None)
