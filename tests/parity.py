"""Parity gates shared by the tests.

bf16 outputs: every element within ``2e-2 * max(1, |ref|)`` (the reference's test-fire rule of
``conv_kernel.py:99-101`` applied per element: one bf16 ulp at |y| in [4, 8) is 0.03125, so a fixed 2e-2 would
fail on a single rounding flip there) and relative L2 error <= 1e-2.  fp32 checks use 1e-5.

Every bf16 comparison is also recorded with its plain max-abs error and whether that alone meets a literal 2e-2
bound; conftest prints the records as a table at the end of the session.
"""
from __future__ import annotations

import numpy as np
import torch

ATOL_BF16 = 2e-2
REL_L2_BF16 = 1e-2
TOL_FP32 = 1e-5


def to_np(t) -> np.ndarray:
    if isinstance(t, torch.Tensor):
        return t.detach().float().cpu().numpy()
    return np.asarray(t, dtype=np.float32)


def stats(out, ref) -> dict:
    o = to_np(out).astype(np.float64)
    r = to_np(ref).astype(np.float64)
    d = np.abs(o - r)
    bound = ATOL_BF16 * np.maximum(1.0, np.abs(r))
    den = np.linalg.norm(r)
    return {
        "max_abs": float(d.max()) if d.size else 0.0,
        "worst_ratio": float((d / bound).max()) if d.size else 0.0,
        "rel_l2": float(np.linalg.norm(o - r) / den) if den > 0 else float(np.linalg.norm(o - r)),
        "exact_frac": float((d == 0).mean()) if d.size else 1.0,
    }


RECORDS: list[tuple[str, dict]] = []     # (what, stats) of every bf16 comparison in this session


def assert_bf16_close(out, ref, what: str = "", rel_l2: float = REL_L2_BF16) -> dict:
    s = stats(out, ref)
    s["max_ref"] = float(np.abs(to_np(ref)).max()) if to_np(ref).size else 0.0
    RECORDS.append((what, s))
    assert to_np(out).shape == to_np(ref).shape, f"{what}: shape {to_np(out).shape} vs {to_np(ref).shape}"
    assert np.isfinite(to_np(out)).all(), f"{what}: non-finite output"
    assert s["worst_ratio"] <= 1.0, f"{what}: element beyond 2e-2*max(1,|ref|): {s}"
    assert s["rel_l2"] <= rel_l2, f"{what}: rel-L2 {s['rel_l2']:.3e} > {rel_l2}: {s}"
    return s
