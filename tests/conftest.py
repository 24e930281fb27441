"""Shared test setup.

Markers: ``gpu`` tests need a CUDA device (a B200) and call the kernels
through the C ABI; everything else runs on CPU.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a); parity through the C ABI")


def has_gpu():
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


# ---------------------------------------------------------------- helpers ----
def u16(t):
    """torch 2-byte tensor -> numpy uint16 view (host copy)."""
    import torch

    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def dev(a, dtype):
    """numpy uint16 -> CUDA torch tensor of `dtype` (float16/bfloat16)."""
    import torch

    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(dtype).cuda()


def dcode(dtype):
    import torch

    return 0 if dtype == torch.float16 else 1


def assert_close(got_u16, ref_u16, dtype_code=0, max_abs=2e-2, rel_l2=1e-3, ulps=1.0, what=""):
    """Parity bar for 2-byte float outputs against the oracle.

    rel-L2 <= rel_l2 and, elementwise, |got - ref| <= max_abs + ulps * ulp(ref)
    where ulp(ref) is the storage format's spacing at |ref| (fp16: 2^-10
    relative, bf16: 2^-7 relative) -- an output rounded once from a slightly
    different fp32 value may land one storage ulp away.
    """
    import oracle

    g = oracle.to_float(got_u16, dtype_code).astype(np.float64)
    r = oracle.to_float(ref_u16, dtype_code).astype(np.float64)
    assert g.shape == r.shape
    fin = np.isfinite(r)
    assert np.array_equal(np.isfinite(g), fin), f"{what}: non-finite mismatch"
    g, r = g[fin], r[fin]
    if r.size == 0:
        return
    rel_ulp = 2.0 ** -10 if dtype_code == 0 else 2.0 ** -7
    tol = max_abs + ulps * rel_ulp * np.abs(r)
    diff = np.abs(g - r)
    bad = diff > tol
    num = np.linalg.norm(g - r)
    den = max(np.linalg.norm(r), 1e-30)
    assert not bad.any(), f"{what}: {bad.sum()} elements out of tolerance, max diff {diff.max():.4g} at ref {r[np.argmax(diff - tol)]:.4g}"
    assert num / den <= rel_l2, f"{what}: rel-L2 {num / den:.3g} > {rel_l2}"
