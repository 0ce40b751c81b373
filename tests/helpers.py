"""Shared helpers for the parity tests."""

from __future__ import annotations

import numpy as np

TOL_MAX_ABS = 2e-2   # north-star bound for bf16/fp16 attention vs the fp32 oracle
TOL_MEAN_ABS = 2e-3


def torch_dtype(name):
    import torch

    return {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}[name]


def to_dev(a, dtype=None, device="cuda"):
    """numpy -> torch on device; float arrays are cast to ``dtype`` (exactly,
    since the seeded values are representable)."""
    import torch

    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(torch_dtype(dtype) if isinstance(dtype, str) else dtype)
    return t.to(device)


def to_np(t):
    return t.detach().float().cpu().numpy()


def assert_attention_close(actual, expected_fp32, max_abs=TOL_MAX_ABS, mean_abs=TOL_MEAN_ABS):
    """Attention output within the north-star tolerance of the fp32 oracle."""
    a = np.asarray(actual, np.float32)
    e = np.asarray(expected_fp32, np.float32)
    assert a.shape == e.shape, (a.shape, e.shape)
    assert np.isfinite(a).all(), "non-finite output"
    d = np.abs(a - e)
    assert d.max() <= max_abs, f"max abs err {d.max():.3g} > {max_abs}"
    assert d.mean() <= mean_abs, f"mean abs err {d.mean():.3g} > {mean_abs}"


def decode_golden(arr, dtype):
    from oracle.numerics import bf16_from_bits

    if dtype == "float32":
        return np.asarray(arr, np.float32)
    if dtype == "float16":
        return np.asarray(arr, np.uint16).view(np.float16).astype(np.float32)
    return bf16_from_bits(arr)
