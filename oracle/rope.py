"""numpy restatement of FlashDec's split-half RoPE and the one-token K/V append.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).
"""

from __future__ import annotations

import math

import numpy as np

from .numerics import round_to_dtype


def inv_freq_table(rotary_dim: int, base: float) -> np.ndarray:
    """``inv_freq = base ** (-arange(0, rd, 2) / rd)`` as float32.

    Follows ``flashdec/rope.py:66-67``: the exponent is formed in float32
    (``arange`` fp32, negated, divided by ``rotary_dim``).  The reference then
    takes ``torch.pow`` in float32, which is not correctly rounded (it differs
    from the correctly rounded value by one ulp in a few entries, and numpy's
    float32 power differs from both).  The oracle uses the correctly rounded
    power (float64 pow, rounded once to float32) so that it does not depend on
    the host's libm; callers that must reproduce a specific table pass it to
    :func:`apply_rope` as ``inv_freq``.
    """
    steps = np.arange(0, rotary_dim, 2, dtype=np.float32)
    expo = (-steps / np.float32(rotary_dim)).astype(np.float32)
    return np.power(np.float64(np.float32(base)), expo.astype(np.float64)).astype(np.float32)


def apply_rope(x, positions, rotary_dim=None, base=10_000.0, dtype="float32", inv_freq=None):
    """Split-half (neox) rotary embedding with fp32 math.

    Follows ``flashdec/rope.py:26-85``: validation (:39-64), angles
    ``pos_f32 * inv_freq`` (:68), ``cos``/``sin`` (:69-70), rotation
    ``[x1 cos - x2 sin, x2 cos + x1 sin]`` over the first ``rotary_dim`` dims
    (:72-83) with the tail copied unchanged (:84-85), result cast to ``dtype``.

    ``inv_freq`` may be passed to pin the exact table (the reference computes
    it with ``torch.pow``; see :func:`inv_freq_table`).
    """
    x = np.asarray(x, dtype=np.float32)
    positions = np.asarray(positions)
    if x.ndim != 3:
        raise ValueError("x must have shape [batch, num_heads, head_dim]")
    if positions.ndim != 1 or positions.size != x.shape[0]:
        raise ValueError("positions must have shape [batch]")
    if (positions < 0).any():
        raise ValueError("positions must be non-negative")
    head_dim = x.shape[-1]
    if rotary_dim is None:
        rotary_dim = head_dim
    if isinstance(rotary_dim, bool) or not isinstance(rotary_dim, int):
        raise ValueError("rotary_dim must be an even integer")
    if rotary_dim <= 0 or rotary_dim > head_dim or rotary_dim % 2 != 0:
        raise ValueError("rotary_dim must be positive, even, and no larger than head_dim")
    base = float(base)
    if not math.isfinite(base) or base <= 0.0:
        raise ValueError("base must be a positive finite number")

    if inv_freq is None:
        inv_freq = inv_freq_table(rotary_dim, base)
    inv_freq = np.asarray(inv_freq, dtype=np.float32)
    angles = positions.astype(np.float32)[:, None] * inv_freq[None, :]
    cos = np.cos(angles).astype(np.float32)[:, None, :]
    sin = np.sin(angles).astype(np.float32)[:, None, :]
    half = rotary_dim // 2
    x1 = x[..., :half]
    x2 = x[..., half:rotary_dim]
    # Separate multiplies then add/sub, as torch evaluates the expression.
    first = (x1 * cos).astype(np.float32) - (x2 * sin).astype(np.float32)
    second = (x2 * cos).astype(np.float32) + (x1 * sin).astype(np.float32)
    rotated = round_to_dtype(np.concatenate([first, second], axis=-1), dtype)
    return np.concatenate([rotated, x[..., rotary_dim:]], axis=-1)


def rope_kv_append_ref(q, k, v, k_cache, v_cache, block_ids, block_offsets, positions,
                       rotary_dim=None, base=10_000.0, dtype="float32", inv_freq=None):
    """Fused RoPE + one-token paged append, as the reference's CUDA primitive.

    Follows ``flashdec/_fused_rope_kv_append.py:210-258`` /
    ``flashdec/csrc/fused_rope_kv_append_kernel.cu:38-82``:
    ``q_out = rope(q)``; for every request row ``r`` and KV head ``h``:
    ``k_cache[block_ids[r], h, block_offsets[r], :] = rope(k)[r, h]`` and
    ``v_cache[...] = v[r, h]`` (V copied bit-exactly).  Cache layout is
    token-major ``[blocks, kv_heads, block_size, head_dim]``.
    Returns ``(q_out, k_cache_after, v_cache_after)``.
    """
    q_out = apply_rope(q, positions, rotary_dim, base, dtype, inv_freq)
    k_rot = apply_rope(k, positions, rotary_dim, base, dtype, inv_freq)
    k_after = np.array(k_cache, dtype=np.float32, copy=True)
    v_after = np.array(v_cache, dtype=np.float32, copy=True)
    for r, (b, o) in enumerate(zip(np.asarray(block_ids).tolist(), np.asarray(block_offsets).tolist())):
        k_after[b, :, o, :] = k_rot[r]
        v_after[b, :, o, :] = np.asarray(v, dtype=np.float32)[r]
    return q_out, k_after, v_after
