"""Decode-time RoPE and the RoPE + paged K/V append step, on B200 kernels.

Drop-in for ``flashdec/rope.py`` (cysong2025/flashdec): same names, argument
meaning, validation order and error messages.

* :func:`apply_rope` keeps the reference's checks (rope.py:26-64) and runs
  the rotation in ``fd_rope_kv_append`` with no cache rows (q only).  The
  frequency table is the reference's fp32 ``torch.pow`` table (rope.py:66-67)
  computed once on the host, the angle is ``float(pos) * inv_freq`` and the
  products and sums are rounded separately, as torch evaluates rope.py:68-79.
* :func:`rope_paged_kv_append` follows rope.py:124-168: next positions from
  the cache ledger, rotate Q/K, append rotated K and raw V.  Every backend
  name runs native kernels: ``'fused_cuda'`` one fused launch,
  ``'torch'``/``'cuda'`` a RoPE launch for Q, one for K and a K/V copy launch
  (the reference's unfused order, kept for callers that select it).

Inputs must be CUDA tensors; there is no CPU path in this package.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any

import torch

from . import _native


@dataclass(frozen=True)
class RopeAppendResult:
    """Outputs required by the next paged decode attention call."""

    q: Any
    positions: Any
    block_tables: Any
    seq_lens: Any


def _check_rotary(rotary_dim, head_dim, base):
    if rotary_dim is None:
        rotary_dim = head_dim
    if isinstance(rotary_dim, bool) or not isinstance(rotary_dim, int):
        raise ValueError("rotary_dim must be an even integer")
    if rotary_dim <= 0 or rotary_dim > head_dim or rotary_dim % 2 != 0:
        raise ValueError("rotary_dim must be positive, even, and no larger than head_dim")
    base = float(base)
    if not math.isfinite(base) or base <= 0.0:
        raise ValueError("base must be a positive finite number")
    return rotary_dim, base


def apply_rope(x, positions, rotary_dim=None, base=10_000.0):
    """Split-half rotary embedding with fp32 math (reference rope.py:26-85).

    ``x`` is ``[batch, num_heads, head_dim]`` (fp16 / bf16 / fp32, CUDA),
    ``positions`` ``[batch]`` int32/int64 non-negative.  Returns a new tensor
    of ``x``'s shape and dtype; dimensions at and after ``rotary_dim`` are
    copied unchanged.
    """
    if not isinstance(x, torch.Tensor) or not isinstance(positions, torch.Tensor):
        raise TypeError("x and positions must be torch tensors")
    if x.dim() != 3:
        raise ValueError("x must have shape [batch, num_heads, head_dim]")
    if positions.dim() != 1 or positions.numel() != x.shape[0]:
        raise ValueError("positions must have shape [batch]")
    if x.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise ValueError("apply_rope supports float16, bfloat16, and float32")
    if positions.dtype not in (torch.int32, torch.int64):
        raise ValueError("positions must use int32 or int64")
    if positions.device != x.device:
        raise ValueError("x and positions must be on the same device")
    if bool(torch.any(positions < 0).item()):
        raise ValueError("positions must be non-negative")
    rotary_dim, base = _check_rotary(rotary_dim, x.shape[-1], base)
    if not x.is_cuda:
        raise ValueError("flashdec_b200.apply_rope requires CUDA tensors")
    return _apply_rope_trusted(x, positions, rotary_dim, base)


def _apply_rope_trusted(x, positions, rotary_dim, base):
    """Launch the rotation for checked arguments (no value reductions)."""
    out = torch.empty_like(x)
    if x.shape[0] == 0 or x.shape[1] == 0:
        return out
    with torch.cuda.device(x.device):
        inv_freq = _native.inv_freq_device(rotary_dim, base, x.device)
        _native.rope_kv_append(x, out, None, None, None, None, None, None, positions,
                               rotary_dim, inv_freq)
    return out


def _prepare_rope_paged_kv_append_inputs(cache, request_ids, q, k, v):
    """Validate one RoPE + paged append batch (reference rope.py:86-121)."""
    from .cache import PagedKVCache

    if not isinstance(cache, PagedKVCache):
        raise TypeError("cache must be a PagedKVCache")
    ids = cache._normalize_request_ids(request_ids)
    if not ids:
        raise ValueError("request_ids must be non-empty")
    if len(set(ids)) != len(ids):
        raise ValueError("request_ids must be unique")
    if q.dim() != 3:
        raise ValueError("q must have shape [num_requests, num_q_heads, head_dim]")
    if k.dim() == 2 and len(ids) == 1:
        k = k.unsqueeze(0)
    if v.dim() == 2 and len(ids) == 1:
        v = v.unsqueeze(0)
    if k.dim() != 3 or v.dim() != 3:
        raise ValueError("k and v must have shape [num_requests, num_kv_heads, head_dim]")
    if q.shape[0] != len(ids) or q.shape[1] <= 0 or q.shape[2] != cache.head_dim:
        raise ValueError("q shape must match request count and cache head_dim")
    expected_kv_shape = (len(ids), cache.num_kv_heads, cache.head_dim)
    if k.shape != expected_kv_shape or v.shape != expected_kv_shape:
        raise ValueError("k and v shapes must match request count and cache dimensions")
    if q.device != cache.device or k.device != cache.device or v.device != cache.device:
        raise ValueError("q, k, and v must be on the cache device")
    if q.dtype != cache.dtype or k.dtype != cache.dtype or v.dtype != cache.dtype:
        raise ValueError("q, k, and v must use the cache dtype")
    return ids, k, v


def rope_paged_kv_append(cache, layer_idx, request_ids, q, k, v, rotary_dim=None,
                         base=10_000.0, append_backend="torch"):
    """Rotate Q/K and append rotated K / raw V at the allocator's next slots.

    Returns :class:`RopeAppendResult` (rotated q, positions, padded int32
    block tables, int32 sequence lengths after the append), as reference
    rope.py:124-168 does.
    """
    if append_backend not in ("torch", "cuda", "fused_cuda"):
        raise ValueError("append_backend must be 'torch', 'cuda', or 'fused_cuda'")
    ids, k, v = _prepare_rope_paged_kv_append_inputs(cache, request_ids, q, k, v)
    positions = cache.next_positions(ids, device=cache.device)
    if append_backend == "fused_cuda":
        q_rotated, block_tables = cache.append_fused_cuda(layer_idx, ids, q, k, v, positions,
                                                          rotary_dim=rotary_dim, base=base)
    else:
        q_rotated = apply_rope(q, positions, rotary_dim=rotary_dim, base=base)
        k_rotated = apply_rope(k, positions, rotary_dim=rotary_dim, base=base)
        if append_backend == "torch":
            block_tables = cache.append(layer_idx, ids, k_rotated, v)
        else:
            block_tables = cache.append_cuda(layer_idx, ids, k_rotated, v)
    seq_lens = cache.seq_lens_tensor(ids)
    return RopeAppendResult(q=q_rotated, positions=positions, block_tables=block_tables,
                            seq_lens=seq_lens)
