"""Fused RoPE + paged K/V append: the reference's public primitive on B200.

Drop-in for ``flashdec/_fused_rope_kv_append.py`` (cysong2025/flashdec):
``fused_rope_kv_append`` keeps its signature, validation order and messages
(:62-146, :210-258) and ``_fused_rope_kv_append_trusted`` its reduced checks
(:261-309).  The JIT-built extension of the reference is replaced by
``fd_rope_kv_append`` in the prebuilt ``libflashdec_b200.so``;
``load_fused_rope_kv_append_extension`` returns that library.

The RoPE table ``inv_freq`` is computed once per (rotary_dim, base) on the
host exactly as ``flashdec/rope.py:66-67`` does (fp32 torch.pow) and kept
resident per device, so the angles the kernel forms (``float(pos) *
inv_freq``) are the reference's angles bit for bit.
"""

from __future__ import annotations

import math

import torch

from . import _lib, _native


def _require_cuda():
    if not torch.cuda.is_available():
        raise RuntimeError("fused RoPE + KV append requires torch.cuda.is_available()")


def load_fused_rope_kv_append_extension():
    """Return the native library that implements the primitive (no JIT build)."""
    _require_cuda()
    return _lib.load_library()


def _check_cuda_contiguous_tensor(name, tensor):
    if not tensor.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if not tensor.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _validate_structure(q, k, v, k_cache, v_cache, block_ids, block_offsets, positions,
                        rotary_dim, base):
    for name, tensor in [
        ("q", q), ("k", k), ("v", v), ("k_cache", k_cache), ("v_cache", v_cache),
        ("block_ids", block_ids), ("block_offsets", block_offsets), ("positions", positions),
    ]:
        if not isinstance(tensor, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        _check_cuda_contiguous_tensor(name, tensor)

    if q.dim() != 3 or k.dim() != 3 or v.dim() != 3:
        raise ValueError("q, k, and v must have shape [batch, heads, head_dim]")
    if q.shape[1] <= 0 or k.shape[1] <= 0:
        raise ValueError("q and k must have at least one head")
    if v.shape != k.shape:
        raise ValueError("v must match k shape")
    if k_cache.dim() != 4 or v_cache.shape != k_cache.shape:
        raise ValueError("K/V caches must match shape [blocks, kv_heads, block_size, head_dim]")
    if q.shape[0] != k.shape[0] or q.shape[2] != k.shape[2]:
        raise ValueError("q batch and head_dim must match k/v")
    if k.shape[1] != k_cache.shape[1] or k.shape[2] != k_cache.shape[3]:
        raise ValueError("k/v heads and head_dim must match cache")
    if block_ids.dim() != 1 or block_offsets.dim() != 1 or positions.dim() != 1:
        raise ValueError("block_ids, block_offsets, and positions must be rank-1 tensors")
    if block_ids.numel() != q.shape[0] or block_offsets.numel() != q.shape[0]:
        raise ValueError("block_ids and block_offsets lengths must match batch")
    if positions.numel() != q.shape[0]:
        raise ValueError("positions length must match batch")
    if any(t.dtype not in (torch.int32, torch.int64) for t in (block_ids, block_offsets, positions)):
        raise ValueError("block_ids, block_offsets, and positions must use int32 or int64")
    if any(t.device != q.device for t in (k, v, k_cache, v_cache, block_ids, block_offsets, positions)):
        raise ValueError("all fused RoPE + KV append inputs must share one CUDA device")
    if any(t.dtype != q.dtype for t in (k, v, k_cache, v_cache)):
        raise ValueError("q, k, v, and K/V caches must share one dtype")
    if q.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise ValueError("fused RoPE + KV append supports float16, bfloat16, and float32")

    head_dim = q.shape[-1]
    if isinstance(rotary_dim, bool) or not isinstance(rotary_dim, int):
        raise ValueError("rotary_dim must be an even integer")
    if rotary_dim <= 0 or rotary_dim > head_dim or rotary_dim % 2 != 0:
        raise ValueError("rotary_dim must be positive, even, and no larger than head_dim")
    base = float(base)
    if not math.isfinite(base) or base <= 0.0:
        raise ValueError("base must be a positive finite number")
    return base


def _validate_index_values(block_ids, block_offsets, positions, num_blocks, block_size):
    """Value checks of caller-owned indices (reference :128-146): the same
    checks in the same order, evaluated with one host synchronisation."""
    rb, ro, rp = _native.index_ranges(block_ids, block_offsets, positions)
    if rb is not None and (rb[0] < 0 or rb[1] >= num_blocks):
        raise ValueError("block_ids must be within [0, num_blocks)")
    if ro is not None and (ro[0] < 0 or ro[1] >= block_size):
        raise ValueError("block_offsets must be within [0, block_size)")
    if rp is not None and rp[0] < 0:
        raise ValueError("positions must be non-negative")


def _launch_fused_rope_kv_append(q, k, v, k_cache, v_cache, block_ids, block_offsets, positions,
                                 rotary_dim, base, q_out=None):
    if q_out is None:
        q_out = torch.empty_like(q)
    with torch.cuda.device(q.device):
        inv_freq = _native.inv_freq_device(rotary_dim, base, q.device)
        _native.rope_kv_append(q, q_out, k, v, k_cache, v_cache, block_ids, block_offsets,
                               positions, rotary_dim, inv_freq)
    return q_out


def _prepare_fused_rope_kv_append(q, k, v, k_cache, v_cache, block_ids, block_offsets,
                                  positions, rotary_dim, base):
    if rotary_dim is None:
        if not isinstance(q, torch.Tensor):
            raise TypeError("q must be a torch.Tensor")
        rotary_dim = q.shape[-1]
    base = _validate_structure(q, k, v, k_cache, v_cache, block_ids, block_offsets, positions,
                               rotary_dim, base)
    return rotary_dim, base


def fused_rope_kv_append(q, k, v, k_cache, v_cache, block_ids, block_offsets, positions,
                         rotary_dim=None, base=10_000.0):
    """Rotate Q/K and append rotated K / raw V through one kernel.

    The caller supplies already allocated physical ``block_ids`` and offsets.
    Returns the rotated Q (same shape/dtype as ``q``); the K/V cache writes
    happen in place.  Request/allocator state is not touched.
    """
    rotary_dim, base = _prepare_fused_rope_kv_append(
        q, k, v, k_cache, v_cache, block_ids, block_offsets, positions, rotary_dim, base
    )
    _validate_index_values(block_ids, block_offsets, positions, k_cache.shape[0],
                           k_cache.shape[2])
    return _launch_fused_rope_kv_append(q, k, v, k_cache, v_cache, block_ids, block_offsets,
                                        positions, rotary_dim, base)


def _fused_rope_kv_append_trusted(q, k, v, k_cache, v_cache, block_ids, block_offsets,
                                  positions, rotary_dim=None, base=10_000.0, q_out=None):
    """Launch with cache-owned transaction metadata (no device value reductions).

    Private: ``PagedKVCache`` uses it only for the current open transaction,
    whose block ids, offsets and positions were proven on the host.  Shape,
    dtype, device, contiguity and RoPE argument checks stay enabled; the
    metadata must be int64 (reference :261-309).
    """
    rotary_dim, base = _prepare_fused_rope_kv_append(
        q, k, v, k_cache, v_cache, block_ids, block_offsets, positions, rotary_dim, base
    )
    if any(t.dtype != torch.int64 for t in (block_ids, block_offsets, positions)):
        raise ValueError("trusted transaction metadata must use int64")
    return _launch_fused_rope_kv_append(q, k, v, k_cache, v_cache, block_ids, block_offsets,
                                        positions, rotary_dim, base, q_out=q_out)
