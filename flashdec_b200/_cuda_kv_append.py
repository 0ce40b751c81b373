"""One-token paged K/V copy (no RoPE): the reference's ``cuda_kv_append``.

Drop-in for ``flashdec/_cuda_kv_append.py`` (cysong2025/flashdec), same
validation and messages (:60-114).  It runs ``fd_rope_kv_append`` with no q
and ``rotary_dim == 0`` (a pure copy of K and V into their slots).
"""

from __future__ import annotations

import torch

from . import _lib, _native

_SUPPORTED_DTYPES = ("float16", "bfloat16", "float32")


def load_cuda_kv_append_extension():
    """Return the native library that implements the copy (no JIT build)."""
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA KV append requires torch.cuda.is_available()")
    return _lib.load_library()


def _check_cuda_tensor(name, tensor):
    if not tensor.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if not tensor.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _validate_inputs(k_cache, v_cache, block_ids, block_offsets, k, v):
    for name, tensor in [("k_cache", k_cache), ("v_cache", v_cache), ("block_ids", block_ids),
                         ("block_offsets", block_offsets), ("k", k), ("v", v)]:
        if not isinstance(tensor, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        _check_cuda_tensor(name, tensor)
    if k_cache.device != v_cache.device or k_cache.device != k.device or k_cache.device != v.device:
        raise ValueError("K/V caches and values must share one CUDA device")
    if block_ids.device != k_cache.device or block_offsets.device != k_cache.device:
        raise ValueError("block_ids and block_offsets must be on the cache CUDA device")
    if k_cache.dim() != 4:
        raise ValueError("k_cache must have shape [blocks, heads, block_size, head_dim]")
    if v_cache.shape != k_cache.shape:
        raise ValueError("v_cache must match k_cache shape")
    if k.dim() != 3 or v.dim() != 3:
        raise ValueError("k and v must have shape [batch, heads, head_dim]")
    if v.shape != k.shape:
        raise ValueError("v must match k shape")
    if k.shape[1:] != (k_cache.shape[1], k_cache.shape[3]):
        raise ValueError("k/v heads and head_dim must match cache")
    if block_ids.dim() != 1 or block_offsets.dim() != 1:
        raise ValueError("block_ids and block_offsets must be rank-1 tensors")
    if block_ids.numel() != k.shape[0] or block_offsets.numel() != k.shape[0]:
        raise ValueError("block_ids and block_offsets lengths must match batch")
    if block_ids.dtype not in (torch.int32, torch.int64):
        raise ValueError("block_ids must use int32 or int64")
    if block_offsets.dtype not in (torch.int32, torch.int64):
        raise ValueError("block_offsets must use int32 or int64")
    if k_cache.dtype != v_cache.dtype or k_cache.dtype != k.dtype or k_cache.dtype != v.dtype:
        raise ValueError("K/V caches and values must share one dtype")
    if str(k_cache.dtype).removeprefix("torch.") not in _SUPPORTED_DTYPES:
        raise ValueError("CUDA KV append supports float16, bfloat16, and float32")
    rb, ro = _native.index_ranges(block_ids, block_offsets)  # one synchronisation
    if rb is not None and (rb[0] < 0 or rb[1] >= k_cache.shape[0]):
        raise ValueError("block_ids must be within [0, num_blocks)")
    if ro is not None and (ro[0] < 0 or ro[1] >= k_cache.shape[2]):
        raise ValueError("block_offsets must be within [0, block_size)")


def cuda_kv_append(k_cache, v_cache, block_ids, block_offsets, k, v):
    """Write one K/V token per request into token-major physical cache blocks.

    ``k_cache``/``v_cache``: contiguous ``[num_blocks, num_kv_heads,
    block_size, head_dim]``; ``block_ids``/``block_offsets``: ``[batch]``;
    ``k``/``v``: ``[batch, num_kv_heads, head_dim]``.  Returns None.
    """
    _validate_inputs(k_cache, v_cache, block_ids, block_offsets, k, v)
    with torch.cuda.device(k.device):
        _native.rope_kv_append(None, None, k, v, k_cache, v_cache, block_ids, block_offsets,
                               None, 0, None)
