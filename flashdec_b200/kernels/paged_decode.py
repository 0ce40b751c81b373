"""Paged single-token decode attention on B200: the reference's public API.

Drop-in for ``flashdec/kernels/paged_decode.py`` of cysong2025/flashdec:
same function names, signatures, defaults, shape/dtype contract and
``ValueError`` messages (``_validate_inputs`` :645-725, ``_into`` :1020-1096).
The Triton kernels are replaced by one launch of ``fd_paged_decode`` (and,
for an explicit reference-style split workspace, ``fd_split_kv_reduce``) from
``libflashdec_b200.so``.

Differences that are deliberate (numerics agree within the tolerances the
reference's tests use):

* ``num_warps`` / ``num_stages`` are validated exactly as before but are
  tuning hints of the Triton kernels; the sm_100a kernel ignores them.
* with the default ``num_splits=1`` the reference runs one program per
  (sequence, KV head) -- 16 CTAs at B8/Hkv2.  Here the default is the
  length-balanced schedule over all SMs with the split merge inside the
  kernel; an explicit ``split_kv_workspace`` + ``num_splits > 1`` keeps the
  reference's fixed split (S chunks per sequence, partials written to the
  caller's workspace, then the reducer).
"""

from __future__ import annotations

import ctypes
import math

import torch

from .. import _lib, _native

_KV_LAYOUT_AXES = {
    "token_major": (2, 3),
    "dim_major": (3, 2),
}


# Prepared launches of the common call (no split workspace, no fused append),
# keyed by everything the checks and the launch arguments depend on: shapes,
# strides, dtypes and devices of every tensor plus the scalar arguments.  A
# signature that passed the full checks once passes them again, so a hit only
# sets the data pointers and launches.
_PREPARED: dict = {}
_PREPARED_LIMIT = 256


def _signature(q, k_cache, v_cache, block_tables, seq_lens, out, sm_scale, block_size, num_warps,
               kv_layout, num_stages):
    return (q.shape, q.stride(), q.dtype, q.device,
            k_cache.shape, k_cache.stride(), k_cache.dtype, k_cache.device,
            v_cache.shape, v_cache.stride(), v_cache.dtype, v_cache.device,
            block_tables.shape, block_tables.stride(), block_tables.dtype, block_tables.device,
            seq_lens.shape, seq_lens.stride(), seq_lens.dtype, seq_lens.device,
            out.shape, out.stride(), out.dtype, out.device,
            sm_scale, block_size, num_warps, kv_layout, num_stages)


def _launch_prepared(prep, q, k_cache, v_cache, block_tables, seq_lens, out):
    dev = q.device
    if torch.cuda.current_device() == dev.index:
        prep.launch(q, k_cache, v_cache, block_tables, seq_lens, out, _native.stream_handle(dev))
    else:
        with torch.cuda.device(dev):
            prep.launch(q, k_cache, v_cache, block_tables, seq_lens, out,
                        _native.stream_handle(dev))


_FAST = None  # (C++ decode_into, its miss code), bound on first use


def _fast_entry():
    global _FAST
    hp = _lib.load_hostpath()
    _FAST = (hp.decode_into, hp.MISS)
    return _FAST


# prepared vLLM launches registered with the C++ host path (kept alive with
# the per-stream workspaces their structs point at)
_VLLM_PREPARED: list = []
_VLLM_FAST = None


def _vllm_fast_entry():
    global _VLLM_FAST
    hp = _lib.load_hostpath()
    _VLLM_FAST = (hp.vllm_into, hp.MISS)
    return _VLLM_FAST


def _register(prep, q, k_cache, v_cache, block_tables, seq_lens, out):
    """Hand the struct that just launched (bound to the current stream's
    workspace, which ``prep`` keeps alive while it is in ``_PREPARED``) to
    the C++ host path under this call's signature."""
    with prep.lock:
        _lib.load_hostpath().register_decode(q, k_cache, v_cache, block_tables, seq_lens, out,
                                             ctypes.addressof(prep.args))


def _layout_axes(kv_layout):
    try:
        return _KV_LAYOUT_AXES[kv_layout]
    except KeyError as exc:
        raise ValueError("kv_layout must be 'token_major' or 'dim_major'") from exc


def _logical_view(cache, kv_layout):
    """[block, kv_head, token, dim] view of a 4-D cache (no copy)."""
    return cache if kv_layout == "token_major" else cache.permute(0, 1, 3, 2)


def _validate_inputs(q, k_cache, v_cache, block_tables, seq_lens, block_size, num_warps,
                     num_stages, kv_layout):
    """Shape/dtype/device contract of the reference (paged_decode.py:645-725)."""
    token_axis, dim_axis = _layout_axes(kv_layout)
    if q.device.type != "cuda" or k_cache.device.type != "cuda" or v_cache.device.type != "cuda":
        raise ValueError("q, k_cache, and v_cache must be CUDA tensors")
    if block_tables.device.type != "cuda" or seq_lens.device.type != "cuda":
        raise ValueError("block_tables and seq_lens must be CUDA tensors")
    if (
        q.device != k_cache.device
        or q.device != v_cache.device
        or q.device != block_tables.device
        or q.device != seq_lens.device
    ):
        raise ValueError(
            "q, k_cache, v_cache, block_tables, and seq_lens must be on the same CUDA device"
        )
    if q.dim() != 3:
        raise ValueError("q must have shape [num_seqs, num_q_heads, head_dim]")
    if k_cache.dim() != 4 or v_cache.dim() != 4:
        raise ValueError("k_cache and v_cache must be 4D tensors")
    if block_tables.dim() != 2:
        raise ValueError("block_tables must have shape [num_seqs, max_blocks_per_seq]")
    if seq_lens.dim() != 1:
        raise ValueError("seq_lens must have shape [num_seqs]")
    if q.dtype != k_cache.dtype or q.dtype != v_cache.dtype:
        raise ValueError("q, k_cache, and v_cache must have the same dtype")
    if q.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("paged_decode_attention currently supports float16 and bfloat16 tensors")
    if block_tables.dtype not in (torch.int32, torch.int64):
        raise ValueError("block_tables must be int32 or int64")
    if seq_lens.dtype not in (torch.int32, torch.int64):
        raise ValueError("seq_lens must be int32 or int64")

    num_seqs, num_q_heads, head_dim = q.shape
    num_blocks, num_kv_heads = k_cache.shape[:2]
    v_num_blocks, v_num_kv_heads = v_cache.shape[:2]
    cache_block_size = k_cache.shape[token_axis]
    k_head_dim = k_cache.shape[dim_axis]
    v_block_size = v_cache.shape[token_axis]
    v_head_dim = v_cache.shape[dim_axis]
    if block_tables.shape[0] != num_seqs or seq_lens.numel() != num_seqs:
        raise ValueError("block_tables and seq_lens must have one row/value per sequence")
    if v_num_blocks != num_blocks:
        raise ValueError("k_cache and v_cache must have the same num_blocks")
    if num_blocks <= 0:
        raise ValueError("num_blocks must be positive")
    if num_seqs <= 0:
        raise ValueError("num_seqs must be positive")
    if num_q_heads <= 0 or num_kv_heads <= 0:
        raise ValueError("num_q_heads and num_kv_heads must be positive")
    if block_tables.shape[1] <= 0:
        raise ValueError("max_blocks_per_seq must be positive")
    if v_num_kv_heads != num_kv_heads:
        raise ValueError("k_cache and v_cache must have the same num_kv_heads")
    if v_block_size != cache_block_size:
        raise ValueError("k_cache and v_cache must have the same block_size")
    if cache_block_size != block_size:
        raise ValueError("block_size must match k_cache/v_cache shape")
    if block_size not in (8, 16, 32):
        raise ValueError("paged_decode_attention currently supports block_size 8, 16, or 32")
    if k_head_dim != head_dim or v_head_dim != head_dim:
        raise ValueError("q, k_cache, and v_cache must have the same head_dim")
    if head_dim not in (64, 128):
        raise ValueError("paged_decode_attention currently supports head_dim 64 or 128")
    if num_q_heads % num_kv_heads != 0:
        raise ValueError("num_q_heads must be divisible by num_kv_heads")
    if isinstance(num_warps, bool) or not isinstance(num_warps, int) or num_warps not in (1, 2, 4, 8):
        raise ValueError("num_warps must be one of 1, 2, 4, or 8")
    if num_stages is not None and (
        isinstance(num_stages, bool)
        or not isinstance(num_stages, int)
        or num_stages not in (1, 2, 3, 4)
    ):
        raise ValueError("num_stages must be None or one of 1, 2, 3, or 4")


def paged_decode_attention(
    q,
    k_cache,
    v_cache,
    block_tables,
    seq_lens,
    sm_scale=None,
    block_size=None,
    num_warps=2,
    kv_layout="token_major",
    num_stages=None,
):
    """Return paged single-token decode attention (``flashdec.decode``).

    Shapes:
    - q: [num_seqs, num_q_heads, head_dim]
    - token_major k_cache/v_cache: [num_blocks, num_kv_heads, block_size, head_dim]
    - dim_major k_cache/v_cache: [num_blocks, num_kv_heads, head_dim, block_size]
    - block_tables: [num_seqs, max_blocks_per_seq] (int32/int64)
    - seq_lens: [num_seqs] (int32/int64)
    - return: [num_seqs, num_q_heads, head_dim]

    Mirrors reference paged_decode.py:922-969 (block_size inferred from the
    cache when omitted; output allocated with ``torch.empty_like(q)``).
    """
    token_axis, _ = _layout_axes(kv_layout)
    if block_size is None:
        if k_cache.dim() != 4:
            raise ValueError("k_cache must be a 4D tensor")
        block_size = k_cache.shape[token_axis]
    else:
        block_size = int(block_size)
    out = torch.empty_like(q)
    return paged_decode_attention_into(
        q, k_cache, v_cache, block_tables, seq_lens, out,
        sm_scale=sm_scale, block_size=block_size, num_warps=num_warps,
        kv_layout=kv_layout, num_stages=num_stages,
    )


def paged_decode_attention_into(
    q,
    k_cache,
    v_cache,
    block_tables,
    seq_lens,
    out,
    sm_scale=None,
    block_size=None,
    num_warps=2,
    kv_layout="token_major",
    num_stages=None,
    split_kv_workspace=None,
    num_splits=1,
    append_k=None,
    append_v=None,
    slot_mapping=None,
):
    """Write paged single-token decode attention into ``out`` and return it.

    Mirrors reference paged_decode.py:972-1264: no output allocation; K/V,
    block tables, seq_lens and out may be strided views (strides go to the
    kernel, nothing cache-sized is copied).  ``append_k``/``append_v``/
    ``slot_mapping`` (together) fuse the current token's K/V store into the
    attention launch; rows with ``slot_mapping < 0`` get a zero output and no
    store.
    """
    # The call with every scalar at its default goes to the C++ host path
    # first: a signature it has seen on this stream launches there.
    # (the chained identities hold only when all seven are None)
    default_call = (sm_scale is block_size is num_stages is split_kv_workspace is append_k
                    is append_v is slot_mapping is None
                    and num_warps.__class__ is int and num_warps == 2
                    and num_splits.__class__ is int and num_splits == 1
                    and kv_layout == "token_major")
    if default_call:
        decode_into, miss = _FAST or _fast_entry()
        try:
            rc = decode_into(q, k_cache, v_cache, block_tables, seq_lens, out)
        except TypeError:  # not tensors: the checks below raise the reference's errors
            rc = miss
        if rc == 0:
            return out
        if rc < 0:
            _lib.check(rc, "fd_paged_decode")
    key = None
    if (split_kv_workspace is None and type(num_splits) is int and num_splits == 1
            and append_k is None and append_v is None and slot_mapping is None):
        try:
            key = _signature(q, k_cache, v_cache, block_tables, seq_lens, out, sm_scale,
                             block_size, num_warps, kv_layout, num_stages)
            hash(key)
        except (AttributeError, TypeError):
            key = None
        if key is not None:
            prep = _PREPARED.get(key)
            if prep is not None:
                _launch_prepared(prep, q, k_cache, v_cache, block_tables, seq_lens, out)
                if default_call:
                    _register(prep, q, k_cache, v_cache, block_tables, seq_lens, out)
                return out

    token_axis, _ = _layout_axes(kv_layout)
    if block_size is None:
        if k_cache.dim() != 4:
            raise ValueError("k_cache must be a 4D tensor")
        block_size = k_cache.shape[token_axis]
    else:
        block_size = int(block_size)

    _validate_inputs(q, k_cache, v_cache, block_tables, seq_lens, block_size, num_warps,
                     num_stages, kv_layout)
    if out.shape != q.shape:
        raise ValueError("out must have the same shape as q")
    if out.dtype != q.dtype:
        raise ValueError("out must have the same dtype as q")
    if out.device != q.device:
        raise ValueError("out must be on the same device as q")
    if isinstance(num_splits, bool) or not isinstance(num_splits, int) or num_splits <= 0:
        raise ValueError("num_splits must be a positive integer")

    num_seqs, num_q_heads, head_dim = q.shape
    _, num_kv_heads = k_cache.shape[:2]
    group_size = num_q_heads // num_kv_heads
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(head_dim)

    use_grouped_gqa = head_dim == 128 and group_size in (4, 8, 16) and block_size in (16, 32)
    append_values = (append_k, append_v, slot_mapping)
    fuse_kv_append = all(value is not None for value in append_values)
    if any(value is not None for value in append_values) and not fuse_kv_append:
        raise ValueError("append_k, append_v, and slot_mapping must be provided together")
    if fuse_kv_append:
        if not use_grouped_gqa:
            raise ValueError("fused KV append requires grouped GQA decode")
        expected_append_shape = (num_seqs, num_kv_heads, head_dim)
        if append_k.shape != expected_append_shape or append_v.shape != expected_append_shape:
            raise ValueError(
                "append_k and append_v must have shape [num_seqs, num_kv_heads, head_dim]"
            )
        if append_k.dtype != q.dtype or append_v.dtype != q.dtype:
            raise ValueError("append_k and append_v must match q.dtype")
        if append_k.device != q.device or append_v.device != q.device:
            raise ValueError("append_k and append_v must be on q.device")
        if slot_mapping.dim() != 1 or slot_mapping.numel() < num_seqs:
            raise ValueError("slot_mapping must have at least one entry per sequence")
        if slot_mapping.dtype not in (torch.int32, torch.int64):
            raise ValueError("slot_mapping must be int32 or int64")
        if slot_mapping.device != q.device:
            raise ValueError("slot_mapping must be on q.device")

    k4 = _logical_view(k_cache, kv_layout)
    v4 = _logical_view(v_cache, kv_layout)
    fused = dict(append_k=append_k, append_v=append_v, slot_mapping=slot_mapping) \
        if fuse_kv_append else {}
    with torch.cuda.device(q.device):
        if use_grouped_gqa and num_splits > 1:
            if split_kv_workspace is None or len(split_kv_workspace) != 3:
                raise ValueError("split_kv_workspace must contain acc, max, and sum tensors")
            split_acc, split_max, split_sum = split_kv_workspace
            expected_acc = (num_seqs, num_q_heads, num_splits, head_dim)
            expected_stats = (num_seqs, num_q_heads, num_splits)
            if split_acc.dim() != 4 or split_max.dim() != 3 or split_sum.dim() != 3:
                raise ValueError("split KV workspace ranks must be 4, 3, and 3")
            if any(t.device != q.device or t.dtype != torch.float32 for t in split_kv_workspace):
                raise ValueError("split KV workspace tensors must be float32 on q.device")
            if any(a < e for a, e in zip(split_acc.shape, expected_acc)):
                raise ValueError("split acc workspace is too small")
            if any(a < e for a, e in zip(split_max.shape, expected_stats)):
                raise ValueError("split max workspace is too small")
            if any(a < e for a, e in zip(split_sum.shape, expected_stats)):
                raise ValueError("split sum workspace is too small")
            if split_sum.stride() != split_max.stride():
                raise ValueError("split max and sum workspaces must have identical strides")
            acc = split_acc[:num_seqs, :num_q_heads, :num_splits, :head_dim]
            mx = split_max[:num_seqs, :num_q_heads, :num_splits]
            sm = split_sum[:num_seqs, :num_q_heads, :num_splits]
            _native.paged_decode(
                q, k4, v4, block_tables, seq_lens, out, sm_scale=sm_scale,
                block_size=block_size, num_seqs=num_seqs, num_splits=num_splits,
                epilogue=_lib.FD_EPILOGUE_PARTIALS, partials=(acc, mx, sm), **fused,
            )
            _native.split_kv_reduce(acc, mx, sm, seq_lens, out, num_seqs=num_seqs,
                                    slot_mapping=slot_mapping if fuse_kv_append else None)
            return out
        if key is not None:
            prep = _native.prepare_paged_decode(
                q, k4, v4, block_tables, seq_lens, out, sm_scale=sm_scale,
                block_size=block_size, num_seqs=num_seqs, num_splits=0)
            if len(_PREPARED) >= _PREPARED_LIMIT:
                _PREPARED.clear()
                _lib.load_hostpath().clear()  # its entries use the dropped workspaces
            _PREPARED[key] = prep
            prep.launch(q, k_cache, v_cache, block_tables, seq_lens, out,
                        _native.stream_handle(q.device))
            if default_call:
                _register(prep, q, k_cache, v_cache, block_tables, seq_lens, out)
            return out
        _native.paged_decode(
            q, k4, v4, block_tables, seq_lens, out, sm_scale=sm_scale,
            block_size=block_size, num_seqs=num_seqs, num_splits=0, **fused,
        )
    return out


def _vllm_paged_decode_attention_into(
    q,
    append_k,
    append_v,
    kv_cache,
    block_tables,
    seq_lens,
    out,
    slot_mapping,
    split_acc,
    split_max,
    split_sum,
    *,
    num_reqs,
    num_q_heads,
    num_kv_heads,
    head_dim,
    block_size,
    sm_scale,
    num_splits,
):
    """Checked-by-caller vLLM decode launcher (reference paged_decode.py:728-919).

    No validation, allocation, slicing of caller tensors or copies, so it is
    CUDA-graph capturable once the per-device workspace is sized.
    ``kv_cache`` is vLLM's complete ``[block, 2, token, kv_head, dim]``
    allocation (NHD or an HND-permuted view); K is plane 0, V plane 1.
    ``num_reqs`` may include CUDA-graph padding rows, which carry
    ``slot_mapping == -1`` and get zero output; tensor rows beyond
    ``num_reqs`` are not touched.

    ``num_splits``: 0 selects the length-balanced in-kernel-merge schedule;
    1 one CTA per (request, KV head); S >= 2 the reference's fixed split
    using vLLM's ``softmax_segm_*`` buffers as the split workspace, followed
    by the reducer (``MASK_INVALID_SLOT`` semantics).
    """
    # the auto plan (num_splits 0, vLLM's default here) goes to the C++ host
    # path first: a signature it has seen on this stream only sets pointers
    if num_splits == 0:
        decode, miss = _VLLM_FAST or _vllm_fast_entry()
        try:
            rc = decode(q, append_k, append_v, kv_cache, block_tables, seq_lens, out,
                        slot_mapping, num_reqs, num_q_heads, num_kv_heads, head_dim,
                        block_size, float(sm_scale))
        except TypeError:
            rc = miss
        if rc == 0:
            return out
        if rc < 0:
            _lib.check(rc, "fd_paged_decode")
    k4 = kv_cache[:, 0].permute(0, 2, 1, 3)
    v4 = kv_cache[:, 1].permute(0, 2, 1, 3)
    fused = dict(append_k=append_k, append_v=append_v, slot_mapping=slot_mapping)
    if num_splits == 0:
        prep = _native.prepare_paged_decode(
            q, k4, v4, block_tables, seq_lens, out, sm_scale=sm_scale, block_size=block_size,
            num_seqs=num_reqs, num_splits=0, **fused)
        prep.launch(q, k4, v4, block_tables, seq_lens, out, _native.stream_handle(q.device))
        hp = _lib.load_hostpath()
        if len(_VLLM_PREPARED) >= _PREPARED_LIMIT:
            _VLLM_PREPARED.clear()
            hp.clear_vllm()  # its entries use the dropped workspaces
        if hp.register_vllm(q, append_k, append_v, kv_cache, block_tables, seq_lens, out,
                            slot_mapping, num_reqs, num_q_heads, num_kv_heads, head_dim,
                            block_size, float(sm_scale), ctypes.addressof(prep.args)):
            _VLLM_PREPARED.append(prep)
        return out
    if num_splits >= 2:
        acc = split_acc[:, :, :num_splits, :]
        mx = split_max[:, :, :num_splits]
        sm = split_sum[:, :, :num_splits]
        _native.paged_decode(
            q, k4, v4, block_tables, seq_lens, out, sm_scale=sm_scale, block_size=block_size,
            num_seqs=num_reqs, num_splits=num_splits, epilogue=_lib.FD_EPILOGUE_PARTIALS,
            partials=(acc, mx, sm), **fused,
        )
        _native.split_kv_reduce(acc, mx, sm, seq_lens, out, num_seqs=num_reqs,
                                slot_mapping=slot_mapping)
        return out
    _native.paged_decode(
        q, k4, v4, block_tables, seq_lens, out, sm_scale=sm_scale, block_size=block_size,
        num_seqs=num_reqs, num_splits=int(num_splits), **fused,
    )
    return out
