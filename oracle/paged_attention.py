"""numpy restatement of FlashDec's paged decode attention oracle.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

All arrays are numpy.  Floating inputs are float32 arrays whose values are
exactly representable in the logical dtype (bf16 / fp16 / fp32); the logical
dtype is passed as a string and only controls the final output rounding, as
``.to(out.dtype)`` does in the reference.
"""

from __future__ import annotations

import math

import numpy as np

from .numerics import round_to_dtype

# flashdec/paged_reference.py:6-9 -- (token_axis, dim_axis) of a 4-D cache.
_KV_LAYOUT_AXES = {"token_major": (2, 3), "dim_major": (3, 2)}


def _layout_axes(kv_layout):
    try:
        return _KV_LAYOUT_AXES[kv_layout]
    except KeyError as exc:  # flashdec/paged_reference.py:12-16
        raise ValueError("kv_layout must be 'token_major' or 'dim_major'") from exc


def paged_decode_attention_ref(
    q,
    k_cache,
    v_cache,
    block_tables,
    seq_lens,
    sm_scale=None,
    kv_layout="token_major",
    dtype="float32",
):
    """Single-token decode attention over a paged KV cache.

    Follows ``flashdec/paged_reference.py:19-125``:

    * shapes / validation: :39-84 (``ValueError`` with the same messages);
    * ``sm_scale`` defaults to ``head_dim ** -0.5`` (:86-87);
    * zero-length rows produce zeros (:93-95);
    * only the first ``ceil(seq_len / block_size)`` block-table entries are
      read and must be valid physical ids (:97-100);
    * blocks are gathered, laid out token-major and sliced to ``seq_len``
      (:102-112);
    * per query head: fp32 ``scores = k @ q * sm_scale``, max-subtracted
      softmax, ``probs @ v`` and a cast to ``dtype`` (:114-123);
    * query head ``h`` reads KV head ``h // (num_q_heads // num_kv_heads)``.

    Returns a float32 array ``[num_seqs, num_q_heads, head_dim]`` rounded to
    ``dtype``.
    """
    token_axis, dim_axis = _layout_axes(kv_layout)
    q = np.asarray(q, dtype=np.float32)
    k_cache = np.asarray(k_cache, dtype=np.float32)
    v_cache = np.asarray(v_cache, dtype=np.float32)
    block_tables = np.asarray(block_tables)
    seq_lens = np.asarray(seq_lens)
    if q.ndim != 3:
        raise ValueError("q must have shape [num_seqs, num_q_heads, head_dim]")
    if k_cache.ndim != 4 or v_cache.ndim != 4:
        raise ValueError("k_cache and v_cache must be 4D tensors")
    if block_tables.ndim != 2:
        raise ValueError("block_tables must have shape [num_seqs, max_blocks_per_seq]")
    if seq_lens.ndim != 1:
        raise ValueError("seq_lens must be a 1D tensor")
    if not np.issubdtype(block_tables.dtype, np.integer):
        raise ValueError("block_tables must contain integer physical block ids")

    num_seqs, num_q_heads, head_dim = q.shape
    num_blocks, num_kv_heads = k_cache.shape[:2]
    block_size = k_cache.shape[token_axis]
    if v_cache.shape[:2] != (num_blocks, num_kv_heads):
        raise ValueError("k_cache and v_cache must have the same num_blocks")
    if v_cache.shape[token_axis] != block_size:
        raise ValueError("k_cache and v_cache must have the same block_size")
    if k_cache.shape[dim_axis] != head_dim or v_cache.shape[dim_axis] != head_dim:
        raise ValueError("q, k_cache, and v_cache must have the same head_dim")
    if block_tables.shape[0] != num_seqs or seq_lens.size != num_seqs:
        raise ValueError("block_tables and seq_lens must have one row/value per sequence")
    if num_q_heads % num_kv_heads != 0:
        raise ValueError("num_q_heads must be divisible by num_kv_heads")
    max_seq_len = block_tables.shape[1] * block_size
    lens = [int(x) for x in seq_lens.tolist()]
    if any(n < 0 or n > max_seq_len for n in lens):
        raise ValueError("seq_lens values must be in [0, max_blocks_per_seq * block_size]")

    if sm_scale is None:
        sm_scale = head_dim ** -0.5
    scale = np.float32(sm_scale)
    group = num_q_heads // num_kv_heads
    out = np.zeros((num_seqs, num_q_heads, head_dim), dtype=np.float32)

    if kv_layout == "token_major":
        k_tm, v_tm = k_cache, v_cache
    else:  # dim_major [NB, Hkv, D, bs] -> token-major view
        k_tm = np.swapaxes(k_cache, 2, 3)
        v_tm = np.swapaxes(v_cache, 2, 3)

    for s, n in enumerate(lens):
        if n == 0:
            continue
        nblk = (n + block_size - 1) // block_size
        ids = [int(x) for x in block_tables[s, :nblk].tolist()]
        if any(b < 0 or b >= num_blocks for b in ids):
            raise ValueError(
                "block_tables contains invalid physical block ids for a non-empty sequence"
            )
        # [nblk, Hkv, bs, D] -> [nblk*bs, Hkv, D] -> first n tokens
        k_seq = k_tm[ids].transpose(0, 2, 1, 3).reshape(-1, num_kv_heads, head_dim)[:n]
        v_seq = v_tm[ids].transpose(0, 2, 1, 3).reshape(-1, num_kv_heads, head_dim)[:n]
        for h in range(num_q_heads):
            kvh = h // group
            k = k_seq[:, kvh]
            v = v_seq[:, kvh]
            scores = (k @ q[s, h]) * scale
            scores = scores - np.max(scores)
            probs = np.exp(scores)
            probs = probs / np.sum(probs)
            out[s, h] = probs @ v
    return round_to_dtype(out, dtype)


def apply_fused_append_ref(
    k_cache, v_cache, append_k, append_v, slot_mapping, seq_lens, block_size
):
    """Cache writes of the fused current-token append (token-major cache).

    Follows ``flashdec/kernels/paged_decode.py:193-221``: for every row with
    ``slot >= 0`` and ``seq_len > 0`` the token's K/V are stored at
    ``(slot // block_size, :, slot % block_size, :)``; other rows write
    nothing.  Returns new (k_cache, v_cache) arrays.
    """
    k_out = np.array(k_cache, dtype=np.float32, copy=True)
    v_out = np.array(v_cache, dtype=np.float32, copy=True)
    for row, (slot, n) in enumerate(zip(np.asarray(slot_mapping).tolist(), np.asarray(seq_lens).tolist())):
        if slot < 0 or n <= 0:
            continue
        blk, off = slot // block_size, slot % block_size
        k_out[blk, :, off, :] = append_k[row]
        v_out[blk, :, off, :] = append_v[row]
    return k_out, v_out


def paged_decode_with_append_ref(
    q,
    k_cache,
    v_cache,
    block_tables,
    seq_lens,
    append_k,
    append_v,
    slot_mapping,
    sm_scale=None,
    dtype="float32",
):
    """Fused current-token append + decode (token-major cache).

    The reference fuses the store of the current token into the attention
    kernel (``flashdec/kernels/paged_decode.py:193-257`` and the split variant
    :400-476) and masks rows whose slot is negative
    (``MASK_INVALID_SLOT``, :586-591).  Semantically that equals: write the
    token, run :func:`paged_decode_attention_ref`, and zero the output rows
    with ``slot < 0``.  Returns ``(out, k_cache_after, v_cache_after)``.
    """
    block_size = np.asarray(k_cache).shape[2]
    k_after, v_after = apply_fused_append_ref(
        k_cache, v_cache, append_k, append_v, slot_mapping, seq_lens, block_size
    )
    out = paged_decode_attention_ref(
        q, k_after, v_after, block_tables, seq_lens, sm_scale=sm_scale, dtype=dtype
    )
    for row, slot in enumerate(np.asarray(slot_mapping).tolist()[: out.shape[0]]):
        if slot < 0:
            out[row] = 0.0
    return out, k_after, v_after


def split_partials_ref(q, k_cache, v_cache, block_tables, seq_lens, num_splits,
                       sm_scale=None, token_block=32):
    """Split-KV partial triples ``(acc, max, sum)`` per (seq, q head, split).

    Follows the partition of ``flashdec/kernels/paged_decode.py:395-411``:
    the ``cdiv(seq_len, TOKEN_BLOCK)`` token blocks are cut into
    ``num_splits`` chunks of ``cdiv(blocks, num_splits)`` blocks; split ``s``
    covers token blocks ``[s*bps, min((s+1)*bps, blocks))``.  Each split keeps
    an un-normalised accumulator, its running max (natural-log domain) and its
    exp-sum (:528-543).  Empty splits hold ``(0, -inf, 0)``.
    Token-major cache only.  fp32 math throughout.
    """
    q = np.asarray(q, dtype=np.float32)
    num_seqs, num_q_heads, head_dim = q.shape
    num_kv_heads = k_cache.shape[1]
    block_size = k_cache.shape[2]
    group = num_q_heads // num_kv_heads
    scale = np.float32(head_dim ** -0.5 if sm_scale is None else sm_scale)
    acc = np.zeros((num_seqs, num_q_heads, num_splits, head_dim), np.float32)
    mx = np.full((num_seqs, num_q_heads, num_splits), -np.inf, np.float32)
    sm = np.zeros((num_seqs, num_q_heads, num_splits), np.float32)
    for s in range(num_seqs):
        n = int(seq_lens[s])
        nblocks = -(-n // token_block)
        bps = -(-nblocks // num_splits)
        for sp in range(num_splits):
            t0 = sp * bps * token_block
            t1 = min((sp + 1) * bps, nblocks) * token_block
            t1 = min(t1, n)
            if t1 <= t0:
                continue
            toks = np.arange(t0, t1)
            blk = np.asarray(block_tables)[s, toks // block_size]
            off = toks % block_size
            for h in range(num_q_heads):
                kvh = h // group
                k = k_cache[blk, kvh, off]
                v = v_cache[blk, kvh, off]
                sc = (k @ q[s, h]) * scale
                m = np.max(sc)
                p = np.exp(sc - m)
                acc[s, h, sp] = p @ v
                mx[s, h, sp] = m
                sm[s, h, sp] = np.sum(p)
    return acc, mx, sm


def merge_split_partials(acc, mx, sm, seq_lens, slot_mapping=None, dtype="float32"):
    """The split-KV query-head reducer.

    Follows ``flashdec/kernels/paged_decode.py:546-642``: ``gmax = max_s m_s``;
    ``w_s = exp(m_s - gmax)``; ``out = sum_s w_s acc_s / sum_s w_s l_s``.
    Rows with ``seq_len == 0`` -- or, when ``slot_mapping`` is given
    (``MASK_INVALID_SLOT``), ``slot < 0`` -- produce zeros.
    """
    acc = np.asarray(acc, np.float32)
    mx = np.asarray(mx, np.float32)
    sm = np.asarray(sm, np.float32)
    num_seqs, num_heads, _, head_dim = acc.shape
    out = np.zeros((num_seqs, num_heads, head_dim), np.float32)
    for s in range(num_seqs):
        has = int(seq_lens[s]) > 0
        if slot_mapping is not None:
            has = has and int(slot_mapping[s]) >= 0
        if not has:
            continue
        for h in range(num_heads):
            g = np.max(mx[s, h])
            w = np.where(np.isneginf(mx[s, h]), 0.0, np.exp(mx[s, h] - g)).astype(np.float32)
            den = np.sum(sm[s, h] * w)
            out[s, h] = (w[:, None] * acc[s, h]).sum(axis=0) / den
    return round_to_dtype(out, dtype)


def attention_bytes(seq_lens, num_q_heads, num_kv_heads, head_dim, block_size,
                    elem_bytes=2, index_bytes=4, fused_append=False):
    """Algorithmic HBM bytes of one paged-decode call (the roofline numerator).

    K and V are counted once per KV head over the exact tokens read, plus q,
    out, the block-table entries used and seq_lens.  With a fused append the
    current token's K/V are read once and written once.
    """
    lens = [int(n) for n in np.asarray(seq_lens).tolist()]
    b = len(lens)
    kv = sum(lens) * num_kv_heads * head_dim * 2 * elem_bytes
    qo = 2 * b * num_q_heads * head_dim * elem_bytes
    bt = sum(math.ceil(n / block_size) for n in lens) * index_bytes
    total = kv + qo + bt + b * index_bytes
    if fused_append:
        total += 2 * b * num_kv_heads * head_dim * 2 * elem_bytes
    return total
