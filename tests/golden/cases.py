"""Seeded, platform-independent input generators for the parity cases.

Used by ``make_golden.py`` (which feeds them to the reference implementation)
and by the tests (which feed the same values to the oracle and to the CUDA
kernels).  Everything is generated with ``numpy.random.default_rng(seed)``,
whose streams are stable across platforms, and floating values are rounded to
the case dtype so that every consumer sees bit-identical inputs.

Shapes follow BASELINE.json's configs and the reference's own GPU tests
(``tests/test_paged_decode.py``, ``tests/test_fused_rope_kv_append.py``,
``tests/test_rope_append.py`` of cysong2025/flashdec).
"""

from __future__ import annotations

import numpy as np

from oracle.numerics import round_to_dtype


def _normal(rng, shape, dtype):
    return round_to_dtype(rng.standard_normal(shape, dtype=np.float32), dtype)


def c4_lengths(seed=4, batch=64):
    """BASELINE config 4's request lengths: log-uniform in [512, 131072]."""
    rng = np.random.default_rng(seed)
    return [int(x) for x in np.exp(rng.uniform(np.log(512), np.log(131072), size=batch))]


# --------------------------------------------------------------------------
# paged decode attention
# --------------------------------------------------------------------------

ATTN_CASES = {
    # B4, 16q/2kv, D128, bs32, fp32, seq U[64,512],
    # block tables from a seeded permutation of a 128-block pool.
    "c1": dict(seed=1, seq_lens=("uniform", 4, 64, 512), hq=16, hkv=2, d=128, bs=32,
               dtype="float32", pool=128, maxblk=16, layout="token_major"),
    # BASELINE config 2 (Qwen2.5-3B shape), pool = 2x needed blocks.
    "c2_ctx1024": dict(seed=2, seq_lens=[1024] * 8, hq=16, hkv=2, d=128, bs=32,
                       dtype="bfloat16", pool=512, maxblk=32, layout="token_major"),
    "c2_ctx2048": dict(seed=3, seq_lens=[2048] * 8, hq=16, hkv=2, d=128, bs=32,
                       dtype="bfloat16", pool=1024, maxblk=64, layout="token_major"),
    # reference tests/test_paged_decode.py:99-128 (lengths 33/1/47, MHA)
    "var_d64_bs8_bf16": dict(seed=61, seq_lens=[33, 1, 47], hq=4, hkv=4, d=64, bs=8,
                             dtype="bfloat16", layout="token_major"),
    "var_d128_bs16_fp16_dim": dict(seed=62, seq_lens=[33, 1, 47], hq=4, hkv=4, d=128, bs=16,
                                   dtype="float16", layout="dim_major"),
    "var_d64_bs32_fp16": dict(seed=63, seq_lens=[33, 1, 47], hq=4, hkv=4, d=64, bs=32,
                              dtype="float16", layout="token_major"),
    # :131-152 GQA 32q/2kv (group 16)
    "gqa_32_2": dict(seed=64, seq_lens=[16, 31], hq=32, hkv=2, d=64, bs=16,
                     dtype="bfloat16", layout="token_major"),
    # :155-176 MQA 16q/1kv
    "mqa_16_1": dict(seed=65, seq_lens=[32, 45], hq=16, hkv=1, d=64, bs=8,
                     dtype="float16", layout="token_major"),
    # :179-193 zero length
    "zero_len": dict(seed=66, seq_lens=[0, 17], hq=2, hkv=2, d=64, bs=16,
                     dtype="bfloat16", layout="token_major"),
    # :196-209 custom scale
    "custom_scale": dict(seed=67, seq_lens=[19], hq=2, hkv=1, d=64, bs=16,
                         dtype="float16", layout="token_major", sm_scale=0.25),
    # :303-341 split-KV shape
    "split_257_193": dict(seed=68, seq_lens=[257, 193], hq=16, hkv=2, d=128, bs=16,
                          dtype="bfloat16", layout="token_major"),
    # BASELINE config 4 attention shape (Llama-3-8B 32q/8kv, bs16) at small lengths
    "llama_shape": dict(seed=69, seq_lens=[512, 700, 1500, 3], hq=32, hkv=8, d=128, bs=16,
                        dtype="bfloat16", layout="token_major"),
    # group 4, D64, dim-major, bf16
    "g4_d64_dim": dict(seed=70, seq_lens=[100, 64, 1], hq=8, hkv=2, d=64, bs=32,
                       dtype="bfloat16", layout="dim_major"),
}


def attn_seq_lens(spec):
    sl = spec["seq_lens"]
    if isinstance(sl, tuple) and sl[0] == "uniform":
        _, b, lo, hi = sl
        rng = np.random.default_rng(spec["seed"] + 1000)
        return [int(x) for x in rng.integers(lo, hi + 1, size=b)]
    return list(sl)


def make_attn_case(name):
    """Return a dict of numpy inputs for attention case ``name``.

    Caches are produced in the case's layout (token-major
    ``[NB, Hkv, bs, D]`` or dim-major ``[NB, Hkv, D, bs]``); block tables are
    int32, padded with -1 past each sequence's blocks.
    """
    spec = ATTN_CASES[name]
    rng = np.random.default_rng(spec["seed"])
    seq_lens = attn_seq_lens(spec)
    b, hq, hkv, d, bs = len(seq_lens), spec["hq"], spec["hkv"], spec["d"], spec["bs"]
    nblk = [-(-n // bs) for n in seq_lens]
    maxblk = spec.get("maxblk", max(1, max(nblk)))
    pool = spec.get("pool", sum(nblk) + 3)
    dtype = spec["dtype"]
    q = _normal(rng, (b, hq, d), dtype)
    k_tm = _normal(rng, (pool, hkv, bs, d), dtype)
    v_tm = _normal(rng, (pool, hkv, bs, d), dtype)
    perm = rng.permutation(pool)
    bt = np.full((b, maxblk), -1, dtype=np.int32)
    pos = 0
    for i, n in enumerate(nblk):
        bt[i, :n] = perm[pos:pos + n]
        pos += n
    if spec["layout"] == "dim_major":
        k = np.ascontiguousarray(np.swapaxes(k_tm, 2, 3))
        v = np.ascontiguousarray(np.swapaxes(v_tm, 2, 3))
    else:
        k, v = k_tm, v_tm
    return dict(q=q, k_cache=k, v_cache=v, block_tables=bt,
                seq_lens=np.asarray(seq_lens, dtype=np.int32),
                sm_scale=spec.get("sm_scale"), kv_layout=spec["layout"], dtype=dtype,
                block_size=bs)


# --------------------------------------------------------------------------
# fused append + attention (reference tests/test_paged_decode.py:344-421,
# :424-554): the current token's K/V come with the call.
# --------------------------------------------------------------------------

APPEND_ATTN_CASES = {
    "append_0_17": dict(seed=80, prior=[0, 17], hq=16, hkv=2, d=128, bs=16, dtype="bfloat16"),
    "append_256_193": dict(seed=81, prior=[256, 193], hq=16, hkv=2, d=128, bs=16, dtype="float16"),
    "append_c2": dict(seed=82, prior=[2047] * 8, hq=16, hkv=2, d=128, bs=32, dtype="bfloat16"),
}


def make_append_attn_case(name):
    """Inputs for a fused-append decode: prior tokens are resident, the current
    token (position ``prior``) arrives in ``append_k``/``append_v`` and its slot
    is already reserved in the block table; the cache slot itself holds stale
    zeros."""
    spec = APPEND_ATTN_CASES[name]
    rng = np.random.default_rng(spec["seed"])
    prior = spec["prior"]
    b, hq, hkv, d, bs, dtype = len(prior), spec["hq"], spec["hkv"], spec["d"], spec["bs"], spec["dtype"]
    seq_lens = [n + 1 for n in prior]
    nblk = [-(-n // bs) for n in seq_lens]
    pool = sum(nblk) + 5
    q = _normal(rng, (b, hq, d), dtype)
    k = _normal(rng, (pool, hkv, bs, d), dtype)
    v = _normal(rng, (pool, hkv, bs, d), dtype)
    append_k = _normal(rng, (b, hkv, d), dtype)
    append_v = _normal(rng, (b, hkv, d), dtype)
    perm = rng.permutation(pool)
    bt = np.full((b, max(nblk)), -1, dtype=np.int32)
    pos = 0
    slots = []
    for i, n in enumerate(nblk):
        bt[i, :n] = perm[pos:pos + n]
        pos += n
        p = seq_lens[i] - 1
        blk = int(bt[i, p // bs])
        slots.append(blk * bs + p % bs)
        k[blk, :, p % bs, :] = 0.0
        v[blk, :, p % bs, :] = 0.0
    return dict(q=q, k_cache=k, v_cache=v, block_tables=bt,
                seq_lens=np.asarray(seq_lens, np.int32), append_k=append_k,
                append_v=append_v, slot_mapping=np.asarray(slots, np.int64),
                dtype=dtype, block_size=bs)


# --------------------------------------------------------------------------
# RoPE + append
# --------------------------------------------------------------------------

ROPE_CASES = {
    # 64 tokens, 16q + 2kv heads, D128, theta 1e6,
    # positions U[0, 32768), distinct slots in a 4096-block x 32-token pool.
    "c3": dict(seed=5, b=64, hq=16, hkv=2, d=128, rd=128, base=1e6, dtype="bfloat16",
               pos=("uniform", 0, 32767), pool=4096, bs=32),
    "c3_fp16": dict(seed=6, b=16, hq=16, hkv=2, d=128, rd=128, base=1e6, dtype="float16",
                    pos=("uniform", 0, 32767), pool=4096, bs=32),
    "c3_fp32": dict(seed=7, b=16, hq=16, hkv=2, d=128, rd=128, base=1e6, dtype="float32",
                    pos=("uniform", 0, 32767), pool=4096, bs=32),
    # reference tests/test_fused_rope_kv_append.py:201-235
    "small_rd4_bf16": dict(seed=241, b=2, hq=4, hkv=2, d=8, rd=4, base=10000.0, dtype="bfloat16",
                           pos=[0, 7], pool=4, bs=3, slots=[(3, 2), (1, 0)]),
    "small_rd4_fp32": dict(seed=242, b=2, hq=4, hkv=2, d=8, rd=4, base=10000.0, dtype="float32",
                           pos=[0, 7], pool=4, bs=3, slots=[(3, 2), (1, 0)]),
    # partial rotary on a Llama-ish shape, theta 1e4, D64
    "partial_d64_rd32": dict(seed=243, b=9, hq=8, hkv=4, d=64, rd=32, base=10000.0,
                             dtype="bfloat16", pos=("uniform", 0, 5000), pool=64, bs=16),
}


def make_rope_case(name):
    spec = ROPE_CASES[name]
    rng = np.random.default_rng(spec["seed"])
    b, hq, hkv, d, dtype = spec["b"], spec["hq"], spec["hkv"], spec["d"], spec["dtype"]
    q = _normal(rng, (b, hq, d), dtype)
    k = _normal(rng, (b, hkv, d), dtype)
    v = _normal(rng, (b, hkv, d), dtype)
    pos = spec["pos"]
    if isinstance(pos, tuple):
        positions = rng.integers(pos[1], pos[2] + 1, size=b).astype(np.int64)
    else:
        positions = np.asarray(pos, dtype=np.int64)
    if "slots" in spec:
        block_ids = np.asarray([s[0] for s in spec["slots"]], np.int64)
        offsets = np.asarray([s[1] for s in spec["slots"]], np.int64)
    else:
        flat = rng.permutation(spec["pool"] * spec["bs"])[:b].astype(np.int64)
        block_ids, offsets = flat // spec["bs"], flat % spec["bs"]
    return dict(q=q, k=k, v=v, positions=positions, block_ids=block_ids,
                block_offsets=offsets, rotary_dim=spec["rd"], base=spec["base"],
                dtype=dtype, num_blocks=spec["pool"], block_size=spec["bs"])
