"""Pin the numpy oracle against fixtures produced by the reference itself.

The fixtures under tests/golden/ were written by tests/golden/make_golden.py,
which ran cysong2025/flashdec's own PyTorch oracles (paged_reference.py,
rope.py) on the seeded inputs of tests/golden/cases.py.  CPU only.
"""

import hashlib
import math

import numpy as np
import pytest

from oracle import apply_rope, inv_freq_table, paged_decode_attention_ref
from oracle.numerics import bf16_from_bits, bf16_round, round_to_dtype
from oracle.paged_attention import (
    merge_split_partials,
    paged_decode_with_append_ref,
    split_partials_ref,
)
from tests.golden import cases


def _digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()[:16]


def _decode_golden(arr, dtype):
    if dtype == "float32":
        return np.asarray(arr, np.float32)
    if dtype == "float16":
        return np.asarray(arr, np.uint16).view(np.float16).astype(np.float32)
    return bf16_from_bits(arr)


def _ulp(x, dtype):
    """Spacing of the target dtype at |x| (for <=1-ulp rounding-flip checks)."""
    mant = {"bfloat16": 7, "float16": 10, "float32": 23}[dtype]
    e = np.floor(np.log2(np.maximum(np.abs(x), 2.0 ** -14)))
    return 2.0 ** (e - mant)


@pytest.fixture(scope="module")
def attn_golden(golden_dir):
    return np.load(golden_dir / "attn_golden.npz")


@pytest.fixture(scope="module")
def rope_golden(golden_dir):
    return np.load(golden_dir / "rope_golden.npz")


def _assert_matches_reference(ours, ref, dtype, fp32_atol=2e-6):
    if dtype == "float32":
        np.testing.assert_allclose(ours, ref, rtol=1e-5, atol=fp32_atol)
        return
    diff = np.abs(ours - ref)
    # fp32 summation order differs between torch and numpy; after rounding to
    # a 16-bit type the results may differ by at most one ulp, rarely.
    assert np.all(diff <= _ulp(ref, dtype) + 1e-12), float(diff.max())
    assert np.mean(diff > 0) < 0.01


@pytest.mark.parametrize("name", list(cases.ATTN_CASES))
def test_oracle_attention_matches_reference(name, attn_golden):
    c = cases.make_attn_case(name)
    assert str(attn_golden[f"{name}/digest"]) == _digest(
        c["q"], c["k_cache"], c["v_cache"], c["block_tables"]
    ), "seeded inputs drifted from the ones the fixture was generated with"
    ours = paged_decode_attention_ref(
        c["q"], c["k_cache"], c["v_cache"], c["block_tables"], c["seq_lens"],
        sm_scale=c["sm_scale"], kv_layout=c["kv_layout"], dtype=c["dtype"],
    )
    ref = _decode_golden(attn_golden[f"{name}/out"], c["dtype"])
    assert ref.shape == ours.shape
    _assert_matches_reference(ours, ref, c["dtype"])


@pytest.mark.parametrize("name", list(cases.APPEND_ATTN_CASES))
def test_oracle_fused_append_matches_reference(name, attn_golden):
    c = cases.make_append_attn_case(name)
    assert str(attn_golden[f"{name}/digest"]) == _digest(
        c["q"], c["k_cache"], c["append_k"], c["block_tables"]
    )
    out, k_after, v_after = paged_decode_with_append_ref(
        c["q"], c["k_cache"], c["v_cache"], c["block_tables"], c["seq_lens"],
        c["append_k"], c["append_v"], c["slot_mapping"], dtype=c["dtype"],
    )
    ref = _decode_golden(attn_golden[f"{name}/out"], c["dtype"])
    _assert_matches_reference(out, ref, c["dtype"])
    bs = c["block_size"]
    for row, slot in enumerate(c["slot_mapping"].tolist()):
        np.testing.assert_array_equal(k_after[slot // bs, :, slot % bs], c["append_k"][row])
        np.testing.assert_array_equal(v_after[slot // bs, :, slot % bs], c["append_v"][row])


@pytest.mark.parametrize("name", list(cases.ROPE_CASES))
def test_oracle_rope_matches_reference(name, rope_golden):
    c = cases.make_rope_case(name)
    assert str(rope_golden[f"{name}/digest"]) == _digest(c["q"], c["k"], c["positions"])
    # Rotate with the reference's own fp32 torch.pow table so the comparison
    # isolates the rotation arithmetic (the table itself is pinned below).
    table = rope_golden[f"inv_freq/{c['rotary_dim']}/{c['base']:g}"]
    for src, key in ((c["q"], "q_rot"), (c["k"], "k_rot")):
        ours = apply_rope(src, c["positions"], c["rotary_dim"], c["base"], c["dtype"],
                          inv_freq=table)
        ref = _decode_golden(rope_golden[f"{name}/{key}"], c["dtype"])
        if c["dtype"] == "float32":
            np.testing.assert_allclose(ours, ref, rtol=0, atol=2e-5)
        else:
            _assert_matches_reference(ours, ref, c["dtype"])


@pytest.mark.parametrize("rd,base", [(128, 1e6), (128, 1e4), (4, 1e4), (32, 1e4), (64, 5e5)])
def test_inv_freq_table_matches_torch_pow(rd, base, rope_golden):
    ref = rope_golden[f"inv_freq/{rd}/{base:g}"]
    ours = inv_freq_table(rd, base)
    # torch.pow (fp32) vs numpy.power (fp32): allow one ulp
    np.testing.assert_array_max_ulp(ours, ref, maxulp=1)


def test_rope_known_answer():
    """reference tests/test_rope_append.py:73-95 (split-half hand calculation)."""
    x = np.array([[[1.0, 2.0, 3.0, 4.0]], [[1.0, 2.0, 3.0, 4.0]]], np.float32)
    actual = apply_rope(x, np.array([0, 1]))
    expected = np.array([
        1.0 * math.cos(1.0) - 3.0 * math.sin(1.0),
        2.0 * math.cos(0.01) - 4.0 * math.sin(0.01),
        3.0 * math.cos(1.0) + 1.0 * math.sin(1.0),
        4.0 * math.cos(0.01) + 2.0 * math.sin(0.01),
    ], np.float32)
    np.testing.assert_array_equal(actual[0], x[0])
    np.testing.assert_allclose(actual[1, 0], expected, rtol=1e-6, atol=1e-6)


def test_rope_known_answer_matches_reference_fixture(rope_golden):
    x = np.array([[[1.0, 2.0, 3.0, 4.0]], [[1.0, 2.0, 3.0, 4.0]]], np.float32)
    # one fp32 ulp of sin/cos at |x| <= 4
    np.testing.assert_allclose(apply_rope(x, np.array([0, 1])), rope_golden["known_answer/out"],
                               rtol=0, atol=5e-7)


def test_softmax_known_answer_ignores_padding_tokens():
    """reference tests/test_decode_reference.py:38-54 restated on a paged cache."""
    q = np.array([[[1.0, 0.0]]], np.float32)
    k = np.zeros((1, 1, 4, 2), np.float32)
    v = np.zeros((1, 1, 4, 2), np.float32)
    k[0, 0, :3] = [[1, 0], [0, 1], [1000, 1000]]
    v[0, 0, :3] = [[10, 0], [0, 20], [999, 999]]
    out = paged_decode_attention_ref(q, k, v, np.array([[0]]), np.array([2]), sm_scale=1.0)
    w = np.exp([1.0, 0.0]) / np.exp([1.0, 0.0]).sum()
    np.testing.assert_allclose(out[0, 0], w[0] * v[0, 0, 0] + w[1] * v[0, 0, 1], rtol=1e-6)


def test_oracle_rejects_invalid_block_ids_and_layouts():
    c = cases.make_attn_case("zero_len")
    bt = c["block_tables"].copy()
    bt[1, 0] = 10_000
    with pytest.raises(ValueError, match="invalid physical block ids"):
        paged_decode_attention_ref(c["q"], c["k_cache"], c["v_cache"], bt, c["seq_lens"])
    with pytest.raises(ValueError, match="kv_layout"):
        paged_decode_attention_ref(c["q"], c["k_cache"], c["v_cache"], c["block_tables"],
                                   c["seq_lens"], kv_layout="nope")


@pytest.mark.parametrize("num_splits", [1, 2, 8, 16])
def test_split_partials_merge_to_the_unsplit_oracle(num_splits):
    c = cases.make_attn_case("split_257_193")
    acc, mx, sm = split_partials_ref(c["q"], c["k_cache"], c["v_cache"], c["block_tables"],
                                     c["seq_lens"], num_splits)
    merged = merge_split_partials(acc, mx, sm, c["seq_lens"])
    full = paged_decode_attention_ref(c["q"], c["k_cache"], c["v_cache"], c["block_tables"],
                                      c["seq_lens"])
    np.testing.assert_allclose(merged, full, rtol=1e-5, atol=1e-6)


def test_merge_masks_invalid_slots_and_empty_rows():
    acc = np.ones((3, 2, 4, 8), np.float32)
    mx = np.zeros((3, 2, 4), np.float32)
    sm = np.ones((3, 2, 4), np.float32)
    out = merge_split_partials(acc, mx, sm, np.array([5, 0, 5]), slot_mapping=np.array([1, 1, -1]))
    np.testing.assert_array_equal(out[1], 0.0)
    np.testing.assert_array_equal(out[2], 0.0)
    np.testing.assert_allclose(out[0], 1.0)


def test_bf16_rounding_is_round_to_nearest_even():
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, 3.0e38, np.inf], np.float32)
    r = bf16_round(x)
    assert r[0] == 1.0 and r[1] == 1.0 and r[2] == 1.0 + 2 ** -6
    assert r[3] == -2.5 and np.isinf(r[5])
    assert np.isnan(bf16_round(np.array([np.nan], np.float32)))[0]
    np.testing.assert_array_equal(round_to_dtype(x[:4], "float32"), x[:4])
