"""GPU parity of the paged decode attention against the numpy oracle.

Every call goes through the public API (flashdec_b200.decode /
paged_decode_attention_into / the vLLM launcher) and therefore through the
C ABI of libflashdec_b200.so.  Cases mirror the reference's own GPU tests
(tests/test_paged_decode.py of cysong2025/flashdec) and BASELINE configs.
"""

import math

import numpy as np
import pytest

from oracle import paged_decode_attention_ref
from oracle.numerics import round_to_dtype
from oracle.paged_attention import paged_decode_with_append_ref
from tests.golden import cases
from tests.helpers import assert_attention_close, decode_golden, to_dev, to_np

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _lib_and_status():
    import flashdec_b200

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    flashdec_b200.device_status(clear=True)
    yield
    assert flashdec_b200.device_status(clear=True) == 0


def _case_on_device(name, force_dtype=None):
    c = cases.make_attn_case(name)
    dt = force_dtype or c["dtype"]
    if force_dtype:
        for key in ("q", "k_cache", "v_cache"):
            c[key] = round_to_dtype(c[key], dt)
        c["dtype"] = dt
    dev = dict(
        q=to_dev(c["q"], dt), k=to_dev(c["k_cache"], dt), v=to_dev(c["v_cache"], dt),
        bt=to_dev(c["block_tables"]), sl=to_dev(c["seq_lens"]),
    )
    return c, dev


ATTN = [n for n in cases.ATTN_CASES if n != "c1"]


@pytest.mark.parametrize("name", ATTN + ["c1"])
def test_decode_matches_fp32_oracle(name):
    import flashdec_b200

    c, d = _case_on_device(name, force_dtype="bfloat16" if name == "c1" else None)
    out = flashdec_b200.decode(d["q"], d["k"], d["v"], d["bt"], d["sl"], sm_scale=c["sm_scale"],
                               kv_layout=c["kv_layout"])
    torch.cuda.synchronize()
    ref = paged_decode_attention_ref(c["q"], c["k_cache"], c["v_cache"], c["block_tables"],
                                     c["seq_lens"], sm_scale=c["sm_scale"],
                                     kv_layout=c["kv_layout"], dtype="float32")
    assert out.dtype == d["q"].dtype and out.shape == d["q"].shape
    assert_attention_close(to_np(out), ref)


@pytest.mark.parametrize("name", ATTN)
def test_decode_matches_reference_golden(name, golden_dir):
    """Against the reference implementation's own output (rtol=atol=3e-2, the
    bf16 tolerance of the reference's tests/test_paged_decode.py:28-32)."""
    import flashdec_b200

    golden = np.load(golden_dir / "attn_golden.npz")
    c, d = _case_on_device(name)
    out = flashdec_b200.decode(d["q"], d["k"], d["v"], d["bt"], d["sl"], sm_scale=c["sm_scale"],
                               kv_layout=c["kv_layout"])
    ref = decode_golden(golden[f"{name}/out"], c["dtype"])
    np.testing.assert_allclose(to_np(out), ref, rtol=3e-2, atol=3e-2)


def test_decode_is_deterministic_and_reusable():
    import flashdec_b200

    c, d = _case_on_device("c2_ctx2048")
    a = flashdec_b200.decode(d["q"], d["k"], d["v"], d["bt"], d["sl"])
    b = flashdec_b200.decode(d["q"], d["k"], d["v"], d["bt"], d["sl"])
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("max_ctas", [1, 2, 3, 7, 16, 61, 148, 1000])
@pytest.mark.parametrize("min_tiles", [1, 3])
def test_length_balanced_schedule_any_grid(max_ctas, min_tiles):
    """Every grid size cuts the batch at different tile boundaries; results
    must not depend on where the cuts fall."""
    from flashdec_b200 import _native

    c, d = _case_on_device("llama_shape")
    out = torch.empty_like(d["q"])
    _native.paged_decode(d["q"], d["k"], d["v"], d["bt"], d["sl"], out,
                         sm_scale=1 / math.sqrt(128), block_size=c["block_size"],
                         num_seqs=d["q"].shape[0], num_splits=0, max_ctas=max_ctas,
                         min_tiles_per_cta=min_tiles)
    ref = paged_decode_attention_ref(c["q"], c["k_cache"], c["v_cache"], c["block_tables"],
                                     c["seq_lens"], dtype="float32")
    assert_attention_close(to_np(out), ref)


@pytest.mark.parametrize("num_splits", [2, 8, 16])
@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
def test_explicit_split_workspace_matches_oracle(num_splits, dtype):
    """Reference tests/test_paged_decode.py:303-341: caller-owned split
    workspace, fixed split count, then the query-head reducer."""
    import flashdec_b200

    c, d = _case_on_device("split_257_193", force_dtype=dtype)
    ws = (torch.empty((2, 16, 16, 128), device="cuda", dtype=torch.float32),
          torch.empty((2, 16, 16), device="cuda", dtype=torch.float32),
          torch.empty((2, 16, 16), device="cuda", dtype=torch.float32))
    out = torch.empty_like(d["q"])
    ret = flashdec_b200.paged_decode_attention_into(d["q"], d["k"], d["v"], d["bt"], d["sl"], out,
                                                    block_size=16, split_kv_workspace=ws,
                                                    num_splits=num_splits)
    assert ret is out
    ref = paged_decode_attention_ref(c["q"], c["k_cache"], c["v_cache"], c["block_tables"],
                                     c["seq_lens"], dtype="float32")
    assert_attention_close(to_np(out), ref)


def test_split_partials_match_oracle_partials():
    """The split kernel's (acc, max, sum) triples themselves, before the
    reducer, against the oracle's split partials."""
    from flashdec_b200 import _lib, _native
    from oracle.paged_attention import split_partials_ref

    c, d = _case_on_device("split_257_193")
    S = 8
    acc = torch.zeros((2, 16, S, 128), device="cuda")
    mx = torch.zeros((2, 16, S), device="cuda")
    sm = torch.zeros((2, 16, S), device="cuda")
    out = torch.empty_like(d["q"])
    _native.paged_decode(d["q"], d["k"], d["v"], d["bt"], d["sl"], out,
                         sm_scale=1 / math.sqrt(128), block_size=16, num_seqs=2, num_splits=S,
                         epilogue=_lib.FD_EPILOGUE_PARTIALS, partials=(acc, mx, sm))
    r_acc, r_mx, r_sm = split_partials_ref(c["q"], c["k_cache"], c["v_cache"], c["block_tables"],
                                           c["seq_lens"], S)
    finite = np.isfinite(r_mx)
    np.testing.assert_array_equal(np.isfinite(to_np(mx)), finite)
    np.testing.assert_allclose(to_np(mx)[finite], r_mx[finite], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(to_np(sm), r_sm, rtol=2e-3, atol=2e-3)
    np.testing.assert_allclose(to_np(acc), r_acc, rtol=2e-2, atol=5e-2)


def test_fp32_is_rejected_like_the_reference():
    import flashdec_b200

    c, d = _case_on_device("c1")
    with pytest.raises(ValueError, match="float16 and bfloat16"):
        flashdec_b200.decode(d["q"], d["k"], d["v"], d["bt"], d["sl"])


def test_strided_nhd_cache_view():
    """Reference :212-251: [block, head, token, dim] view of an NHD buffer."""
    import flashdec_b200

    c, d = _case_on_device("split_257_193")
    k_nhd = d["k"].permute(0, 2, 1, 3).contiguous()
    v_nhd = d["v"].permute(0, 2, 1, 3).contiguous()
    k_view = k_nhd.permute(0, 2, 1, 3)
    v_view = v_nhd.permute(0, 2, 1, 3)
    assert not k_view.is_contiguous()
    out = torch.empty_like(d["q"])
    ret = flashdec_b200.paged_decode_attention_into(d["q"], k_view, v_view, d["bt"], d["sl"], out,
                                                    block_size=16)
    assert ret is out
    ref = paged_decode_attention_ref(c["q"], c["k_cache"], c["v_cache"], c["block_tables"],
                                     c["seq_lens"], dtype="float32")
    assert_attention_close(to_np(out), ref)


def test_unused_block_table_entries_are_never_read():
    """Reference :254-282: entries past ceil(seq_len/bs) hold 2**30."""
    import flashdec_b200

    c, d = _case_on_device("var_d64_bs8_bf16")
    ext = torch.full((3, 64), 2 ** 30, device="cuda", dtype=torch.int32)
    ext[:, : d["bt"].shape[1]] = d["bt"]
    nb = [-(-int(n) // 8) for n in c["seq_lens"]]
    for row, n in enumerate(nb):
        ext[row, n:] = 2 ** 30
    out = flashdec_b200.decode(d["q"], d["k"], d["v"], ext, d["sl"], block_size=8)
    ref = paged_decode_attention_ref(c["q"], c["k_cache"], c["v_cache"], c["block_tables"],
                                     c["seq_lens"], dtype="float32")
    assert_attention_close(to_np(out), ref)


def test_nan_in_unwritten_slots_does_not_leak():
    """Slots past seq_len inside the last page (never written in a real cache,
    e.g. torch.empty in vLLM) may hold NaN; the output must stay finite."""
    import flashdec_b200

    c, d = _case_on_device("var_d64_bs32_fp16")
    k, v = d["k"].clone(), d["v"].clone()
    for row, n in enumerate(c["seq_lens"].tolist()):
        last = int(c["block_tables"][row, (n - 1) // 32])
        off = n % 32
        if off:
            k[last, :, off:, :] = float("nan")
            v[last, :, off:, :] = float("nan")
    out = flashdec_b200.decode(d["q"], k, v, d["bt"], d["sl"])
    ref = paged_decode_attention_ref(c["q"], c["k_cache"], c["v_cache"], c["block_tables"],
                                     c["seq_lens"], dtype="float32")
    assert_attention_close(to_np(out), ref)


def test_int64_metadata_and_noncontiguous_seq_lens():
    import flashdec_b200

    c, d = _case_on_device("llama_shape")
    bt64 = d["bt"].to(torch.int64)
    sl_store = torch.zeros((4, 3), device="cuda", dtype=torch.int64)
    sl_store[:, 1] = d["sl"]
    sl = sl_store[:, 1]
    assert not sl.is_contiguous()
    out = flashdec_b200.decode(d["q"], d["k"], d["v"], bt64, sl)
    ref = paged_decode_attention_ref(c["q"], c["k_cache"], c["v_cache"], c["block_tables"],
                                     c["seq_lens"], dtype="float32")
    assert_attention_close(to_np(out), ref)


@pytest.mark.parametrize("name", list(cases.APPEND_ATTN_CASES))
@pytest.mark.parametrize("num_splits", [1, 8])
def test_fused_current_token_append(name, num_splits, golden_dir):
    """Reference :344-421: the token's K/V arrive with the call, its cache
    slot holds stale zeros; attention must use the new token and the slot
    must hold it afterwards (bit-exact)."""
    import flashdec_b200

    c = cases.make_append_attn_case(name)
    dt = c["dtype"]
    q, k, v = to_dev(c["q"], dt), to_dev(c["k_cache"], dt), to_dev(c["v_cache"], dt)
    ak, av = to_dev(c["append_k"], dt), to_dev(c["append_v"], dt)
    bt, sl, slots = to_dev(c["block_tables"]), to_dev(c["seq_lens"]), to_dev(c["slot_mapping"])
    b = q.shape[0]
    ws = (torch.empty((b, 16, 16, 128), device="cuda"), torch.empty((b, 16, 16), device="cuda"),
          torch.empty((b, 16, 16), device="cuda"))
    out = torch.empty_like(q)
    flashdec_b200.paged_decode_attention_into(q, k, v, bt, sl, out, block_size=c["block_size"],
                                              split_kv_workspace=ws, num_splits=num_splits,
                                              append_k=ak, append_v=av, slot_mapping=slots)
    ref_out, k_after, v_after = paged_decode_with_append_ref(
        c["q"], c["k_cache"], c["v_cache"], c["block_tables"], c["seq_lens"], c["append_k"],
        c["append_v"], c["slot_mapping"], dtype="float32")
    assert_attention_close(to_np(out), ref_out)
    np.testing.assert_array_equal(to_np(k), k_after)
    np.testing.assert_array_equal(to_np(v), v_after)
    golden = decode_golden(np.load(golden_dir / "attn_golden.npz")[f"{name}/out"], dt)
    np.testing.assert_allclose(to_np(out), golden, rtol=3e-2, atol=3e-2)


@pytest.mark.parametrize("num_splits,layout", [(0, "NHD"), (1, "NHD"), (8, "NHD"), (8, "HND"),
                                               (0, "HND")])
@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
def test_vllm_launcher_full_cache_and_graph_padding(num_splits, layout, dtype):
    """Reference :424-554: vLLM's 5-D cache, a padding row (slot = -1) that
    must produce zeros and write nothing, a row past num_reqs left untouched."""
    from flashdec_b200.kernels.paged_decode import _vllm_paged_decode_attention_into

    c = cases.make_append_attn_case("append_256_193")
    dt = dtype
    for key in ("q", "k_cache", "v_cache", "append_k", "append_v"):
        c[key] = round_to_dtype(c[key], dt)
    bs = c["block_size"]
    ref_out, k_after, v_after = paged_decode_with_append_ref(
        c["q"], c["k_cache"], c["v_cache"], c["block_tables"], c["seq_lens"], c["append_k"],
        c["append_v"], c["slot_mapping"], dtype="float32")
    nb = c["k_cache"].shape[0]
    # expected full cache [NB, 2, bs, Hkv, D] after the append
    expected = np.stack([k_after.transpose(0, 2, 1, 3), v_after.transpose(0, 2, 1, 3)], axis=1)
    start = np.stack([c["k_cache"].transpose(0, 2, 1, 3), c["v_cache"].transpose(0, 2, 1, 3)], axis=1)
    if layout == "NHD":
        full = to_dev(start, dt)
    else:
        storage = torch.empty((nb, 2, 2, bs, 128), device="cuda", dtype=getattr(torch, dt))
        full = storage.permute(0, 1, 3, 2, 4)
        full.copy_(to_dev(start, dt))
        assert not full.is_contiguous()
    rng = np.random.default_rng(5)
    q = torch.cat((to_dev(c["q"], dt), to_dev(rng.standard_normal((2, 16, 128), dtype=np.float32), dt)))
    ak = torch.cat((to_dev(c["append_k"], dt), to_dev(rng.standard_normal((2, 2, 128), dtype=np.float32), dt)))
    av = torch.cat((to_dev(c["append_v"], dt), to_dev(rng.standard_normal((2, 2, 128), dtype=np.float32), dt)))
    bt = to_dev(c["block_tables"])
    bt = torch.cat((bt, torch.zeros_like(bt[:1])))
    sl_store = torch.zeros((3, 2), device="cuda", dtype=torch.int32)
    sl_store[:2, 1] = to_dev(c["seq_lens"])
    sl_store[2, 1] = 17
    sl = sl_store[:, 1]
    slots = torch.tensor([*c["slot_mapping"].tolist(), -1], device="cuda", dtype=torch.int64)
    ws = (torch.empty((4, 16, 16, 128), device="cuda"), torch.empty((4, 16, 16), device="cuda"),
          torch.empty((4, 16, 16), device="cuda"))
    out = torch.full_like(q, 37)
    ret = _vllm_paged_decode_attention_into(
        q, ak, av, full, bt, sl, out, slots, *ws, num_reqs=3, num_q_heads=16, num_kv_heads=2,
        head_dim=128, block_size=bs, sm_scale=1.0 / math.sqrt(128), num_splits=num_splits)
    assert ret is out
    torch.cuda.synchronize()
    assert_attention_close(to_np(out[:2]), ref_out)
    assert torch.count_nonzero(out[2]).item() == 0
    assert torch.all(out[3] == 37).item()
    np.testing.assert_array_equal(to_np(full), expected)


def test_zero_length_and_inactive_rows_are_zero():
    import flashdec_b200

    c, d = _case_on_device("zero_len")
    out = flashdec_b200.decode(d["q"], d["k"], d["v"], d["bt"], d["sl"])
    assert torch.count_nonzero(out[0]).item() == 0


def test_validation_errors_match_reference_messages():
    import flashdec_b200

    q = torch.randn((1, 1, 64), device="cuda", dtype=torch.float16)
    k = torch.randn((1, 1, 8, 64), device="cuda", dtype=torch.float16)
    bt = torch.tensor([[0]], device="cuda", dtype=torch.int32)
    sl = torch.tensor([7], device="cuda", dtype=torch.int32)
    with pytest.raises(ValueError, match="same shape"):
        flashdec_b200.paged_decode_attention_into(q, k, k, bt, sl, torch.empty((1, 64), device="cuda",
                                                                            dtype=torch.float16))
    with pytest.raises(ValueError, match="block_size 8, 16, or 32"):
        flashdec_b200.decode(q, torch.randn((1, 1, 4, 64), device="cuda", dtype=torch.float16),
                             torch.randn((1, 1, 4, 64), device="cuda", dtype=torch.float16), bt,
                             sl, block_size=4)
    with pytest.raises(ValueError, match="num_warps"):
        flashdec_b200.decode(q, k, k, bt, sl, num_warps=3)
    with pytest.raises(ValueError, match="num_stages"):
        flashdec_b200.decode(q, k, k, bt, sl, num_stages=5)
    with pytest.raises(ValueError, match="kv_layout"):
        flashdec_b200.decode(q, k, k, bt, sl, kv_layout="unknown")
    with pytest.raises(ValueError, match="must be provided together"):
        flashdec_b200.paged_decode_attention_into(q, k, k, bt, sl, torch.empty_like(q),
                                                  append_k=torch.empty((1, 1, 64), device="cuda",
                                                                       dtype=torch.float16))


def test_prepared_signature_reuses_checks_but_reads_new_data():
    """Calls with an already-seen signature take the prepared launch: new
    values in new tensors (q, caches, block tables, lengths) are read, and
    arguments outside the prepared case still get the reference's errors."""
    from flashdec_b200.kernels import paged_decode as pd

    c1 = cases.make_attn_case("split_257_193")
    rng = np.random.default_rng(123)
    for trial in range(3):
        c = dict(c1)
        if trial:
            c["q"] = cases._normal(rng, c1["q"].shape, c1["dtype"])
            c["k_cache"] = cases._normal(rng, c1["k_cache"].shape, c1["dtype"])
            c["v_cache"] = cases._normal(rng, c1["v_cache"].shape, c1["dtype"])
            order = rng.permutation(c1["k_cache"].shape[0])
            c["block_tables"] = np.where(c1["block_tables"] >= 0, order[c1["block_tables"]], -1
                                         ).astype(np.int32)
            c["seq_lens"] = np.asarray([255 - trial, 190 + trial], np.int32)
        q = to_dev(c["q"], c["dtype"])
        out = torch.empty_like(q)
        pd.paged_decode_attention_into(q, to_dev(c["k_cache"], c["dtype"]),
                                       to_dev(c["v_cache"], c["dtype"]),
                                       to_dev(c["block_tables"]), to_dev(c["seq_lens"]), out)
        want = paged_decode_attention_ref(c["q"], c["k_cache"], c["v_cache"], c["block_tables"],
                                          c["seq_lens"])
        assert_attention_close(to_np(out), want)
    assert len(pd._PREPARED) >= 1
    with pytest.raises(ValueError, match="num_splits must be a positive integer"):
        pd.paged_decode_attention_into(q, to_dev(c1["k_cache"], c1["dtype"]),
                                       to_dev(c1["v_cache"], c1["dtype"]),
                                       to_dev(c1["block_tables"]), to_dev(c1["seq_lens"]), out,
                                       num_splits=True)


def test_cpp_host_path_hits_match_python_path_and_follow_streams():
    """The C++ host path (flashdec_b200._hostpath) launches a default-argument
    call whose signature the Python path prepared on the same stream: its
    output is bit-identical to the Python path's, a new stream or a new shape
    goes through the Python path first (and is then registered), and a
    changed shape still gets the reference's errors."""
    from flashdec_b200 import _lib
    from flashdec_b200.kernels import paged_decode as pd

    hp = _lib.load_hostpath()
    c = cases.make_attn_case("split_257_193")
    q = to_dev(c["q"], c["dtype"])
    k, v = to_dev(c["k_cache"], c["dtype"]), to_dev(c["v_cache"], c["dtype"])
    bt, sl = to_dev(c["block_tables"]), to_dev(c["seq_lens"])
    pd._PREPARED.clear()
    hp.clear()
    ref = torch.empty_like(q)
    pd.paged_decode_attention_into(q, k, v, bt, sl, ref)  # Python path: prepares, registers
    assert hp.table_size() == 1
    assert hp.decode_into(q, k, v, bt, sl, torch.empty_like(q)) == 0
    fast = torch.empty_like(q)
    pd.paged_decode_attention_into(q, k, v, bt, sl, fast)
    torch.cuda.synchronize()
    assert torch.equal(fast, ref)
    # another stream: a miss, then the Python path binds that stream's workspace
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        assert hp.decode_into(q, k, v, bt, sl, fast) == hp.MISS
        out2 = torch.empty_like(q)
        pd.paged_decode_attention_into(q, k, v, bt, sl, out2)
        assert hp.table_size() == 2
        out3 = torch.empty_like(q)
        pd.paged_decode_attention_into(q, k, v, bt, sl, out3)
    side.synchronize()
    assert torch.equal(out2, ref) and torch.equal(out3, ref)
    # a different shape is not a hit and is checked by the Python path
    with pytest.raises(ValueError, match="out must have the same shape as q"):
        pd.paged_decode_attention_into(q, k, v, bt, sl, torch.empty_like(q[:1]))
    # non-tensor arguments fall through to the reference's checks, which
    # fail on them the way the reference's do (attribute access on a list)
    with pytest.raises(AttributeError):
        pd.paged_decode_attention_into(q, k, v, bt.tolist(), sl, fast)
    want = paged_decode_attention_ref(c["q"], c["k_cache"], c["v_cache"], c["block_tables"],
                                      c["seq_lens"])
    assert_attention_close(to_np(fast), want)
