"""PagedKVCache / DecodeEngine / RoPE helpers on the GPU, checked against the
numpy oracle.

The oracle keeps its own copy of every request's token history (rotated K,
raw V) per layer and computes attention with ``paged_decode_attention_ref``
(a restatement of flashdec/paged_reference.py:19-125); RoPE comes from
``oracle.rope.apply_rope`` with the same fp32 frequency table the library
uploads.  Slot placement is integer work and must match bit for bit; V must
be stored exactly; rotated K within the RoPE tolerance; attention within the
bf16 tolerance of the fp32 oracle (reference tests/test_decode_engine.py,
tests/test_multi_layer_transaction.py, tests/test_rope_append.py)."""

from __future__ import annotations

import json

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle.numerics import round_to_dtype  # noqa: E402
from oracle.paged_attention import paged_decode_attention_ref  # noqa: E402
from oracle.rope import apply_rope as apply_rope_ref  # noqa: E402
from tests.golden.cases import _normal  # noqa: E402
from tests.helpers import assert_attention_close, to_dev, to_np  # noqa: E402

pytestmark = pytest.mark.gpu

ROPE_K_TOL = 1e-2


@pytest.fixture(scope="module", autouse=True)
def _device_ok():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required")
    import flashdec_b200

    flashdec_b200.device_status(clear=True)
    yield
    assert flashdec_b200.device_status() == 0


def _table(rd, base):
    from flashdec_b200 import _native

    return _native.inv_freq_host(rd, base).numpy()


class OracleStore:
    """Host-side history of every request: per layer lists of K/V rows."""

    def __init__(self, num_layers):
        self.k = {}
        self.v = {}
        self.num_layers = num_layers

    def add(self, rid, k_layers=None, v_layers=None):
        self.k[rid] = [[] for _ in range(self.num_layers)]
        self.v[rid] = [[] for _ in range(self.num_layers)]
        if k_layers is not None:
            for layer in range(self.num_layers):
                self.k[rid][layer].extend(list(k_layers[layer]))
                self.v[rid][layer].extend(list(v_layers[layer]))

    def attention(self, layer, ids, q, sm_scale=None):
        lens = [len(self.k[r][layer]) for r in ids]
        t = max(max(lens), 1)
        hkv, d = np.asarray(self.k[ids[0]][layer][0]).shape
        kc = np.zeros((len(ids), hkv, t, d), np.float32)
        vc = np.zeros_like(kc)
        for i, r in enumerate(ids):
            if lens[i]:
                kc[i, :, : lens[i]] = np.stack(self.k[r][layer], axis=1)
                vc[i, :, : lens[i]] = np.stack(self.v[r][layer], axis=1)
        bt = np.arange(len(ids), dtype=np.int32)[:, None]
        return paged_decode_attention_ref(q, kc, vc, bt, np.asarray(lens, np.int32),
                                          sm_scale=sm_scale)


def _check_cache_contents(cache, store, ids, dtype):
    """Every committed token of every request sits at the slot the ledger
    assigned, K within RoPE tolerance, V exact."""
    kc = to_np(cache.k_cache)
    vc = to_np(cache.v_cache)
    bs = cache.block_size
    for r in ids:
        st = cache.request_state(r)
        for layer in range(cache.num_layers):
            want_k = np.stack(store.k[r][layer])
            want_v = np.stack(store.v[r][layer])
            assert len(want_k) == st["seq_len"]
            pos = np.arange(st["seq_len"])
            blocks = np.asarray(st["block_ids"])[pos // bs]
            got_k = kc[layer, blocks, :, pos % bs]
            got_v = vc[layer, blocks, :, pos % bs]
            np.testing.assert_array_equal(got_v, want_v)
            np.testing.assert_allclose(got_k, want_k, atol=ROPE_K_TOL, rtol=0)


@pytest.mark.parametrize("append_backend", ["fused_cuda", "torch"])
@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
def test_multi_layer_engine_matches_oracle(append_backend, dtype):
    from flashdec_b200 import DecodeEngine, PagedKVCache
    from tests.helpers import torch_dtype

    L, hq, hkv, d, bs, rd, base = 3, 16, 2, 128, 16, 64, 1e6
    rng = np.random.default_rng(11)
    cache = PagedKVCache(L, hkv, d, bs, max_blocks=64, dtype=torch_dtype(dtype), device="cuda")
    eng = DecodeEngine(cache, append_backend=append_backend)
    store = OracleStore(L)
    ids = ["a", "b", "c"]
    for r in ids:
        eng.add_request(r)
        store.add(r)
    eng.admit()
    table = _table(rd, base)
    for step in range(37):
        order = ids[::-1] if step % 4 == 1 else ids
        if step == 20:  # a request finishes, a new one joins
            eng.finish_request("b")
            ids = ["a", "c", "d"]
            eng.add_request("d")
            eng.admit("d")
            store.add("d")
            order = ids
        tx = eng.begin_step(order)
        pos = tx.positions.cpu().numpy()
        assert pos.tolist() == [len(store.k[r][0]) for r in order]
        abort_at = 1 if step in (7, 30) else None
        pending = []
        for layer in range(L):
            q = _normal(rng, (len(order), hq, d), dtype)
            k = _normal(rng, (len(order), hkv, d), dtype)
            v = _normal(rng, (len(order), hkv, d), dtype)
            res = eng.step_layer(tx, layer, to_dev(q, dtype), to_dev(k, dtype), to_dev(v, dtype),
                                 rotary_dim=rd, base=base)
            q_rot = apply_rope_ref(q, pos, rd, base, dtype, table)
            k_rot = apply_rope_ref(k, pos, rd, base, dtype, table)
            for i, r in enumerate(order):
                store.k[r][layer].append(k_rot[i])
                store.v[r][layer].append(np.asarray(v[i], np.float32))
            pending.append(layer)
            want = store.attention(layer, order, q_rot)
            assert_attention_close(to_np(res.output), want)
            assert res.effective_seq_lens.tolist() == [p + 1 for p in pos]
            if abort_at == layer:
                break
        if abort_at is not None:
            eng.abort_step(tx)
            for r in order:
                for layer in pending:
                    store.k[r][layer].pop()
                    store.v[r][layer].pop()
            continue
        out = eng.commit_step(tx)
        assert out.status == "ok"
        assert out.seq_lens.tolist() == [len(store.k[r][0]) for r in order]
    assert eng.validate_invariants()
    _check_cache_contents(cache, store, ids, dtype)


def test_shared_prefix_engine_matches_oracle():
    from flashdec_b200 import DecodeEngine, PagedKVCache

    L, hq, hkv, d, bs, dtype = 2, 16, 2, 128, 32, "bfloat16"
    rng = np.random.default_rng(5)
    cache = PagedKVCache(L, hkv, d, bs, max_blocks=32, dtype=torch.bfloat16, device="cuda",
                         prefix_cache_capacity_blocks=4)
    eng = DecodeEngine(cache, append_backend="fused_cuda")
    nb = 3
    pk = _normal(rng, (L, nb, hkv, bs, d), dtype)
    pv = _normal(rng, (L, nb, hkv, bs, d), dtype)
    eng.register_prefix("sys", to_dev(pk, dtype), to_dev(pv, dtype))
    # token-major prefix history: [L, nb*bs, hkv, d]
    pk_tok = pk.transpose(0, 1, 3, 2, 4).reshape(L, nb * bs, hkv, d)
    pv_tok = pv.transpose(0, 1, 3, 2, 4).reshape(L, nb * bs, hkv, d)
    store = OracleStore(L)
    for r in ("p1", "p2", "solo"):
        eng.add_request(r)
    eng.admit()
    for r in ("p1", "p2"):
        cache.attach_prefix(r, "sys")
        store.add(r, pk_tok, pv_tok)
    store.add("solo")
    ids = ["p1", "p2", "solo"]
    for step in range(40):
        tx = eng.begin_step(ids)
        pos = tx.positions.cpu().numpy()
        for layer in range(L):
            q = _normal(rng, (3, hq, d), dtype)
            k = _normal(rng, (3, hkv, d), dtype)
            v = _normal(rng, (3, hkv, d), dtype)
            res = eng.step_layer(tx, layer, to_dev(q, dtype), to_dev(k, dtype), to_dev(v, dtype))
            q_rot = apply_rope_ref(q, pos, None, 1e4, dtype, _table(d, 1e4))
            k_rot = apply_rope_ref(k, pos, None, 1e4, dtype, _table(d, 1e4))
            for i, r in enumerate(ids):
                store.k[r][layer].append(k_rot[i])
                store.v[r][layer].append(np.asarray(v[i], np.float32))
            assert_attention_close(to_np(res.output), store.attention(layer, ids, q_rot))
        eng.commit_step(tx)
    # the shared blocks were never written by the decode tokens
    np.testing.assert_array_equal(
        to_np(cache.k_cache[:, list(cache.prefix_state("sys")["block_ids"])]), pk)
    _check_cache_contents(cache, store, ids, dtype)
    assert cache.metrics()["active_prefix_references"] == 2


@pytest.mark.parametrize("bs,nb", [(32, 8), (16, 12)])
def test_shared_prefix_cascade_engine_matches_oracle(bs, nb, monkeypatch):
    """Rows sharing a registered prefix of >= 128 tokens take the cascade
    path (prefix pass + tail pass + merge); outputs against the oracle over
    the full histories, cache contents exact."""
    from flashdec_b200 import DecodeEngine, PagedKVCache

    monkeypatch.setenv("FLASHDEC_B200_CASCADE", "1")  # the engine's opt-in
    L, hq, hkv, d, dtype = 2, 16, 2, 128, "bfloat16"
    rng = np.random.default_rng(15)
    cache = PagedKVCache(L, hkv, d, bs, max_blocks=96, dtype=torch.bfloat16, device="cuda",
                         prefix_cache_capacity_blocks=nb)
    eng = DecodeEngine(cache, append_backend="fused_cuda")
    pk = _normal(rng, (L, nb, hkv, bs, d), dtype)
    pv = _normal(rng, (L, nb, hkv, bs, d), dtype)
    eng.register_prefix("sys", to_dev(pk, dtype), to_dev(pv, dtype))
    pk_tok = pk.transpose(0, 1, 3, 2, 4).reshape(L, nb * bs, hkv, d)
    pv_tok = pv.transpose(0, 1, 3, 2, 4).reshape(L, nb * bs, hkv, d)
    store = OracleStore(L)
    ids = ["p1", "solo", "p2", "p3", "p4"]
    for r in ids:
        eng.add_request(r)
    eng.admit()
    for r in ids:
        if r == "solo":
            store.add(r)
        else:
            cache.attach_prefix(r, "sys")
            store.add(r, pk_tok, pv_tok)
    table = _table(96, 1e6)
    for step in range(45):
        tx = eng.begin_step(ids)
        assert cache._cascades.groups is not None  # the cascade path is taken
        pos = tx.positions.cpu().numpy()
        for layer in range(L):
            q = _normal(rng, (len(ids), hq, d), dtype)
            k = _normal(rng, (len(ids), hkv, d), dtype)
            v = _normal(rng, (len(ids), hkv, d), dtype)
            res = eng.step_layer(tx, layer, to_dev(q, dtype), to_dev(k, dtype), to_dev(v, dtype),
                                 rotary_dim=96, base=1e6)
            q_rot = apply_rope_ref(q, pos, 96, 1e6, dtype, table)
            k_rot = apply_rope_ref(k, pos, 96, 1e6, dtype, table)
            for i, r in enumerate(ids):
                store.k[r][layer].append(k_rot[i])
                store.v[r][layer].append(np.asarray(v[i], np.float32))
            assert_attention_close(to_np(res.output), store.attention(layer, ids, q_rot))
        eng.commit_step(tx)
    np.testing.assert_array_equal(
        to_np(cache.k_cache[:, list(cache.prefix_state("sys")["block_ids"])]), pk)
    _check_cache_contents(cache, store, ids, dtype)


def test_single_layer_step_backends_agree_bitwise():
    from flashdec_b200 import DecodeEngine, PagedKVCache

    rng = np.random.default_rng(3)
    outs = {}
    for backend in ("torch", "cuda", "fused_cuda"):
        cache = PagedKVCache(1, 2, 128, 16, max_blocks=16, dtype=torch.bfloat16, device="cuda")
        eng = DecodeEngine(cache, append_backend=backend)
        for r in (1, 2):
            eng.add_request(r)
        eng.admit()
        seq = []
        rng = np.random.default_rng(3)
        for _ in range(20):
            q = to_dev(_normal(rng, (2, 8, 128), "bfloat16"), "bfloat16")
            k = to_dev(_normal(rng, (2, 2, 128), "bfloat16"), "bfloat16")
            v = to_dev(_normal(rng, (2, 2, 128), "bfloat16"), "bfloat16")
            res = eng.step(q, k, v, rotary_dim=128, base=5e5)
            assert res.status == "ok"
            seq.append(res.output.clone())
        outs[backend] = (torch.stack(seq), cache.k_cache.clone(), cache.v_cache.clone())
    for backend in ("cuda", "fused_cuda"):
        for a, b in zip(outs["torch"], outs[backend]):
            assert torch.equal(a, b), backend


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
@pytest.mark.parametrize("rd", [128, 64, 2])
def test_apply_rope_matches_oracle(dtype, rd):
    import flashdec_b200

    rng = np.random.default_rng(rd)
    x = _normal(rng, (9, 5, 128), dtype)
    pos = rng.integers(0, 32768, size=9)
    got = flashdec_b200.apply_rope(to_dev(x, dtype), torch.as_tensor(pos, device="cuda"),
                                   rotary_dim=rd, base=1e6)
    want = apply_rope_ref(x, pos, rd, 1e6, dtype, _table(rd, 1e6))
    np.testing.assert_allclose(to_np(got), want, atol=ROPE_K_TOL, rtol=0)
    # the untouched tail is copied bit for bit
    np.testing.assert_array_equal(to_np(got)[..., rd:], np.asarray(x, np.float32)[..., rd:])


def test_apply_rope_validation():
    import flashdec_b200

    x = torch.zeros((2, 1, 8), device="cuda")
    pos = torch.zeros(2, dtype=torch.int64, device="cuda")
    with pytest.raises(ValueError, match="non-negative"):
        flashdec_b200.apply_rope(x, pos - 1)
    with pytest.raises(ValueError, match="rotary_dim"):
        flashdec_b200.apply_rope(x, pos, rotary_dim=3)
    with pytest.raises(ValueError, match="base"):
        flashdec_b200.apply_rope(x, pos, base=float("inf"))
    with pytest.raises(ValueError, match="int32 or int64"):
        flashdec_b200.apply_rope(x, pos.float())


@pytest.mark.parametrize("backend", ["torch", "cuda", "fused_cuda"])
def test_rope_paged_kv_append_matches_oracle(backend):
    from flashdec_b200 import PagedKVCache, RopeAppendResult, rope_paged_kv_append

    rng = np.random.default_rng(17)
    cache = PagedKVCache(1, 2, 64, 8, max_blocks=16, dtype=torch.float16, device="cuda")
    for r in ("x", "y"):
        cache.add_request(r)
    store = OracleStore(1)
    store.add("x")
    store.add("y")
    for step in range(11):
        q = _normal(rng, (2, 4, 64), "float16")
        k = _normal(rng, (2, 2, 64), "float16")
        v = _normal(rng, (2, 2, 64), "float16")
        res = rope_paged_kv_append(cache, 0, ["x", "y"], to_dev(q, "float16"),
                                   to_dev(k, "float16"), to_dev(v, "float16"), rotary_dim=32,
                                   base=1e4, append_backend=backend)
        assert isinstance(res, RopeAppendResult)
        assert res.positions.tolist() == [step, step]
        assert res.seq_lens.tolist() == [step + 1, step + 1]
        want_q = apply_rope_ref(q, [step, step], 32, 1e4, "float16", _table(32, 1e4))
        np.testing.assert_allclose(to_np(res.q), want_q, atol=ROPE_K_TOL, rtol=0)
        k_rot = apply_rope_ref(k, [step, step], 32, 1e4, "float16", _table(32, 1e4))
        for i, r in enumerate(("x", "y")):
            store.k[r][0].append(k_rot[i])
            store.v[r][0].append(np.asarray(v[i], np.float32))
        assert res.block_tables.tolist() == cache.block_tables(["x", "y"]).tolist()
    _check_cache_contents(cache, store, ["x", "y"], "float16")


def test_cache_replays_reference_ledger_trace_with_data(golden_dir):
    """The reference PagedKVCache trace (tests/golden/ledger_golden.json)
    replayed through the product cache on the GPU: same integers, and each
    layer's K/V land at the recorded slots."""
    from flashdec_b200 import PagedKVCache
    from tests.golden.make_golden import LEDGER_METRICS

    golden = json.loads((golden_dir / "ledger_golden.json").read_text())
    cache = PagedKVCache(num_layers=2, num_kv_heads=1, head_dim=2, block_size=8, max_blocks=24,
                         dtype=torch.float32, device="cuda", prefix_cache_capacity_blocks=6)
    recs = [g for g in golden if g["tag"].startswith(("commit_", "abort_"))]
    prefix_k = torch.arange(2 * 2 * 1 * 8 * 2, dtype=torch.float32).reshape(2, 2, 1, 8, 2)
    cache.register_prefix("sys", prefix_k.cuda(), (prefix_k + 1000).cuda())
    for rid in ("a", "b", "c"):
        cache.add_request(rid)
    cache.attach_prefix("c", "sys")

    def active():
        return [r for r, st in cache._requests.items() if st.status == "active"]

    for step, want in zip(range(30), recs):
        ids = active()
        if step % 3 == 1:
            ids = list(reversed(ids))
        tx = cache.begin_token(ids)
        assert [str(r) for r in ids] == want["ids"]
        assert tx.positions.tolist() == want["positions"]
        assert tx.physical_block_ids.tolist() == want["physical_block_ids"]
        assert tx.block_offsets.tolist() == want["block_offsets"]
        assert tx.effective_seq_lens.tolist() == want["effective_seq_lens"]
        assert tx.block_tables.tolist() == want["tx_block_tables"]
        for layer in range(2):
            kv = torch.full((len(ids), 1, 2), float(step), device="cuda")
            cache.write_token_layer(tx, layer, kv + layer, -kv)
        kc = cache.k_cache.cpu()
        for b, o in zip(want["physical_block_ids"], want["block_offsets"]):
            for layer in range(2):
                assert kc[layer, b, 0, o].tolist() == [float(step + layer)] * 2
        if step in (4, 11, 20):
            cache.abort_token(tx)
        else:
            cache.commit_token(tx)
        assert list(cache._free_blocks) == want["free"]
        m = cache.metrics()
        assert {k: m[k] for k in LEDGER_METRICS} == want["metrics"]
        if step == 6:
            cache.finish_request("b")
            cache.add_request("d")
        if step == 12:
            cache.cancel_request("a")
            cache.add_request("e")
            cache.attach_prefix("e", "sys")
            cache.add_request("f")
        if step == 24:
            cache.finish_request(active()[0])
    assert cache.validate_invariants()


def test_fused_layer_shape_errors_abort_the_token():
    """The fused layer launch (C++ host path) rejects a non-contiguous q and
    k/v of the wrong shape with the engine's ValueError; the open token is
    aborted, committed lengths are unchanged and the next token runs."""
    from flashdec_b200 import DecodeEngine, PagedKVCache

    L, hq, hkv, d = 2, 8, 2, 128
    cache = PagedKVCache(L, hkv, d, 16, max_blocks=16, dtype=torch.bfloat16, device="cuda")
    eng = DecodeEngine(cache, append_backend="fused_cuda")
    ids = ["a", "b"]
    for r in ids:
        eng.add_request(r)
    eng.admit()
    g = torch.Generator(device="cuda").manual_seed(3)
    q = torch.randn((2, hq, d), device="cuda", dtype=torch.bfloat16, generator=g)
    k = torch.randn((2, hkv, d), device="cuda", dtype=torch.bfloat16, generator=g)
    v = torch.randn_like(k)
    for _ in range(2):
        tx = eng.begin_step(ids)
        for layer in range(L):
            eng.step_layer(tx, layer, q, k, v)
        eng.commit_step(tx)
    lens = [cache.request_state(r)["seq_len"] for r in ids]
    tx = eng.begin_step(ids)
    q_strided = torch.randn((hq, 2, d), device="cuda", dtype=torch.bfloat16,
                            generator=g).transpose(0, 1)
    with pytest.raises(ValueError, match="q must be a contiguous"):
        eng.step_layer(tx, 0, q_strided, k, v)
    assert [cache.request_state(r)["seq_len"] for r in ids] == lens
    tx = eng.begin_step(ids)
    eng.step_layer(tx, 0, q, k, v)
    with pytest.raises(ValueError, match="k and v must be contiguous"):
        eng.step_layer(tx, 1, q, k, v.transpose(1, 2).contiguous().transpose(1, 2))
    assert [cache.request_state(r)["seq_len"] for r in ids] == lens
    tx = eng.begin_step(ids)
    for layer in range(L):
        res = eng.step_layer(tx, layer, q, k, v)
    eng.commit_step(tx)
    torch.cuda.synchronize()
    assert torch.isfinite(res.output.float()).all()
    assert [cache.request_state(r)["seq_len"] for r in ids] == [n + 1 for n in lens]
