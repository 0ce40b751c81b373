"""One-launch RoPE + K/V append + decode (``fd_paged_decode`` with its rope
fields) against the two-launch path it replaces: ``fd_rope_kv_append`` (RoPE
of q and K, K/V stored at the slot) followed by ``fd_paged_decode`` over the
cache.  Both use one rotation routine and the same tiles, so the caches and
the outputs must agree bit for bit, over every schedule (cluster merge,
explicit splits, the persistent schedule), page sizes 8/16/32, head_dim
64/128, partial rotary dims and GQA groups.  The engine path built on it is
checked against the numpy oracle in ``tests/test_engine_gpu.py``."""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from tests.golden.cases import _normal  # noqa: E402
from tests.helpers import to_dev  # noqa: E402

pytestmark = pytest.mark.gpu

CASES = [
    # batch, hq, hkv, d, bs, rd, dtype, max_len, schedule
    (8, 16, 2, 128, 32, 128, "bfloat16", 2048, "auto"),      # c2 shape: cluster merge
    (3, 16, 2, 128, 16, 64, "bfloat16", 300, "auto"),
    (16, 16, 2, 128, 32, 128, "bfloat16", 4600, "auto"),     # c5 shape: persistent
    (5, 32, 8, 128, 16, 128, "float16", 5000, "streamk"),
    (4, 8, 8, 64, 8, 32, "bfloat16", 700, "splits"),
    (6, 32, 4, 128, 8, 128, "bfloat16", 900, "splits"),
    (1, 4, 1, 64, 32, 64, "float16", 33, "auto"),
    (40, 16, 2, 128, 32, 128, "bfloat16", 1200, "streamk"),
]


def _case(idx):
    b, hq, hkv, d, bs, rd, dtype, max_len, sched = CASES[idx]
    rng = np.random.default_rng(900 + idx)
    lens = rng.integers(1, max_len + 1, size=b)
    lens[0] = max_len
    nblk = [-(-int(n) // bs) for n in lens]
    pool = sum(nblk) + 5
    perm = rng.permutation(pool)
    bt = np.full((b, max(nblk) + 1), -1, np.int32)
    at = 0
    for i, n in enumerate(nblk):
        bt[i, :n] = perm[at:at + n]
        at += n
    pos = (lens - 1).astype(np.int64)
    blk = bt[np.arange(b), pos // bs].astype(np.int64)
    off = (pos % bs).astype(np.int64)
    return dict(
        b=b, hq=hq, hkv=hkv, d=d, bs=bs, rd=rd, dtype=dtype, sched=sched,
        q=_normal(rng, (b, hq, d), dtype), k=_normal(rng, (b, hkv, d), dtype),
        v=_normal(rng, (b, hkv, d), dtype),
        kc=_normal(rng, (pool, hkv, bs, d), dtype), vc=_normal(rng, (pool, hkv, bs, d), dtype),
        bt=bt, lens=lens.astype(np.int32), pos=pos, blk=blk, off=off, slot=blk * bs + off)


def _sched_kw(c):
    if c["sched"] == "streamk":
        return dict(num_splits=0, max_ctas=37)
    if c["sched"] == "splits":
        return dict(num_splits=3)
    return dict(num_splits=0)


@pytest.mark.parametrize("idx", range(len(CASES)))
def test_one_launch_matches_rope_append_then_decode(idx):
    import flashdec_b200
    from flashdec_b200 import _lib, _native

    c = _case(idx)
    dt = c["dtype"]
    q, k, v = to_dev(c["q"], dt), to_dev(c["k"], dt), to_dev(c["v"], dt)
    bt, sl = to_dev(c["bt"]), to_dev(c["lens"])
    pos, blk, off, slot = (to_dev(c[n]) for n in ("pos", "blk", "off", "slot"))
    invf = _native.inv_freq_device(c["rd"], 1e6, q.device)
    scale = c["d"] ** -0.5
    kw = dict(sm_scale=scale, block_size=c["bs"], num_seqs=c["b"], **_sched_kw(c))
    flashdec_b200.device_status(clear=True)

    # two launches: RoPE + append, then decode over the cache
    kc_a, vc_a = to_dev(c["kc"], dt), to_dev(c["vc"], dt)
    q_rot = torch.empty_like(q)
    _native.rope_kv_append(q, q_rot, k, v, kc_a, vc_a, blk, off, pos, c["rd"], invf)
    out_a = torch.empty_like(q)
    _native.paged_decode(q_rot, kc_a, vc_a, bt, sl, out_a, **kw)

    # one launch
    kc_b, vc_b = to_dev(c["kc"], dt), to_dev(c["vc"], dt)
    out_b = torch.empty_like(q)
    _native.paged_decode(q, kc_b, vc_b, bt, sl, out_b, append_k=k, append_v=v, slot_mapping=slot,
                         rope=(c["rd"], invf, pos), **kw)
    torch.cuda.synchronize()
    assert flashdec_b200.device_status(clear=True) == 0
    assert torch.equal(kc_a, kc_b)
    assert torch.equal(vc_a, vc_b)
    assert torch.equal(out_a, out_b)


def test_rope_fields_are_validated():
    from flashdec_b200 import _lib, _native

    c = _case(1)
    dt = c["dtype"]
    q = to_dev(c["q"], dt)
    kc, vc = to_dev(c["kc"], dt), to_dev(c["vc"], dt)
    bt, sl, pos = to_dev(c["bt"]), to_dev(c["lens"]), to_dev(c["pos"])
    invf = _native.inv_freq_device(64, 1e6, q.device)
    out = torch.empty_like(q)
    kw = dict(sm_scale=0.1, block_size=c["bs"], num_seqs=c["b"])
    # rope without a fused append
    with pytest.raises(_lib.FlashDecNativeError, match="invalid argument"):
        _native.paged_decode(q, kc, vc, bt, sl, out, rope=(64, invf, pos), **kw)
    k, v, slot = to_dev(c["k"], dt), to_dev(c["v"], dt), to_dev(c["slot"])
    # odd rotary dim
    with pytest.raises(_lib.FlashDecNativeError, match="invalid argument"):
        _native.paged_decode(q, kc, vc, bt, sl, out, append_k=k, append_v=v, slot_mapping=slot,
                             rope=(63, invf, pos), **kw)


def test_engine_transaction_one_launch_matches_two_launch_backend(monkeypatch):
    """DecodeEngine with append_backend='fused_cuda' (one launch per layer)
    and 'torch' (RoPE + append launch, then decode) on the same inputs,
    with a shared prefix: identical outputs and caches.  (The cascade path,
    which sums in another order, is off here; tests/test_engine_gpu.py checks
    it against the oracle.)"""
    from flashdec_b200 import DecodeEngine, PagedKVCache

    monkeypatch.setenv("FLASHDEC_B200_CASCADE", "0")

    L, hq, hkv, d, bs = 3, 16, 2, 128, 32
    results = {}
    for backend in ("torch", "fused_cuda"):
        rng = np.random.default_rng(21)
        cache = PagedKVCache(L, hkv, d, bs, max_blocks=96, dtype=torch.bfloat16, device="cuda",
                             prefix_cache_capacity_blocks=8)
        eng = DecodeEngine(cache, append_backend=backend)
        shape = (L, 8, hkv, bs, d)
        eng.register_prefix("sys", to_dev(_normal(rng, shape, "bfloat16"), "bfloat16"),
                            to_dev(_normal(rng, shape, "bfloat16"), "bfloat16"))
        ids = list(range(6))
        for r in ids:
            eng.add_request(r)
        eng.admit()
        for r in ids[:4]:
            cache.attach_prefix(r, "sys")
        outs = []
        for _ in range(40):
            tx = eng.begin_step(ids)
            for layer in range(L):
                q = to_dev(_normal(rng, (6, hq, d), "bfloat16"), "bfloat16")
                k = to_dev(_normal(rng, (6, hkv, d), "bfloat16"), "bfloat16")
                v = to_dev(_normal(rng, (6, hkv, d), "bfloat16"), "bfloat16")
                outs.append(eng.step_layer(tx, layer, q, k, v, rotary_dim=96, base=1e6).output)
            eng.commit_step(tx)
        results[backend] = (torch.stack(outs), cache.k_cache.clone(), cache.v_cache.clone())
    for a, b in zip(results["torch"], results["fused_cuda"]):
        assert torch.equal(a, b)
