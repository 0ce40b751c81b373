"""Seeded randomized parity of the decode kernel against the numpy oracle.

Covers the schedule space the planner chooses from automatically -- the
cluster merge (small batches), the balanced split, the persistent
length-balanced schedule with pair-aligned cuts (large batches), explicit
grids and explicit reference splits -- over GQA groups 1..32, head_dim
64/128, page sizes 8/16/32, fp16/bf16, token-/dim-major caches, ragged and
zero lengths.  Every case is reproducible from its index."""

from __future__ import annotations

import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import paged_decode_attention_ref  # noqa: E402
from tests.golden.cases import _normal  # noqa: E402
from tests.helpers import assert_attention_close, to_dev, to_np  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _status_clean():
    import flashdec_b200

    flashdec_b200.device_status(clear=True)
    yield
    assert flashdec_b200.device_status(clear=True) == 0


def make_case(idx):
    rng = np.random.default_rng(1000 + idx)
    hkv = int(rng.choice([1, 2, 4, 8]))
    group = int(rng.choice([g for g in (1, 2, 4, 8, 16, 32) if g * hkv <= 64]))
    hq = group * hkv
    d = int(rng.choice([64, 128]))
    bs = int(rng.choice([8, 16, 32]))
    dtype = str(rng.choice(["bfloat16", "float16"]))
    layout = str(rng.choice(["token_major", "token_major", "dim_major"]))
    batch = int(np.exp(rng.uniform(0, math.log(160))))
    max_len = int(rng.choice([64, 300, 1500, 4000]))
    budget = 50_000 // max(1, hkv)  # keep the CPU oracle quick
    kind = rng.integers(0, 3)
    if kind == 0:  # uniform
        lens = np.full(batch, int(rng.integers(1, max_len + 1)))
    elif kind == 1:  # ragged, log-uniform
        lens = np.exp(rng.uniform(0, math.log(max_len), size=batch)).astype(np.int64)
    else:  # ragged with zero-length rows
        lens = rng.integers(0, max_len + 1, size=batch)
        lens[rng.random(batch) < 0.2] = 0
    while lens.sum() > budget and batch > 1:
        batch = max(1, batch // 2)
        lens = lens[:batch]
    lens = np.minimum(lens, max(1, budget // max(1, batch)))
    nblk = [-(-int(n) // bs) for n in lens]
    maxblk = max(1, max(nblk)) + int(rng.integers(0, 3))  # unused tail entries
    pool = sum(nblk) + 4
    q = _normal(rng, (batch, hq, d), dtype)
    k = _normal(rng, (pool, hkv, bs, d), dtype)
    v = _normal(rng, (pool, hkv, bs, d), dtype)
    perm = rng.permutation(pool)
    bt = np.full((batch, maxblk), -1, np.int32)
    pos = 0
    for i, n in enumerate(nblk):
        bt[i, :n] = perm[pos:pos + n]
        pos += n
    sched = rng.integers(0, 4)
    return dict(hkv=hkv, hq=hq, d=d, bs=bs, dtype=dtype, layout=layout, q=q, k=k, v=v, bt=bt,
                lens=lens.astype(np.int32), sched=int(sched),
                max_ctas=int(rng.choice([1, 5, 37, 148, 300])),
                splits=int(rng.choice([2, 3, 8])))


@pytest.mark.parametrize("idx", range(48))
def test_random_shapes_match_oracle(idx):
    import flashdec_b200
    from flashdec_b200 import _native

    c = make_case(idx)
    dt = c["dtype"]
    if c["layout"] == "dim_major":
        k_np, v_np = np.swapaxes(c["k"], 2, 3).copy(), np.swapaxes(c["v"], 2, 3).copy()
    else:
        k_np, v_np = c["k"], c["v"]
    q, k, v = to_dev(c["q"], dt), to_dev(k_np, dt), to_dev(v_np, dt)
    bt, sl = to_dev(c["bt"]), to_dev(c["lens"])
    want = paged_decode_attention_ref(c["q"], c["k"], c["v"], c["bt"], c["lens"])
    scale = c["d"] ** -0.5
    if c["sched"] == 0 or c["layout"] == "dim_major":
        out = flashdec_b200.decode(q, k, v, bt, sl, kv_layout=c["layout"])
    elif c["sched"] == 1:  # persistent schedule on an explicit grid
        out = torch.empty_like(q)
        _native.paged_decode(q, k, v, bt, sl, out, sm_scale=scale, block_size=c["bs"],
                             num_seqs=q.shape[0], num_splits=0, max_ctas=c["max_ctas"])
    elif c["sched"] == 2 and c["d"] == 128 and c["hq"] // c["hkv"] in (4, 8, 16) \
            and c["bs"] in (16, 32):
        # the reference's explicit split with a caller-owned workspace
        s = c["splits"]
        b = q.shape[0]
        ws = (torch.empty((b, c["hq"], s, 128), device="cuda", dtype=torch.float32),
              torch.empty((b, c["hq"], s), device="cuda", dtype=torch.float32),
              torch.empty((b, c["hq"], s), device="cuda", dtype=torch.float32))
        out = torch.empty_like(q)
        flashdec_b200.paged_decode_attention_into(q, k, v, bt, sl, out, split_kv_workspace=ws,
                                                  num_splits=s)
    else:  # fused split merge inside the kernel (tickets)
        out = torch.empty_like(q)
        _native.paged_decode(q, k, v, bt, sl, out, sm_scale=scale, block_size=c["bs"],
                             num_seqs=q.shape[0], num_splits=c["splits"])
    torch.cuda.synchronize()
    assert_attention_close(to_np(out), want)
