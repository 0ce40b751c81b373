"""Cascade (shared-prefix) decode against the numpy oracle and the plain
decode.

``fd_cascade_decode`` must give what ``paged_decode_attention_ref`` (a
restatement of flashdec/paged_reference.py:19-125) gives for the full
sequences: the prefix pass attends the shared leading pages of each group,
the tail pass the rest, and the split reducer merges them.  Cases cover one
and several groups, sequences outside any group, page sizes 8/16/32, head_dim
64/128, GQA groups 1..16 (1 or 2 row blocks of 128 query rows), more chunks
than prefix tiles (empty chunks), fp16/bf16, and the engine's fused append
with RoPE (cache bytes identical to the plain fused launch)."""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import paged_decode_attention_ref  # noqa: E402
from tests.golden.cases import _normal  # noqa: E402
from tests.helpers import assert_attention_close, to_dev, to_np  # noqa: E402

pytestmark = pytest.mark.gpu

# (name, batch, hq, hkv, d, bs, groups [(members, prefix pages)], tail max, dtype, chunks)
CASES = [
    ("c5_like", 16, 16, 2, 128, 32, [(list(range(16)), 64)], 300, "bfloat16", 0),
    ("two_groups_and_loners", 10, 16, 2, 128, 32, [([0, 2, 5], 8), ([1, 3], 4)], 500,
     "bfloat16", 0),
    ("bs16", 6, 32, 8, 128, 16, [([0, 1, 2, 3, 4], 6)], 200, "float16", 0),
    ("bs8_d64_mha", 7, 4, 4, 64, 8, [([1, 2, 3, 4, 5], 12)], 90, "bfloat16", 0),
    ("g16_three_row_blocks", 9, 32, 2, 128, 32, [(list(range(9)), 10)], 120, "bfloat16", 0),
    ("empty_chunks", 4, 16, 2, 128, 32, [([0, 1, 2, 3], 3)], 64, "bfloat16", 7),
]


def _build(batch, hkv, d, bs, groups, tail_max, dtype, seed):
    rng = np.random.default_rng(seed)
    nxt = 0
    member_pages = {}
    for members, pages in groups:
        ids = list(range(nxt, nxt + pages))
        nxt += pages
        for b in members:
            member_pages[b] = ids
    tails = rng.integers(1, tail_max + 1, size=batch)
    rows, lens = [], []
    for b in range(batch):
        pre = member_pages.get(b, [])
        n_tail_pages = -(-int(tails[b]) // bs)
        priv = list(range(nxt, nxt + n_tail_pages))
        nxt += n_tail_pages
        rows.append(pre + priv)
        lens.append(len(pre) * bs + int(tails[b]))
    width = max(len(r) for r in rows) + 1
    perm = rng.permutation(nxt + 3)  # scatter logical pages over the pool
    bt = np.full((batch, width), -1, np.int32)
    for b, r in enumerate(rows):
        bt[b, :len(r)] = perm[r]
    pool = nxt + 3
    k = _normal(rng, (pool, hkv, bs, d), dtype)
    v = _normal(rng, (pool, hkv, bs, d), dtype)
    return rng, bt, np.asarray(lens, np.int32), k, v


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_cascade_matches_oracle(case):
    import flashdec_b200
    from flashdec_b200 import _native

    name, batch, hq, hkv, d, bs, groups, tail_max, dtype, chunks = case
    rng, bt, lens, k, v = _build(batch, hkv, d, bs, groups, tail_max, dtype, seed=len(name))
    q = _normal(rng, (batch, hq, d), dtype)
    want = paged_decode_attention_ref(q, k, v, bt, lens)
    qd, kd, vd = to_dev(q, dtype), to_dev(k, dtype), to_dev(v, dtype)
    btd, sld = to_dev(bt), to_dev(lens)
    cg = _native.CascadeGroups([m for m, _ in groups], [p for _, p in groups], batch, bs,
                               qd.device)
    flashdec_b200.device_status(clear=True)
    out = torch.empty_like(qd)
    _native.cascade_decode(qd, kd, vd, btd, sld, out, cg, sm_scale=d ** -0.5, block_size=bs,
                           num_seqs=batch, chunks=chunks)
    plain = flashdec_b200.decode(qd, kd, vd, btd, sld)
    torch.cuda.synchronize()
    assert flashdec_b200.device_status(clear=True) == 0
    assert_attention_close(to_np(out), want)
    # the two schedules differ only in summation order
    assert float((out.float() - plain.float()).abs().max()) <= 1.6e-2


# (rotary_dim, batch, hq, hkv, groups): full rotation with the per-block cos/sin
# table; partial rotations whose half is (64 -> 32) and is not (40 -> 20) a
# multiple of 8 elements; GQA group 2 with 40 members in one 128-row block
# (more members than the table holds: cos/sin per element)
ROPE_CASES = [
    (128, 12, 16, 2, [(list(range(8)), 16), ([9, 10], 2)]),
    (64, 12, 16, 2, [(list(range(8)), 16), ([9, 10], 2)]),
    (40, 12, 16, 2, [(list(range(8)), 16), ([9, 10], 2)]),
    (128, 44, 4, 2, [(list(range(40)), 6)]),
]


@pytest.mark.parametrize("rope_case", ROPE_CASES,
                         ids=["rot128", "rot64", "rot40", "g2_40_members"])
def test_cascade_fused_append_rope_matches_plain_fused_launch(rope_case):
    """Engine shape: every row appends its current token (RoPE'd K) and
    rotates q in the kernels; the cache bytes must equal those of the plain
    one-launch path and the outputs agree to the bf16 summation-order bound."""
    import flashdec_b200
    from flashdec_b200 import _native

    rot, batch, hq, hkv, groups = rope_case
    d, bs, dtype = 128, 32, "bfloat16"
    rng, bt, lens, k, v = _build(batch, hkv, d, bs, groups, 200, dtype, seed=77)
    q = to_dev(_normal(rng, (batch, hq, d), dtype), dtype)
    ak = to_dev(_normal(rng, (batch, hkv, d), dtype), dtype)
    av = to_dev(_normal(rng, (batch, hkv, d), dtype), dtype)
    btd, sld = to_dev(bt), to_dev(lens)
    pos = to_dev((lens - 1).astype(np.int64))
    slot = to_dev((bt[np.arange(batch), (lens - 1) // bs].astype(np.int64) * bs
                   + (lens - 1) % bs).astype(np.int64))
    invf = _native.inv_freq_device(rot, 1e6, q.device)
    rope = (rot, invf, pos)
    cg = _native.CascadeGroups([m for m, _ in groups], [p for _, p in groups], batch, bs,
                               q.device)
    flashdec_b200.device_status(clear=True)
    kc_a, vc_a = to_dev(k, dtype), to_dev(v, dtype)
    out_a = torch.empty_like(q)
    _native.paged_decode(q, kc_a, vc_a, btd, sld, out_a, sm_scale=d ** -0.5, block_size=bs,
                         num_seqs=batch, append_k=ak, append_v=av, slot_mapping=slot, rope=rope)
    kc_b, vc_b = to_dev(k, dtype), to_dev(v, dtype)
    out_b = torch.empty_like(q)
    _native.cascade_decode(q, kc_b, vc_b, btd, sld, out_b, cg, sm_scale=d ** -0.5,
                           block_size=bs, num_seqs=batch, append_k=ak, append_v=av,
                           slot_mapping=slot, rope=rope)
    torch.cuda.synchronize()
    assert flashdec_b200.device_status(clear=True) == 0
    assert torch.equal(kc_a, kc_b) and torch.equal(vc_a, vc_b)
    assert float((out_a.float() - out_b.float()).abs().max()) <= 1.6e-2
    # and both against the oracle over the updated caches with rotated q
    from oracle.rope import apply_rope
    from tests.test_engine_gpu import _table

    q_rot = apply_rope(to_np(q), to_np(pos), rot, 1e6, dtype, _table(rot, 1e6))
    want = paged_decode_attention_ref(q_rot, to_np(kc_b), to_np(vc_b), bt, lens)
    assert_attention_close(to_np(out_b), want)



@pytest.mark.parametrize("env", [{"FLASHDEC_B200_CASCADE_CONCURRENT": "0"},
                                 {"FLASHDEC_B200_CASCADE_CONCURRENT": "0",
                                  "FLASHDEC_B200_PREFIX_UMMA": "0"}],
                         ids=["serial_tcgen05_prefix", "serial_mma_sync_prefix"])
def test_serial_cascade_paths(env):
    """The default cascade runs the prefix and tail passes concurrently and
    merges in one reduction (the other tests here).  With
    FLASHDEC_B200_CASCADE_CONCURRENT=0 the passes run one after the other and
    the tail merges through tickets; head_dim 128 / 32-token pages then take
    the tcgen05 prefix pass unless FLASHDEC_B200_PREFIX_UMMA=0.  The switches
    are read once per process, so the cases run in a child process."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    code = (
        "import sys, numpy as np, torch\n"
        "sys.path.insert(0, %r)\n"
        "import flashdec_b200\n"
        "from flashdec_b200 import _native\n"
        "from oracle import paged_decode_attention_ref\n"
        "from tests.test_cascade_gpu import CASES, _build\n"
        "from tests.golden.cases import _normal\n"
        "from tests.helpers import assert_attention_close, to_dev, to_np\n"
        "for case in CASES[:2]:\n"
        "    name, batch, hq, hkv, d, bs, groups, tail_max, dtype, chunks = case\n"
        "    rng, bt, lens, k, v = _build(batch, hkv, d, bs, groups, tail_max, dtype, seed=3)\n"
        "    q = _normal(rng, (batch, hq, d), dtype)\n"
        "    want = paged_decode_attention_ref(q, k, v, bt, lens)\n"
        "    qd, kd, vd = to_dev(q, dtype), to_dev(k, dtype), to_dev(v, dtype)\n"
        "    cg = _native.CascadeGroups([m for m, _ in groups], [p for _, p in groups], batch,"
        " bs, qd.device)\n"
        "    out = torch.empty_like(qd)\n"
        "    _native.cascade_decode(qd, kd, vd, to_dev(bt), to_dev(lens), out, cg,"
        " sm_scale=d ** -0.5, block_size=bs, num_seqs=batch)\n"
        "    torch.cuda.synchronize()\n"
        "    assert flashdec_b200.device_status(clear=True) == 0\n"
        "    assert_attention_close(to_np(out), want)\n"
        "print('ok')\n" % str(Path(__file__).resolve().parents[1]))
    res = subprocess.run([sys.executable, "-c", code], env=dict(os.environ, **env),
                         capture_output=True, text=True, timeout=300)
    assert res.returncode == 0 and res.stdout.strip().endswith("ok"), res.stderr[-2000:]


def test_concurrent_cascade_replays_from_a_cuda_graph():
    """The concurrent cascade forks a second stream and joins it back with
    events, so it can be captured: a graph of the call replays to the eager
    call's output, bit for bit (same kernels, same partial order)."""
    import flashdec_b200
    from flashdec_b200 import _native

    name, batch, hq, hkv, d, bs, groups, tail_max, dtype, chunks = CASES[0]
    rng, bt, lens, k, v = _build(batch, hkv, d, bs, groups, tail_max, dtype, seed=11)
    q = _normal(rng, (batch, hq, d), dtype)
    qd, kd, vd = to_dev(q, dtype), to_dev(k, dtype), to_dev(v, dtype)
    btd, sld = to_dev(bt), to_dev(lens)
    cg = _native.CascadeGroups([m for m, _ in groups], [p for _, p in groups], batch, bs,
                               qd.device)
    eager = torch.empty_like(qd)
    kw = dict(sm_scale=d ** -0.5, block_size=bs, num_seqs=batch)
    _native.cascade_decode(qd, kd, vd, btd, sld, eager, cg, **kw)  # also sets up the streams
    torch.cuda.synchronize()
    out = torch.full_like(qd, float("nan"))
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        _native.cascade_decode(qd, kd, vd, btd, sld, out, cg, **kw)
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    assert flashdec_b200.device_status(clear=True) == 0
    assert torch.equal(out, eager)
    del graph
