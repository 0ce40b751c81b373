"""fd_paged_decode_static (the entry point that allocates nothing) against
fd_paged_decode, both called through the C ABI.

Two static calls in a row must agree with the regular entry point (same
kernel, same plan) and with the numpy oracle.  The cases include plans that
merge through the tickets and the fp32 partials of the static storage (the
length-balanced schedule, an explicit split, and the small-batch split with
clusters off), so the second call proves the first left its tickets at zero
and the storage holds correct partials.  This file is collected last and
builds everything it needs itself, so it passes alone in a fresh process as
well as after the other GPU tests."""

from __future__ import annotations

import ctypes
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle.paged_attention import paged_decode_attention_ref  # noqa: E402
from tests.golden.cases import _normal  # noqa: E402
from tests.helpers import assert_attention_close, to_dev, to_np  # noqa: E402

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def _args(q, k4, v4, bt, sl, out, sm_scale, block_size):
    from flashdec_b200 import _lib

    a = _lib.PagedDecodeArgs()
    a.struct_size = ctypes.sizeof(a)
    a.dtype = _lib.FD_DTYPE_BF16 if q.dtype == torch.bfloat16 else _lib.FD_DTYPE_F16
    a.num_seqs, a.num_q_heads, a.head_dim = q.shape
    a.num_kv_heads = k4.shape[1]
    a.block_size = block_size
    a.num_blocks = k4.shape[0]
    a.max_blocks_per_seq = bt.shape[1]
    a.sm_scale = sm_scale
    a.q, a.out = q.data_ptr(), out.data_ptr()
    a.q_stride[:] = q.stride()
    a.out_stride[:] = out.stride()
    a.k_cache, a.v_cache = k4.data_ptr(), v4.data_ptr()
    a.k_stride[:] = k4.stride()
    a.v_stride[:] = v4.stride()
    a.block_tables = bt.data_ptr()
    a.block_tables_index = _lib.FD_INDEX_I32
    a.block_tables_stride[:] = bt.stride()
    a.seq_lens = sl.data_ptr()
    a.seq_lens_index = _lib.FD_INDEX_I32
    a.seq_lens_stride = sl.stride(0)
    return a


def _case(seed, lens, hq=16, hkv=2, d=128, bs=32):
    rng = np.random.default_rng(seed)
    nblk = [max(1, -(-n // bs)) for n in lens]
    pool = 2 * sum(nblk)
    q = _normal(rng, (len(lens), hq, d), "bfloat16")
    k = _normal(rng, (pool, hkv, bs, d), "bfloat16")
    v = _normal(rng, (pool, hkv, bs, d), "bfloat16")
    perm = rng.permutation(pool)
    bt = np.zeros((len(lens), max(nblk)), np.int32)
    pos = 0
    for i, n in enumerate(nblk):
        bt[i, :n] = perm[pos:pos + n]
        pos += n
    return q, k, v, bt, np.asarray(lens, np.int32)


def _regular_and_static(lens, hq=16, hkv=2, bs=32, num_splits=0, seed=7):
    """One call of fd_paged_decode with a caller-owned zero-filled workspace
    and two static calls in a row; returns (regular out, [static outs],
    workspace need, inputs)."""
    from flashdec_b200 import _lib

    lib = _lib.load_library()
    q, k, v, bt, sl = _case(seed, lens, hq=hq, hkv=hkv, bs=bs)
    dq, dk, dv = to_dev(q, "bfloat16"), to_dev(k, "bfloat16"), to_dev(v, "bfloat16")
    dbt, dsl = to_dev(bt), to_dev(sl)
    scale = 128 ** -0.5
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    ref_out = torch.empty_like(dq)
    a = _args(dq, dk, dv, dbt, dsl, ref_out, scale, bs)
    a.num_splits = num_splits
    scratch_bytes, tickets_needed = ctypes.c_size_t(0), ctypes.c_int64(0)
    _lib.check(lib.fd_paged_decode_workspace(ctypes.byref(a), ctypes.byref(scratch_bytes),
                                             ctypes.byref(tickets_needed)), "workspace")
    tickets = torch.zeros(max(1, tickets_needed.value), dtype=torch.int32, device="cuda")
    scratch = torch.empty(max(1, (scratch_bytes.value + 3) // 4), dtype=torch.float32,
                          device="cuda")
    a.tickets, a.tickets_capacity = tickets.data_ptr(), tickets.numel()
    a.scratch, a.scratch_bytes = scratch.data_ptr(), scratch.numel() * 4
    _lib.check(lib.fd_paged_decode(ctypes.byref(a), stream), "fd_paged_decode")

    outs = []
    for _ in range(2):  # two calls in a row: the static tickets must be re-armed
        out = torch.full_like(dq, float("nan"))
        s = _args(dq, dk, dv, dbt, dsl, out, scale, bs)
        s.num_splits = num_splits
        _lib.check(lib.fd_paged_decode_static(ctypes.byref(s), stream), "static")
        outs.append(out)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    return ref_out, outs, (scratch_bytes.value, tickets_needed.value), (q, k, v, bt, sl, scale)


def _check(lens, **kw):
    ref_out, outs, need, (q, k, v, bt, sl, scale) = _regular_and_static(lens, **kw)
    want = paged_decode_attention_ref(q, k, v, bt, sl, sm_scale=scale)
    for out in outs:
        assert_attention_close(to_np(out), want)
        assert torch.equal(out, ref_out)
    return need


@pytest.mark.parametrize("lens", [[2048] * 8, [1, 517, 4096, 33, 2000, 0, 129]])
def test_static_entry_point_matches_regular_entry_point(lens):
    _check(lens)


def test_static_storage_carries_stream_k_tickets_and_partials():
    # 64 sequences x 8 KV heads = 512 (sequence, KV head) pairs: more pairs
    # than SMs, so the length-balanced schedule cuts pairs across CTAs, which
    # merge through the tickets and the fp32 partial slots of the storage
    rng = np.random.default_rng(3)
    lens = [int(x) for x in rng.integers(200, 1400, size=64)]
    scratch_bytes, tickets = _check(lens, hq=32, hkv=8, bs=16)
    assert tickets > 0 and scratch_bytes > 0


def test_static_storage_carries_explicit_split_merge():
    # the reference's fixed split (3 chunks per sequence), merged in the
    # kernel through the tickets and the partials of the storage
    scratch_bytes, tickets = _check([2048] * 8, num_splits=3)
    assert tickets > 0 and scratch_bytes > 0


def test_static_storage_carries_the_small_batch_ticket_merge():
    # with thread-block clusters off, the small-batch plan merges its splits
    # through the tickets and partials as well; run in a fresh process (the
    # switch is read once per process)
    code = (
        "import sys; sys.path.insert(0, %r)\n"
        "from tests.test_zz_no_alloc import _check\n"
        "need = _check([2048] * 8)\n"
        "assert need[0] > 0 and need[1] > 0, need\n"
        "need = _check([1, 517, 4096, 33, 2000, 0, 129])\n"
        "print('ok')\n" % str(ROOT)
    )
    env = dict(os.environ, FLASHDEC_B200_CLUSTER="0")
    res = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True,
                         text=True, timeout=600)
    assert res.returncode == 0 and "ok" in res.stdout, res.stderr[-3000:]


def test_static_entry_point_rejects_requests_beyond_its_storage():
    from flashdec_b200 import _lib

    lib = _lib.load_library()
    # 4097 sequences x 8 KV heads need > 4096 tickets and > 8 MiB of slots
    q = torch.zeros((4097, 8, 128), dtype=torch.bfloat16, device="cuda")
    k4 = torch.zeros((1, 8, 16, 128), dtype=torch.bfloat16, device="cuda")
    bt = torch.zeros((4097, 1), dtype=torch.int32, device="cuda")
    sl = torch.ones(4097, dtype=torch.int32, device="cuda")
    out = torch.full_like(q, 7.0)
    a = _args(q, k4, k4, bt, sl, out, 1.0, 16)
    rc = lib.fd_paged_decode_static(ctypes.byref(a),
                                    ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == _lib.FD_ERR_CAPACITY
    assert b"static storage" in lib.fd_error_string(rc)
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())  # nothing was launched
