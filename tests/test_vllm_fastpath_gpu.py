"""The vLLM launcher's C++ host path (auto plan): a call whose signature was
prepared on this stream launches from C++ with only its pointers replaced.
On new data (new q, cache, append rows and slots, same shapes) its output and
the cache bytes it appends must equal the Python path's bit for bit (the
Python path is forced by clearing the C++ table)."""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from tests.golden.cases import _normal  # noqa: E402

pytestmark = pytest.mark.gpu

B, HQ, HKV, D, BS = 6, 16, 2, 128, 16
POOL, WIDTH = 300, 48  # every case: the same cache and table shapes


def _case(seed):
    rng = np.random.default_rng(seed)
    lens = [int(x) for x in rng.integers(1, 700, size=B)]
    nblk = [-(-n // BS) for n in lens]
    perm = rng.permutation(POOL)
    bt = np.zeros((B, WIDTH), np.int32)
    at = 0
    for i, n in enumerate(nblk):
        bt[i, :n] = perm[at:at + n]
        at += n
    pos = np.asarray(lens, np.int64) - 1
    slots = bt[np.arange(B), pos // BS].astype(np.int64) * BS + pos % BS

    def t(shape):
        return torch.from_numpy(_normal(rng, shape, "bfloat16")).to(torch.bfloat16).cuda()

    return dict(q=t((B, HQ, D)), ak=t((B, HKV, D)), av=t((B, HKV, D)),
                kv=t((POOL, 2, BS, HKV, D)),
                bt=torch.from_numpy(bt).cuda(), sl=torch.tensor(lens, dtype=torch.int32).cuda(),
                slot=torch.from_numpy(slots).cuda())


def _call(c, kv, out):
    from flashdec_b200.kernels.paged_decode import _vllm_paged_decode_attention_into

    acc = torch.empty((B, HQ, 16, D), dtype=torch.float32, device="cuda")
    mx = torch.empty((B, HQ, 16), dtype=torch.float32, device="cuda")
    _vllm_paged_decode_attention_into(c["q"], c["ak"], c["av"], kv, c["bt"], c["sl"], out,
                                      c["slot"], acc, mx, torch.empty_like(mx), num_reqs=B,
                                      num_q_heads=HQ, num_kv_heads=HKV, head_dim=D,
                                      block_size=BS, sm_scale=D ** -0.5, num_splits=0)


def test_cpp_hit_matches_python_path_bit_for_bit():
    import flashdec_b200
    from flashdec_b200 import _lib

    hp = _lib.load_hostpath()
    hp.clear_vllm()
    first = _case(1)
    _call(first, first["kv"].clone(), torch.empty_like(first["q"]))  # Python path, registers
    for seed in (2, 3):
        c = _case(seed)
        kv_fast, out_fast = c["kv"].clone(), torch.empty_like(c["q"])
        _call(c, kv_fast, out_fast)  # C++ hit
        hp.clear_vllm()
        kv_py, out_py = c["kv"].clone(), torch.empty_like(c["q"])
        _call(c, kv_py, out_py)  # Python path (registers again)
        torch.cuda.synchronize()
        assert flashdec_b200.device_status(clear=True) == 0
        assert torch.equal(out_fast, out_py)
        assert torch.equal(kv_fast, kv_py)
    # a hit returns 0 straight from the C++ call
    c = _case(4)
    rc = hp.vllm_into(c["q"], c["ak"], c["av"], c["kv"], c["bt"], c["sl"], torch.empty_like(c["q"]),
                      c["slot"], B, HQ, HKV, D, BS, float(D ** -0.5))
    torch.cuda.synchronize()
    assert rc == 0
