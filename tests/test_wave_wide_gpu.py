"""The length-balanced one-wave plan past the plain balanced limit (pairs x
tiles above 148 x 32, up to 148 x 64, when the even split covers every SM):
a near-uniform c5-shaped batch (16 requests of 4096 + U[1,1024] tokens,
Qwen2.5-3B attention shape) and a ragged one (one 9000-token request and 15
short ones) against the numpy oracle (flashdec/paged_reference.py:19-125),
against the stream-K plan of the same batch (``max_ctas=148``), and with the
fused current-token append against a manual store followed by a plain
decode (cache bytes equal, outputs within the attention tolerance)."""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle.paged_attention import paged_decode_attention_ref  # noqa: E402
from tests.helpers import assert_attention_close, to_np  # noqa: E402

pytestmark = pytest.mark.gpu

HQ, HKV, D, BS = 16, 2, 128, 32


def _lengths(kind):
    rng = np.random.default_rng(17)
    if kind == "c5like":
        return [4096 + int(x) for x in rng.integers(1, 1025, size=16)]
    return [9000] + [int(x) for x in rng.integers(1, 201, size=15)]


def _batch(lens, seed):
    nblk = [-(-n // BS) for n in lens]
    total = sum(nblk) + 4
    g = torch.Generator(device="cuda").manual_seed(seed)
    k = torch.randn((total, HKV, BS, D), device="cuda", dtype=torch.bfloat16, generator=g)
    v = torch.randn((total, HKV, BS, D), device="cuda", dtype=torch.bfloat16, generator=g)
    perm = torch.randperm(total, device="cuda", generator=g).to(torch.int32)
    bt = torch.full((len(lens), max(nblk)), -1, device="cuda", dtype=torch.int32)
    at = 0
    for i, n in enumerate(nblk):
        bt[i, :n] = perm[at:at + n]
        at += n
    sl = torch.tensor(lens, device="cuda", dtype=torch.int32)
    q = torch.randn((len(lens), HQ, D), device="cuda", dtype=torch.bfloat16, generator=g)
    return dict(lens=lens, nblk=nblk, k=k, v=v, bt=bt, sl=sl, q=q)


def _oracle_row(b, i, k=None, v=None):
    k = b["k"] if k is None else k
    v = b["v"] if v is None else v
    n, nb = b["lens"][i], b["nblk"][i]
    blocks = b["bt"][i, :nb].long()
    kc = k.index_select(0, blocks).float().cpu().numpy()
    vc = v.index_select(0, blocks).float().cpu().numpy()
    q = b["q"][i:i + 1].float().cpu().numpy()
    return paged_decode_attention_ref(q, kc, vc, np.arange(nb, dtype=np.int32)[None],
                                      np.asarray([n], np.int32), sm_scale=D ** -0.5)


def _stream_k(b, k=None, v=None):
    from flashdec_b200 import _native

    out = torch.empty_like(b["q"])
    _native.paged_decode(b["q"], b["k"] if k is None else k, b["v"] if v is None else v,
                         b["bt"], b["sl"], out, sm_scale=D ** -0.5, block_size=BS,
                         num_seqs=len(b["lens"]), num_splits=0, max_ctas=148)
    return out


@pytest.mark.parametrize("kind", ["c5like", "ragged"])
def test_wide_balanced_plan_matches_oracle_and_stream_k(kind):
    import flashdec_b200

    b = _batch(_lengths(kind), seed=5 if kind == "c5like" else 6)
    out = torch.empty_like(b["q"])
    flashdec_b200.paged_decode_attention_into(b["q"], b["k"], b["v"], b["bt"], b["sl"], out)
    ref = _stream_k(b)
    torch.cuda.synchronize()
    assert flashdec_b200.device_status(clear=True) == 0
    got, sk = to_np(out), to_np(ref)
    for i in range(len(b["lens"])):
        assert_attention_close(got[i:i + 1], _oracle_row(b, i))
    assert_attention_close(got, sk)


@pytest.mark.parametrize("kind", ["c5like", "ragged"])
def test_wide_balanced_plan_fused_append(kind):
    """Fused append on the wide plan: the current token (position seq_len-1)
    of every row is stored at its slot by the decode launch itself."""
    import flashdec_b200

    b = _batch(_lengths(kind), seed=7)
    g = torch.Generator(device="cuda").manual_seed(8)
    ak = torch.randn((len(b["lens"]), HKV, D), device="cuda", dtype=torch.bfloat16, generator=g)
    av = torch.randn_like(ak)
    pos = torch.tensor(b["lens"], device="cuda", dtype=torch.int64) - 1
    blk = b["bt"].long().gather(1, (pos // BS)[:, None])[:, 0]
    slots = blk * BS + pos % BS
    k_fused, v_fused = b["k"].clone(), b["v"].clone()
    out = torch.empty_like(b["q"])
    flashdec_b200.paged_decode_attention_into(b["q"], k_fused, v_fused, b["bt"], b["sl"], out,
                                              append_k=ak, append_v=av, slot_mapping=slots)
    # the same store by hand, then the stream-K decode
    k_ref, v_ref = b["k"].clone(), b["v"].clone()
    k_ref[blk, :, pos % BS] = ak
    v_ref[blk, :, pos % BS] = av
    ref = _stream_k(b, k_ref, v_ref)
    torch.cuda.synchronize()
    assert flashdec_b200.device_status(clear=True) == 0
    assert torch.equal(k_fused, k_ref) and torch.equal(v_fused, v_ref)
    got = to_np(out)
    assert_attention_close(got, to_np(ref))
    for i in (0, len(b["lens"]) - 1):
        assert_attention_close(got[i:i + 1], _oracle_row(b, i, k_ref, v_ref))
